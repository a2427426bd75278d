"""Convert the output of oracle/_ref/ref_rng_probe (the reference's own rng_uniform and
mono_key, csrc/fused_sampling.cuh:8-11,65-71, evaluated on a GPU) into ref_rng_vectors.npz.

Run on a GPU machine:  make -f oracle/Makefile && ./oracle/_ref/ref_rng_probe > probe.txt
then:                  python tests/golden/make_rng_golden.py probe.txt
"""

import sys
from pathlib import Path

import numpy as np


def main(path: str) -> None:
    seeds, offs, rows, ubits = [], [], [], []
    keys = np.zeros(65536, dtype=np.uint16)
    for line in Path(path).read_text().splitlines():
        parts = line.split()
        if not parts or parts[0].startswith("#"):
            continue
        if parts[0] == "u":
            seeds.append(int(parts[1]))
            offs.append(int(parts[2]))
            rows.append(int(parts[3]))
            ubits.append(int(parts[4], 16))
        elif parts[0] == "k":
            keys[int(parts[1])] = int(parts[2])
    out = Path(__file__).resolve().parent / "ref_rng_vectors.npz"
    np.savez_compressed(out, seed=np.array(seeds, dtype=np.uint64), offset=np.array(offs, dtype=np.uint64),
                        row=np.array(rows, dtype=np.uint32), u_bits=np.array(ubits, dtype=np.uint32),
                        mono_key=keys)
    print(f"wrote {len(seeds)} uniforms and 65536 keys to {out}")


if __name__ == "__main__":
    main(sys.argv[1])
