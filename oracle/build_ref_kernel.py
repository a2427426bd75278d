"""Builds the reference's own CUDA extension, unchanged, for sm_100a into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: a comparison rung for bench.py (``--rungs``), never the product. The
sources are compiled where they lie in the reference checkout (csrc/bindings.cpp,
csrc/fused_sampling.cu, csrc/probes.cu) with the reference's own compiler flags (setup.py:16-21:
-O3 -std=c++17 --expt-relaxed-constexpr -lineinfo) under the module name ``fused_sampling_ref``;
nothing of them is copied into this repository. The built module keeps the reference's limits
(top_k <= 128).

    python oracle/build_ref_kernel.py [reference checkout]
"""

from __future__ import annotations

import glob
import os
import shutil
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def build(reference: Path) -> Path:
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils import cpp_extension

    csrc = reference / "csrc"
    sources = [str(csrc / n) for n in ("bindings.cpp", "fused_sampling.cu", "probes.cu")]
    bdir = OUT / "build_ref_kernel"
    bdir.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name="fused_sampling_ref",
        sources=sources,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "-std=c++17", "--expt-relaxed-constexpr", "-lineinfo"],
        build_directory=str(bdir),
        with_cuda=True,
        is_python_module=True,
        verbose=False,
    )
    built = sorted(glob.glob(str(bdir / "fused_sampling_ref*.so")))
    if not built:
        raise RuntimeError("the reference extension build produced no shared object")
    target = OUT / ("fused_sampling_ref" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
    shutil.copy2(built[0], target)
    return target


if __name__ == "__main__":
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference")
    print(build(ref))
