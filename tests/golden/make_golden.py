"""Generate golden vectors by running the reference's own CPU oracle.

Imports ``benchmarks/reference.py`` of sathviknookala/llm_sampling_kernel from a local checkout
(``--reference PATH``; the default is the checkout location of the build machine) and records, for seeded inputs, every
stage ``sample_eager(..., return_stages=True)`` returns. The output ``golden_stages.npz`` is
committed; the tests read it and never need the reference itself.

Run:  python tests/golden/make_golden.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    """benchmarks/reference.py uses a relative import, so import it as benchmarks.reference."""
    sys.path.insert(0, str(root))
    return importlib.import_module("benchmarks.reference")


def cases():
    """(name, logits, k, p) tuples; logits are CPU tensors."""
    out = []
    g = torch.Generator().manual_seed(20261201)
    for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        x = (torch.randn(4, 4000, generator=g) * 4).to(dtype)
        for k in (1, 20, 50, 100, 256):
            for p in (0.5, 0.9, 1.0):
                out.append((f"randn4_{tag}_k{k}_p{p}", x, k, p))
        # 30% of entries on a 0.25 grid: ties and signed zeros everywhere
        y = torch.randn(4, 4000, generator=g)
        m = torch.rand(4, 4000, generator=g) < 0.3
        y = torch.where(m, torch.round(y * 4) / 4, y).to(dtype)
        for k in (50, 256):
            out.append((f"grid_{tag}_k{k}_p0.9", y, k, 0.9))
        # narrow range: dense ties at the k boundary
        z = (torch.randn(4, 4000, generator=g) * 0.05).to(dtype)
        for k in (20, 100):
            out.append((f"dense_{tag}_k{k}_p0.95", z, k, 0.95))
        # signed zeros straddling the k boundary
        s = torch.full((2, 64), -1.0)
        s[0, ::3] = 0.0
        s[0, 1::3] = -0.0
        s[1, 10:20] = -0.0
        s[1, 30:40] = 0.0
        out.append((f"signed_zero_{tag}_k12_p1.0", s.to(dtype), 12, 1.0))
        # -inf masked tail, k larger than the finite count
        w = torch.randn(3, 200, generator=g)
        w[:, 100:] = float("-inf")
        out.append((f"neginf_tail_{tag}_k150_p1.0", w.to(dtype), 150, 1.0))
        out.append((f"neginf_tail_{tag}_k150_p0.9", w.to(dtype), 150, 0.9))
    # known answers of the reference tests (tests/test_reference.py, tests/test_fused_kernel.py)
    probs = torch.tensor([0.40, 0.30, 0.15, 0.10, 0.05])
    out.append(("hand_cut_f32", probs.log().unsqueeze(0), 5, 0.9))
    out.append(("equal4_f32", torch.zeros(1, 4), 4, 0.5))
    alt = torch.zeros(1, 64)
    alt[0, ::2] = 1.0
    out.append(("alternating_f32", alt, 8, 1.0))
    bt = torch.zeros(1, 20)
    bt[0, 3:12] = 5.0
    out.append(("boundary_tie_f32", bt, 5, 1.0))
    for p in (0.25, 0.5, 0.75, 0.875):
        e8 = torch.full((2, 4000), -30.0)
        e8[:, :8] = 10.0
        out.append((f"equal8_bf16_p{p}", e8.to(torch.bfloat16), 8, p))
    out.append(("small_vocab_bf16_k10", (torch.randn(3, 7, generator=g) * 2).to(torch.bfloat16), 10, 0.9))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--out", default=str(HERE / "golden_stages.npz"))
    args = ap.parse_args()
    ref = load_reference(Path(args.reference))
    arrays = {}
    names = []
    for name, x, k, p in cases():
        st = ref.sample_eager(x, k, p, generator=torch.Generator().manual_seed(0), check_inputs=True,
                              return_stages=True)
        names.append(name)
        if x.dtype in (torch.float16, torch.bfloat16):
            arrays[f"{name}/bits"] = x.contiguous().view(torch.int16).numpy().view(np.uint16)
            arrays[f"{name}/dtype"] = np.array("bf16" if x.dtype == torch.bfloat16 else "f16")
        else:
            arrays[f"{name}/f32"] = x.numpy().astype(np.float32)
            arrays[f"{name}/dtype"] = np.array("f32")
        arrays[f"{name}/k"] = np.array(k)
        arrays[f"{name}/p"] = np.array(p)
        arrays[f"{name}/topk_ids"] = st.topk_ids.numpy().astype(np.int32)
        arrays[f"{name}/topk_logits"] = st.topk_logits.numpy().astype(np.float32)
        arrays[f"{name}/probs"] = st.probs.numpy().astype(np.float32)
        arrays[f"{name}/cumsum"] = st.cumsum.numpy().astype(np.float32)
        arrays[f"{name}/keep"] = st.keep.numpy()
        arrays[f"{name}/cutoff"] = st.cutoff.numpy().astype(np.int32)
        arrays[f"{name}/renormed"] = st.renormed.numpy().astype(np.float32)
    arrays["names"] = np.array(names)
    arrays["torch_version"] = np.array(torch.__version__)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {len(names)} cases to {args.out}")


if __name__ == "__main__":
    main()
