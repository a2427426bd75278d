"""Python front end of the B200 fused sampler.

``sample_fused`` and ``topk_fused`` keep the signatures of the reference's
``benchmarks/fused.py:13-21``: ``offset=None`` routes the draw through torch's default CUDA
generator (graph-capture safe: replays advance it), an explicit ``offset`` gives a reproducible
stream, ``splits`` overrides the number of CTAs per row (0 = the measured plan).

``sample`` is the general serving-engine form: per-row ``top_k`` / ``top_p`` tensors,
caller-supplied uniforms, stage outputs and per-row input status.

Every entry point also takes logits in pinned host memory (``tensor.pin_memory()``): the current
CUDA device's kernels read them in place over PCIe (no copy-engine transfer, no staging buffer)
and write the results into pinned host tensors, which hold their values once the current stream
has reached the call (``torch.cuda.current_stream().synchronize()``), as after a non_blocking
copy to the host.
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch

from . import ops

DEFAULT_SEED = 0x5EED

ROW_OK, ROW_NAN, ROW_POSINF, ROW_ALL_NEGINF, ROW_BAD_PARAM, ROW_TIMEOUT = 0, 1, 2, 3, 4, 5
_ROW_MESSAGES = {
    ROW_NAN: "logits contain NaN",
    ROW_POSINF: "logits contain +inf",
    ROW_ALL_NEGINF: "logits contain a row that is entirely -inf",
    ROW_BAD_PARAM: "a per-row top_k < 1 or top_p outside (0, 1]",
}


def sample_fused(logits, top_k, top_p, seed=DEFAULT_SEED, offset=None, splits=0):
    off = -1 if offset is None else offset
    return ops().sample_fused(logits, int(top_k), float(top_p), int(seed), int(off), int(splits))


def topk_fused(logits, top_k, splits=0):
    return ops().topk_fused(logits, int(top_k), int(splits))


def stages_fused(logits, top_k, top_p, seed=0, offset=0, splits=0):
    return ops().stages_fused(logits, int(top_k), float(top_p), int(seed), int(offset), int(splits))


class SampleResult(NamedTuple):
    token_ids: torch.Tensor  # [B] int64 (-1 for rejected rows)
    status: torch.Tensor  # [B] int32 (ROW_*)
    topk_ids: Optional[torch.Tensor]  # [B, K] int64 when stages were requested
    keep: Optional[torch.Tensor]  # [B, K] bool
    renormed: Optional[torch.Tensor]  # [B, K] float32


def sample(
    logits: torch.Tensor,
    top_k,
    top_p,
    *,
    uniforms: Optional[torch.Tensor] = None,
    seed: int = DEFAULT_SEED,
    offset: Optional[int] = None,
    splits: int = 0,
    id_base: int = 0,
    row_base: int = 0,
    return_stages: bool = False,
    check_inputs: bool = False,
    temperature: float = 1.0,
) -> SampleResult:
    """General sampler.

    top_k: int, or an int32 [B] tensor of per-row k (the bound K is its maximum, read on host).
    top_p: float, or a float32 [B] tensor of per-row p.
    uniforms: optional float32 [B] tensor of caller-supplied u in [0, 1).
    check_inputs: raise ValueError (the reference's messages) for NaN / +inf / all -inf rows;
    this synchronises with the device, so keep it off in timed loops.
    temperature: T > 0 divides the selected candidates' logits (IEEE fp32) before the softmax,
    as sampling fp32 ``logits / T`` would; the top-k selection is that of the raw logits
    (fp32 division by T > 0 keeps their order). 1 (or 0) means none.
    """
    k_rows = p_rows = None
    # per-row tensors live on the device the call runs on (logits in pinned host memory are read
    # in place by the current CUDA device)
    dev = logits.device if logits.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if isinstance(top_k, torch.Tensor):
        k_rows = top_k.to(device=dev, dtype=torch.int32).contiguous()
        k_bound = int(k_rows.max().item()) if k_rows.numel() else 1
        k_bound = max(1, k_bound)
    else:
        k_bound = int(top_k)
    if isinstance(top_p, torch.Tensor):
        p_rows = top_p.to(device=dev, dtype=torch.float32).contiguous()
        p_scalar = 1.0
    else:
        p_scalar = float(top_p)
    off = -1 if offset is None else int(offset)
    if uniforms is not None:
        uniforms = uniforms.to(device=dev, dtype=torch.float32).contiguous()
    ids, tk, keep, ren, status = ops().sample_ex(
        logits, k_bound, p_scalar, k_rows, p_rows, uniforms, int(seed), off, int(splits), int(id_base),
        int(row_base), bool(return_stages), 0, float(temperature))
    if check_inputs:
        if not status.is_cuda:
            torch.cuda.current_stream(dev).synchronize()  # host outputs are written by the launch
        bad = status[status != ROW_OK]
        if bad.numel():
            code = int(bad.min().item())
            if code == ROW_TIMEOUT:
                raise RuntimeError("a bounded device wait of the sampling launch ran out")
            raise ValueError(_ROW_MESSAGES.get(code, f"row status {code}"))
    return SampleResult(ids, status, tk, keep, ren)
