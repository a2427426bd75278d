"""CPU oracle of the fused top-k / top-p sampling path.

TEST INFRASTRUCTURE ONLY. This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``
arm) may import it. The package ``llm_sampling_kernel_b200`` never does, and has no CPU
fallback.

It restates the reference's semantics (sathviknookala/llm_sampling_kernel):

* selection -- ``benchmarks/reference.py:47-54``: cast to FP32, stable descending sort, keep the
  first ``k = min(top_k, V)``; equal values keep the lowest token id first. Restated here on the
  16-bit order key of the input (integer radix sort), which orders FP16/BF16 values exactly as
  their FP32 casts do (both zeros tie).
* probabilities -- ``benchmarks/reference.py:55-65``: softmax over the k survivors, cumulative
  sum, exclusive-prefix top-p mask ``(cumsum - probs) < top_p`` (all kept when ``top_p >= 1``),
  renormalisation. Computed with torch's CPU FP32 operators so the values are those of the
  reference on a CPU.
* validation -- ``benchmarks/reference.py:20-26``.
* the seeded uniform -- ``csrc/fused_sampling.cuh:65-71`` (splitmix64 of
  ``seed + offset * 0x9E3779B97F4A7C15 + row * 0xD1B54A32D192ED03``, top 24 bits / 2**24).
* the draw -- ``csrc/fused_sampling.cu:285-309``: ``r`` = last kept index, target
  ``u * cumsum[r]``, pick the first ``i <= r`` with ``cumsum[i] >= target``.

Pinned by ``tests/test_oracle.py`` against golden vectors made by running the reference's own
``sample_eager`` (``tests/golden/make_golden.py``), the reference tests' known answers, and the
published first output of splitmix64 from state 0.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

MASK64 = (1 << 64) - 1
GOLDEN_GAMMA = 0x9E3779B97F4A7C15
ROW_MULT = 0xD1B54A32D192ED03


# ---------------------------------------------------------------------------------------------
# integer keys and selection
# ---------------------------------------------------------------------------------------------


def bits16(logits: torch.Tensor) -> np.ndarray:
    """Raw 16-bit patterns of an FP16/BF16 tensor as uint16 numpy."""
    if logits.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("logits must be float16 or bfloat16")
    return logits.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def order_keys32(x: np.ndarray) -> np.ndarray:
    """Order-preserving 32-bit key of float32 values (-0 folded onto +0), for FP32 inputs."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = np.where(b == 0x80000000, 0, b)
    neg = (b & 0x80000000) != 0
    return np.where(neg, (~b) & 0xFFFFFFFF, b | 0x80000000).astype(np.uint32)


def topk_ids_any(logits: torch.Tensor, k: int) -> np.ndarray:
    """[B, k] ids for FP16/BF16 (16-bit keys) or FP32 (32-bit keys) logits."""
    if logits.dtype == torch.float32:
        inv = (np.uint64(0xFFFFFFFF) - order_keys32(logits.detach().cpu().numpy()).astype(np.uint64))
        return np.argsort(inv, axis=-1, kind="stable")[:, :k].astype(np.int64)
    return topk_order(bits16(logits), k)


def order_keys(bits: np.ndarray) -> np.ndarray:
    """Order-preserving 16-bit key; -0 (0x8000) is folded onto +0 first (both zeros tie).

    Negative patterns map to ~bits, non-negative ones to bits | 0x8000, so a larger key is a
    larger value -- the reference kernel's mono_key (csrc/fused_sampling.cuh:8-11) plus the fold.
    """
    b = bits.astype(np.uint32)
    b = np.where(b == 0x8000, 0, b)
    neg = (b & 0x8000) != 0
    return np.where(neg, (~b) & 0xFFFF, b | 0x8000).astype(np.uint16)


def topk_order(bits: np.ndarray, k: int) -> np.ndarray:
    """[B, k] token ids: value descending, id ascending (a stable sort on the inverted key)."""
    inv = (0xFFFF - order_keys(bits).astype(np.int32)).astype(np.uint16)
    order = np.argsort(inv, axis=-1, kind="stable")
    return order[:, :k].astype(np.int64)


def packed(keys: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """Packed candidates (key << 32) | (0xFFFFFFFF - id) as uint64 (the shard exchange format)."""
    return (keys.astype(np.uint64) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))


# ---------------------------------------------------------------------------------------------
# validation
# ---------------------------------------------------------------------------------------------

ROW_OK, ROW_NAN, ROW_POSINF, ROW_ALL_NEGINF, ROW_BAD_PARAM = 0, 1, 2, 3, 4


def row_status(logits: torch.Tensor) -> np.ndarray:
    """Per-row rejection code, in the reference's order of checks (benchmarks/reference.py:20-26)."""
    x = logits.detach().cpu().float()
    st = np.zeros(x.shape[0], dtype=np.int32)
    ninf = torch.isneginf(x).all(dim=-1).numpy()
    pinf = torch.isposinf(x).any(dim=-1).numpy()
    nan = torch.isnan(x).any(dim=-1).numpy()
    st[ninf] = ROW_ALL_NEGINF
    st[pinf] = ROW_POSINF
    st[nan] = ROW_NAN
    return st


def validate_logits(logits: torch.Tensor) -> None:
    """Raises ValueError with the reference's messages."""
    st = row_status(logits)
    if (st == ROW_NAN).any():
        raise ValueError("logits contain NaN")
    if (st == ROW_POSINF).any():
        raise ValueError("logits contain +inf")
    if (st == ROW_ALL_NEGINF).any():
        raise ValueError("logits contain a row that is entirely -inf")


# ---------------------------------------------------------------------------------------------
# stages
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class Stages:
    topk_logits: torch.Tensor  # [B, K] float32
    topk_ids: torch.Tensor  # [B, K] int64
    probs: torch.Tensor  # [B, K] float32
    cumsum: torch.Tensor  # [B, K] float32
    keep: torch.Tensor  # [B, K] bool
    cutoff: torch.Tensor  # [B] int64
    renormed: torch.Tensor  # [B, K] float32


def _check_args(logits: torch.Tensor, top_k: int, top_p: float) -> None:
    if logits.dim() != 2:
        raise ValueError(f"logits must be [B, V], got shape {tuple(logits.shape)}")
    if top_k < 1:
        raise ValueError(f"top_k must be >= 1, got {top_k}")
    if not 0.0 < top_p <= 1.0:
        raise ValueError(f"top_p must be in (0, 1], got {top_p}")


def stages(logits: torch.Tensor, top_k: int, top_p: float, check_inputs: bool = False,
           temperature: float = 1.0) -> Stages:
    """Every intermediate of the reference pipeline, on CPU.

    temperature (not in the reference, which leaves it to the caller): the top-k logits are divided
    by T in fp32 before the softmax, i.e. the pipeline run on fp32 ``logits / T``; the top-k order
    is that of the raw logits, since fp32 division by T > 0 keeps the order of 16-bit values."""
    _check_args(logits, top_k, top_p)
    if check_inputs:
        validate_logits(logits)
    k = min(top_k, logits.shape[-1])
    ids = torch.from_numpy(topk_ids_any(logits, k))
    x = logits.detach().cpu().float()
    topk_logits = x.gather(-1, ids)
    if temperature != 1.0:
        topk_logits = topk_logits / temperature
    probs = torch.softmax(topk_logits, dim=-1)
    cumsum = probs.cumsum(dim=-1)
    if top_p >= 1.0:
        keep = torch.ones_like(probs, dtype=torch.bool)
    else:
        keep = (cumsum - probs) < top_p
    filtered = torch.where(keep, probs, torch.zeros_like(probs))
    renormed = filtered / filtered.sum(dim=-1, keepdim=True)
    return Stages(topk_logits, ids, probs, cumsum, keep, keep.sum(dim=-1), renormed)


# ---------------------------------------------------------------------------------------------
# the seeded uniform and the draw
# ---------------------------------------------------------------------------------------------


def splitmix64_finalize(z: int) -> int:
    z &= MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def splitmix_uniform(seed: int, offset: int, row: int) -> np.float32:
    """The reference kernel's per-row uniform (csrc/fused_sampling.cuh:65-71), bit-exact."""
    z = (seed + offset * GOLDEN_GAMMA + row * ROW_MULT) & MASK64
    top24 = splitmix64_finalize(z) >> 40
    return np.float32(top24) * np.float32(1.0 / 16777216.0)


def splitmix_uniforms(seed: int, offset: int, rows: int, row_base: int = 0) -> np.ndarray:
    return np.array([splitmix_uniform(seed, offset, row_base + r) for r in range(rows)], dtype=np.float32)


@dataclass(frozen=True)
class Draw:
    ids: np.ndarray  # [B] int64 sampled token ids
    pick: np.ndarray  # [B] rank of the sampled token inside the top-k order
    near_boundary: np.ndarray  # [B] bool: u * Z_p within rel_tol of a CDF step, or a cut tie
    stages: Stages


def draw(st: Stages, u: np.ndarray, top_p: float | np.ndarray, rel_tol: float | np.ndarray = 1e-6,
         cut_tol: float | np.ndarray | None = None) -> Draw:
    """Inverse-CDF draw with the reference kernel's rule over the oracle's stages.

    r is the last index of the exclusive-prefix keep mask, Z_p = cumsum[r], target = u * Z_p,
    pick = first i <= r with cumsum[i] >= target. A row is flagged near a boundary when the
    target is within rel_tol * Z_p of cumsum[pick] or cumsum[pick - 1], or when some exclusive
    prefix lies within cut_tol of top_p (default 4 ulp of top_p: the cut itself is then
    rounding-sensitive). rel_tol and cut_tol may be per-row arrays.
    """
    cum = st.cumsum.numpy().astype(np.float32)
    probs = st.probs.numpy().astype(np.float32)
    keep = st.keep.numpy()
    B, K = cum.shape
    p_rows = np.broadcast_to(np.asarray(top_p, dtype=np.float64), (B,))
    rel_rows = np.broadcast_to(np.asarray(rel_tol, dtype=np.float64), (B,))
    cut_rows = None if cut_tol is None else np.broadcast_to(np.asarray(cut_tol, dtype=np.float64), (B,))
    ids = np.empty(B, dtype=np.int64)
    picks = np.empty(B, dtype=np.int64)
    near = np.zeros(B, dtype=bool)
    topk_ids = st.topk_ids.numpy()
    for b in range(B):
        r = int(keep[b].sum()) - 1
        # the kernel's r is the first failing index - 1 (prefix form)
        fails = np.nonzero(~keep[b])[0]
        if fails.size:
            r = int(fails[0]) - 1
        zp = np.float32(cum[b, r])
        target = np.float32(np.float32(u[b]) * zp)
        hits = np.nonzero(cum[b, : r + 1] >= target)[0]
        pick = int(hits[0]) if hits.size else r
        picks[b] = pick
        ids[b] = topk_ids[b, pick]
        tol = float(rel_rows[b]) * float(zp)
        if abs(float(cum[b, pick]) - float(target)) <= tol:
            near[b] = True
        if pick > 0 and abs(float(cum[b, pick - 1]) - float(target)) <= tol:
            near[b] = True
        if p_rows[b] < 1.0:
            excl = (cum[b] - probs[b]).astype(np.float32)
            pf = np.float32(p_rows[b])
            window = 4 * float(np.spacing(pf)) if cut_rows is None else max(4 * float(np.spacing(pf)), float(cut_rows[b]))
            if np.any(np.abs(excl.astype(np.float64) - float(pf)) <= window):
                near[b] = True
    return Draw(ids, picks, near, st)


def fp32_cumsum_error(st: Stages) -> np.ndarray:
    """Per row, the largest relative deviation of the stages' FP32 cumulative sum (torch's CPU
    softmax over the top-k, then cumsum) from the same quantity in FP64. Over tens of thousands of
    candidates torch's FP32 softmax normaliser drifts by several 1e-6, so this bounds how far the
    reference's own CDF can sit from any other correct implementation's."""
    x = st.topk_logits.double()
    p64 = torch.softmax(x, dim=-1)
    c64 = p64.cumsum(dim=-1)
    c32 = st.cumsum.double()
    rel = ((c32 - c64).abs() / c64.clamp_min(1e-300)).max(dim=-1).values
    return rel.numpy()


def pick_consistent(st: Stages, ids: np.ndarray, u: np.ndarray, top_p: float | np.ndarray,
                    rel_tol: float | np.ndarray = 1e-6, fp64: bool = True) -> np.ndarray:
    """Per row: is token ids[b] a pick the draw rule allows up to rounding? With k near V the
    CDF steps near the target are far below any useful tolerance, so comparing picks by index
    says little; this checks the pick's CDF interval instead. With c the cumulative sum (FP64 of
    the same top-k logits when fp64, else the stages' FP32 one) and the cut r (first i >= 1 with
    c_i - p_i >= top_p, minus 1), allowing every r whose exclusive prefix is within 4 ulp (FP32)
    of top_p plus rel_tol * top_p: the token is in the top-k at a position pos <= the largest
    allowed r, and c[pos-1] - tol <= u * Z_p and c[pos] + tol >= u * Z_p for some allowed Z_p,
    with tol = rel_tol * Z_p."""
    if fp64:
        p = torch.softmax(st.topk_logits.double(), dim=-1).numpy()
        c = np.cumsum(p, axis=-1)
    else:
        p = st.probs.numpy().astype(np.float64)
        c = st.cumsum.numpy().astype(np.float64)
    B, K = c.shape
    p_rows = np.broadcast_to(np.asarray(top_p, dtype=np.float64), (B,))
    rel_rows = np.broadcast_to(np.asarray(rel_tol, dtype=np.float64), (B,))
    topk_ids = st.topk_ids.numpy()
    ok = np.zeros(B, dtype=bool)
    for b in range(B):
        where = np.nonzero(topk_ids[b] == ids[b])[0]
        if where.size != 1:
            continue
        pos = int(where[0])
        if p_rows[b] >= 1.0:
            r_lo = r_hi = K - 1
        else:
            excl = c[b] - p[b]
            band = 4 * float(np.spacing(np.float32(p_rows[b]))) + rel_rows[b] * p_rows[b]
            lo_fail = np.nonzero(excl[1:] >= p_rows[b] - band)[0]  # earliest possible cut
            hi_fail = np.nonzero(excl[1:] >= p_rows[b] + band)[0]  # latest possible cut
            r_lo = int(lo_fail[0]) if lo_fail.size else K - 1
            r_hi = int(hi_fail[0]) if hi_fail.size else K - 1
        if pos > r_hi:
            continue
        z_lo, z_hi = c[b, r_lo], c[b, r_hi]
        tol = rel_rows[b] * z_hi
        t_lo, t_hi = float(u[b]) * z_lo, float(u[b]) * z_hi
        below = c[b, pos - 1] if pos > 0 else 0.0
        ok[b] = below - tol <= t_hi and c[b, pos] + tol >= t_lo
    return ok


def draw_fp64(st: Stages, u: np.ndarray, top_p: float | np.ndarray, rel_tol: float = 1e-6) -> Draw:
    """The same cut and draw over FP64 probabilities of the same top-k logits (the exact
    distribution the reference's FP32 arithmetic approximates). A row is flagged when the target
    lies within rel_tol * Z_p of a CDF step, or some exclusive prefix within 4 ulp (FP32) of
    top_p."""
    x = st.topk_logits.double()
    p64 = torch.softmax(x, dim=-1).numpy()
    c64 = np.cumsum(p64, axis=-1)
    B, K = c64.shape
    p_rows = np.broadcast_to(np.asarray(top_p, dtype=np.float64), (B,))
    ids = np.empty(B, dtype=np.int64)
    picks = np.empty(B, dtype=np.int64)
    near = np.zeros(B, dtype=bool)
    topk_ids = st.topk_ids.numpy()
    for b in range(B):
        excl = c64[b] - p64[b]
        r = K - 1
        if p_rows[b] < 1.0:
            fails = np.nonzero(excl[1:] >= p_rows[b])[0]
            if fails.size:
                r = int(fails[0])  # (index fails[0] + 1) - 1
            if np.any(np.abs(excl - p_rows[b]) <= 4 * float(np.spacing(np.float32(p_rows[b])))):
                near[b] = True
        zp = c64[b, r]
        target = float(u[b]) * zp
        hits = np.nonzero(c64[b, : r + 1] >= target)[0]
        pick = int(hits[0]) if hits.size else r
        picks[b] = pick
        ids[b] = topk_ids[b, pick]
        tol = rel_tol * zp
        if abs(c64[b, pick] - target) <= tol or (pick > 0 and abs(c64[b, pick - 1] - target) <= tol):
            near[b] = True
    return Draw(ids, picks, near, st)


def sample(
    logits: torch.Tensor,
    top_k: int,
    top_p: float,
    seed: int = 0,
    offset: int = 0,
    uniforms: np.ndarray | None = None,
    row_base: int = 0,
    temperature: float = 1.0,
) -> Draw:
    """Token ids for the same per-row uniform the kernel draws (or the caller supplies)."""
    st = stages(logits, top_k, top_p, temperature=temperature)
    B = logits.shape[0]
    u = uniforms if uniforms is not None else splitmix_uniforms(seed, offset, B, row_base)
    return draw(st, np.asarray(u, dtype=np.float32), top_p)


# ---------------------------------------------------------------------------------------------
# exact FP64 categorical (for chi-square tests of the sampled frequencies)
# ---------------------------------------------------------------------------------------------


def categorical_fp64(logits_row: torch.Tensor, top_k: int, top_p: float) -> tuple[np.ndarray, np.ndarray]:
    """(ids, probabilities) of the nucleus in FP64: top-k by the tie rule, softmax, exclusive
    prefix cut, renormalisation."""
    bits = bits16(logits_row.reshape(1, -1))
    k = min(top_k, bits.shape[-1])
    ids = topk_order(bits, k)[0]
    x = logits_row.detach().cpu().double().reshape(-1)[torch.from_numpy(ids)].numpy()
    w = np.exp(x - x.max())
    p = w / w.sum()
    if top_p < 1.0:
        excl = np.cumsum(p) - p
        keep = excl < top_p
        keep[0] = True
        p = np.where(keep, p, 0.0)
    p = p / p.sum()
    nz = p > 0
    return ids[nz], p[nz]


# ---------------------------------------------------------------------------------------------
# synthetic inputs of the benchmark configurations (seeded)
# ---------------------------------------------------------------------------------------------


def anchor_logits(B: int = 1, V: int = 151936, seed: int = 1234, sigma: float = 2.0, boosted: int = 20,
                  boost: float = 8.0, dtype=torch.bfloat16) -> torch.Tensor:
    """C1: i.i.d. N(0, sigma^2) with `boosted` random ids raised by `boost`."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, V, generator=g) * sigma
    for b in range(B):
        idx = torch.randperm(V, generator=g)[:boosted]
        x[b, idx] += boost
    return x.to(dtype)


def grid_logits(B: int, V: int, sigma: float, dtype, seed: int = 0, tie_frac: float = 0.3) -> torch.Tensor:
    """C2: N(0, sigma^2) with a fraction of entries rounded to a 0.25 grid (ties, signed zeros)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, V, generator=g) * sigma
    mask = torch.rand(B, V, generator=g) < tie_frac
    x = torch.where(mask, torch.round(x * 4.0) / 4.0, x)
    return x.to(dtype)


def zipf_logits(B: int, V: int, sigma: float = 3.0, s: float = 1.1, seed: int = 0,
                dtype=torch.bfloat16) -> torch.Tensor:
    """C3: N(0, sigma^2) plus a per-row Zipf(s) log-bias over a random permutation of ids."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, V, generator=g) * sigma
    ranks = torch.arange(1, V + 1, dtype=torch.float32)
    bias = -s * torch.log(ranks)
    bias = bias - bias.mean()
    for b in range(B):
        perm = torch.randperm(V, generator=g)
        x[b, perm] += bias
    return x.to(dtype)


def adversarial_logits(case: int, B: int = 8, V: int = 151936, seed: int = 0, dtype=torch.float16) -> torch.Tensor:
    """C5 cases: 1 = 16 distinct values, 2 = near-flat N(0, 0.1^2), 3 = N(0, 4) (greedy),
    4 = rows mixing +-inf with the most negative finite value."""
    g = torch.Generator().manual_seed(seed)
    if case == 1:
        levels = torch.linspace(-4.0, 4.0, 16)
        x = levels[torch.randint(0, 16, (B, V), generator=g)]
    elif case == 2:
        x = torch.randn(B, V, generator=g) * 0.1
    elif case == 3:
        x = torch.randn(B, V, generator=g) * 2.0
    elif case == 4:
        x = torch.randn(B, V, generator=g) * 2.0
        lowest = torch.finfo(dtype).min
        for b in range(B):
            idx = torch.randperm(V, generator=g)[:64]
            if b % 4 == 0:
                x[b, idx[:32]] = float("-inf")
                x[b, idx[32:]] = lowest
            elif b % 4 == 1:
                x[b, idx[0]] = float("inf")
            elif b % 4 == 2:
                x[b, :] = float("-inf")
            else:
                x[b, :] = lowest
                x[b, idx[:8]] = float("-inf")
    else:
        raise ValueError("case must be 1..4")
    return x.to(dtype)
