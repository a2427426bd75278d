"""CPU model of the cluster kernel's heavy-tie fallback (`exact_select` in csrc/fs_sample.cu).

When more keys reach the filter threshold L than the survivor buffer holds, every rank of the
cluster counts its keys at L, L+1, L+2, L+3 and at or above L+4; the per-rank totals give the k-th
key T, the count above it and each rank's offsets without a radix select whenever T lies in
[L, L+3]. The keys above T are stored at (rank, thread, chunk) positions and the ties at T are
ranked in (rank, chunk, thread, lane) order, which is id order, and the lowest-id ones kept.

These tests restate that bookkeeping in numpy, skipping the ranks and chunks the kernel skips, and
check on tie-heavy rows that the positions it assigns fill [0, k) exactly once and hold the
oracle's top-k set. They run on the CPU; the kernel itself is compared with
the oracle on the same kinds of rows by the GPU tests.
"""

import numpy as np
import pytest
import torch

from oracle import sampler_oracle as orc

NT = 256
BINS = 5


def slice_layout(V, S, C):
    """ids of the row as [S, C, NT, 8] (rank, chunk, thread, lane); -1 past the row end."""
    ids = np.arange(S * C * NT * 8, dtype=np.int64).reshape(S, C, NT, 8)
    return np.where(ids < V, ids, -1)


def fallback(keys, k, L, S, C):
    """The kernel's decision and positions. Returns (T, positions dict id -> slot) or None when T
    lies above L + 3 (the kernel then runs its radix levels)."""
    V = keys.shape[0]
    ids = slice_layout(V, S, C)
    valid = ids >= 0
    kk = keys[np.where(valid, ids, 0)].astype(np.int64)
    kk = np.where(valid, kk, -1)
    # per-thread bins: [S, NT, BINS]
    d = np.where(kk >= L, np.minimum(kk - L, BINS - 1), -1)
    per_thread = np.stack([(d == j).sum(axis=(1, 3)) for j in range(BINS)], axis=-1)  # [S, NT, 5]
    per_rank = per_thread.sum(axis=1)  # [S, 5]
    row = per_rank.sum(axis=0)
    known = None
    above = row[BINS - 1]
    for j in range(BINS - 2, -1, -1):
        if above < k <= above + row[j]:
            known = j
            break
        above += row[j]
    if known is None:
        return None
    j = known
    T = L + j
    n_gt = int(row[j + 1:].sum())
    need = k - n_gt
    pos = {}
    for s in range(S):
        gt_base = int(per_rank[:s, j + 1:].sum())
        tie_base = int(per_rank[:s, j].sum())
        ngt = per_thread[s, :, j + 1:].sum(axis=-1)
        gt_rank = int(ngt.sum())
        gt_off = np.cumsum(ngt) - ngt
        if gt_rank == 0 and tie_base >= need:
            continue  # the kernel skips this rank (the caller checks that [0, k) still fills)
        slot = gt_base + gt_off  # per thread, advanced in chunk order
        chunk_base = tie_base
        for c in range(C):
            for t in range(NT):
                for lane in range(8):
                    if kk[s, c, t, lane] > T:
                        pos[int(ids[s, c, t, lane])] = int(slot[t])
                        slot[t] += 1
            if chunk_base < need:
                tie = kk[s, c] == T  # [NT, 8]
                cnt = tie.sum(axis=1)
                excl = np.cumsum(cnt) - cnt
                for t in np.nonzero(cnt)[0]:
                    r = chunk_base + excl[t]
                    for lane in np.nonzero(tie[t])[0]:
                        if r < need:
                            pos[int(ids[s, c, t, lane])] = n_gt + int(r)
                        r += 1
                chunk_base += int(cnt.sum())
            # else: the kernel skips the ranking; every later tie ranks past the kept ones
    return T, pos


def adjacent_key_row(V, counts, dtype, rng):
    one = int(torch.tensor(1.0, dtype=dtype).view(torch.int16).item())
    r = torch.full((V,), -1.0, dtype=dtype).view(torch.int16)
    perm = torch.from_numpy(rng.permutation(V))
    p = 0
    for i, c in enumerate(counts):
        r[perm[p:p + c]] = one + i
        p += c
    return r.view(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("V,S,C", [(20000, 4, 3), (40000, 8, 3), (151936, 16, 5)])
def test_positions_fill_the_top_k_exactly(dtype, V, S, C):
    assert S * C * NT * 8 >= V
    rng = np.random.default_rng(V + S)
    profiles = [[V // 16] * 8, [0] * 7 + [V // 10], [V // 20] * 4 + [40, 10, 5, 1],
                [0, 0, 0, V // 8, 0, 0, 0, 1], [V // 8] + [0] * 6 + [30], [0, V // 30, 0, V // 30, 0, V // 30, 0, V // 30]]
    resolved = fell_back = 0
    for counts in profiles:
        x = adjacent_key_row(V, counts, dtype, rng)
        keys = orc.order_keys(orc.bits16(x[None]))[0].astype(np.int64)
        for k in (1, 20, 50, 256, 1024):
            want = orc.topk_order(orc.bits16(x[None]), k)[0]
            kth = int(keys[want[-1]])
            for back in range(0, 7):
                L = kth - back
                if (keys >= L).sum() < k:
                    continue
                out = fallback(keys, k, L, S, C)
                if out is None:
                    assert (keys >= L + 4).sum() >= k  # T above L + 3: the radix levels run
                    fell_back += 1
                    continue
                T, pos = out
                assert T == kth
                slots = sorted(pos.values())
                assert slots == list(range(k))
                assert set(pos) == set(int(i) for i in want)
                resolved += 1
    assert resolved > 0 and fell_back > 0


def test_sixteen_value_rows_resolve_without_the_radix_levels():
    # the FP16 anchored threshold is the floor of a four-key bin below the top value
    g = torch.Generator().manual_seed(5)
    levels = torch.linspace(-3.0, 3.0, 16)
    x = levels[torch.randint(0, 16, (1, 151936), generator=g)].to(torch.float16)
    keys = orc.order_keys(orc.bits16(x))[0].astype(np.int64)
    top = int(keys.max())
    for k in (20, 50, 1024):
        T, pos = fallback(keys, k, top - 3, 16, 5)
        assert T == top
        assert set(pos) == set(int(i) for i in orc.topk_order(orc.bits16(x), k)[0])
