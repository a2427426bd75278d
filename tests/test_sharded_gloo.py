"""Multi-process host logic of the sharded layouts, world_size 2 over gloo on CPU.

The CUDA kernels are replaced by an oracle-backed implementation of the same four operator
calls (test infrastructure), so these tests cover the plumbing: shard ranges, the global row
base of the uniform, the shard id base, the candidate exchange layout and rank agreement.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_sampling_kernel_b200.sharded import BatchShardedSampler, VocabShardedSampler, shard_range
from oracle import sampler_oracle as orc


class OracleOps:
    """CPU stand-in for the operator module, built on the oracle."""

    def sample_ex(self, logits, top_k, top_p, k_rows, p_rows, uniforms, seed, offset, splits, id_base, row_base,
                  return_stages):
        u = uniforms.numpy() if uniforms is not None else orc.splitmix_uniforms(seed, offset, logits.shape[0],
                                                                                  row_base)
        d = orc.sample(logits, top_k, top_p, uniforms=u)
        ids = torch.from_numpy(d.ids + id_base)
        return ids, None, None, None, torch.zeros(logits.shape[0], dtype=torch.int32)

    def shard_candidates(self, logits, top_k, id_base, splits):
        bits = orc.bits16(logits)
        ids = orc.topk_order(bits, top_k)
        keys = np.take_along_axis(orc.order_keys(bits), ids, axis=1)
        packed = orc.packed(keys, ids + id_base).view(np.int64)
        status = orc.row_status(logits).astype(np.int64)[:, None]
        return torch.from_numpy(np.concatenate([packed, status], axis=1))

    def merge_sample(self, cand, bf16, top_k, top_p, k_rows, p_rows, uniforms, seed, offset, row_base,
                     temperature=1.0):
        c = cand.numpy()
        parts, B, _ = c.shape
        words = c[:, :, :top_k].transpose(1, 0, 2).reshape(B, parts * top_k).view(np.uint64)
        # exact descending order of the uint64 words
        order = np.argsort(~words, axis=1, kind="stable")
        best = np.take_along_axis(words, order, axis=1)[:, :top_k]
        keys = (best >> np.uint64(32)).astype(np.uint32)
        gid = (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)
        neg = (keys & 0x8000) == 0
        bits = np.where(neg, (~keys) & 0xFFFF, keys & 0x7FFF).astype(np.uint16)
        x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16 if bf16 else torch.float16)
        u = uniforms.numpy() if uniforms is not None else orc.splitmix_uniforms(seed, offset, B, row_base)
        d = orc.sample(x, top_k, top_p, uniforms=u, temperature=temperature)
        ids = gid[np.arange(B), d.ids]
        return torch.from_numpy(ids), torch.zeros(B, dtype=torch.int32)


def test_shard_range_covers_everything_once():
    for n in (1, 7, 32, 1024, 256000):
        for w in (1, 2, 3, 4, 8):
            spans = [shard_range(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [h - l for l, h in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops = OracleOps()
        # batch-sharded rows
        x = orc.anchor_logits(B=6, V=3000, seed=5)
        bs = BatchShardedSampler(batch=6, ops=ops)
        lo, hi = bs.rows
        ids = bs.sample(x[lo:hi], 50, 0.9, seed=3, offset=4, gather=True)
        # vocab-sharded tensor parallel
        y = orc.grid_logits(4, 4000, 2.0, torch.bfloat16, seed=6)
        vs = VocabShardedSampler(vocab=4000, top_k=40, ops=ops)
        c0, c1 = vs.cols
        tp_ids, _ = vs.sample(y[:, c0:c1].contiguous(), 0.9, seed=3, offset=4)
        results[rank] = (ids.tolist(), tp_ids.tolist())
    finally:
        dist.destroy_process_group()


def test_sharded_layouts_match_the_unsharded_oracle_over_gloo():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
    x = orc.anchor_logits(B=6, V=3000, seed=5)
    want = orc.sample(x, 50, 0.9, seed=3, offset=4).ids.tolist()
    y = orc.grid_logits(4, 4000, 2.0, torch.bfloat16, seed=6)
    want_tp = orc.sample(y, 40, 0.9, seed=3, offset=4).ids.tolist()
    for r in range(world):
        ids, tp_ids = results[r]
        assert ids == want, f"rank {r}: batch-sharded ids differ"
        assert tp_ids == want_tp, f"rank {r}: vocab-sharded ids differ"
