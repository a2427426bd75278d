"""Two-GPU runs of the sharded samplers over NCCL (skipped on a box with fewer than two GPUs).

Each rank builds the same seeded logits, samples its shard, and rank 0 checks the result against
the unsharded single-GPU call:

* batch-sharded rows (no collective on the data path, ids all-gathered for the check) draw exactly
  what one GPU draws over the whole batch, because the uniform is evaluated at the global row;
* vocab-sharded tensor parallelism (local top-k as packed candidates, exchanged by an NCCL
  all-gather or pushed into every rank's buffers over NVLink by the p2p kernel, merge on every
  rank) gives identical ids on both ranks, equal to the unsharded call.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from llm_sampling_kernel_b200 import ops
        from llm_sampling_kernel_b200.sharded import BatchShardedSampler, VocabShardedSampler, shard_range

        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(21)
        # batch-sharded rows
        B, V = 300, 151936
        full = (torch.randn(B, V, generator=g) * 3.0).to(torch.bfloat16).to(dev)
        bs = BatchShardedSampler(batch=B)
        lo, hi = bs.rows
        ids = bs.sample(full[lo:hi], 50, 0.9, seed=7, offset=3, gather=True)
        want = ops().sample_ex(full, 50, 0.9, None, None, None, 7, 3, 0, 0, 0, False)[0]
        assert torch.equal(ids, want), "batch-sharded ids differ from the single-GPU call"
        # vocab-sharded tensor parallelism
        B, V = 32, 256000
        full = (torch.randn(B, V, generator=g) * 2.5).to(torch.bfloat16).to(dev)
        for backend in ("nccl", "p2p"):
            tp = VocabShardedSampler(vocab=V, top_k=64, backend=backend)
            c0, c1 = tp.cols
            for off in range(5):
                tids, status = tp.sample(full[:, c0:c1].contiguous(), 0.9, seed=11, offset=off)
                ref = ops().sample_ex(full, 64, 0.9, None, None, None, 11, off, 0, 0, 0, False)[0]
                assert torch.equal(tids, ref), f"vocab-sharded ids ({backend}) differ from the unsharded call"
                assert (status == 0).all()
                others = [torch.empty_like(tids) for _ in range(world)]
                dist.all_gather(others, tids)
                assert all(torch.equal(o, tids) for o in others), "ranks disagree"
            # a tempered step: the merged candidates' logits / T before the softmax
            tids, status = tp.sample(full[:, c0:c1].contiguous(), 0.9, seed=11, offset=9, temperature=0.6)
            ref = ops().sample_ex(full, 64, 0.9, None, None, None, 11, 9, 0, 0, 0, False, 0, 0.6)[0]
            assert torch.equal(tids, ref), f"tempered vocab-sharded ids ({backend}) differ from the unsharded call"
            assert (status == 0).all()
            tp.close()
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_batch_and_vocab_sharding_match_one_gpu():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_one_process_driving_two_gpus_grants_kernel_attributes_per_device():
    """Function attributes (dynamic shared memory, non-portable cluster size) are per device: a
    size granted on one GPU must not be assumed on the other. The order below (small on GPU 0,
    large on GPU 1, then large on GPU 0, small on GPU 1) is the one a single per-kernel record
    would get wrong."""
    from llm_sampling_kernel_b200 import fused
    from oracle import sampler_oracle as orc

    xs = {d: orc.anchor_logits(B=4, V=151936, seed=d) for d in (0, 1)}
    for d, k in ((0, 50), (1, 2048), (0, 2048), (1, 50), (1, 8192)):
        with torch.cuda.device(d):
            got = fused.topk_fused(xs[d].cuda(d), k).cpu()
        want = torch.from_numpy(orc.topk_order(orc.bits16(xs[d]), k))
        assert torch.equal(got, want), (d, k)
