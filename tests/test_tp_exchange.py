"""The peer-to-peer exchange + merge (fs_tp_merge_sample) on one GPU.

Nothing here waits on another kernel: a second rank is emulated by filling its slot of the
receive buffer and its flags before the launch (as its own kernel would have), or by never
filling them, which must end in the bounded wait's FS_ROW_TIMEOUT status, not a hang.
"""

import pytest
import torch

from llm_sampling_kernel_b200 import abi, fused

pytestmark = pytest.mark.gpu

K = 64


def setup(world, B, V):
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(B, V, generator=g) * 2.5).to(torch.bfloat16).cuda()
    recv, recv_ptr = abi.ipc_alloc((2, world, B, K + 1), torch.int64)
    flags, flags_ptr = abi.ipc_alloc((2, world, B), torch.int32)
    return x, recv, recv_ptr, flags, flags_ptr


def shard_cands(x, world):
    vs = x.shape[1] // world
    return [fused.ops().shard_candidates(x[:, r * vs:(r + 1) * vs].contiguous(), K, r * vs) for r in range(world)]


def test_two_ranks_emulated_on_one_gpu_merge_to_the_unsharded_result():
    B, V = 16, 256000
    x, recv, recv_ptr, flags, flags_ptr = setup(2, B, V)
    try:
        cands = shard_cands(x, 2)
        ptrs = torch.tensor([recv_ptr, recv_ptr], dtype=torch.int64, device="cuda")
        fptrs = torch.tensor([flags_ptr, flags_ptr], dtype=torch.int64, device="cuda")
        for epoch in (1, 2, 3):
            slot = epoch & 1
            recv[slot, 1].copy_(cands[1])   # what rank 1's kernel pushes
            flags[slot, 1].fill_(epoch)     # and the flags it raises
            ids, status = fused.ops().tp_merge(cands[0], True, K, 0.9, recv, flags, ptrs, fptrs, 2, 0, epoch,
                                               seed=3, offset=epoch)
            want = fused.ops().sample_ex(x, K, 0.9, None, None, None, 3, epoch, 0, 0, 0, False)[0]
            assert torch.equal(ids, want)
            assert (status == 0).all()
            assert (flags[slot, 0] == epoch).all()  # this rank raised its own flags
    finally:
        torch.cuda.synchronize()
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)


def test_a_rank_that_never_pushes_times_out_with_a_row_status():
    B, V = 8, 256000
    x, recv, recv_ptr, flags, flags_ptr = setup(2, B, V)
    try:
        cands = shard_cands(x, 2)
        ptrs = torch.tensor([recv_ptr, recv_ptr], dtype=torch.int64, device="cuda")
        fptrs = torch.tensor([flags_ptr, flags_ptr], dtype=torch.int64, device="cuda")
        ids, status = fused.ops().tp_merge(cands[0], True, K, 0.9, recv, flags, ptrs, fptrs, 2, 0, 1,
                                           seed=3, offset=1, wait_polls=2000)
        torch.cuda.synchronize()
        assert (status == 5).all()  # FS_ROW_TIMEOUT
        assert (ids == -1).all()
        # the context is still usable
        assert torch.equal(fused.topk_fused(x, 5), fused.topk_fused(x, 5))
    finally:
        torch.cuda.synchronize()
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)


def test_one_rank_exchange_equals_the_plain_sampler():
    B, V = 8, 151936
    x, recv, recv_ptr, flags, flags_ptr = setup(1, B, V)
    try:
        cand = fused.ops().shard_candidates(x, K, 0)
        ptrs = torch.tensor([recv_ptr], dtype=torch.int64, device="cuda")
        fptrs = torch.tensor([flags_ptr], dtype=torch.int64, device="cuda")
        ids, status = fused.ops().tp_merge(cand, True, K, 0.95, recv, flags, ptrs, fptrs, 1, 0, 7, seed=1, offset=2)
        assert torch.equal(ids, fused.sample_fused(x, K, 0.95, seed=1, offset=2))
        assert (status == 0).all()
    finally:
        torch.cuda.synchronize()
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)


def test_the_device_epoch_counter_advances_per_call_wraps_and_replays_in_a_graph():
    """With an epoch counter the launch reads its epoch from device memory and advances it, so a
    step (shard top-k + exchange-merge) captured in a CUDA graph runs a new epoch on every replay."""
    B, V = 8, 151936
    x, recv, recv_ptr, flags, flags_ptr = setup(1, B, V)
    try:
        ops = fused.ops()
        ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
        ptrs = torch.tensor([recv_ptr], dtype=torch.int64, device="cuda")
        fptrs = torch.tensor([flags_ptr], dtype=torch.int64, device="cuda")
        want = fused.sample_fused(x, K, 0.95, seed=1, offset=2)

        def step():
            cand = ops.shard_candidates(x, K, 0)
            return ops.tp_merge(cand, True, K, 0.95, recv, flags, ptrs, fptrs, 1, 0, 0, seed=1, offset=2,
                                epoch_counter=ctr)

        for k in (1, 2, 3):
            ids, status = step()
            assert torch.equal(ids, want) and (status == 0).all()
            assert ctr.tolist() == [k, 0]
            assert (flags[k & 1, 0] == k).all()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                ids_g, status_g = step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        assert ctr.tolist() == [3, 0]  # capture runs nothing
        for k in (4, 5, 6):
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(ids_g, want) and (status_g == 0).all()
            assert ctr.tolist() == [k, 0]
        del g
        # after 2^32 - 1 the epoch wraps to 2 (never 0, and the slot parity still alternates)
        ctr.copy_(torch.tensor([-1, 0], dtype=torch.int32))
        ids, status = step()
        assert torch.equal(ids, want) and (status == 0).all()
        assert ctr.tolist() == [2, 0]
        assert (flags[0, 0] == 2).all()
    finally:
        torch.cuda.synchronize()
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)
