"""Logits in pinned host memory: the kernels read them in place over PCIe and write the results
into pinned host tensors. Every path (cluster, streaming, wide) gives the ids of the same call on
a device copy of the logits; the host blocks stay reserved until the stream has passed the call."""

import numpy as np
import pytest
import torch

from llm_sampling_kernel_b200 import abi
from llm_sampling_kernel_b200 import fused
from oracle import sampler_oracle as orc

V = 151936


def anchor(B, seed, dtype=torch.bfloat16, V=V):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, V, generator=g) * 2.0).to(dtype)


def test_unpinned_host_logits_are_rejected():
    x = torch.zeros(1, 100, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned host memory"):
        fused.sample_fused(x, 5, 0.9)


@pytest.mark.gpu
def test_anchor_ids_equal_the_device_call_and_the_oracle():
    x = anchor(1, 11)
    h = x.pin_memory()
    d = x.cuda()
    for off in range(32):
        got = fused.sample_fused(h, 50, 0.9, seed=0x5EED, offset=off)
        assert got.device.type == "cpu" and got.is_pinned()
        torch.cuda.current_stream().synchronize()
        want = fused.sample_fused(d, 50, 0.9, seed=0x5EED, offset=off).cpu()
        assert torch.equal(got, want), off
        o = orc.sample(x, 50, 0.9, seed=0x5EED, offset=off)
        assert ((got.numpy() == o.ids) | o.near_boundary).all()


@pytest.mark.gpu
@pytest.mark.parametrize("B,top_k,top_p,path", [(8, 50, 0.9, abi.FS_PATH_CLUSTER), (192, 50, 0.95, abi.FS_PATH_STREAM),
                                                (2, V, 0.5, abi.FS_PATH_WIDE)])
def test_every_path_reads_host_logits(B, top_k, top_p, path):
    x = anchor(B, B, dtype=torch.float16)
    assert abi.plan(B, V, top_k).path == path
    h = x.pin_memory()
    d = x.cuda()
    u = torch.rand(B, generator=torch.Generator().manual_seed(5))
    res = fused.sample(h, top_k, top_p, uniforms=u)
    torch.cuda.current_stream().synchronize()
    want = fused.sample(d, top_k, top_p, uniforms=u.cuda())
    assert res.token_ids.device.type == "cpu" and res.status.device.type == "cpu"
    assert torch.equal(res.token_ids, want.token_ids.cpu())
    assert torch.equal(res.status, want.status.cpu())


@pytest.mark.gpu
def test_stage_outputs_and_topk_from_host_logits():
    x = anchor(4, 3)
    h = x.pin_memory()
    d = x.cuda()
    ids = fused.topk_fused(h, 256)
    out, keep, ren = fused.stages_fused(h, 100, 0.9, seed=1, offset=2)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(ids, fused.topk_fused(d, 256).cpu())
    w_out, w_keep, w_ren = fused.stages_fused(d, 100, 0.9, seed=1, offset=2)
    assert torch.equal(out, w_out.cpu()) and torch.equal(keep, w_keep.cpu()) and torch.equal(ren, w_ren.cpu())
    assert np.array_equal(ids.numpy(), orc.topk_order(orc.bits16(x), 256))


@pytest.mark.gpu
def test_per_row_parameters_and_input_checks_with_host_logits():
    x = anchor(6, 7)
    x[2, 10] = float("nan")
    h = x.pin_memory()
    k_rows = torch.tensor([1, 50, 50, 256, 1024, 7], dtype=torch.int32)  # host tensors, moved to the device
    p_rows = torch.tensor([0.9, 0.5, 0.9, 1.0, 0.95, 0.3])
    res = fused.sample(h, k_rows, p_rows, seed=3, offset=4)
    torch.cuda.current_stream().synchronize()
    want = fused.sample(x.cuda(), k_rows.cuda(), p_rows.cuda(), seed=3, offset=4)
    assert torch.equal(res.token_ids, want.token_ids.cpu())
    assert res.status.tolist() == [0, 0, fused.ROW_NAN, 0, 0, 0]
    with pytest.raises(ValueError, match="NaN"):
        fused.sample(h, 50, 0.9, check_inputs=True)


@pytest.mark.gpu
def test_cuda_only_entry_points_reject_host_logits():
    h = anchor(2, 1, V=4000).pin_memory()
    with pytest.raises(RuntimeError, match="contiguous cuda"):
        fused.ops().shard_candidates(h, 10, 0)
    with pytest.raises(RuntimeError, match="contiguous cuda"):
        fused.ops().probe_scan_rowblock(h)


@pytest.mark.gpu
def test_a_released_input_block_is_not_reused_before_the_call_has_run():
    x = anchor(64, 21)
    want = fused.sample_fused(x.cuda(), 50, 0.9, seed=9, offset=1).cpu()
    torch.cuda.synchronize()
    # keep the stream busy so the sampling call is still queued when its input is released
    busy = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(20):
        busy.add_(1)
    h = x.pin_memory()
    got = fused.sample_fused(h, 50, 0.9, seed=9, offset=1)
    del h
    # a new pinned block of the same size, filled with other logits, must not alias the old one
    other = torch.full((64, V), -3.0, dtype=torch.bfloat16).pin_memory()
    other[:, 0] = 5.0
    torch.cuda.current_stream().synchronize()
    assert torch.equal(got, want)
    del other


@pytest.mark.gpu
def test_ready_input_flag_changes_only_when_the_logits_are_read():
    """FS_INPUT_READY (set by the operators for pinned host logits) lets the cluster kernel read
    the logits before it waits for the previous kernel; the ids are those of the unflagged call."""
    import ctypes

    x = anchor(8, 31).cuda()
    lib = abi.lib()
    outs = []
    for flags in (0, abi.FS_INPUT_READY):
        out = torch.empty(8, dtype=torch.int64, device="cuda")
        ids = []
        for off in range(4):  # back to back on one stream
            a = abi.make_args(x, 50, 0.9, seed=0x5EED, offset=off, out_ids=out, path=abi.FS_PATH_CLUSTER)
            a.input_flags = flags
            abi.check(lib.fs_sample(ctypes.byref(a), abi._stream()), "fs_sample")
            ids.append(out.clone())
        outs.append(torch.stack(ids).cpu())
    assert torch.equal(outs[0], outs[1])
