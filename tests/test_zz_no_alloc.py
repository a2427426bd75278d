"""fs_sample_noalloc (the allocation-free entry point) against fs_sample, through the C ABI.

The entry point keeps the streaming path's scratch in a static device array, so two calls in a
row reuse the same memory: both must give exactly what fs_sample gives with its own workspace.
"""

import ctypes

import pytest
import torch

from llm_sampling_kernel_b200 import abi

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 16 << 20


def noalloc_call(x, top_k, top_p, *, seed, offset, path=abi.FS_PATH_AUTO):
    B, V = x.shape
    K = min(top_k, V)
    dev = x.device
    out = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    ids = torch.empty(B, K, dtype=torch.int64, device=dev)
    keep = torch.empty(B, K, dtype=torch.uint8, device=dev)
    ren = torch.empty(B, K, dtype=torch.float32, device=dev)
    a = abi.make_args(x, top_k, top_p, seed=seed, offset=offset, out_ids=out, topk_ids=ids, keep=keep,
                      renormed=ren, row_status=status, path=path)
    st = abi.lib().fs_sample_noalloc(ctypes.byref(a), abi._stream())
    abi.check(st, "fs_sample_noalloc")
    return out, ids, keep.bool(), ren, status


@pytest.mark.parametrize("B,path", [(256, abi.FS_PATH_AUTO), (40, abi.FS_PATH_STREAM), (4, abi.FS_PATH_AUTO)])
def test_two_calls_in_a_row_equal_fs_sample(B, path):
    g = torch.Generator().manual_seed(B)
    x = (torch.randn(B, 151936, generator=g) * 3.0).to(torch.bfloat16).cuda()
    y = (torch.randn(B, 151936, generator=g) * 2.0).to(torch.bfloat16).cuda()
    for inp, off in ((x, 3), (y, 4)):
        want = abi.sample(inp, 50, 0.9, seed=7, offset=off, stages=True, path=path)
        got = noalloc_call(inp, 50, 0.9, seed=7, offset=off, path=path)
        for name, p, q in zip(("ids", "topk", "keep", "renormed", "status"), want, got):
            assert torch.equal(p, q), name


def test_a_call_beyond_the_static_scratch_is_rejected():
    x = torch.zeros(1024, 151936, dtype=torch.bfloat16, device="cuda")
    a = abi.make_args(x, 256, 0.9, path=abi.FS_PATH_STREAM)
    assert abi.lib().fs_workspace_size(ctypes.byref(a)) > STATIC_SCRATCH_BYTES
    with pytest.raises(abi.FsError) as e:
        noalloc_call(x, 256, 0.9, seed=1, offset=0, path=abi.FS_PATH_STREAM)
    assert e.value.status == abi.FS_EWORKSPACE
    assert "static scratch" in str(e.value)
