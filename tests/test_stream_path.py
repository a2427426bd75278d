"""CUDA parity tests of the large-batch streaming path (slice launch + row-merge launch).

The streaming path must give exactly what the cluster path gives: the same top-k set and order
(checked against the oracle), and, because both end in the same row tail over the same
candidates, the same ids, keep mask, renormed probabilities and row status, bit for bit.
`path=2` forces it at any batch (k <= 256); batches of 128 rows and more take it by default when
k <= 128.
"""

import numpy as np
import pytest
import torch

from llm_sampling_kernel_b200 import abi
from llm_sampling_kernel_b200 import fused
from oracle import sampler_oracle as orc

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]
CLUSTER, STREAM = abi.FS_PATH_CLUSTER, abi.FS_PATH_STREAM


def dev_randn(B, V, scale, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, V, generator=g) * scale).to(dtype).cuda()


def oracle_topk(x, k):
    return torch.from_numpy(orc.topk_order(orc.bits16(x.cpu()), min(k, x.shape[1])))


def run(x, top_k, top_p, path, **kw):
    out, ids, keep, ren, status = fused.ops().sample_ex(x, top_k, top_p, return_stages=True, path=path, **kw)
    return out, ids, keep, ren, status


def assert_paths_agree(x, top_k, top_p, **kw):
    a = run(x, top_k, top_p, CLUSTER, **kw)
    b = run(x, top_k, top_p, STREAM, **kw)
    for name, p, q in zip(("ids", "topk", "keep", "renormed", "status"), a, b):
        assert torch.equal(p, q), name
    return b


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k", [1, 20, 50, 100, 256])
@pytest.mark.parametrize("vocab", [2000, 4001, 32000, 128256, 151936])
def test_streaming_candidate_set_matches_the_oracle_exactly(vocab, top_k, dtype):
    x = dev_randn(24, vocab, 4.0, dtype, seed=vocab + top_k)
    got = abi.topk(x, top_k, path=STREAM).cpu()
    assert torch.equal(got, oracle_topk(x, top_k))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k", [1, 50, 256])
def test_all_equal_rows_take_the_exact_slice_fallback(top_k, dtype):
    # every slice overflows its slots: each writes its exact top-k (lowest ids first)
    x = torch.zeros(3, 151936, device="cuda", dtype=dtype)
    assert torch.equal(abi.topk(x, top_k, path=STREAM).cpu(), torch.arange(top_k).expand(3, top_k))


@pytest.mark.parametrize("vocab", [20000, 151936])
def test_dense_ties_and_grid_rounded_values(vocab):
    x = dev_randn(16, vocab, 0.05, torch.bfloat16, seed=3)
    for top_k in (20, 50, 100, 256):
        assert torch.equal(abi.topk(x, top_k, path=STREAM).cpu(), oracle_topk(x, top_k))
    for dtype in DTYPES:
        g = orc.grid_logits(16, vocab, 1.0, dtype, seed=vocab).cuda()
        for top_k in (1, 50, 256):
            assert torch.equal(abi.topk(g, top_k, path=STREAM).cpu(), oracle_topk(g, top_k))


def test_ties_straddling_slice_boundaries_keep_the_lowest_ids():
    # a block of equal maxima across a slice boundary, plus heavy ties at the k-th value
    x = torch.full((4, 151936), -5.0)
    x[0, 10000:12000] = 3.0
    x[1, ::7] = 1.0
    x[2, 151000:] = 2.0
    x[2, :40] = 2.0
    x[3, 5:9] = 7.0
    x[3, 70000:150000:3] = 6.0
    for dtype in DTYPES:
        xd = x.to(dtype).cuda()
        for k in (1, 7, 50, 256):
            assert torch.equal(abi.topk(xd, k, path=STREAM).cpu(), oracle_topk(xd, k))


def test_signed_zeros_tie_across_slices():
    x = torch.full((2, 40000), -1.0)
    x[0, ::3] = 0.0
    x[0, 1::3] = -0.0
    x[1, 100:20000:5] = -0.0
    x[1, 20000:] = 0.0
    for dtype in DTYPES:
        xd = x.to(dtype).cuda()
        for k in (5, 150, 256):
            assert torch.equal(abi.topk(xd, k, path=STREAM).cpu(), oracle_topk(xd, k))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k,top_p", [(1, 1.0), (50, 0.9), (100, 0.95), (256, 0.5), (256, 1.0)])
def test_stages_and_ids_equal_the_cluster_path(top_k, top_p, dtype):
    x = dev_randn(96, 151936, 3.0, dtype, seed=top_k)
    u = torch.rand(96, generator=torch.Generator().manual_seed(top_k)).cuda()
    assert_paths_agree(x, top_k, top_p, uniforms=u)
    assert_paths_agree(x, top_k, top_p, seed=17, offset=top_k)


def test_anchor_batch_takes_the_streaming_path_and_matches_the_oracle():
    assert abi.plan(256, 151936, 50).path == STREAM
    x = orc.anchor_logits(B=256, V=151936, seed=5).cuda()
    u = torch.rand(256, generator=torch.Generator().manual_seed(6))
    got = fused.sample(x, 50, 0.9, uniforms=u.cuda()).token_ids.cpu().numpy()
    d = orc.sample(x.cpu(), 50, 0.9, uniforms=u.numpy())
    ok = (got == d.ids) | d.near_boundary
    assert ok.all()
    assert int(d.near_boundary.sum()) <= 2


def test_zipf_rows_match_the_oracle():
    x = orc.zipf_logits(64, 151936, seed=2).cuda()
    for k in (50, 256):
        assert torch.equal(abi.topk(x, k, path=STREAM).cpu(), oracle_topk(x, k))


def test_per_row_k_and_p_and_bad_rows():
    B = 80
    x = dev_randn(B, 151936, 3.0, torch.bfloat16, seed=8)
    g = torch.Generator().manual_seed(3)
    ks = torch.randint(1, 257, (B,), generator=g, dtype=torch.int32)
    ps = torch.rand(B, generator=g) * 0.9 + 0.1
    ks[5] = 0       # bad parameter
    ps[7] = 1.5     # bad parameter
    u = torch.rand(B, generator=g).cuda()
    out = assert_paths_agree(x, 256, 1.0, top_k_rows=ks.cuda(), top_p_rows=ps.cuda(), uniforms=u)
    status = out[4].cpu()
    assert status[5] == 4 and status[7] == 4


def test_invalid_rows_report_the_same_status():
    x = orc.adversarial_logits(4, B=8, V=151936).cuda()
    y = x.clone()
    y[1, 77] = float("nan")
    y[2, :] = float("-inf")
    for z in (x, y):
        out = assert_paths_agree(z, 50, 0.9, seed=1, offset=1)
        assert out[4].cpu().numpy().tolist() == orc.row_status(z.cpu()).tolist()


def test_strided_unaligned_and_odd_vocab_rows():
    base = dev_randn(8, 151936 + 24, 3.0, torch.bfloat16, seed=10)
    view = base[:, 8:8 + 151936]
    odd = base[:, 3:3 + 151936]
    for v in (view, odd):
        assert torch.equal(abi.topk(v, 50, path=STREAM).cpu(), oracle_topk(v.contiguous(), 50))
    y = dev_randn(8, 100003, 3.0, torch.float16, seed=11)
    assert torch.equal(abi.topk(y, 100, path=STREAM).cpu(), oracle_topk(y, 100))
    u = torch.rand(8, generator=torch.Generator().manual_seed(4)).cuda()
    assert_paths_agree(odd, 50, 0.9, uniforms=u)


def test_vocab_shard_candidates_from_the_streaming_path_merge_exactly():
    x = dev_randn(128, 256000, 2.5, torch.bfloat16, seed=4)
    u = torch.rand(128, generator=torch.Generator().manual_seed(3)).cuda()
    want = run(x, 64, 0.9, CLUSTER, uniforms=u)[0]
    ops = fused.ops()
    world, vs = 4, 64000
    assert abi.plan(128, vs, 64).path == STREAM
    parts = [ops.shard_candidates(x[:, r * vs:(r + 1) * vs], 64, r * vs) for r in range(world)]
    ids, status = ops.merge_sample(torch.stack(parts), True, 64, 0.9, uniforms=u)
    assert torch.equal(ids, want)
    assert (status == 0).all()


def test_repeated_calls_reuse_no_state():
    x = dev_randn(70, 151936, 2.0, torch.float16, seed=12)
    a = abi.sample(x, 50, 0.9, seed=5, offset=6, path=STREAM)
    y = torch.zeros_like(x)
    abi.sample(y, 50, 0.9, seed=5, offset=6, path=STREAM)
    b = abi.sample(x, 50, 0.9, seed=5, offset=6, path=STREAM)
    assert torch.equal(a, b)
    assert torch.equal(a, abi.sample(x, 50, 0.9, seed=5, offset=6, path=CLUSTER))
