"""CUDA parity tests of the large-batch path: STREAM (slice launch + row-merge launch).

It must give exactly what the cluster path gives: the same top-k set and order (checked against
the oracle), and, because all end in the same row tail over the same candidates, the same ids,
keep mask, renormed probabilities and row status, bit for bit. `path=` forces a path at any batch
(k <= 256); batches of 96 rows and more take STREAM by default when k <= 128.
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
PATHS = [STREAM]


def dev_randn(B, V, scale, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, V, generator=g) * scale).to(dtype).cuda()


def oracle_topk(x, k):
    return torch.from_numpy(orc.topk_order(orc.bits16(x.cpu()), min(k, x.shape[1])))


def run(x, top_k, top_p, path, **kw):
    out, ids, keep, ren, status = fused.ops().sample_ex(x, top_k, top_p, return_stages=True, path=path, **kw)
    return out, ids, keep, ren, status


def assert_paths_agree(x, top_k, top_p, path=STREAM, **kw):
    a = run(x, top_k, top_p, CLUSTER, **kw)
    b = run(x, top_k, top_p, path, **kw)
    for name, p, q in zip(("ids", "topk", "keep", "renormed", "status"), a, b):
        assert torch.equal(p, q), name
    return b


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k", [1, 20, 50, 100, 256])
@pytest.mark.parametrize("vocab", [2000, 4001, 32000, 128256, 151936])
@pytest.mark.parametrize("path", PATHS)
def test_streaming_candidate_set_matches_the_oracle_exactly(vocab, top_k, dtype, path):
    x = dev_randn(24, vocab, 4.0, dtype, seed=vocab + top_k)
    got = abi.topk(x, top_k, path=path).cpu()
    assert torch.equal(got, oracle_topk(x, top_k))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k", [1, 50, 256])
@pytest.mark.parametrize("path", PATHS)
def test_all_equal_rows_take_the_exact_slice_fallback(top_k, dtype, path):
    # every slice overflows its slots: each writes its exact top-k (lowest ids first)
    x = torch.zeros(3, 151936, device="cuda", dtype=dtype)
    assert torch.equal(abi.topk(x, top_k, path=path).cpu(), torch.arange(top_k).expand(3, top_k))


@pytest.mark.parametrize("vocab", [20000, 151936])
@pytest.mark.parametrize("path", PATHS)
def test_dense_ties_and_grid_rounded_values(vocab, path):
    x = dev_randn(16, vocab, 0.05, torch.bfloat16, seed=3)
    for top_k in (20, 50, 100, 256):
        assert torch.equal(abi.topk(x, top_k, path=path).cpu(), oracle_topk(x, top_k))
    for dtype in DTYPES:
        g = orc.grid_logits(16, vocab, 1.0, dtype, seed=vocab).cuda()
        for top_k in (1, 50, 256):
            assert torch.equal(abi.topk(g, top_k, path=path).cpu(), oracle_topk(g, top_k))


@pytest.mark.parametrize("path", PATHS)
def test_ties_straddling_slice_boundaries_keep_the_lowest_ids(path):
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
            assert torch.equal(abi.topk(xd, k, path=path).cpu(), oracle_topk(xd, k))


@pytest.mark.parametrize("path", PATHS)
def test_signed_zeros_tie_across_slices(path):
    x = torch.full((2, 40000), -1.0)
    x[0, ::3] = 0.0
    x[0, 1::3] = -0.0
    x[1, 100:20000:5] = -0.0
    x[1, 20000:] = 0.0
    for dtype in DTYPES:
        xd = x.to(dtype).cuda()
        for k in (5, 150, 256):
            assert torch.equal(abi.topk(xd, k, path=path).cpu(), oracle_topk(xd, k))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("top_k,top_p", [(1, 1.0), (50, 0.9), (100, 0.95), (256, 0.5), (256, 1.0)])
@pytest.mark.parametrize("path", PATHS)
def test_stages_and_ids_equal_the_cluster_path(top_k, top_p, dtype, path):
    x = dev_randn(96, 151936, 3.0, dtype, seed=top_k)
    u = torch.rand(96, generator=torch.Generator().manual_seed(top_k)).cuda()
    assert_paths_agree(x, top_k, top_p, path, uniforms=u)
    assert_paths_agree(x, top_k, top_p, path, seed=17, offset=top_k)


def test_anchor_batch_takes_the_streaming_path_and_matches_the_oracle():
    assert abi.plan(256, 151936, 50).path == STREAM
    x = orc.anchor_logits(B=256, V=151936, seed=5).cuda()
    u = torch.rand(256, generator=torch.Generator().manual_seed(6))
    got = fused.sample(x, 50, 0.9, uniforms=u.cuda()).token_ids.cpu().numpy()
    d = orc.sample(x.cpu(), 50, 0.9, uniforms=u.numpy())
    ok = (got == d.ids) | d.near_boundary
    assert ok.all()
    assert int(d.near_boundary.sum()) <= 2


@pytest.mark.parametrize("path", PATHS)
def test_zipf_rows_match_the_oracle(path):
    x = orc.zipf_logits(64, 151936, seed=2).cuda()
    for k in (50, 256):
        assert torch.equal(abi.topk(x, k, path=path).cpu(), oracle_topk(x, k))


@pytest.mark.parametrize("path", PATHS)
def test_per_row_k_and_p_and_bad_rows(path):
    B = 80
    x = dev_randn(B, 151936, 3.0, torch.bfloat16, seed=8)
    g = torch.Generator().manual_seed(3)
    ks = torch.randint(1, 257, (B,), generator=g, dtype=torch.int32)
    ps = torch.rand(B, generator=g) * 0.9 + 0.1
    ks[5] = 0       # bad parameter
    ps[7] = 1.5     # bad parameter
    u = torch.rand(B, generator=g).cuda()
    out = assert_paths_agree(x, 256, 1.0, path, top_k_rows=ks.cuda(), top_p_rows=ps.cuda(), uniforms=u)
    status = out[4].cpu()
    assert status[5] == 4 and status[7] == 4


@pytest.mark.parametrize("path", PATHS)
def test_invalid_rows_report_the_same_status(path):
    x = orc.adversarial_logits(4, B=8, V=151936).cuda()
    y = x.clone()
    y[1, 77] = float("nan")
    y[2, :] = float("-inf")
    for z in (x, y):
        out = assert_paths_agree(z, 50, 0.9, path, seed=1, offset=1)
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


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch", [1, 149, 300, 1024])
def test_streaming_batches_up_to_the_large_batch_config(batch, dtype):
    # more rows than SMs; 1024 rows is the large-batch config's batch
    x = dev_randn(batch, 151936, 3.0, dtype, seed=batch)
    u = torch.rand(batch, generator=torch.Generator().manual_seed(batch)).cuda()
    assert_paths_agree(x, 50, 0.9, STREAM, uniforms=u)
    rows = torch.arange(0, batch, max(1, batch // 7))
    assert torch.equal(abi.topk(x, 50, path=STREAM).cpu()[rows], oracle_topk(x[rows], 50))


@pytest.mark.parametrize("top_k", [1, 50, 128, 256])
def test_rising_rows_concentrate_candidates_in_the_last_slices(top_k):
    # the row rises by about one sigma every 16384 ids: the last slices hold every candidate
    B, V = 8, 151936
    g = torch.Generator().manual_seed(top_k)
    trend = torch.arange(V, dtype=torch.float32) // 16384 * 0.95
    x = (torch.randn(B, V, generator=g) + trend).to(torch.bfloat16).cuda()
    assert torch.equal(abi.topk(x, top_k, path=STREAM).cpu(), oracle_topk(x, top_k))
    u = torch.rand(B, generator=g).cuda()
    assert_paths_agree(x, top_k, 0.9, STREAM, uniforms=u)
    steep = (torch.randn(B, V, generator=g) * 0.3 + trend * 3).to(torch.float16).cuda()
    assert torch.equal(abi.topk(steep, top_k, path=STREAM).cpu(), oracle_topk(steep, top_k))


def test_late_stage_ties_overflow_into_the_exact_fallback():
    # a tie block in the last slices: their candidate slots overflow
    x = torch.randn(4, 151936, generator=torch.Generator().manual_seed(1))
    x[:, 140000:] = 3.5
    x[1, 5] = 9.0
    x[2, 100000:100600] = 3.5
    for dtype in DTYPES:
        xd = x.to(dtype).cuda()
        for k in (1, 50, 256):
            assert torch.equal(abi.topk(xd, k, path=STREAM).cpu(), oracle_topk(xd, k))
        u = torch.rand(4, generator=torch.Generator().manual_seed(2)).cuda()
        assert_paths_agree(xd, 50, 0.9, STREAM, uniforms=u)


def test_nan_and_inf_in_the_last_slices_are_reported():
    x = dev_randn(6, 151936, 2.0, torch.bfloat16, seed=15)
    x[0, 151000] = float("nan")
    x[1, 140001] = float("inf")
    x[2, :] = float("-inf")
    x[3, :150000] = float("-inf")  # finite values only in the last slice
    x[4, 16384 * 3 + 7] = float("-inf")
    out = assert_paths_agree(x, 50, 0.9, STREAM, seed=3, offset=4)
    assert out[4].cpu().tolist() == orc.row_status(x.cpu()).tolist()
    assert out[4].cpu().tolist()[:4] == [1, 2, 3, 0]


def test_vocab_shard_candidates_from_the_streaming_path_merge_exactly():
    x = dev_randn(192, 256000, 2.5, torch.bfloat16, seed=4)
    u = torch.rand(192, generator=torch.Generator().manual_seed(3)).cuda()
    want = run(x, 64, 0.9, CLUSTER, uniforms=u)[0]
    ops = fused.ops()
    world, vs = 4, 64000
    assert abi.plan(192, vs, 64).path == STREAM
    parts = [ops.shard_candidates(x[:, r * vs:(r + 1) * vs], 64, r * vs) for r in range(world)]
    ids, status = ops.merge_sample(torch.stack(parts), True, 64, 0.9, uniforms=u)
    assert torch.equal(ids, want)
    assert (status == 0).all()


@pytest.mark.parametrize("path", PATHS)
def test_repeated_calls_reuse_no_state(path):
    x = dev_randn(70, 151936, 2.0, torch.float16, seed=12)
    a = abi.sample(x, 50, 0.9, seed=5, offset=6, path=path)
    y = torch.zeros_like(x)
    abi.sample(y, 50, 0.9, seed=5, offset=6, path=path)
    b = abi.sample(x, 50, 0.9, seed=5, offset=6, path=path)
    assert torch.equal(a, b)
    assert torch.equal(a, abi.sample(x, 50, 0.9, seed=5, offset=6, path=CLUSTER))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("path", PATHS)
def test_masked_vocabulary_regions(dtype, path):
    """Whole slices of -inf (their threshold ladders carry no bound), rows with fewer finite
    logits than k (-inf elements enter the top k), and rows finite in one slice only."""
    B, V, k = 8, 151936, 50
    x = dev_randn(B, V, 3.0, dtype, seed=31)
    ninf = float("-inf")
    x[0, : V // 2] = ninf                      # half the slices masked
    x[1, 20480:] = ninf                        # one slice finite
    x[2] = ninf
    x[2, torch.randperm(V, generator=torch.Generator().manual_seed(2))[:30].cuda()] = 1.0  # 30 finite < k
    x[3, ::2] = ninf                           # every other id masked
    x[4, 20480 * 3: 20480 * 3 + 40] = 50.0     # a tight cluster inside one slice
    ids_out = assert_paths_agree(x, k, 0.9, path, seed=5, offset=1)[1]
    for r in range(B):
        assert torch.equal(ids_out[r].cpu(), oracle_topk(x[r:r + 1], k)[0]), r


@pytest.mark.parametrize("path", PATHS)
def test_survivor_keys_spanning_more_than_256_values(path):
    """fp16 keys of the top k spread over far more than 256 key values: the row merge's counting
    sort declines and the comparison rank (or the histogram path) must give the same order."""
    B, V = 4, 65536
    g = torch.Generator().manual_seed(9)
    x = (torch.rand(B, V, generator=g) * 2.0 ** torch.randint(-8, 8, (B, V), generator=g)).to(torch.float16).cuda()
    for k in (20, 50, 128):
        ids = assert_paths_agree(x, k, 1.0, path, seed=6, offset=k)[1]
        for r in range(B):
            assert torch.equal(ids[r].cpu(), oracle_topk(x[r:r + 1], k)[0])


def test_kernel_attribute_queries_leave_the_granted_launch_limits_alone():
    """kernel_attrs computes occupancy at a typical shared-memory size; it must not lower the
    limit a launch path granted (and remembers granting) for a larger row merge."""
    x = dev_randn(24, 151936, 2.0, torch.bfloat16, seed=41)
    assert torch.equal(abi.topk(x, 256, path=STREAM).cpu(), oracle_topk(x, 256))
    fused.ops().kernel_attrs()
    assert torch.equal(abi.topk(x, 256, path=STREAM).cpu(), oracle_topk(x, 256))
    assert torch.equal(abi.topk(x, 100, path=STREAM).cpu(), oracle_topk(x, 100))
