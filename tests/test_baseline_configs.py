"""CUDA parity at the benchmark configurations' stated shapes (the reference's Gate A grid,
tests/test_fused_kernel.py:29-37,211-220, and the adversarial and large-batch configurations).

* C2: every cell of B {1, 4, 16, 64} x V {128256, 151936} x sigma {1, 4} x k {1, 50, 256, 1024}
  x p {0.5, 0.9, 1.0} x {FP16, BF16}, with 30% of the logits on a 0.25 grid: token ids equal to the
  oracle's for the same uniform (boundary exemption as in test_kernel_parity), top-k set exact.
* C3: the full B=1024 Zipf-biased launch under AUTO (the streaming path), ids and keep mask
  against the oracle on a fixed subset of rows.
* C5 (B=8, V=151936, FP16): 16 distinct values at k=1024, p=0.99; k=V at p=0.5 on N(0, 0.1^2);
  greedy k=1; rows with +-inf and the most negative finite value.
"""

import numpy as np
import pytest
import torch

from llm_sampling_kernel_b200 import abi
from llm_sampling_kernel_b200 import fused
from oracle import sampler_oracle as orc

pytestmark = pytest.mark.gpu

V5 = 151936


def ids_match(got, d, max_exempt):
    got = np.asarray(got)
    ok = (got == d.ids) | d.near_boundary
    assert ok.all(), f"rows {np.nonzero(~ok)[0][:8]}: kernel {got[~ok][:8]} oracle {d.ids[~ok][:8]}"
    assert int(d.near_boundary.sum()) <= max_exempt


def ids_match_whole_vocab(got, d, u, top_p):
    """k near V: each pick checked by its CDF interval against the FP64-exact cumulative sums
    (1e-6 tolerance) and against the reference's FP32 ones (tolerance widened by the row's own FP32
    drift: torch's FP32 softmax over ~1e5 candidates is off by several 1e-6 relative)."""
    got = np.asarray(got)
    assert orc.pick_consistent(d.stages, got, u, top_p).all()
    err = orc.fp32_cumsum_error(d.stages)
    assert orc.pick_consistent(d.stages, got, u, top_p, rel_tol=1e-6 + 2 * err, fp64=False).all()


# ---- C2 ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("sigma", [1.0, 4.0])
@pytest.mark.parametrize("vocab", [128256, 151936])
@pytest.mark.parametrize("batch", [1, 4, 16, 64])
def test_grid_config_every_cell(batch, vocab, sigma, dtype):
    x = orc.grid_logits(batch, vocab, sigma, dtype, seed=batch * 7 + int(sigma)).cuda()
    xc = x.cpu()
    full = orc.topk_order(orc.bits16(xc), 1024)
    for top_k in (1, 50, 256, 1024):
        assert np.array_equal(fused.topk_fused(x, top_k).cpu().numpy(), full[:, :top_k]), top_k
        for top_p in (0.5, 0.9, 1.0):
            off = top_k * 10 + int(top_p * 10)
            got = fused.sample_fused(x, top_k, top_p, seed=0x5EED, offset=off).cpu().numpy()
            d = orc.sample(xc, top_k, top_p, seed=0x5EED, offset=off)
            ids_match(got, d, max_exempt=max(1, batch // 16))


# ---- C3 ----------------------------------------------------------------------------------------


@pytest.fixture(scope="module")
def c3_logits():
    return orc.zipf_logits(1024, V5, seed=7)


def test_large_batch_config_ids_and_keep_mask(c3_logits):
    x = c3_logits.cuda()
    assert abi.plan(1024, V5, 50).path == abi.FS_PATH_STREAM
    u = torch.rand(1024, generator=torch.Generator().manual_seed(31))
    res = fused.sample(x, 50, 0.95, uniforms=u.cuda(), return_stages=True)
    rows = torch.arange(0, 1024, 8)  # the oracle on every 8th row; the launch is the full batch
    st = orc.stages(c3_logits[rows], 50, 0.95)
    d = orc.draw(st, u[rows].numpy(), 0.95)
    ids_match(res.token_ids.cpu()[rows].numpy(), d, max_exempt=2)
    assert torch.equal(res.topk_ids.cpu()[rows], st.topk_ids)
    keep = res.keep.cpu()[rows]
    assert torch.equal(keep[~torch.from_numpy(d.near_boundary)], st.keep[~torch.from_numpy(d.near_boundary)])
    assert (res.status == 0).all()


def test_large_batch_config_seeded_draws(c3_logits):
    x = c3_logits.cuda()
    rows = torch.arange(3, 1024, 16)
    for off in (0, 1):
        got = fused.sample_fused(x, 50, 0.95, seed=0x5EED, offset=off).cpu()[rows].numpy()
        st = orc.stages(c3_logits[rows], 50, 0.95)
        u = np.array([orc.splitmix_uniform(0x5EED, off, int(r)) for r in rows], dtype=np.float32)
        ids_match(got, orc.draw(st, u, 0.95), max_exempt=1)


# ---- C5 ----------------------------------------------------------------------------------------


def test_adversarial_case1_sixteen_values_k1024_p099():
    x = orc.adversarial_logits(1, B=8, V=V5, seed=1)
    xd = x.cuda()
    want = orc.topk_order(orc.bits16(x), 1024)
    assert np.array_equal(fused.topk_fused(xd, 1024).cpu().numpy(), want)
    u = torch.rand(8, generator=torch.Generator().manual_seed(1))
    res = fused.sample(xd, 1024, 0.99, uniforms=u.cuda(), return_stages=True)
    st = orc.stages(x, 1024, 0.99)
    d = orc.draw(st, u.numpy(), 0.99)
    ids_match(res.token_ids.cpu().numpy(), d, max_exempt=1)
    assert torch.equal(res.topk_ids.cpu(), st.topk_ids)
    near = torch.from_numpy(d.near_boundary)
    assert torch.equal(res.keep.cpu()[~near], st.keep[~near])
    for off in range(4):
        got = fused.sample_fused(xd, 1024, 0.99, seed=0x5EED, offset=off).cpu().numpy()
        ids_match(got, orc.sample(x, 1024, 0.99, seed=0x5EED, offset=off), max_exempt=1)


def test_adversarial_case2_top_p_only_on_a_near_flat_row():
    x = orc.adversarial_logits(2, B=8, V=V5, seed=2)
    xd = x.cuda()
    assert abi.plan(8, V5, V5).path == abi.FS_PATH_WIDE
    for off in range(3):
        got = fused.sample_fused(xd, V5, 0.5, seed=0x5EED, offset=off).cpu().numpy()
        d = orc.sample(x, V5, 0.5, seed=0x5EED, offset=off)
        ids_match_whole_vocab(got, d, orc.splitmix_uniforms(0x5EED, off, 8), 0.5)
        assert (d.stages.cutoff.numpy() > 20000).all()  # the nucleus spans a large part of V


def test_adversarial_case3_greedy():
    x = orc.adversarial_logits(3, B=8, V=V5, seed=3)
    xd = x.cuda()
    want = orc.topk_order(orc.bits16(x), 1)[:, 0]
    for top_p in (0.5, 0.9, 1.0):
        got = fused.sample_fused(xd, 1, top_p, seed=1, offset=2).cpu().numpy()
        assert np.array_equal(got, want)
    # the first maximum of the FP32 view, lowest id on ties
    assert np.array_equal(want, x.float().argmax(dim=-1).numpy())


@pytest.mark.parametrize("top_k", [1, 50, 1024, V5])
def test_adversarial_case4_infinities_and_the_lowest_finite_value(top_k):
    x = orc.adversarial_logits(4, B=8, V=V5, seed=4)
    xd = x.cuda()
    res = fused.sample(xd, top_k, 0.9, seed=0x5EED, offset=5)
    status = orc.row_status(x)
    assert res.status.cpu().numpy().tolist() == status.tolist()
    ok_rows = np.nonzero(status == 0)[0]
    got = res.token_ids.cpu().numpy()
    assert (got[status != 0] == -1).all()
    u = orc.splitmix_uniforms(0x5EED, 5, 8)[ok_rows]
    d = orc.sample(x[ok_rows], top_k, 0.9, uniforms=u)
    if top_k <= 1024:
        # the two constant rows (every logit the most negative finite value) put exclusive
        # prefixes exactly on multiples of 1/n: the oracle may flag both
        ids_match(got[ok_rows], d, max_exempt=2)
    else:
        ids_match_whole_vocab(got[ok_rows], d, u, 0.9)
    with pytest.raises(ValueError, match="NaN|inf"):
        fused.sample(xd, top_k, 0.9, check_inputs=True)
