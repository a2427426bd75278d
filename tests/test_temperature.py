"""Temperature (an extension of the reference's operator, which leaves it to the caller): the
selected candidates' logits are divided by T in fp32 before the softmax. Checked against the
oracle run on the same rows with the same T, on the cluster path (small batches) and the
streaming path (B >= 96), and against T = 1 being exactly the untempered call."""

import numpy as np
import pytest
import torch

from llm_sampling_kernel_b200 import abi, fused
from oracle import sampler_oracle as orc


def test_oracle_temperature_is_the_pipeline_on_scaled_fp32_logits():
    x = orc.anchor_logits(B=2, V=4096, seed=3)
    for T in (0.5, 2.0):
        st = orc.stages(x, 50, 0.9, temperature=T)
        ref = orc.stages(x, 50, 0.9)
        assert torch.equal(st.topk_ids, ref.topk_ids)  # the selection does not move
        assert torch.equal(st.topk_logits, ref.topk_logits / T)
        assert torch.allclose(st.probs.sum(-1), torch.ones(2), atol=1e-5)
    # a lower temperature sharpens: the top probability grows
    assert (orc.stages(x, 50, 1.0, temperature=0.5).probs[:, 0] > orc.stages(x, 50, 1.0).probs[:, 0]).all()


def test_the_args_struct_carries_the_temperature():
    a = abi.make_args(None, 50, 0.9, temperature=0.7)
    assert abs(a.temperature - 0.7) < 1e-7


@pytest.mark.gpu
@pytest.mark.parametrize("B", [4, 128])
@pytest.mark.parametrize("T", [0.3, 0.7, 1.5, 4.0])
def test_tempered_draws_and_stages_match_the_oracle(B, T):
    x = orc.anchor_logits(B=B, V=151936, seed=40 + B).cuda()
    u = torch.rand(B, generator=torch.Generator().manual_seed(7)).cuda()
    res = fused.sample(x, 50, 0.9, uniforms=u, return_stages=True, temperature=T)
    d = orc.sample(x.cpu(), 50, 0.9, uniforms=u.cpu().numpy(), temperature=T)
    got = res.token_ids.cpu().numpy()
    ok = (got == d.ids) | d.near_boundary
    assert ok.all(), (np.nonzero(~ok)[0][:8], got[~ok][:8], d.ids[~ok][:8])
    st = d.stages
    assert torch.equal(res.topk_ids.cpu(), st.topk_ids)
    # the same bars as the untempered parity tests: keep exact outside near-boundary rows,
    # renormed probabilities within 64 ulp and 2e-6 absolute
    rows = ~torch.from_numpy(d.near_boundary)
    keep = res.keep.cpu()
    assert torch.equal(keep[rows], st.keep[rows])
    both = keep & st.keep
    ren = res.renormed.cpu()
    ulp = (ren[both].view(torch.int32) - st.renormed[both].view(torch.int32)).abs()
    assert ulp.max().item() <= 64
    assert torch.allclose(ren[both], st.renormed[both], atol=2e-6, rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [2, 128])
def test_temperature_one_and_zero_are_the_untempered_call(B):
    x = orc.anchor_logits(B=B, V=151936, seed=9).cuda()
    base = fused.sample(x, 50, 0.9, seed=5, offset=3, return_stages=True)
    for T in (1.0, 0.0):
        r = fused.sample(x, 50, 0.9, seed=5, offset=3, return_stages=True, temperature=T)
        for p, q in zip(base, r):
            assert (p is None and q is None) or torch.equal(p, q)


@pytest.mark.gpu
def test_a_scaled_maximum_that_overflows_reports_posinf_and_bad_temperatures_are_rejected():
    x = torch.full((2, 4096), -1.0, dtype=torch.bfloat16, device="cuda")
    x[:, 7] = 3.0e38
    r = fused.sample(x, 10, 1.0, seed=1, temperature=1e-3)
    assert (r.status.cpu() == 2).all()  # FS_ROW_POSINF
    assert (r.token_ids.cpu() == -1).all()
    for T in (-1.0, float("nan"), float("inf")):
        with pytest.raises(RuntimeError, match="temperature"):
            fused.sample(x, 10, 1.0, seed=1, temperature=T)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [0.5, 2.0])
def test_vocab_sharded_merge_applies_the_same_temperature(T):
    """Two vocabulary shards merged on one GPU (the all-gather emulated by a stack) give the ids
    of the unsharded tempered call; the peer-memory exchange with one rank does too."""
    ops = fused.ops()
    B, V, K = 16, 256000, 64
    x = (torch.randn(B, V, generator=torch.Generator().manual_seed(12)) * 2.5).to(torch.bfloat16).cuda()
    vs = V // 2
    cands = torch.stack([ops.shard_candidates(x[:, r * vs:(r + 1) * vs].contiguous(), K, r * vs) for r in range(2)])
    want = ops.sample_ex(x, K, 0.9, seed=3, offset=5, temperature=T)[0]
    ids, status = ops.merge_sample(cands, True, K, 0.9, seed=3, offset=5, temperature=T)
    assert torch.equal(ids, want) and (status == 0).all()
    assert not torch.equal(want, ops.sample_ex(x, K, 0.9, seed=3, offset=5)[0])  # T changes the draws
    recv, recv_ptr = abi.ipc_alloc((2, 1, B, K + 1), torch.int64)
    flags, flags_ptr = abi.ipc_alloc((2, 1, B), torch.int32)
    try:
        cand = ops.shard_candidates(x, K, 0)
        ptrs = torch.tensor([recv_ptr], dtype=torch.int64, device="cuda")
        fptrs = torch.tensor([flags_ptr], dtype=torch.int64, device="cuda")
        ids1, st1 = ops.tp_merge(cand, True, K, 0.9, recv, flags, ptrs, fptrs, 1, 0, 1, seed=3, offset=5,
                                 temperature=T)
        assert torch.equal(ids1, want) and (st1 == 0).all()
    finally:
        torch.cuda.synchronize()
        abi.ipc_free(recv_ptr)
        abi.ipc_free(flags_ptr)
