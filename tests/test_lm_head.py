"""The LM-head pipeline (bf16 GEMM in vocabulary chunks, each chunk's top-K taken while it is in
L2, one merge and draw): its ids equal the plain sampler's over the same chunk logits, and the
oracle's over them."""

import numpy as np
import pytest
import torch

from llm_sampling_kernel_b200 import fused
from llm_sampling_kernel_b200.lm_head import LMHeadSampler
from oracle import sampler_oracle as orc

pytestmark = pytest.mark.gpu


def weights(V, H, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(V, H, generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    return w


def hidden_states(B, H, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(B, H, generator=g, device="cuda") * 2.0).to(torch.bfloat16)


@pytest.mark.parametrize("B,V,H,k,chunk", [(1, 151936, 1024, 50, None), (8, 151936, 1024, 50, 16384),
                                           (64, 128256, 512, 256, 8192), (300, 151936, 256, 50, None),
                                           (4, 50000, 512, 1024, 12288)])
def test_pipeline_ids_equal_the_plain_sampler_over_the_chunk_logits(B, V, H, k, chunk):
    w = weights(V, H)
    h = hidden_states(B, H)
    lm = LMHeadSampler(w, k, max_batch=max(B, 8), chunk=chunk)
    u = torch.rand(B, generator=torch.Generator().manual_seed(B)).cuda()
    ids, status = lm.sample(h, 0.9, uniforms=u)
    # the same logits the pipeline consumed: the same GEMM calls, concatenated
    full = torch.cat([lm.chunk_logits(h, c).clone() for c in range(lm.parts)], dim=1)
    want = fused.sample(full, k, 0.9, uniforms=u)
    assert torch.equal(ids, want.token_ids)
    assert (status == 0).all()
    d = orc.sample(full.cpu(), k, 0.9, uniforms=u.cpu().numpy())
    got = ids.cpu().numpy()
    assert ((got == d.ids) | d.near_boundary).all()


def test_seeded_and_tempered_calls_match_the_plain_sampler():
    V, H, B = 151936, 512, 16
    w = weights(V, H, seed=3)
    h = hidden_states(B, H, seed=4)
    lm = LMHeadSampler(w, 64, max_batch=B)
    full = torch.cat([lm.chunk_logits(h, c).clone() for c in range(lm.parts)], dim=1)
    for off, t in ((0, 1.0), (5, 0.7), (9, 1.8)):
        ids, _ = lm.sample(h, 0.95, seed=11, offset=off, temperature=t)
        want = fused.sample(full, 64, 0.95, seed=11, offset=off, temperature=t).token_ids
        assert torch.equal(ids, want), (off, t)


def test_candidate_block_holds_each_chunks_exact_top_k():
    V, H, B, k = 40000, 256, 4, 20
    w = weights(V, H, seed=5)
    h = hidden_states(B, H, seed=6)
    lm = LMHeadSampler(w, k, max_batch=B, chunk=10000)
    cand = lm.candidates(h).cpu().numpy().view(np.uint64)
    for c, (lo, hi) in enumerate(lm.bounds):
        logits = lm.chunk_logits(h, c).cpu()
        ids = orc.topk_order(orc.bits16(logits), k) + lo
        got = (np.uint64(0xFFFFFFFF) - (cand[c, :, :k] & np.uint64(0xFFFFFFFF))).astype(np.int64)
        assert np.array_equal(got, ids), c
        assert (cand[c, :, k] == 0).all()


def test_a_tail_narrower_than_top_k_joins_the_chunk_before_it():
    lm = LMHeadSampler(weights(50000, 64), 1024, max_batch=4, chunk=12288)
    assert lm.bounds[-1] == (36864, 50000) and lm.parts == 4


def test_arguments_are_checked():
    w = weights(1000, 64)
    with pytest.raises(ValueError):
        LMHeadSampler(w.float(), 10)
    with pytest.raises(ValueError):
        LMHeadSampler(w, 300, chunk=256)  # a chunk narrower than top_k
    lm = LMHeadSampler(w, 10, max_batch=4)
    with pytest.raises(ValueError):
        lm.sample(hidden_states(5, 64), 0.9)
