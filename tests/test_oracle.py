"""The CPU oracle pinned against the reference: golden vectors produced by the reference's own
``sample_eager`` (tests/golden/make_golden.py), the reference tests' known answers, and the
published splitmix64 output. CPU only."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sampler_oracle as orc

GOLDEN = np.load(Path(__file__).parent / "golden" / "golden_stages.npz")
NAMES = [str(n) for n in GOLDEN["names"]]


def golden_logits(name):
    dt = str(GOLDEN[f"{name}/dtype"])
    if dt == "f32":
        return torch.from_numpy(GOLDEN[f"{name}/f32"])
    bits = torch.from_numpy(GOLDEN[f"{name}/bits"].view(np.int16))
    return bits.view(torch.bfloat16 if dt == "bf16" else torch.float16)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_reproduces_reference_stages_exactly(name):
    x = golden_logits(name)
    k, p = int(GOLDEN[f"{name}/k"]), float(GOLDEN[f"{name}/p"])
    st = orc.stages(x, k, p)
    assert np.array_equal(st.topk_ids.numpy(), GOLDEN[f"{name}/topk_ids"])
    assert np.array_equal(st.topk_logits.numpy(), GOLDEN[f"{name}/topk_logits"])
    assert np.array_equal(st.probs.numpy(), GOLDEN[f"{name}/probs"])
    assert np.array_equal(st.cumsum.numpy(), GOLDEN[f"{name}/cumsum"])
    assert np.array_equal(st.keep.numpy(), GOLDEN[f"{name}/keep"])
    assert np.array_equal(st.cutoff.numpy(), GOLDEN[f"{name}/cutoff"])
    assert np.array_equal(st.renormed.numpy(), GOLDEN[f"{name}/renormed"], equal_nan=False)


def test_known_answer_hand_cut():
    # 0.40 0.30 0.15 0.10 0.05 at p=0.9 keeps four (reference tests/test_reference.py:69-74)
    x = torch.tensor([[0.40, 0.30, 0.15, 0.10, 0.05]]).log()
    st = orc.stages(x, 5, 0.9)
    assert st.cutoff.item() == 4
    assert st.keep.tolist() == [[True, True, True, True, False]]


def test_known_answer_equal_logits_cut_is_inclusive():
    # tests/test_reference.py:77-83
    st = orc.stages(torch.zeros(1, 4), 4, 0.5)
    assert st.cumsum.tolist() == [[0.25, 0.5, 0.75, 1.0]]
    assert st.cutoff.item() == 2


@pytest.mark.parametrize("p,kept", [(0.25, 2), (0.5, 4), (0.75, 6), (0.875, 7)])
def test_known_answer_eight_equal_logits(p, kept):
    # tests/test_fused_kernel.py:244-257
    x = torch.full((4, 4000), -30.0)
    x[:, :8] = 10.0
    st = orc.stages(x.to(torch.bfloat16), 8, p)
    assert st.keep.sum(-1).tolist() == [kept] * 4


def test_known_answer_ties_lowest_id():
    x = torch.zeros(1, 64)
    x[0, ::2] = 1.0
    assert orc.stages(x.to(torch.bfloat16), 8, 1.0).topk_ids[0].tolist() == list(range(0, 16, 2))
    y = torch.zeros(1, 20)
    y[0, 3:12] = 5.0
    assert orc.stages(y.to(torch.float16), 5, 1.0).topk_ids[0].tolist() == [3, 4, 5, 6, 7]
    z = torch.zeros(4, 4000, dtype=torch.bfloat16)
    assert torch.equal(orc.stages(z, 50, 0.9).topk_ids, torch.arange(50).expand(4, 50))


def test_signed_zeros_tie():
    # -0 and +0 are one value: lowest id first regardless of sign
    x = torch.tensor([[-1.0, -0.0, 0.0, -0.0, 0.0, -1.0]], dtype=torch.bfloat16)
    assert orc.topk_order(orc.bits16(x), 4)[0].tolist() == [1, 2, 3, 4]
    keys = orc.order_keys(np.array([0x8000, 0x0000], dtype=np.uint16))
    assert keys[0] == keys[1] == 0x8000


def test_order_keys_are_monotone_for_every_finite_pattern():
    for dtype in (torch.float16, torch.bfloat16):
        bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
        vals = torch.from_numpy(bits.view(np.int16)).view(dtype).float().numpy()
        ok = ~np.isnan(vals)
        keys = orc.order_keys(bits)[ok].astype(np.int64)
        v = vals[ok]
        order = np.argsort(v, kind="stable")
        # keys are non-decreasing along increasing value; equal only for equal values
        dk = np.diff(keys[order])
        dv = np.diff(v[order])
        assert (dk >= 0).all()
        assert ((dk == 0) == (dv == 0)).all()


def test_splitmix_matches_the_published_first_output():
    # splitmix64 from state 0 first returns 0xE220A8397B1DCDAF; the reference's uniform with
    # seed 0, offset 1, row 0 evaluates exactly that finaliser at the golden gamma.
    assert orc.splitmix64_finalize(orc.GOLDEN_GAMMA) == 0xE220A8397B1DCDAF
    u = orc.splitmix_uniform(0, 1, 0)
    assert u == np.float32(0xE220A8) / np.float32(16777216.0)
    assert 0.0 <= orc.splitmix_uniform(0x5EED, 7, 3) < 1.0


def test_splitmix_uniforms_differ_by_row_and_offset():
    a = orc.splitmix_uniforms(7, 3, 64)
    b = orc.splitmix_uniforms(7, 4, 64)
    assert len(set(a.tolist())) > 60
    assert not np.array_equal(a, b)
    assert np.array_equal(orc.splitmix_uniforms(7, 3, 8, row_base=56), a[56:])


def test_draw_picks_inside_the_nucleus():
    x = orc.anchor_logits(B=4, V=4000)
    d = orc.sample(x, 50, 0.9, seed=1, offset=2)
    assert (d.pick < d.stages.cutoff.numpy()).all()
    assert np.array_equal(d.ids, d.stages.topk_ids.numpy()[np.arange(4), d.pick])


def test_draw_frequencies_follow_the_fp64_categorical():
    # reference tests/test_reference.py:397-406, via the oracle's draw rule
    probs = [0.40, 0.30, 0.15, 0.10, 0.05]
    n = 20000
    x = torch.tensor(probs).log().expand(n, 5).contiguous().to(torch.bfloat16)
    u = np.random.default_rng(0).random(n, dtype=np.float32)
    d = orc.draw(orc.stages(x, 5, 1.0), u, 1.0)
    freq = np.bincount(d.pick, minlength=5) / n
    ids, pr = orc.categorical_fp64(x[0], 5, 1.0)
    assert (np.abs(freq - pr) < 4 * np.sqrt(0.4 * 0.6 / n)).all()


def test_validation_messages():
    x = torch.randn(4, 100)
    x[2, 7] = float("nan")
    with pytest.raises(ValueError, match="NaN"):
        orc.validate_logits(x)
    y = torch.randn(4, 100)
    y[1, 3] = float("inf")
    with pytest.raises(ValueError, match=r"\+inf"):
        orc.validate_logits(y)
    z = torch.randn(4, 100)
    z[3] = float("-inf")
    with pytest.raises(ValueError, match="entirely -inf"):
        orc.validate_logits(z)
    assert orc.row_status(x).tolist() == [0, 0, 1, 0]


def test_adversarial_generators_have_their_shapes():
    a = orc.adversarial_logits(1, B=2, V=1000)
    assert len(torch.unique(a.float())) == 16
    d = orc.adversarial_logits(4, B=4, V=1000)
    st = orc.row_status(d)
    assert st.tolist() == [0, 2, 3, 0]


REF_RNG = np.load(Path(__file__).parent / "golden" / "ref_rng_vectors.npz")


def test_splitmix_matches_the_reference_kernel_bit_for_bit():
    # vectors from the reference's own rng_uniform run on a B200 (tests/golden/make_rng_golden.py)
    got = np.array([orc.splitmix_uniform(int(s), int(o), int(r))
                    for s, o, r in zip(REF_RNG["seed"], REF_RNG["offset"], REF_RNG["row"])], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), REF_RNG["u_bits"])


def test_order_keys_match_the_reference_except_the_negative_zero_fold():
    ref = REF_RNG["mono_key"]
    ours = orc.order_keys(np.arange(1 << 16, dtype=np.uint32).astype(np.uint16))
    diff = np.nonzero(ref != ours)[0]
    # the reference keys -0 (0x8000) as 0x7FFF, one below +0; the oracle folds it onto +0
    assert diff.tolist() == [0x8000]
    assert ref[0x8000] == 0x7FFF and ours[0x8000] == 0x8000


def test_pick_consistency_accepts_the_oracle_pick_and_rejects_far_neighbours():
    """The interval check used at k near V: the oracle's own FP32 pick lies inside the exact
    (FP64) CDF interval of the target, a token 50 places later does not, and the FP32 drift of
    torch's softmax over ~1.5e5 candidates is measured in the 1e-7..1e-5 range."""
    x = orc.adversarial_logits(2, B=4, V=151936, seed=2)
    u = orc.splitmix_uniforms(0x5EED, 0, 4)
    d = orc.sample(x, 151936, 0.5, uniforms=u)
    assert orc.pick_consistent(d.stages, d.ids, u, 0.5).all()
    far = d.stages.topk_ids.numpy()[np.arange(4), d.pick + 50]
    assert not orc.pick_consistent(d.stages, far, u, 0.5).any()
    err = orc.fp32_cumsum_error(d.stages)
    assert (err > 0).all() and (err < 1e-4).all()
    d64 = orc.draw_fp64(d.stages, u, 0.5)
    assert orc.pick_consistent(d.stages, d64.ids, u, 0.5).all()
