"""Pin the CPU oracle before trusting it (no GPU).

1. The reference's own known-answer packing tests (tests/test_pack.py in the
   reference), restated here with the same literal words.
2. Golden vectors produced by running the reference's kernels on the same
   seeded inputs (tests/golden/make_golden.py).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.cases import CASES


# --- reference tests/test_pack.py:25-52, 101-111, restated ------------------
def test_pack_2bit_lsb_first_known_words():
    codes = np.zeros((1, 128), dtype=np.uint32)
    codes[0, 0], codes[0, 1], codes[0, 15], codes[0, 16] = 2, 1, 2, 3
    packed = oracle.pack_2bit(codes)
    assert packed.dtype == np.uint32 and packed.shape == (1, 8)
    assert packed[0, 0] == np.uint32((2 << 0) | (1 << 2) | (2 << 30))
    assert packed[0, 1] == np.uint32(3)
    np.testing.assert_array_equal(oracle.unpack_2bit(packed), codes)


def test_pack_2bit_sixteen_codes_one_word():
    codes = (np.arange(16, dtype=np.uint32) % 3).reshape(1, 16)
    expected = 0
    for i, c in enumerate(codes[0]):
        expected |= int(c) << (2 * i)
    assert oracle.pack_2bit(codes)[0, 0] == np.uint32(expected)


def test_pack_4bit_lsb_first_known_word():
    codes = np.zeros((1, 64), dtype=np.uint32)
    codes[0, 0], codes[0, 1], codes[0, 7] = 0xA, 0x3, 0xF
    packed = oracle.pack_4bit(codes)
    assert packed.shape == (1, 8)
    assert packed[0, 0] == np.uint32((0xA << 0) | (0x3 << 4) | (0xF << 28))
    np.testing.assert_array_equal(oracle.unpack_4bit(packed), codes)


def test_ternarize_sign_mask_alpha_zero_row():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((32, 128)).astype(np.float32)
    packed, alpha = oracle.ternarize(w)
    t = oracle.unpack_2bit(packed).astype(np.float32) - 1
    aw = np.abs(w)
    mask = aw > 0.7 * aw.mean(-1, keepdims=True)
    np.testing.assert_array_equal(t, np.sign(w) * mask)
    np.testing.assert_allclose(alpha, (aw * mask).sum(-1) / mask.sum(-1), rtol=1e-6)
    p0, a0 = oracle.ternarize(np.zeros((2, 128), np.float32))
    np.testing.assert_array_equal(oracle.unpack_2bit(p0), np.ones((2, 128), np.uint32))
    np.testing.assert_array_equal(a0, 0)
    with pytest.raises(ValueError, match="multiple"):
        oracle.ternarize(np.ones((4, 64), np.float32))


def test_quantize_rtn_roundtrip_within_half_scale():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((16, 64)).astype(np.float32)
    packed, s, b = oracle.quantize_rtn(w)
    rec = oracle.dequantize_rtn(packed, s, b)
    assert np.all(np.abs(rec - w) <= 0.5 * s[:, :1] + 1e-5)


def test_bf16_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.0e38, np.nan, np.inf], np.float32)
    bits = oracle.bf16_bits(x)
    assert bits[0] == 0x3F80 and bits[1] == 0x3F80 and bits[2] == 0x3F81
    assert bits[4] == 0x7FC0 and bits[5] == 0x7F80


def test_oracle_exp_accuracy():
    x = np.linspace(-100, 80, 20001, dtype=np.float32)
    got = oracle.mexp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ok = ref > 1e-37
    rel = np.abs(got[ok] - ref[ok]) / ref[ok]
    assert rel.max() < 3e-7, rel.max()
    assert oracle.mexp(np.zeros(1))[0] == 1.0


# --- oracle vs the reference's own kernels on identical inputs ---------------
@pytest.mark.parametrize("name", [n for n, c in CASES.items() if c.kind == "ternary_gemv"])
def test_oracle_ternary_gemv_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    y_ref = golden[f"{name}/y"]
    y = oracle.ternary_gemv(d["x"], d["packed"], d["alpha"], d["rms_weight"], 1e-6, out_bf16=False)
    # Both accumulate in >= fp32; the reference's tl.rsqrt is approximate.
    np.testing.assert_allclose(y, y_ref, rtol=2e-5, atol=2e-6 * np.abs(y_ref).max())


def _close(got, want, rtol, what=""):
    """max |got - want| <= rtol * max |want| (a scale-relative bound: values
    near zero carry the row's absolute rounding, not their own)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want).max()
    scale = np.abs(want).max()
    assert err <= rtol * scale, f"{what}: max err {err:.3g} > {rtol:g} * {scale:.3g}"


def _cases(kind):
    return [n for n, c in CASES.items() if c.kind == kind]


# Router: indices bit-exact (ties to the lower index), weights to fp32 rounding.
@pytest.mark.parametrize("name", _cases("router"))
def test_oracle_router_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    idx, wt = oracle.router_topk(d["x"], d["gate"], case.top_k)
    np.testing.assert_array_equal(idx, golden[f"{name}/idx"])
    np.testing.assert_allclose(wt, golden[f"{name}/wt"], rtol=2e-6, atol=1e-7)
    # The margin that makes the selection robust to summation order: the gap
    # between the 8th and 9th logit (exact in float64), reported per token.
    logits = d["x"].astype(np.float64) @ d["gate"].astype(np.float64).T
    srt = -np.sort(-logits, axis=-1)
    gap = srt[:, case.top_k - 1] - srt[:, case.top_k]
    print(f"{name}: min top-{case.top_k}/{case.top_k + 1} logit gap {gap.min():.3e}")
    if case.ties:
        # duplicated gate rows score alike; the lower index must come first
        for t in range(idx.shape[0]):
            pos = {int(e): r for r, e in enumerate(idx[t])}
            for lo, hi in ((5, 9), (3, 40), (17, 30), (30, 61)):
                if lo in pos and hi in pos:
                    assert pos[lo] < pos[hi]


@pytest.mark.parametrize("name", _cases("norms"))
def test_oracle_norms_match_reference(golden, name):
    d = CASES[name].inputs()
    _close(oracle.rms_norm(d["x"], d["w"], 1e-6, out_bf16=False), golden[f"{name}/rms"], 1e-6, "rms_norm")
    res, nrm = oracle.add_rms_norm(d["x"], d["y"], d["w"], 1e-6, out_bf16=False)
    np.testing.assert_array_equal(res, golden[f"{name}/residual"])
    _close(nrm, golden[f"{name}/normed"], 1e-6, "add_rms_norm")
    _close(oracle.moe_reduce_add(d["slots"], d["wt"], d["x"], out_bf16=False), golden[f"{name}/reduce"], 1e-6,
           "moe_reduce_add")
    _close(oracle.moe_reduce_add(d["slots"], d["wt"], None, out_bf16=False), golden[f"{name}/reduce_nores"], 1e-6,
           "moe_reduce_add (no residual)")


@pytest.mark.parametrize("name", _cases("experts"))
def test_oracle_experts_match_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    h = oracle.expert_swiglu(d["x"], d["ug"], d["ug_a"], d["ids"], out_bf16=False)
    _close(h, golden[f"{name}/h"], 2e-6, "expert swiglu")
    T, k = d["ids"].shape
    y = oracle.expert_gemv(d["h_in"].reshape(T * k, -1), d["down"], d["down_a"], d["ids"].reshape(-1),
                           out_bf16=False)
    _close(y.reshape(T, k, -1), golden[f"{name}/down"], 2e-6, "expert down")
    out = oracle.expert_down_reduce(d["h_in"], d["down"], d["down_a"], d["ids"], d["wt"], d["residual"], mode=1,
                                    out_bf16=False)
    _close(out, golden[f"{name}/down_sum"], 2e-6, "expert down_sum")
    if case.alpha_scale > 0.1:  # the clamp case must actually clamp
        up_gate = golden[f"{name}/h"]
        assert np.abs(up_gate).max() > 7.0


@pytest.mark.parametrize("name", _cases("attention"))
def test_oracle_attention_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    kc, vc = d["kc"].copy(), d["vc"].copy()
    q = oracle.apply_qkv_decode(d["qkv"], d["qw"], d["kw"], d["cos"], d["sin"], kc, vc, d["seqlen"], d["row_map"],
                                num_heads=case.hq, num_kv_heads=case.hkv, head_dim=case.d, use_rope=case.use_rope,
                                eps=1e-6, out_bf16=False)
    _close(q, golden[f"{name}/q"], 2e-6, "q (QK-norm + RoPE)")
    rows = np.arange(len(case.lengths)) if d["row_map"] is None else d["row_map"]
    _close(kc[rows, :, d["seqlen"], :], golden[f"{name}/k_new"], 2e-6, "stored K row")
    np.testing.assert_array_equal(vc[rows, :, d["seqlen"], :], golden[f"{name}/v_new"])
    out = oracle.decode_gqa(q, kc, vc, d["seqlen"], d["row_map"], scale=np.float32(case.d ** -0.5),
                            window=case.window, split_len=64, out_bf16=False)
    _close(out, golden[f"{name}/out"], 1e-5, "attention out")


@pytest.mark.parametrize("name", _cases("rtn4"))
def test_oracle_rtn4_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    biases = None if case.symmetric else d["b"]  # symmetric: the oracle's own b = -8 s
    if case.n_clusters:
        S = case.cluster_size
        rows = (d["cids"][:, None] * S + np.arange(S)).reshape(-1)
        y = oracle.rtn4_gemv(d["x"], d["packed"], d["s"], biases, case.group, row_index=rows, out_bf16=False)
    else:
        y = oracle.rtn4_gemv(d["x"], d["packed"], d["s"], biases, case.group, out_bf16=False)
    _close(y, golden[f"{name}/y"], 2e-6, "rtn4")


@pytest.mark.parametrize("name", _cases("sampler"))
def test_oracle_sampler_matches_reference(golden, name):
    case = CASES[name]
    d = case.inputs()
    got = np.stack([oracle.fused_sample(d["logits"], np.full(case.batch, u, np.float32),
                                        temperature=case.temperature, top_p=case.top_p, top_k=case.top_k)
                    for u in d["u"]], axis=1)
    np.testing.assert_array_equal(got, golden[f"{name}/single"])
    np.testing.assert_array_equal(got, golden[f"{name}/batched"])
