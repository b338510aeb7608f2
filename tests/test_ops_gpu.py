"""Every sm_100a decode operator vs the CPU oracle on identical inputs: bit-exact (GPU)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.helpers import alpha_bf, bf, randn_bf, rng, tern_packed, to_dev, to_np

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
BF = None


@pytest.fixture(scope="module")
def K():
    from maple_flash_dgx_spark_b200 import kernels

    return kernels


@pytest.fixture(autouse=True)
def _no_device_errors(cuda):
    from maple_flash_dgx_spark_b200 import _lib

    _lib.take_device_errors(cuda)
    yield


@pytest.mark.parametrize("rows,n", [(1, 2048), (3, 2048), (2, 128), (1, 4096)])
def test_norms(cuda, K, rows, n):
    rs = rng(rows * 7 + n)
    x, y = randn_bf(rs, rows, n), randn_bf(rs, rows, n)
    w = (1 + 0.02 * rs.standard_normal(n)).astype(np.float32)
    xt, yt, wt = to_dev(x, cuda, torch.bfloat16), to_dev(y, cuda, torch.bfloat16), to_dev(w, cuda)
    np.testing.assert_array_equal(to_np(K.rms_norm(xt, wt, 1e-6)), oracle.rms_norm(x, w, 1e-6))
    r, nrm = K.add_rms_norm(xt, yt, wt, 1e-6)
    r_o, n_o = oracle.add_rms_norm(x, y, w, 1e-6)
    np.testing.assert_array_equal(to_np(r), r_o)
    np.testing.assert_array_equal(to_np(nrm), n_o)


@pytest.mark.parametrize("T,E,topk,k", [(1, 64, 8, 2048), (5, 64, 8, 2048), (3, 4, 2, 128), (2, 256, 8, 1024)])
def test_router_topk(cuda, K, T, E, topk, k):
    rs = rng(T * 100 + E)
    x = randn_bf(rs, T, k)
    g = randn_bf(rs, E, k, scale=0.02)
    idx, wt = K.router_topk(to_dev(x, cuda, torch.bfloat16), to_dev(g, cuda, torch.bfloat16), topk)
    idx_o, wt_o = oracle.router_topk(x, g, topk)
    np.testing.assert_array_equal(to_np(idx), idx_o)
    np.testing.assert_array_equal(to_np(wt), wt_o)


def test_router_ties_take_lowest_index(cuda, K):
    x = np.ones((1, 128), np.float32)
    g = np.zeros((8, 128), np.float32)  # all logits equal
    idx, wt = K.router_topk(to_dev(x, cuda, torch.bfloat16), to_dev(g, cuda, torch.bfloat16), 3)
    np.testing.assert_array_equal(to_np(idx), [[0, 1, 2]])


@pytest.mark.parametrize("T,topk,E,inter,k", [(1, 8, 64, 1024, 2048), (3, 2, 4, 128, 128), (2, 8, 16, 96, 1024)])
def test_expert_swiglu(cuda, K, T, topk, E, inter, k):
    rs = rng(T + topk + inter)
    x = randn_bf(rs, T, k)
    packed = tern_packed(rs, E, 2 * inter, k)
    alpha = bf(alpha_bf(rs, E, 2 * inter) * 40)  # larger scales exercise the clamp
    ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    h = K.ternary_expert_swiglu(to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda),
                                to_dev(alpha, cuda, torch.bfloat16), to_dev(ids, cuda))
    h_o = oracle.expert_swiglu(x, packed, alpha, ids)
    np.testing.assert_array_equal(to_np(h), h_o)


@pytest.mark.parametrize("per_slot", [False, True])
def test_expert_gemv(cuda, K, per_slot):
    rs = rng(5 + per_slot)
    T, topk, E, N, k = 3, 4, 8, 320, 1024
    x = randn_bf(rs, T, topk, k) if per_slot else randn_bf(rs, T, k)
    packed = tern_packed(rs, E, N, k)
    alpha = alpha_bf(rs, E, N)
    ids = rs.randint(0, E, size=(T, topk)).astype(np.int32)
    y = K.ternary_expert_gemv(to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda), to_dev(alpha, cuda, torch.bfloat16),
                              to_dev(ids, cuda))
    y_o = oracle.expert_gemv(x.reshape(-1, k), packed, alpha, ids, x_rows_per_token=1 if per_slot else topk)
    np.testing.assert_array_equal(to_np(y).reshape(-1, N), y_o)


@pytest.mark.parametrize("mode", ["reduce", "sum"])
@pytest.mark.parametrize("T,topk,E,N,k", [(1, 8, 64, 2048, 1024), (4, 2, 4, 128, 128), (2, 8, 8, 200, 512)])
def test_expert_down(cuda, K, mode, T, topk, E, N, k):
    rs = rng(T * topk + N)
    h = randn_bf(rs, T, topk, k)
    packed = tern_packed(rs, E, N, k)
    alpha = alpha_bf(rs, E, N)
    ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    w = rs.random_sample((T, topk)).astype(np.float32)
    res = randn_bf(rs, T, N)
    fn = K.ternary_expert_down_reduce if mode == "reduce" else K.ternary_expert_down_sum
    out = fn(to_dev(h, cuda, torch.bfloat16), to_dev(packed, cuda), to_dev(alpha, cuda, torch.bfloat16), to_dev(ids, cuda),
             to_dev(w, cuda), to_dev(res, cuda, torch.bfloat16))
    out_o = oracle.expert_down_reduce(h, packed, alpha, ids, w, res, mode=0 if mode == "reduce" else 1)
    np.testing.assert_array_equal(to_np(out), out_o)


@pytest.mark.parametrize("skew", [False, True])
def test_grouped_expert_gemms_decode_sizes(cuda, K, skew):
    """configs[3]'s MoE at batch 64 (64 tokens x top-8 over 64 experts, ~8
    slots per expert: the single-buffer grouped kernels): SwiGLU (K=2048,
    I=1024) and down (K=1024, N=2048) equal the oracle bit for bit.  The
    skewed routing sends many slots to a few experts (several digit chunks
    per expert), leaves others empty, and has one out-of-range id (a NaN
    row)."""
    rs = rng(71 + skew)
    T, topk, E, inter, k = 64, 8, 64, 1024, 2048
    x = randn_bf(rs, T, k)
    up = tern_packed(rs, E, 2 * inter, k)
    a_up = bf(alpha_bf(rs, E, 2 * inter) * 40)
    down = tern_packed(rs, E, k, inter)
    a_dn = alpha_bf(rs, E, k)
    if skew:
        hot = np.array([3, 17, 64, 127])
        ids = np.stack([np.concatenate([hot, rs.permutation(np.setdiff1d(np.arange(40), hot))[:topk - 4]])
                        for _ in range(T)]).astype(np.int32)
        ids[5, 7] = -1
    else:
        ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    h = K.ternary_expert_swiglu(to_dev(x, cuda, torch.bfloat16), to_dev(up, cuda), to_dev(a_up, cuda, torch.bfloat16),
                                to_dev(ids, cuda))
    h_o = oracle.expert_swiglu(x, up, a_up, ids)
    np.testing.assert_array_equal(to_np(h), h_o)
    y = K.ternary_expert_gemv(to_dev(h_o, cuda, torch.bfloat16), to_dev(down, cuda), to_dev(a_dn, cuda, torch.bfloat16),
                              to_dev(ids, cuda))
    y_o = oracle.expert_gemv(h_o.reshape(-1, inter), down, a_dn, ids, x_rows_per_token=1)
    np.testing.assert_array_equal(to_np(y).reshape(-1, k), y_o)
    if skew:
        assert np.isnan(y_o[5 * topk + 7]).all()


def test_moe_reduce_add(cuda, K):
    rs = rng(9)
    x = randn_bf(rs, 3, 8, 2048)
    w = rs.random_sample((3, 8)).astype(np.float32)
    r = randn_bf(rs, 3, 2048)
    y = K.moe_reduce_add(to_dev(x, cuda, torch.bfloat16), to_dev(w, cuda), to_dev(r, cuda, torch.bfloat16))
    np.testing.assert_array_equal(to_np(y), oracle.moe_reduce_add(x, w, r))


def _attn_case(rs, B, Hq, Hkv, D, T, lens, Bc=None):
    Bc = Bc or B
    qkv = randn_bf(rs, B, (Hq + 2 * Hkv) * D)
    qw = (1 + 0.02 * rs.standard_normal(D)).astype(np.float32)
    kw = (1 + 0.02 * rs.standard_normal(D)).astype(np.float32)
    kc = randn_bf(rs, Bc, Hkv, T, D)
    vc = randn_bf(rs, Bc, Hkv, T, D)
    pos = np.asarray(lens, np.int64) - 1
    inv = 1.0 / (1e6 ** (np.arange(0, D, 2, dtype=np.float32) / D))
    ang = np.outer(pos.astype(np.float32), inv)
    emb = np.concatenate([ang, ang], -1).astype(np.float32)
    cos, sin = bf(np.cos(emb)), bf(np.sin(emb))
    return qkv, qw, kw, kc, vc, pos, cos, sin


@pytest.mark.parametrize("B,Hq,Hkv,D,T,lens,split,window", [
    (1, 32, 4, 128, 4096, [4096], 64, 0),
    (1, 32, 4, 128, 768, [640], 32, 0),
    (7, 32, 4, 128, 1024, [1, 63, 64, 65, 300, 511, 1000], 64, 0),
    (2, 2, 2, 64, 64, [20, 64], 32, 0),
    (3, 16, 2, 128, 600, [600, 17, 333], 128, 0),
    (2, 8, 8, 128, 512, [512, 100], 64, 96),
    (1, 32, 4, 128, 512, [512], 32, 0),
    (2, 32, 4, 128, 1024, [1024, 700], 64, 0),
    (1, 32, 4, 128, 8192, [8192], 64, 0),
    (3, 16, 2, 128, 16384, [16384, 9000, 1], 128, 0),
])
@pytest.mark.parametrize("kv_final", [False, True])
def test_qkv_decode_and_attention(cuda, K, B, Hq, Hkv, D, T, lens, split, window, kv_final):
    """Up to 16 splits merge inside a thread-block cluster (sizes 1-16, idle
    ranks included), more through the workspace; kv_final loads the
    already-final rows before the PDL wait."""
    rs = rng(B * 31 + T)
    qkv, qw, kw, kc, vc, pos, cos, sin = _attn_case(rs, B, Hq, Hkv, D, T, lens)
    kc_d, vc_d = to_dev(kc, cuda, torch.bfloat16), to_dev(vc, cuda, torch.bfloat16)
    sl = to_dev(pos, cuda)
    q = K.apply_qkv_decode(to_dev(qkv, cuda, torch.bfloat16), to_dev(qw, cuda), to_dev(kw, cuda),
                           to_dev(cos, cuda, torch.bfloat16), to_dev(sin, cuda, torch.bfloat16), kc_d, vc_d, sl,
                           num_heads=Hq, num_kv_heads=Hkv, head_dim=D, rotary_dim=D, use_rope=True,
                           use_qk_norm=True, eps=1e-6)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = oracle.apply_qkv_decode(qkv, qw, kw, cos, sin, kc_o, vc_o, pos, num_heads=Hq, num_kv_heads=Hkv,
                                  head_dim=D)
    np.testing.assert_array_equal(to_np(q)[:, :, 0], q_o)
    np.testing.assert_array_equal(to_np(kc_d), kc_o)
    np.testing.assert_array_equal(to_np(vc_d), vc_o)
    out = K.decode_gqa_attn(q, kc_d, vc_d, sl, scale=D ** -0.5, window=window or None, split_len=split,
                            kv_final=kv_final)
    out_o = oracle.decode_gqa(q_o, kc_o, vc_o, pos, scale=np.float32(D ** -0.5), window=window, split_len=split)
    np.testing.assert_array_equal(to_np(out)[:, :, 0], out_o)


def test_attention_row_map_equals_gathered_cache(cuda, K):
    """Reference tests/test_fused_decode.py:364-402: row_map reads the mapped cache rows."""
    rs = rng(77)
    B, Bc, Hq, Hkv, D, T = 3, 5, 8, 2, 128, 256
    qkv, qw, kw, kc, vc, pos, cos, sin = _attn_case(rs, B, Hq, Hkv, D, T, [200, 31, 256], Bc=Bc)
    rmap = np.array([4, 0, 2], np.int32)
    kc_d, vc_d = to_dev(kc, cuda, torch.bfloat16), to_dev(vc, cuda, torch.bfloat16)
    sl, rm = to_dev(pos, cuda), to_dev(rmap, cuda)
    q = K.apply_qkv_decode(to_dev(qkv, cuda, torch.bfloat16), to_dev(qw, cuda), to_dev(kw, cuda),
                           to_dev(cos, cuda, torch.bfloat16), to_dev(sin, cuda, torch.bfloat16), kc_d, vc_d, sl,
                           row_map=rm, num_heads=Hq, num_kv_heads=Hkv, head_dim=D, rotary_dim=D, use_rope=True,
                           use_qk_norm=True, eps=1e-6)
    out = K.decode_gqa_attn(q, kc_d, vc_d, sl, row_map=rm, scale=D ** -0.5, window=None, split_len=64)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = oracle.apply_qkv_decode(qkv, qw, kw, cos, sin, kc_o, vc_o, pos, rmap, num_heads=Hq, num_kv_heads=Hkv,
                                  head_dim=D)
    out_o = oracle.decode_gqa(q_o, kc_o, vc_o, pos, rmap, scale=np.float32(D ** -0.5), split_len=64)
    np.testing.assert_array_equal(to_np(out)[:, :, 0], out_o)
    untouched = [1, 3]
    np.testing.assert_array_equal(to_np(kc_d)[untouched], kc[untouched])


def test_attention_vs_sdpa(cuda, K):
    """Within the reference's 1e-3 tolerance of torch SDPA (test_fused_decode.py:104-222)."""
    rs = rng(3)
    B, Hq, Hkv, D, T = 2, 32, 4, 128, 1000
    q = to_dev(randn_bf(rs, B, Hq, 1, D), cuda, torch.bfloat16)
    kc = to_dev(randn_bf(rs, B, Hkv, T, D), cuda, torch.bfloat16)
    vc = to_dev(randn_bf(rs, B, Hkv, T, D), cuda, torch.bfloat16)
    sl = torch.tensor([T - 1, 499], device=cuda)
    out = K.decode_gqa_attn(q, kc, vc, sl, scale=D ** -0.5, window=None)
    for b, n in enumerate([T, 500]):
        ref = torch.nn.functional.scaled_dot_product_attention(
            q[b:b + 1].float(), kc[b:b + 1, :, :n].float(), vc[b:b + 1, :, :n].float(), enable_gqa=True)
        torch.testing.assert_close(out[b:b + 1].float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("group,symmetric,B,k", [(128, True, 1, 2048), (64, False, 1, 2048), (128, False, 3, 2048),
                                                (256, True, 2, 2048), (128, True, 17, 2048), (64, True, 5, 2048),
                                                (128, True, 64, 2048), (128, False, 9, 4096)])
def test_rtn4_gemv(cuda, K, group, symmetric, B, k):
    """Batch >= 2 runs the batched head (rows encoded once, head streamed per
    16-row chunk); every row equals the batch-1 kernel's row."""
    rs = rng(group + B)
    N = 1000
    x = randn_bf(rs, B, k)
    codes = rs.randint(0, 16, size=(N, k)).astype(np.uint32)
    packed = oracle.pack_4bit(codes)
    s = bf(np.abs(rs.standard_normal((N, k // group))) * 0.003 + 1e-4)
    b = None if symmetric else bf(rs.standard_normal((N, k // group)) * 0.01)
    xd, pd = to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda)
    sd, bd = to_dev(s, cuda, torch.bfloat16), None if b is None else to_dev(b, cuda, torch.bfloat16)
    y = K.rtn4_gemv(xd, pd, sd, bd, group_size=group)
    np.testing.assert_array_equal(to_np(y), oracle.rtn4_gemv(x, packed, s, b, group))
    for r in {0, B - 1}:
        torch.testing.assert_close(y[r:r + 1], K.rtn4_gemv(xd[r:r + 1], pd, sd, bd, group_size=group), rtol=0, atol=0)


def test_rtn4_indexed_gemv(cuda, K):
    rs = rng(44)
    nc, C, k, P = 50, 32, 2048, 7
    x = randn_bf(rs, 1, k)
    packed = oracle.pack_4bit(rs.randint(0, 16, size=(nc * C, k)).astype(np.uint32))
    s = bf(np.abs(rs.standard_normal((nc * C, k // 64))) * 0.003)
    b = bf(rs.standard_normal((nc * C, k // 64)) * 0.01)
    cids = rs.permutation(nc)[:P].astype(np.int32)
    y = K.rtn4_indexed_gemv(to_dev(x, cuda, torch.bfloat16), to_dev(packed.reshape(nc, C, -1), cuda),
                            to_dev(s.reshape(nc, C, -1), cuda, torch.bfloat16),
                            to_dev(b.reshape(nc, C, -1), cuda, torch.bfloat16), to_dev(cids, cuda), group_size=64)
    rows = (cids[:, None].astype(np.int64) * C + np.arange(C)).reshape(-1)
    np.testing.assert_array_equal(to_np(y), oracle.rtn4_gemv(x, packed, s, b, 64, row_index=rows))


@pytest.mark.parametrize("V", [151936, 1000, 8192])
def test_argmax(cuda, K, V):
    rs = rng(V)
    logits = randn_bf(rs, 3, V)
    logits[1, 17] = logits[1].max()   # a tie: the first index wins
    logits[1, 5] = logits[1].max()
    got = K.argmax(to_dev(logits, cuda, torch.bfloat16))
    np.testing.assert_array_equal(to_np(got), oracle.argmax(logits))


@pytest.mark.parametrize("top_k,top_p,temp", [(20, 0.95, 1.0), (2, 1.0, 0.8), (64, 0.5, 1.3)])
def test_fused_sampler(cuda, K, top_k, top_p, temp):
    rs = rng(top_k)
    V = 151936
    logits = (rs.standard_normal((4, V)) * 3).astype(np.float32)
    for u in (0.0, 0.25, 0.5, 0.75, 0.999):
        uu = np.full(4, u, np.float32)
        got = K.fused_sample_batched(to_dev(logits, cuda), to_dev(uu, cuda), temperature=temp, top_p=top_p,
                                     top_k=top_k)
        np.testing.assert_array_equal(to_np(got), oracle.fused_sample(logits, uu, temperature=temp, top_p=top_p,
                                                                      top_k=top_k))
    one = K.fused_sample(to_dev(logits[2], cuda), to_dev(np.float32(0.5), cuda), temperature=temp, top_p=top_p,
                         top_k=top_k)
    assert int(one) == int(oracle.fused_sample(logits[2:3], np.float32([0.5]), temperature=temp, top_p=top_p,
                                               top_k=top_k)[0])


def test_embeddings(cuda, K):
    rs = rng(12)
    V, H = 1000, 2048
    table = randn_bf(rs, V, H, scale=0.02)
    ids = np.array([0, 999, 17], np.int64)
    e = K.embedding(to_dev(ids, cuda), to_dev(table, cuda, torch.bfloat16))
    np.testing.assert_array_equal(to_np(e), table[ids])
    packed = oracle.pack_4bit(rs.randint(0, 16, size=(V, H)).astype(np.uint32))
    s = bf(np.abs(rs.standard_normal((V, H // 64))) * 0.003)
    b = bf(rs.standard_normal((V, H // 64)) * 0.01)
    r = K.rtn4_embedding(to_dev(ids, cuda), to_dev(packed, cuda), to_dev(s, cuda, torch.bfloat16),
                         to_dev(b, cuda, torch.bfloat16), group_size=64)
    np.testing.assert_array_equal(to_np(r), oracle.rtn4_embedding(ids, packed, s, b, 64, out_bf16=False))


def test_synthetic_generator_matches_oracle(cuda):
    """The device generator and the oracle's independent one agree bit for bit."""
    from maple_flash_dgx_spark_b200 import synth as S
    from oracle import model as om

    t = S._ternary(5, 77, (64, 128), cuda)
    np.testing.assert_array_equal(to_np(t.view(torch.int32)).view(np.uint32), om.synth_ternary(5, 77, (64, 128)))
    n = S._normal(5, 78, (3000,), cuda, 0.02, 1e-3, True)
    np.testing.assert_array_equal(to_np(n), om.synth_normal(5, 78, (3000,), 0.02, 1e-3, True))
    f = S._normal(5, 79, (3000,), cuda, 0.02, 1.0, dtype=torch.float32)
    np.testing.assert_array_equal(to_np(f), om.synth_normal(5, 79, (3000,), 0.02, 1.0, bf16=False))
    codes = torch.empty(40, 2048 // 8, dtype=torch.int32, device=cuda).view(torch.uint32)
    scales = torch.empty(40, 16, dtype=torch.bfloat16, device=cuda)
    from maple_flash_dgx_spark_b200._lib import lib, ptr, stream_ptr

    assert lib().maple_synth_rtn4_sym(5, 80, 40, 2048, 128, 0.02, ptr(codes), ptr(scales), stream_ptr(cuda)) == 0
    c_o, s_o = om.synth_rtn4_sym(5, 80, 40, 2048, 128, 0.02)
    np.testing.assert_array_equal(to_np(codes.view(torch.int32)).view(np.uint32), c_o)
    np.testing.assert_array_equal(to_np(scales), s_o)
    tok = S.synthetic_tokens(5, 100, 151936, cuda)
    np.testing.assert_array_equal(to_np(tok), om.synth_tokens(5, 100, 151936))


def test_row_uniform_per_sequence(cuda, K):
    """Counter-based per-row uniforms: in [0, 1), a fresh draw per call, the
    same sequence for the same seeds, independent of the other rows."""
    a = K.RowUniform([7, 8, 9], cuda)
    b = K.RowUniform([7, 100, 9], cuda)
    d1, d2 = a().clone(), a().clone()
    e1 = b().clone()
    assert ((d1 >= 0) & (d1 < 1)).all() and not torch.equal(d1, d2)
    assert d1[0] == e1[0] and d1[2] == e1[2] and d1[1] != e1[1]
    c = K.RowUniform([7, 8, 9], cuda)
    torch.testing.assert_close(c(), d1, rtol=0, atol=0)


@pytest.mark.parametrize("T", [1, 5])
def test_add_norm_router_fused_equals_sequence(cuda, K, T):
    """The fused add + RMSNorm + router launch returns exactly what
    add_rms_norm followed by router_topk returns."""
    rs = rng(60 + T)
    H, E = 2048, 64
    x = to_dev(randn_bf(rs, T, H), cuda, torch.bfloat16)
    y = to_dev(randn_bf(rs, T, H, scale=0.5), cuda, torch.bfloat16)
    w = to_dev((1 + 0.05 * rs.standard_normal(H)).astype(np.float32), cuda)
    g = to_dev(randn_bf(rs, E, H, scale=0.02), cuda, torch.bfloat16)
    res, normed = K.add_rms_norm(x, y, w, 1e-6)
    idx, wt = K.router_topk(normed, g, 8)
    r2, n2, i2, w2 = K.add_rms_norm_router_topk(x, y, w, 1e-6, g, 8)
    for a, b in ((res, r2), (normed, n2), (idx, i2), (wt, w2)):
        torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("B,Hq,Hkv,D,T,lens,split,window,remap", [
    (1, 32, 4, 128, 4096, [4096], 64, 0, False),
    (1, 32, 4, 128, 768, [640], 32, 0, False),
    (7, 32, 4, 128, 1024, [1, 63, 64, 65, 300, 511, 1000], 64, 0, False),
    (2, 2, 2, 64, 64, [20, 64], 32, 0, False),
    (3, 16, 2, 128, 600, [600, 17, 333], 128, 0, True),
    (2, 8, 8, 128, 512, [512, 100], 64, 96, False),
    (1, 32, 4, 128, 8192, [8192], 64, 0, False),
    (3, 16, 2, 128, 16384, [16384, 9000, 1], 128, 0, True),
])
def test_fused_qk_attention_equals_two_launches(cuda, K, B, Hq, Hkv, D, T, lens, split, window, remap):
    """decode_gqa_attn_qk == apply_qkv_decode + decode_gqa_attn (oracle), out
    and caches bit for bit, cluster and workspace merges, through a row map."""
    rs = rng(B * 57 + T)
    Bc = B + 2 if remap else B
    qkv, qw, kw, kc, vc, pos, _, _ = _attn_case(rs, B, Hq, Hkv, D, T, lens, Bc=Bc)
    inv = 1.0 / (1e6 ** (np.arange(0, D, 2, dtype=np.float32) / D))
    ang = np.outer(np.arange(T, dtype=np.float32), inv)
    emb = np.concatenate([ang, ang], -1).astype(np.float32)
    cos_t, sin_t = bf(np.cos(emb)), bf(np.sin(emb))
    rmap = (np.arange(B, dtype=np.int32)[::-1] + 2).copy() if remap else None
    kc_d, vc_d = to_dev(kc, cuda, torch.bfloat16), to_dev(vc, cuda, torch.bfloat16)
    out = K.decode_gqa_attn_qk(to_dev(qkv, cuda, torch.bfloat16), to_dev(qw, cuda), to_dev(kw, cuda),
                               to_dev(cos_t, cuda, torch.bfloat16), to_dev(sin_t, cuda, torch.bfloat16), kc_d, vc_d,
                               to_dev(pos, cuda), row_map=None if rmap is None else to_dev(rmap, cuda),
                               num_heads=Hq, num_kv_heads=Hkv, head_dim=D, rotary_dim=D, use_rope=True, eps=1e-6,
                               scale=D ** -0.5, window=window or None, split_len=split)
    kc_o, vc_o = kc.copy(), vc.copy()
    q_o = oracle.apply_qkv_decode(qkv, qw, kw, cos_t[pos], sin_t[pos], kc_o, vc_o, pos, rmap, num_heads=Hq,
                                  num_kv_heads=Hkv, head_dim=D)
    out_o = oracle.decode_gqa(q_o, kc_o, vc_o, pos, rmap, scale=np.float32(D ** -0.5), window=window,
                              split_len=split)
    np.testing.assert_array_equal(to_np(out)[:, :, 0], out_o)
    np.testing.assert_array_equal(to_np(kc_d), kc_o)
    np.testing.assert_array_equal(to_np(vc_d), vc_o)
