"""Batched ternary GEMM and grouped expert GEMM (weights read once per batch)
vs the CPU oracle and vs the per-row GEMV: bit-exact (GPU).

Reference coverage: tests/test_ternary_gemv.py (batched GEMM branch) and
tests/test_model.py:194-242 (MoE block vs a per-expert loop).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.helpers import alpha_bf, bf, randn_bf, rng, tern_packed, to_dev, to_np

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from maple_flash_dgx_spark_b200 import kernels

    return kernels


@pytest.mark.parametrize("B,n,k,rms", [(4, 5120, 2048, True), (9, 2048, 4096, False), (64, 1000, 1024, False),
                                       (17, 300, 1472, True), (64, 5120, 2048, True), (5, 48, 64, False)])
def test_dense_gemm_vs_oracle_and_rows(cuda, K, B, n, k, rms):
    rs = rng(B * 7 + n + k)
    x = randn_bf(rs, B, k)
    packed = tern_packed(rs, n, k)
    alpha = alpha_bf(rs, n)
    w = (1 + 0.05 * rs.standard_normal(k)).astype(np.float32) if rms else None
    xd = to_dev(x, cuda, torch.bfloat16)
    pd, ad = to_dev(packed, cuda), to_dev(alpha, cuda, torch.bfloat16)
    wd = to_dev(w, cuda) if rms else None
    y = K.ternary_gemv(xd, pd, ad, rms_weight=wd, rms_eps=1e-6)
    y_o = oracle.ternary_gemv(x, packed, alpha, w, 1e-6, out_bf16=True)
    np.testing.assert_array_equal(to_np(y), y_o)
    # each row equals the batch-1 GEMV of that row
    for r in (0, B // 2, B - 1):
        y1 = K.ternary_gemv(xd[r:r + 1], pd, ad, rms_weight=wd, rms_eps=1e-6)
        torch.testing.assert_close(y[r:r + 1], y1, rtol=0, atol=0)


def test_dense_gemm_nonfinite_row_is_nan(cuda, K):
    rs = rng(3)
    x = randn_bf(rs, 6, 256)
    x[2, 17] = np.inf
    packed, alpha = tern_packed(rs, 64, 256), alpha_bf(rs, 64)
    y = to_np(K.ternary_gemv(to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda), to_dev(alpha, cuda, torch.bfloat16)))
    assert np.isnan(y[2]).all()
    np.testing.assert_array_equal(np.delete(y, 2, 0), np.delete(oracle.ternary_gemv(x, packed, alpha, out_bf16=True),
                                                                 2, 0))


def test_moe_plan_sorts_slots(cuda, K):
    rs = rng(4)
    T, topk, E = 37, 8, 64
    ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    ids[5, 3] = 99  # out of range: listed under expert 0, flagged
    plan = K.moe_plan(to_dev(ids, cuda), E)
    off = to_np(plan.offsets)
    lst = to_np(plan.slots).view(np.uint32)
    assert off[0] == 0 and off[-1] == T * topk and (np.diff(off) >= 0).all()
    flat = ids.reshape(-1)
    seen = np.zeros(T * topk, bool)
    for e in range(E):
        for v in lst[off[e]:off[e + 1]]:
            s = int(v & 0x7FFFFFFF)
            assert not seen[s]
            seen[s] = True
            if v & 0x80000000:
                assert e == 0 and not (0 <= flat[s] < E)
            else:
                assert flat[s] == e
    assert seen.all()


@pytest.mark.parametrize("T,topk,E,inter,k", [(4, 8, 64, 1024, 2048), (64, 8, 64, 1024, 2048), (16, 2, 4, 128, 128),
                                              (9, 8, 16, 96, 1024)])
def test_grouped_swiglu(cuda, K, T, topk, E, inter, k):
    rs = rng(T + topk + inter + 1)
    x = randn_bf(rs, T, k)
    packed = tern_packed(rs, E, 2 * inter, k)
    alpha = bf(alpha_bf(rs, E, 2 * inter) * 40)  # larger scales exercise the clamp
    ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    h = K.ternary_expert_swiglu(to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda),
                                to_dev(alpha, cuda, torch.bfloat16), to_dev(ids, cuda))
    np.testing.assert_array_equal(to_np(h), oracle.expert_swiglu(x, packed, alpha, ids))


@pytest.mark.parametrize("per_slot", [False, True])
@pytest.mark.parametrize("T", [4, 33])
def test_grouped_expert_gemv(cuda, K, per_slot, T):
    rs = rng(50 + per_slot + T)
    topk, E, N, k = 4, 8, 320, 1024
    x = randn_bf(rs, T, topk, k) if per_slot else randn_bf(rs, T, k)
    packed = tern_packed(rs, E, N, k)
    alpha = alpha_bf(rs, E, N)
    ids = rs.randint(0, E, size=(T, topk)).astype(np.int32)  # repeats within a token too
    ids[1, 2] = -1  # out of range: NaN row, like the per-row GEMV
    y = to_np(K.ternary_expert_gemv(to_dev(x, cuda, torch.bfloat16), to_dev(packed, cuda),
                                    to_dev(alpha, cuda, torch.bfloat16), to_dev(ids, cuda))).reshape(-1, N)
    y_o = oracle.expert_gemv(x.reshape(-1, k), packed, alpha, ids, x_rows_per_token=1 if per_slot else topk)
    np.testing.assert_array_equal(y, y_o)
    assert np.isnan(y[1 * topk + 2]).all()


@pytest.mark.parametrize("T,topk,E,N,k", [(4, 8, 64, 2048, 1024), (64, 8, 64, 2048, 1024), (6, 2, 4, 128, 128)])
def test_grouped_down_reduce(cuda, K, T, topk, E, N, k):
    rs = rng(T * topk + N + 3)
    h = randn_bf(rs, T, topk, k)
    packed = tern_packed(rs, E, N, k)
    alpha = alpha_bf(rs, E, N)
    ids = np.stack([rs.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    w = rs.random_sample((T, topk)).astype(np.float32)
    res = randn_bf(rs, T, N)
    out = K.ternary_expert_down_reduce(to_dev(h, cuda, torch.bfloat16), to_dev(packed, cuda),
                                       to_dev(alpha, cuda, torch.bfloat16), to_dev(ids, cuda), to_dev(w, cuda),
                                       to_dev(res, cuda, torch.bfloat16))
    np.testing.assert_array_equal(to_np(out), oracle.expert_down_reduce(h, packed, alpha, ids, w, res, mode=0))


def test_moe_block_batched_equals_per_token(cuda, K):
    """Reference tests/test_model.py:194-242: the batched MoE block equals
    running each token alone (per-slot GEMV path), bit for bit."""
    from maple_flash_dgx_spark_b200.linear import PackedTernaryExperts
    from maple_flash_dgx_spark_b200.model import MapleSparseMoeBlock

    rs = rng(9)
    T, E, topk, inter, H = 12, 16, 4, 128, 256
    x = to_dev(randn_bf(rs, T, H), cuda, torch.bfloat16)
    res = to_dev(randn_bf(rs, T, H), cuda, torch.bfloat16)
    gate = to_dev(randn_bf(rs, E, H, scale=0.02), cuda, torch.bfloat16)
    up = PackedTernaryExperts(to_dev(tern_packed(rs, E, 2 * inter, H), cuda),
                              to_dev(alpha_bf(rs, E, 2 * inter), cuda, torch.bfloat16))
    down = PackedTernaryExperts(to_dev(tern_packed(rs, E, H, inter), cuda),
                                to_dev(alpha_bf(rs, E, H), cuda, torch.bfloat16))
    block = MapleSparseMoeBlock(gate, up, down, topk, inter)
    y = block(x, residual=res)
    for t in range(T):
        torch.testing.assert_close(y[t:t + 1], block(x[t:t + 1], residual=res[t:t + 1]), rtol=0, atol=0)
