"""tcgen05 grouped expert GEMM (``maple_ternary_grouped_gemm_tc``) on the GPU.

The tensor-memory kernel contracts the same exact integers (2-bit codes
against the FXA digits of the activations) as the mma.sync grouped GEMM, so
its outputs must equal that path's bit for bit -- SwiGLU (up|gate) and plain
(down) modes, experts with no, few and several chunks of 64 routed slots, an
out-of-range expert id (NaN row in both paths), a rank's local expert range,
a whole prefill through the model, and dense batched GEMMs (with the fused
input RMSNorm) run as one expert.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import alpha_bf, randn_bf, rng, tern_packed, to_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture
def K(monkeypatch):
    from maple_flash_dgx_spark_b200 import kernels

    return kernels


def _routing(rs, tokens, topk, E, skew):
    """Distinct experts per token; with ``skew`` most tokens pick the low
    experts, so some experts get several 64-slot chunks and some none."""
    ids = np.empty((tokens, topk), np.int32)
    for t in range(tokens):
        if skew:
            p = np.exp(-0.6 * np.arange(E))
            ids[t] = rs.choice(E, size=topk, replace=False, p=p / p.sum())
        else:
            ids[t] = rs.permutation(E)[:topk]
    return ids


def _both(K, monkeypatch, fn):
    monkeypatch.setattr(K, "TC_GEMM_MIN_SLOTS", 10 ** 9)  # mma.sync grouped path
    want = fn()
    monkeypatch.setattr(K, "TC_GEMM_MIN_SLOTS", 0)  # tcgen05 path
    got = fn()
    torch.cuda.synchronize()
    return got, want


@pytest.mark.parametrize("tokens,topk,E,inter,H,skew", [
    (100, 4, 8, 256, 2048, True),
    (64, 8, 64, 1024, 2048, False),
    (64, 8, 64, 512, 1024, True),   # decode-sized, skewed: some experts need several 16-slot chunks
    (300, 2, 4, 128, 256, True),
])
def test_tc_swiglu_equals_mma_sync(cuda, K, monkeypatch, tokens, topk, E, inter, H, skew):
    rs = rng(tokens + E)
    x = to_dev(randn_bf(rs, tokens, H), cuda, torch.bfloat16)
    ug = to_dev(tern_packed(rs, E, 2 * inter, H), cuda)
    ug_a = to_dev(alpha_bf(rs, E, 2 * inter), cuda, torch.bfloat16)
    ids = _routing(rs, tokens, topk, E, skew)
    ids[3, 0] = E + 5  # out-of-range: NaN row in both paths
    ids_d = to_dev(ids, cuda)

    def run():
        plan = K.moe_plan(ids_d, E)
        return K.ternary_expert_swiglu(x, ug, ug_a, ids_d, plan=plan)

    got, want = _both(K, monkeypatch, run)
    assert torch.isnan(want[3, 0]).all()
    torch.testing.assert_close(got, want, rtol=0, atol=0, equal_nan=True)
    assert K.lib() is not None and _errors(cuda) == 0


@pytest.mark.parametrize("tokens,topk,E,inter,H", [(96, 4, 8, 1024, 2048), (40, 8, 16, 256, 512),
                                                   (64, 8, 64, 1024, 2048)])
def test_tc_down_equals_mma_sync(cuda, K, monkeypatch, tokens, topk, E, inter, H):
    rs = rng(7 * tokens + E)
    h = to_dev(randn_bf(rs, tokens, topk, inter, scale=0.5), cuda, torch.bfloat16)
    down = to_dev(tern_packed(rs, E, H, inter), cuda)
    down_a = to_dev(alpha_bf(rs, E, H), cuda, torch.bfloat16)
    ids_d = to_dev(_routing(rs, tokens, topk, E, True), cuda)

    def run():
        plan = K.moe_plan(ids_d, E)
        return K.ternary_expert_gemv(h, down, down_a, ids_d, plan=plan)

    got, want = _both(K, monkeypatch, run)
    torch.testing.assert_close(got, want, rtol=0, atol=0)
    assert _errors(cuda) == 0


def test_tc_local_expert_range(cuda, K, monkeypatch):
    """One rank's experts (moe_plan e_first / n_local): only listed slots are
    encoded and written."""
    rs = rng(11)
    tokens, topk, E, inter, H = 128, 4, 16, 256, 1024
    x = to_dev(randn_bf(rs, tokens, H), cuda, torch.bfloat16)
    ug = to_dev(tern_packed(rs, 4, 2 * inter, H), cuda)  # experts 8..11 held here
    ug_a = to_dev(alpha_bf(rs, 4, 2 * inter), cuda, torch.bfloat16)
    ids_d = to_dev(_routing(rs, tokens, topk, E, False), cuda)

    def run():
        plan = K.moe_plan(ids_d, E, e_first=8, n_local=4)
        y = torch.full((tokens * topk, inter), 7.0, dtype=torch.bfloat16, device=cuda)
        return K._grouped("swiglu", x, topk, ug, ug_a, plan, True, tokens * topk, inter, x.dtype, out=y)

    got, want = _both(K, monkeypatch, run)
    torch.testing.assert_close(got, want, rtol=0, atol=0)
    assert _errors(cuda) == 0


def test_prefill_through_tc_gemm_equals_mma_sync(cuda, monkeypatch):
    """A 96-token prompt (24 routed slots per expert on average) prefilled
    with the tcgen05 expert GEMMs gives the same logits and cache."""
    from maple_flash_dgx_spark_b200 import kernels as K
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_weights
    from oracle.model import synth_tokens

    cfg = synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2,
                           inter=128, vocab=1000)
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, 13, cuda), device=cuda)
    prompt = torch.from_numpy(synth_tokens(13, 96, cfg["vocab_size"])).to(cuda).reshape(1, -1)
    outs = []
    for tc in (False, True):
        monkeypatch.setattr(K, "TC_GEMM_MIN_SLOTS", 0 if tc else 10 ** 9)
        cache = model.make_cache(max_len=100)
        outs.append((model.forward(prompt, cache=cache, logits_to_keep=4), cache))
    torch.testing.assert_close(outs[1][0], outs[0][0], rtol=0, atol=0)
    for a, b in zip(outs[1][1].k + outs[1][1].v, outs[0][1].k + outs[0][1].v):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    assert _errors(cuda) == 0


@pytest.mark.parametrize("rows,k,n,rms", [(64, 2048, 5120, True), (512, 4096, 4096, False), (300, 2048, 5120, True),
                                           (80, 1024, 4096, True)])
def test_tc_dense_equals_mma_sync(cuda, K, monkeypatch, rows, k, n, rms):
    """Dense batched GEMMs (QKV with its fused input RMSNorm, O) on the
    tcgen05 kernel as one expert equal the mma.sync GEMM bit for bit."""
    rs = rng(rows + n)
    x = to_dev(randn_bf(rs, rows, k), cuda, torch.bfloat16)
    w = to_dev(tern_packed(rs, n, k), cuda)
    a = to_dev(alpha_bf(rs, n), cuda, torch.bfloat16)
    rw = to_dev((1 + 0.05 * rs.standard_normal(k)).astype(np.float32), cuda) if rms else None
    assert K.use_tc_dense(rows, k, n)
    monkeypatch.setenv("MAPLE_TC_DENSE", "0")
    want = K.ternary_gemv(x, w, a, rms_weight=rw)
    monkeypatch.setenv("MAPLE_TC_DENSE", "1")
    got = K.ternary_gemv(x, w, a, rms_weight=rw)
    torch.cuda.synchronize()
    torch.testing.assert_close(got, want, rtol=0, atol=0)
    assert _errors(cuda) == 0


def _errors(dev):
    from maple_flash_dgx_spark_b200 import _lib

    return _lib.take_device_errors(dev)
