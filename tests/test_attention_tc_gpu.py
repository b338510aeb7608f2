"""Tensor-core decode attention (``maple_decode_gqa_attn_tc``) on the GPU.

The reference's decode attention (kernels/decode_attn.py:166-313) takes
bf16 q.K^T and P.V dots with fp32 accumulation and P rounded to bf16; this
kernel runs the same arithmetic on the tensor pipe, so it is checked to a
tolerance (1e-2 of the output's scale, north_star's attention bound; the
measured error is far smaller) against both the CPU oracle (fp32 sums, P
rounded to bf16) and torch fp32 attention -- at the reference test's ragged
lengths (tests/test_fused_decode.py:245-291), sliding windows, a row map,
head_dim 64 and 128, group sizes 1-8 and contexts up to 16384.  Split
boundaries depend on the cache length only, so a row's result does not depend
on the batch it decodes in.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.helpers import randn_bf, rng, to_dev, to_np

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from maple_flash_dgx_spark_b200 import kernels

    return kernels


def _scale_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)


CASES = [
    # B, Hq, Hkv, D, T, lens, window, row_map
    (7, 32, 4, 128, 1025, [1, 63, 64, 65, 300, 511, 1000], 0, None),
    (3, 32, 4, 128, 8192, [8192, 4097, 17], 0, None),
    (3, 16, 2, 128, 16384, [16384, 9000, 1], 0, None),
    (2, 8, 8, 128, 2048, [2048, 777], 96, None),
    (2, 4, 1, 64, 3000, [3000, 1500], 0, None),
    (3, 32, 4, 128, 4096, [4096, 100, 2500], 0, [2, 0, 1]),
    (2, 16, 4, 64, 2000, [2000, 1999], 700, None),
]


@pytest.mark.parametrize("B,Hq,Hkv,D,T,lens,window,rmap", CASES)
def test_tc_attention_matches_oracle_and_fp32(cuda, K, B, Hq, Hkv, D, T, lens, window, rmap):
    rs = rng(B * 97 + T + D)
    Bc = B if rmap is None else max(rmap) + 1
    q = randn_bf(rs, B, Hq, D)
    kc = randn_bf(rs, Bc, Hkv, T, D)
    vc = randn_bf(rs, Bc, Hkv, T, D)
    pos = np.asarray(lens, np.int64) - 1
    rm = None if rmap is None else np.asarray(rmap, np.int32)
    q_d = to_dev(q, cuda, torch.bfloat16).reshape(B, Hq, 1, D)
    kc_d, vc_d = to_dev(kc, cuda, torch.bfloat16), to_dev(vc, cuda, torch.bfloat16)
    sl = to_dev(pos, cuda)
    rm_d = None if rm is None else to_dev(rm, cuda)
    out = K.decode_gqa_attn(q_d, kc_d, vc_d, sl, row_map=rm_d, scale=D ** -0.5, window=window or None,
                            tensor_cores=True)
    got = to_np(out)[:, :, 0]
    want = oracle.decode_gqa(q, kc, vc, pos, rm, scale=np.float32(D ** -0.5), window=window, split_len=128)
    assert np.isfinite(got).all()
    err_o = _scale_err(got, want)
    # torch fp32 attention over each row's live range
    G = Hq // Hkv
    ref = np.empty_like(want)
    for b in range(B):
        cb = b if rm is None else rm[b]
        n = lens[b]
        lo = max(0, n - window) if window else 0
        k = torch.from_numpy(kc[cb, :, lo:n]).repeat_interleave(G, 0)
        v = torch.from_numpy(vc[cb, :, lo:n]).repeat_interleave(G, 0)
        s = torch.einsum("hd,htd->ht", torch.from_numpy(q[b]), k) * D ** -0.5
        ref[b] = torch.einsum("ht,htd->hd", torch.softmax(s, -1), v).numpy()
    err_r = _scale_err(got, ref)
    print(f"tc attention: scale-relative error vs oracle {err_o:.2e}, vs fp32 {err_r:.2e}")
    assert err_o <= 1e-2 and err_r <= 1e-2
    assert _lib_errors(cuda) == 0


def _lib_errors(dev):
    from maple_flash_dgx_spark_b200 import _lib

    return _lib.take_device_errors(dev)


def test_tc_attention_row_independent_of_batch(cuda, K):
    """A row decoded alone equals the same row inside a batch, bit for bit."""
    rs = rng(5)
    B, Hq, Hkv, D, T = 5, 32, 4, 128, 9000
    q = to_dev(randn_bf(rs, B, Hq, D), cuda, torch.bfloat16).reshape(B, Hq, 1, D)
    kc = to_dev(randn_bf(rs, B, Hkv, T, D), cuda, torch.bfloat16)
    vc = to_dev(randn_bf(rs, B, Hkv, T, D), cuda, torch.bfloat16)
    sl = torch.tensor([8999, 4000, 123, 8191, 6000], device=cuda)
    full = K.decode_gqa_attn(q, kc, vc, sl, scale=D ** -0.5, window=None, tensor_cores=True)
    for b in range(B):
        one = K.decode_gqa_attn(q[b:b + 1], kc[b:b + 1], vc[b:b + 1], sl[b:b + 1], scale=D ** -0.5, window=None,
                                tensor_cores=True)
        torch.testing.assert_close(one, full[b:b + 1], rtol=0, atol=0)


def test_tc_attention_in_long_context_model_step(cuda):
    """A model cache past one cluster's worth of splits decodes through the
    tensor-core kernel, and batched rows equal single-row decode."""
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import fill_kv_cache, synthetic_config, synthetic_weights

    cfg = synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2,
                           inter=128, vocab=1000)
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, 41, cuda), device=cuda)
    ctx, B = 3000, 3
    cache = model.make_cache(max_len=ctx + 8, batch=B)
    assert cache.attn_tc
    fill_kv_cache(cache, 41, ctx)
    toks = torch.tensor([[5], [17], [900]], device=cuda)
    logits = model.forward(toks, cache=cache)
    for b in range(B):
        c1 = model.make_cache(max_len=ctx + 8, batch=1)
        fill_kv_cache(c1, 41, ctx, row0=b, total_rows=B)
        one = model.forward(toks[b:b + 1], cache=c1)
        torch.testing.assert_close(one[0], logits[b], rtol=0, atol=0)
