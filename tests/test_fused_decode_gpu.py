"""Whole-stack batch-1 decode in one launch == the operator-by-operator path (GPU).

``maple_decode_layers`` runs every decoder layer of a decode step in one
persistent launch.  It must give the same logits and the same K/V cache
contents, bit for bit, as the per-operator kernels (which the other GPU tests
pin to the CPU oracle), for one and several attention splits, full-size
layer shapes, and a cache row reached through the row map.
"""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPES = {
    # name: (config kwargs, prompt length, decode steps)
    "tiny_one_split": (dict(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2,
                            inter=128, vocab=1000), 20, 6),
    "tiny_many_splits": (dict(num_layers=3, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2,
                              inter=128, vocab=1000), 250, 5),
    "g4_d128": (dict(num_layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, experts=16, topk=4, inter=256,
                     vocab=2000), 130, 5),
    "full_layers": (dict(num_layers=2, vocab=4096), 300, 4),
}


def _model(kw, seed, dev):
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_weights

    cfg = synthetic_config(**kw)
    return cfg, MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, seed, dev), device=dev)


def _decode(model, prompt, steps, fused, monkeypatch, *, batch=1, slot=None):
    from maple_flash_dgx_spark_b200.kernels import argmax

    monkeypatch.setenv("MAPLE_FUSED_DECODE", "1" if fused else "0")
    cache = model.make_cache(max_len=prompt.numel() + steps + 3, batch=batch)
    if slot is not None:
        cache.remap = True
        with cache.prefill_slot(slot):
            logits = model.forward(prompt.reshape(1, -1), cache=cache)
    else:
        logits = model.forward(prompt.reshape(1, -1), cache=cache)
    outs = []
    tok = argmax(logits[:, -1, :]).reshape(1, 1)
    for _ in range(steps):
        if slot is not None:
            with cache.prefill_slot(slot):
                logits = model.forward(tok, cache=cache)
        else:
            logits = model.forward(tok, cache=cache)
        outs.append(logits[0, -1].clone())
        tok = argmax(logits[:, -1, :]).reshape(1, 1)
    torch.cuda.synchronize()
    return outs, cache


@pytest.mark.parametrize("name", list(SHAPES))
def test_fused_decode_equals_operator_path(cuda, monkeypatch, name):
    from maple_flash_dgx_spark_b200.fused_decode import fused_decode_supported
    from maple_flash_dgx_spark_b200.synth import synthetic_tokens

    kw, plen, steps = SHAPES[name]
    cfg, model = _model(kw, 21, cuda)
    prompt = synthetic_tokens(21, plen, cfg["vocab_size"], cuda)
    ref, c_ref = _decode(model, prompt, steps, False, monkeypatch)
    got, c_got = _decode(model, prompt, steps, True, monkeypatch)
    assert fused_decode_supported(model, c_got)
    assert getattr(c_got, "_fused_plan", None) is not None, "the fused launch did not run"
    assert int(c_got._fused_plan.err.item()) == 0
    for a, b in zip(ref, got):
        torch.testing.assert_close(b, a, rtol=0, atol=0)
    for a, b in zip(c_ref.k + c_ref.v, c_got.k + c_got.v):
        torch.testing.assert_close(b, a, rtol=0, atol=0)
    assert c_ref.seen == c_got.seen


def test_fused_decode_through_row_map(cuda, monkeypatch):
    """A decode slot whose K/V live in another cache row (reference KVCache
    row_map, model.py:116-310) reads and writes that row."""
    from maple_flash_dgx_spark_b200.synth import synthetic_tokens

    kw, plen, steps = SHAPES["tiny_many_splits"]
    cfg, model = _model(kw, 23, cuda)
    prompt = synthetic_tokens(23, 90, cfg["vocab_size"], cuda)
    ref, c_ref = _decode(model, prompt, 4, False, monkeypatch, batch=3, slot=1)
    got, c_got = _decode(model, prompt, 4, True, monkeypatch, batch=3, slot=1)
    assert getattr(c_got, "_fused_plan", None) is not None
    for a, b in zip(ref, got):
        torch.testing.assert_close(b, a, rtol=0, atol=0)
    for a, b in zip(c_ref.k + c_ref.v, c_got.k + c_got.v):
        torch.testing.assert_close(b, a, rtol=0, atol=0)


def test_fused_decode_graph_replay(cuda, monkeypatch):
    """The launch is captured in the decode CUDA graph (generate.py's replay ==
    eager gate passes) and gives the operator path's greedy ids."""
    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.synth import synthetic_tokens

    kw, _, _ = SHAPES["g4_d128"]
    cfg, model = _model(kw, 25, cuda)
    prompt = synthetic_tokens(25, 70, cfg["vocab_size"], cuda).cpu()
    monkeypatch.setenv("MAPLE_FUSED_DECODE", "0")
    a = run_generate(model, prompt, max_tokens=24, temperature=0.0, use_graph=True, log=None)
    monkeypatch.setenv("MAPLE_FUSED_DECODE", "1")
    b = run_generate(model, prompt, max_tokens=24, temperature=0.0, use_graph=True, log=None)
    assert b.used_graph
    assert a.token_ids == b.token_ids
