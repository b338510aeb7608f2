"""Continuous-batching worker (``serve.PackedEngine``) on the GPU.

Mirrors the reference's scheduler tests (tests/test_server.py:566-650):
overlapping jobs give each request the ids it gets alone, decode stops at the
cache's last position, padding rows of a wider graph leave free slots empty;
plus seeded sampled rows that are isolated from their neighbours.
"""

from __future__ import annotations

import threading

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _model(dev, seed=31):
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_weights

    cfg = synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2, inter=128,
                           vocab=1000)
    return MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, seed, dev), device=dev), cfg


def _engine(model, max_batch, max_len):
    from maple_flash_dgx_spark_b200.serve import PackedEngine, ServerDefaults

    eng = PackedEngine(model, None, ServerDefaults(max_batch=max_batch, max_len=max_len, model_id="tiny"), log=None)
    eng.wait_ready()
    return eng


def _prompts(cfg, dev, lens, seed=9):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(1, cfg["vocab_size"], (n,), generator=g).to(dev) for n in lens]


def _concurrently(fns):
    out = [None] * len(fns)
    errs = []

    def go(i):
        try:
            out[i] = fns[i]()
        except BaseException as exc:  # surfaced below
            errs.append(exc)

    threads = [threading.Thread(target=go, args=(i,)) for i in range(len(fns))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
        assert not t.is_alive(), "a request never finished"
    if errs:
        raise errs[0]
    return out


def test_overlapping_jobs_match_solo(cuda):
    """Three jobs, two slots: the waiting job joins a freed slot and nobody's
    ids change (greedy ids == batched_generate of the prompt alone)."""
    from maple_flash_dgx_spark_b200.generate import batched_generate

    model, cfg = _model(cuda)
    prompts = _prompts(cfg, cuda, (4, 9, 6))
    caps = (8, 12, 8)
    solo = [batched_generate(model, [p], max_tokens=m, stop_ids=set(), log=None).token_ids[0]
            for p, m in zip(prompts, caps)]
    eng = _engine(model, 2, 64)
    try:
        got = _concurrently([lambda i=i: eng.run(prompts[i], max_tokens=caps[i], temperature=0.0, top_k=1,
                                                 stop_ids=set()) for i in range(3)])
        for i in range(3):
            assert got[i].token_ids == solo[i], f"job {i} diverged from its solo run"
            assert got[i].finish_reason == "length"
    finally:
        eng.close()


def test_decode_stops_at_max_len(cuda):
    """A huge max_tokens stops at the cache's last position, and the engine
    serves the next request."""
    model, cfg = _model(cuda)
    prompt = _prompts(cfg, cuda, (4,))[0]
    eng = _engine(model, 1, 16)
    try:
        res = eng.run(prompt, max_tokens=64000, temperature=0.0, top_k=1, stop_ids=set())
        assert res.finish_reason == "length"
        assert res.n_new == 12  # max_len 16 - prompt 4
        again = eng.run(prompt, max_tokens=4, temperature=0.0, top_k=1, stop_ids=set())
        assert again.token_ids == res.token_ids[:4]
    finally:
        eng.close()


def test_padding_rows_leave_free_slots_empty(cuda):
    """Four slots (graph widths 1, 2, 4): three live rows replay the width-4
    graph; its padding row must not advance the free slot's length."""
    model, cfg = _model(cuda)
    prompts = _prompts(cfg, cuda, (2, 5, 3))
    eng = _engine(model, 4, 24)
    try:
        _concurrently([lambda i=i: eng.run(prompts[i], max_tokens=10 + i, temperature=0.0, top_k=1, stop_ids=set())
                       for i in range(3)])
        assert eng.live == 0
        for s in range(4):
            assert eng.cache.seen[s] == 0
            assert int(eng.cache.seqlen[s]) == 0
        res = eng.run(prompts[0], max_tokens=12, temperature=0.0, top_k=1, stop_ids=set())
        assert len(res.token_ids) == 12
    finally:
        eng.close()


def test_stop_ids_and_sampled_rows(cuda):
    """A seeded sampled request gives the same ids alone and beside a greedy
    neighbour; a stop id ends a request with reason "stop"."""
    model, cfg = _model(cuda)
    p_s, p_g = _prompts(cfg, cuda, (6, 7), seed=5)
    eng = _engine(model, 2, 48)
    try:
        kw = dict(max_tokens=16, temperature=1.0, top_p=0.95, top_k=20, seed=123, stop_ids=set())
        alone = eng.run(p_s, **kw)
        both = _concurrently([lambda: eng.run(p_s, **kw),
                              lambda: eng.run(p_g, max_tokens=16, temperature=0.0, top_k=1, stop_ids=set())])
        assert both[0].token_ids == alone.token_ids
        greedy = both[1].token_ids
        stop = greedy[5]
        first = greedy.index(stop)
        cut = eng.run(p_g, max_tokens=16, temperature=0.0, top_k=1, stop_ids={stop})
        assert cut.finish_reason == "stop"
        assert cut.token_ids == greedy[:first + 1]
    finally:
        eng.close()
