"""Whole-model decode on the GPU vs the CPU oracle (GPU).

Greedy token ids and logits must equal the oracle's, which feeds prompts one
token at a time through the reference's decode path; the engine prefills the
prompt in one forward, so this also checks prefill == token-by-token.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.model import OracleModel, synth_tokens

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def tiny_config(layers=2):
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    return synthetic_config(num_layers=layers, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2,
                            inter=128, vocab=1000)


def build(cfg, seed, dev):
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_weights

    return MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, seed, dev), device=dev)


@pytest.mark.parametrize("cfg_name,seed,plen,n_new", [("tiny2", 3, 12, 24), ("tiny4", 5, 40, 16),
                                                       ("mid", 7, 33, 12)])
def test_greedy_ids_and_logits_equal_oracle(cuda, cfg_name, seed, plen, n_new):
    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    cfg = {"tiny2": tiny_config(2), "tiny4": tiny_config(4),
           "mid": synthetic_config(num_layers=2, vocab=151936)}[cfg_name]
    model = build(cfg, seed, cuda)
    prompt = synth_tokens(seed, plen, cfg["vocab_size"])
    res = run_generate(model, torch.from_numpy(prompt), max_tokens=n_new, temperature=0.0, log=None)
    cache = model.make_cache(max_len=plen + n_new)
    orc = OracleModel(cfg, seed, max_len=plen + n_new, split_len=cache.split_len)
    want = orc.greedy(prompt, n_new)
    assert res.token_ids == want
    assert res.used_graph
    # logits of the prompt's last position, bit for bit
    orc2 = OracleModel(cfg, seed, max_len=plen + 1, split_len=model.make_cache(max_len=plen + 1).split_len)
    for tok in prompt[:-1]:
        orc2.step(int(tok))
    _, logits_o = orc2.step(int(prompt[-1]), want_logits=True)
    logits = model.forward(torch.from_numpy(prompt).to(cuda).reshape(1, -1), cache=model.make_cache(max_len=plen + 1))
    np.testing.assert_array_equal(logits[0, -1].float().cpu().numpy(), logits_o)


def test_prefill_rows_equal_token_by_token(cuda):
    cfg = tiny_config(2)
    model = build(cfg, 11, cuda)
    prompt = torch.from_numpy(synth_tokens(11, 20, cfg["vocab_size"])).to(cuda)
    c1 = model.make_cache(max_len=32)
    l1 = model.forward(prompt.reshape(1, -1), cache=c1)
    c2 = model.make_cache(max_len=32)
    for t in prompt:
        l2 = model.forward(t.reshape(1, 1), cache=c2)
    torch.testing.assert_close(l1[0, -1], l2[0, -1], rtol=0, atol=0)
    for a, b in zip(c1.k + c1.v, c2.k + c2.v):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    assert c1.seen == c2.seen == [20]


def test_graph_replay_equals_eager(cuda):
    """Reference generate.py:284-373: graph decode == eager decode."""
    from maple_flash_dgx_spark_b200.generate import run_generate

    cfg = tiny_config(2)
    model = build(cfg, 13, cuda)
    prompt = torch.from_numpy(synth_tokens(13, 9, cfg["vocab_size"]))
    a = run_generate(model, prompt, max_tokens=20, temperature=0.0, use_graph=True, log=None)
    b = run_generate(model, prompt, max_tokens=20, temperature=0.0, use_graph=False, log=None)
    assert a.token_ids == b.token_ids
    s1 = run_generate(model, prompt, max_tokens=20, temperature=1.0, top_p=0.95, top_k=20, seed=4, log=None)
    s2 = run_generate(model, prompt, max_tokens=20, temperature=1.0, top_p=0.95, top_k=20, seed=4, use_graph=False,
                      log=None)
    assert s1.token_ids == s2.token_ids


def test_model_generate_api(cuda):
    cfg = tiny_config(2)
    model = build(cfg, 17, cuda)
    out = model.generate(torch.from_numpy(synth_tokens(17, 5, cfg["vocab_size"])), max_tokens=6)
    assert out.shape == (1, 11)


def test_cfg2_first_64_greedy_ids_equal_oracle(cuda):
    """configs[2] (48 layers, V=151936, 512-token prompt): the first 64 greedy
    ids equal the CPU oracle's (tests/golden/cfg2_greedy.json, made by
    tests/golden/make_cfg2_greedy.py)."""
    import json
    from pathlib import Path

    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    gold = json.loads((Path(__file__).parent / "golden" / "cfg2_greedy.json").read_text())
    cfg = synthetic_config()
    model = build(cfg, gold["seed"], cuda)
    assert model.make_cache(max_len=gold["max_len"]).split_len == gold["split_len"]
    prompt = synth_tokens(gold["seed"], gold["prompt_len"], cfg["vocab_size"])
    res = run_generate(model, torch.from_numpy(prompt), max_tokens=gold["n_new"], temperature=0.0, log=None)
    assert res.token_ids == gold["ids"]
    # every step's bf16 logits, bit for bit (SHA-1 of the bit patterns): the
    # whole step, routing of all 48 layers included, equals the oracle's
    import hashlib

    cache = model.make_cache(max_len=gold["max_len"])
    logits = model.forward(torch.from_numpy(prompt).to(cuda).reshape(1, -1), cache=cache)[0, -1]
    for i in range(gold["n_new"]):
        bits = logits.contiguous().view(torch.int16).cpu().numpy().astype("<i2")
        assert hashlib.sha1(bits.tobytes()).hexdigest() == gold["logits_sha1"][i], i
        tok = int(logits.argmax())
        assert tok == gold["ids"][i]
        logits = model.forward(torch.tensor([[tok]], device=cuda), cache=cache)[0, -1]


def test_batched_decode_equals_single_sequences(cuda):
    """Ragged prompts prefilled per slot, then decoded as one batch (batched
    GEMM / grouped experts): every row's greedy ids and logits equal that
    sequence decoded alone at batch 1."""
    cfg = tiny_config(2)
    model = build(cfg, 19, cuda)
    lens = [5, 9, 12, 7, 16]
    prompts = [torch.from_numpy(synth_tokens(100 + i, n, cfg["vocab_size"])).to(cuda) for i, n in enumerate(lens)]
    B, n_new, max_len = len(lens), 10, 40
    cache = model.make_cache(max_len=max_len, batch=B)
    nxt = []
    for b, p in enumerate(prompts):
        with cache.prefill_slot(b):
            nxt.append(int(model.forward(p.reshape(1, -1), cache=cache)[0, -1].argmax()))
    ids = [[t] for t in nxt]
    cur = torch.tensor(nxt, device=cuda).reshape(B, 1)
    for _ in range(n_new):
        logits = model.forward(cur, cache=cache)
        cur = logits[:, -1].argmax(-1).reshape(B, 1)
        for b in range(B):
            ids[b].append(int(cur[b]))
    for b, p in enumerate(prompts):
        c1 = model.make_cache(max_len=max_len, batch=1)
        assert c1.split_len == cache.split_len
        t = int(model.forward(p.reshape(1, -1), cache=c1)[0, -1].argmax())
        seq = [t]
        for _ in range(n_new):
            lg = model.forward(torch.tensor([[t]], device=cuda), cache=c1)
            t = int(lg[0, -1].argmax())
            seq.append(t)
        assert seq == ids[b]
        torch.testing.assert_close(lg[0, -1], logits[b, -1], rtol=0, atol=0)


@pytest.mark.parametrize("graphs", [False, True])
def test_batched_generate_equals_run_generate(cuda, graphs):
    """Reference generate.py:842-1028: batched greedy decode (per-row caps,
    retirement with slot compaction, bucketed graph widths) gives every row
    the ids of decoding that prompt alone."""
    from maple_flash_dgx_spark_b200.generate import batched_generate, run_generate

    cfg = tiny_config(2)
    model = build(cfg, 23, cuda)
    lens = [6, 11, 4, 9, 13, 7]
    caps = [12, 3, 9, 12, 5, 1]
    prompts = [synth_tokens(200 + i, n, cfg["vocab_size"]) for i, n in enumerate(lens)]
    res = batched_generate(model, prompts, max_new=caps, graphs=graphs, stop_ids=set(), log=None)
    assert [len(t) for t in res.token_ids] == caps
    for p, cap, got in zip(prompts, caps, res.token_ids):
        want = run_generate(model, torch.from_numpy(p), max_tokens=cap, temperature=0.0, log=None).token_ids
        assert got == want
    if graphs:
        assert res.widths and res.widths[0] == 6 and res.widths[-1] <= 2  # live rows shrink to narrower graphs


def test_batched_generate_sampled_graph_equals_eager(cuda):
    from maple_flash_dgx_spark_b200.generate import batched_generate

    cfg = tiny_config(2)
    model = build(cfg, 29, cuda)
    prompts = [synth_tokens(300 + i, 5 + i, cfg["vocab_size"]) for i in range(5)]
    kw = dict(max_tokens=10, temperature=0.9, top_p=0.9, top_k=16, seed=7, stop_ids=set(), log=None)
    a = batched_generate(model, prompts, graphs=True, **kw)
    b = batched_generate(model, prompts, graphs=False, **kw)
    assert a.token_ids == b.token_ids
