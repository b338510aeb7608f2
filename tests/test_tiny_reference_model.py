"""The oracle's whole decode step against the reference's own model (no GPU).

``tests/golden/tiny_packed/`` is a checkpoint written by the reference's
converter (convert.py:380-450) from a seeded Hugging Face-style source, and
``tests/golden/tiny_greedy.npz`` holds the greedy ids and per-step logits the
reference's ``MapleForCausalLM`` decoded from it (model.py:848-913), with the
bf16 stores of its GPU kernels applied (``tests/golden/make_tiny_model.py``).
The model exercises what the synthetic benchmark model does not: an RTN-4
embedding, a g64 affine RTN-4 head, fp32 row scales, a sliding-window layer,
a NoPE global layer and partial RoPE.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.model import OracleModel

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_tiny():
    from safetensors.numpy import load_file

    config = json.loads((GOLDEN / "tiny_packed" / "config.json").read_text())
    weights = {}
    for f in sorted((GOLDEN / "tiny_packed").glob("*.safetensors")):
        weights.update(load_file(str(f)))
    return config, weights


@pytest.fixture(scope="module")
def tiny_golden():
    return np.load(GOLDEN / "tiny_greedy.npz")


def test_converted_checkpoint_layout():
    config, w = load_tiny()
    meta = config["maple_run"]
    assert meta["format"] == "packed-ternary-v1" and meta["rtn_4bit"]["group_size"] == 64
    assert w["model.layers.0.mlp.switch_mlp.up_proj.weight"].shape == (8, 128, 256 // 16)
    assert w["model.layers.0.self_attn.q_proj.row_alpha"].dtype == np.float32
    assert w["lm_head.weight"].shape == (512, 256 // 8)
    assert "lm_head.biases" in w and "model.word_embeddings.scales" in w


def test_oracle_greedy_equals_reference(tiny_golden):
    config, weights = load_tiny()
    prompt, want = tiny_golden["prompt"], tiny_golden["ids"]
    ref_logits = tiny_golden["logits"]
    total = len(prompt) + len(want)
    m = OracleModel.from_weights(config, weights, max_len=total, split_len=64)
    got_ids, nxt = [], None
    for i in range(total - 1):
        tok = int(prompt[i]) if i < len(prompt) else nxt
        nxt, logits = m.step(tok, want_logits=True)
        # within 1e-2 of the step's logit scale (measured: 7.5e-3 worst, a
        # third of the logits bit-identical); the remaining difference is
        # the reference's fp32 P in attention (the oracle rounds P to bf16
        # as the reference's bf16 cache path does) and summation order
        err = np.abs(logits - ref_logits[i]).max()
        assert err <= 1e-2 * np.abs(ref_logits[i]).max(), (i, err)
        if i >= len(prompt) - 1:
            got_ids.append(nxt)
    assert got_ids == want.tolist()
    # the reference's generate() (prompt prefilled by its SDPA path) agrees
    assert tiny_golden["generate_ids"].tolist() == want.tolist()


@pytest.mark.gpu
def test_engine_on_reference_checkpoint(cuda, tiny_golden):
    """``MapleForCausalLM.from_packed`` loads the reference-converted directory
    (RTN-4 embedding and g64 affine head, fp32 row scales, sliding-window and
    NoPE layers, partial RoPE); its greedy ids equal the reference's, and every
    step's logits equal the oracle's bit for bit."""
    import torch

    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM

    model = MapleForCausalLM.from_packed(str(GOLDEN / "tiny_packed"), device=cuda)
    prompt, want = tiny_golden["prompt"], tiny_golden["ids"]
    total = len(prompt) + len(want)
    res = run_generate(model, torch.from_numpy(prompt), max_tokens=len(want), temperature=0.0, log=None)
    assert res.token_ids == want.tolist()

    config, weights = load_tiny()
    cache = model.make_cache(max_len=total)
    orc = OracleModel.from_weights(config, weights, max_len=total, split_len=cache.split_len)
    nxt = None
    for i in range(total - 1):
        tok = int(prompt[i]) if i < len(prompt) else nxt
        logits = model.forward(torch.tensor([[tok]], device=cuda), cache=cache)[0, -1].float().cpu().numpy()
        nxt, want_logits = orc.step(tok, want_logits=True)
        np.testing.assert_array_equal(logits, want_logits)
