"""Packed-ternary-v1 checkpoint writer: shards, index and config round trip
(CPU); the model loaded from the written directory decodes like the
in-memory one (GPU)."""

from __future__ import annotations

import json

import pytest
import torch


def _host_weights(cfg, seed=0):
    """Host tensors with the packed-ternary-v1 names and shapes of ``cfg``."""
    g = torch.Generator().manual_seed(seed)
    H, V, E, I = cfg["hidden_size"], cfg["vocab_size"], cfg["num_experts"], cfg["moe_intermediate_size"]
    Hq, Hkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    grp = cfg["maple_run"]["rtn_4bit"]["group_size"]

    def u32(*shape):
        return torch.randint(0, 2**31 - 1, shape, generator=g, dtype=torch.int64).to(torch.int32).view(torch.uint32)

    def f(*shape, dt=torch.bfloat16):
        return torch.randn(*shape, generator=g).to(dt)

    w = {"model.word_embeddings.weight": f(V, H), "lm_head.weight": u32(V, H // 8), "lm_head.scales": f(V, H // grp),
         "model.norm.weight": f(H, dt=torch.float32)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        for n in ("input_layernorm", "post_attention_layernorm"):
            w[f"{p}.{n}.weight"] = f(H, dt=torch.float32)
        for n in ("q_norm", "k_norm"):
            w[f"{p}.self_attn.{n}.weight"] = f(D, dt=torch.float32)
        for n, rows, k in (("q_proj", Hq * D, H), ("k_proj", Hkv * D, H), ("v_proj", Hkv * D, H), ("o_proj", H, Hq * D)):
            w[f"{p}.self_attn.{n}.weight"] = u32(rows, k // 16)
            w[f"{p}.self_attn.{n}.row_alpha"] = f(rows)
        w[f"{p}.mlp.gate.weight"] = f(E, H)
        for n, rows, k in (("up_proj", I, H), ("gate_proj", I, H), ("down_proj", H, I)):
            w[f"{p}.mlp.switch_mlp.{n}.weight"] = u32(E, rows, k // 16)
            w[f"{p}.mlp.switch_mlp.{n}.row_alpha"] = f(E, rows)
    return w


def _tiny():
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    return synthetic_config(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, topk=2, inter=128,
                            vocab=1000)


def test_save_load_round_trip(tmp_path):
    from maple_flash_dgx_spark_b200.checkpoint import load_packed_weights, save_packed

    cfg = _tiny()
    w = _host_weights(cfg)
    w["lm_head_flash.token_map"] = torch.arange(1000, dtype=torch.int32).reshape(125, 8)
    index = save_packed(tmp_path, cfg, w, max_shard_bytes=300_000)
    shards = sorted(set(index["weight_map"].values()))
    assert len(shards) > 2 and "model-flashhead.safetensors" in shards
    assert json.loads((tmp_path / "config.json").read_text()) == cfg
    cfg2, w2 = load_packed_weights(tmp_path)
    assert cfg2 == cfg and "lm_head_flash.token_map" not in w2
    _, w3 = load_packed_weights(tmp_path, flash_head=True)
    assert set(w3) == set(w)
    for k, v in w.items():
        assert w3[k].dtype == v.dtype and torch.equal(w3[k].view(torch.uint8), v.view(torch.uint8)), k


def test_save_rejects_unpacked_config(tmp_path):
    from maple_flash_dgx_spark_b200.checkpoint import save_packed

    with pytest.raises(ValueError):
        save_packed(tmp_path, {"maple_run": {"format": "hf"}}, {})


@pytest.mark.gpu
def test_model_from_written_checkpoint_decodes_identically(cuda, tmp_path):
    from maple_flash_dgx_spark_b200.checkpoint import save_packed
    from maple_flash_dgx_spark_b200.generate import run_generate
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_tokens, synthetic_weights

    cfg = _tiny()
    w = synthetic_weights(cfg, 31, cuda)
    save_packed(tmp_path, cfg, w)
    a = MapleForCausalLM.from_weight_dict(cfg, w, device=cuda)
    b = MapleForCausalLM.from_packed(str(tmp_path), device=cuda)
    prompt = synthetic_tokens(31, 7, cfg["vocab_size"], cuda).cpu()
    ra = run_generate(a, prompt, max_tokens=8, temperature=0.0, log=None)
    rb = run_generate(b, prompt, max_tokens=8, temperature=0.0, log=None)
    assert ra.token_ids == rb.token_ids
