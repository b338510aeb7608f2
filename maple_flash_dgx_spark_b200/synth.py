"""Synthetic packed models of the benchmark architecture (no checkpoint exists).

Weights are generated on the device by ``maple_synth_*`` (csrc/synth.cu): a
counter-based integer hash per element, so any tensor can be regenerated bit
for bit from (seed, stream id, index) by an independent implementation.  The
weight dict uses the reference's packed-ternary-v1 tensor names
(convert.py:180-248, model.py:750-832) so it loads through
``MapleForCausalLM.from_weight_dict`` like a converted checkpoint.

Distributions follow the benchmark configs: ternary codes with P(0)=0.4,
P(+-1)=0.3; row scales bf16 |N(0, 0.02)| + 1e-3; router bf16 N(0, 0.02);
embedding bf16 N(0, 0.02); RMSNorm weights fp32 1 + N(0, 0.02); lm_head RTN-4
g128 symmetric from N(0, 0.02).  "Normal" here is the Irwin-Hall sum of four
16-bit uniforms (bounded, kurtosis 2.7): a seeded stand-in for N(0, s).
"""

from __future__ import annotations

import torch

from maple_flash_dgx_spark_b200._lib import BF16, F32, check, lib, ptr, stream_ptr

# Stream ids of the synthetic tensors (part of the generator's definition).
S_EMB, S_NORM, S_HEAD, S_PROMPT = 1, 2, 3, 50
LAYER_BASE, LAYER_STRIDE = 1000, 64
L_IN_LN, L_POST_LN, L_Q_NORM, L_K_NORM = 0, 1, 2, 3
L_Q, L_QA, L_K, L_KA, L_V, L_VA, L_O, L_OA = 4, 5, 6, 7, 8, 9, 10, 11
L_ROUTER, L_UP, L_UPA, L_GATE, L_GATEA, L_DOWN, L_DOWNA = 12, 13, 14, 15, 16, 17, 18
L_KCACHE, L_VCACHE = 19, 20


def layer_stream(layer: int, kind: int) -> int:
    return LAYER_BASE + LAYER_STRIDE * layer + kind


def synthetic_config(num_layers: int = 48, hidden: int = 2048, heads: int = 32, kv_heads: int = 4,
                     head_dim: int = 128, experts: int = 64, topk: int = 8, inter: int = 1024,
                     vocab: int = 151936, head_group: int = 128) -> dict:
    """The benchmark architecture (configs[1]/[2]): RoPE theta 1e6 on every
    layer, full attention, QK-norm, MLP clamp 7, symmetric RTN-4 g128 head."""
    return {
        "hidden_size": hidden,
        "num_hidden_layers": num_layers,
        "num_attention_heads": heads,
        "num_key_value_heads": kv_heads,
        "head_dim": head_dim,
        "num_experts": experts,
        "num_experts_per_tok": topk,
        "moe_intermediate_size": inter,
        "vocab_size": vocab,
        "rms_norm_eps": 1e-6,
        "sliding_window": 512,
        "layer_types": ["full_attention"] * num_layers,
        "use_qk_norm": True,
        "nope_on_global_attention": False,
        "partial_rotary_factor": 1.0,
        "rope_theta": 1.0e6,
        "eos_token_id": None,
        "maple_run": {
            "format": "packed-ternary-v1",
            "rtn_4bit": {"group_size": head_group, "bits": 4, "mode": "symmetric"},
            "embedding": "dense",
        },
    }


def _ternary(seed, stream, shape, dev):
    t = torch.empty(shape, dtype=torch.int32, device=dev).view(torch.uint32)
    check(lib().maple_synth_ternary(seed, stream, t.numel(), ptr(t), stream_ptr(dev)), "synth_ternary")
    return t


def _normal(seed, stream, shape, dev, scale, offset=0.0, use_abs=False, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=dtype, device=dev)
    check(lib().maple_synth_normal(seed, stream, t.numel(), float(scale), float(offset), int(use_abs),
                                   BF16 if dtype == torch.bfloat16 else F32, ptr(t), stream_ptr(dev)), "synth_normal")
    return t


def _alpha(seed, stream, shape, dev):
    return _normal(seed, stream, shape, dev, 0.02, 1e-3, True)


def synthetic_weights(config: dict, seed: int, device) -> dict[str, torch.Tensor]:
    """Packed-ternary-v1 weight dict of ``config`` generated on ``device``."""
    dev = torch.device(device)
    H, V = config["hidden_size"], config["vocab_size"]
    Hq, Hkv, D = config["num_attention_heads"], config["num_key_value_heads"], config["head_dim"]
    E, I = config["num_experts"], config["moe_intermediate_size"]
    g = config["maple_run"]["rtn_4bit"]["group_size"]
    w: dict[str, torch.Tensor] = {}
    w["model.word_embeddings.weight"] = _normal(seed, S_EMB, (V, H), dev, 0.02)
    codes = torch.empty(V, H // 8, dtype=torch.int32, device=dev).view(torch.uint32)
    scales = torch.empty(V, H // g, dtype=torch.bfloat16, device=dev)
    check(lib().maple_synth_rtn4_sym(seed, S_HEAD, V, H, g, 0.02, ptr(codes), ptr(scales), stream_ptr(dev)),
          "synth_rtn4")
    w["lm_head.weight"], w["lm_head.scales"] = codes, scales
    w["model.norm.weight"] = _normal(seed, S_NORM, (H,), dev, 0.02, 1.0, dtype=torch.float32)
    for i in range(config["num_hidden_layers"]):
        p = f"model.layers.{i}"
        s = lambda kind: layer_stream(i, kind)  # noqa: E731
        w[f"{p}.input_layernorm.weight"] = _normal(seed, s(L_IN_LN), (H,), dev, 0.02, 1.0, dtype=torch.float32)
        w[f"{p}.post_attention_layernorm.weight"] = _normal(seed, s(L_POST_LN), (H,), dev, 0.02, 1.0,
                                                            dtype=torch.float32)
        w[f"{p}.self_attn.q_norm.weight"] = _normal(seed, s(L_Q_NORM), (D,), dev, 0.02, 1.0, dtype=torch.float32)
        w[f"{p}.self_attn.k_norm.weight"] = _normal(seed, s(L_K_NORM), (D,), dev, 0.02, 1.0, dtype=torch.float32)
        for name, kc, ka, n, k in (("q_proj", L_Q, L_QA, Hq * D, H), ("k_proj", L_K, L_KA, Hkv * D, H),
                                   ("v_proj", L_V, L_VA, Hkv * D, H), ("o_proj", L_O, L_OA, H, Hq * D)):
            w[f"{p}.self_attn.{name}.weight"] = _ternary(seed, s(kc), (n, k // 16), dev)
            w[f"{p}.self_attn.{name}.row_alpha"] = _alpha(seed, s(ka), (n,), dev)
        w[f"{p}.mlp.gate.weight"] = _normal(seed, s(L_ROUTER), (E, H), dev, 0.02)
        for name, kc, ka, n, k in (("up_proj", L_UP, L_UPA, I, H), ("gate_proj", L_GATE, L_GATEA, I, H),
                                   ("down_proj", L_DOWN, L_DOWNA, H, I)):
            w[f"{p}.mlp.switch_mlp.{name}.weight"] = _ternary(seed, s(kc), (E, n, k // 16), dev)
            w[f"{p}.mlp.switch_mlp.{name}.row_alpha"] = _alpha(seed, s(ka), (E, n), dev)
    return w


def synthetic_tokens(seed: int, n: int, vocab: int, device, stream: int = S_PROMPT) -> torch.Tensor:
    """``n`` token ids uniform over ``vocab`` (hash % vocab)."""
    dev = torch.device(device)
    t = torch.empty(n, dtype=torch.int64, device=dev)
    check(lib().maple_synth_tokens(seed, stream, n, vocab, ptr(t), stream_ptr(dev)), "synth_tokens")
    return t


def fill_kv_cache(cache, seed: int, length: int, row0: int = 0, total_rows: int | None = None) -> None:
    """Fill positions [0, length) of every layer's K/V with bf16 N(0, 1) (the
    configs' random cached context) and set every row's length to ``length``.
    ``row0`` / ``total_rows``: the cache holds rows [row0, row0 + batch) of a
    ``total_rows``-row batch (a data-parallel rank), with those rows' values."""
    for i in range(len(cache.k)):
        for kind, t in ((L_KCACHE, cache.k[i]), (L_VCACHE, cache.v[i])):
            B, Hkv, T, D = t.shape
            n = B if total_rows is None else int(total_rows)
            tmp = _normal(seed, layer_stream(i, kind), (n, Hkv, length, D), t.device, 1.0)
            t[:, :, :length].copy_(tmp[row0:row0 + B])
            del tmp
    cache.seqlen.fill_(length)
    cache.seen = [length] * cache.batch
