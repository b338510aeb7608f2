"""Golden tiny checkpoint + greedy decode produced by the REFERENCE itself.

Usage (needs the reference checkout; CPU only, about a minute):

    python tests/golden/make_tiny_model.py /path/to/maple-flash-dgx-spark

1. Writes a small Hugging Face-style source checkpoint (per-expert weights,
   seeded numpy draws) to a temporary directory.
2. Converts it with the reference's own ``convert_checkpoint``
   (convert.py:380-450): ternary codes + fp32 row_alpha, RTN-4 g64 affine
   embedding and lm_head, stacked ``switch_mlp`` experts, ``config.json``.
   The converted directory is copied to ``tests/golden/tiny_packed/``.
3. Loads that directory with the reference's ``MapleForCausalLM``
   (model.py:664-832) on the CPU in fp32 under the Triton interpreter and
   decodes greedily, one token per forward (the reference's decode path:
   apply_qkv_decode / decode_gqa_attn / router / experts / rtn4 head).  The
   reference's kernels store bf16 on a GPU; here every kernel output, the
   K/V cache, the RoPE table, the embedding row and the tensors a bf16 model
   holds in bf16 (router, RTN scales and biases) are rounded to bf16 (RNE)
   at exactly those points, so the run follows the reference's arithmetic
   at its GPU rounding points.  It also records ``generate()`` (prompt
   prefilled through the reference's SDPA path) for the same prompt.

Writes ``tests/golden/tiny_packed/`` and ``tests/golden/tiny_greedy.npz``.
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "tiny_packed"
SEED = 7
PROMPT_LEN, N_NEW = 12, 20

TINY = {
    "architectures": ["MapleForCausalLM"],
    "hidden_size": 256,
    "num_hidden_layers": 2,
    "num_attention_heads": 4,
    "num_key_value_heads": 2,
    "head_dim": 64,
    "num_experts": 8,
    "num_experts_per_tok": 2,
    "moe_intermediate_size": 128,
    "vocab_size": 512,
    "tie_word_embeddings": False,
    "rms_norm_eps": 1e-6,
    "sliding_window": 16,
    "layer_types": ["sliding_attention", "full_attention"],
    "use_qk_norm": True,
    "nope_on_global_attention": True,
    "partial_rotary_factor": 0.5,
    "rope_theta": 10000.0,
    "eos_token_id": None,
    "dtype": "float32",
}


def source_weights(cfg: dict, rng: np.random.RandomState) -> dict[str, np.ndarray]:
    """Hugging Face-style tensors (the names convert.py reads), fan-in scaled."""
    h, v, e, inter, d = (cfg["hidden_size"], cfg["vocab_size"], cfg["num_experts"], cfg["moe_intermediate_size"],
                         cfg["head_dim"])
    nq, nkv = cfg["num_attention_heads"] * d, cfg["num_key_value_heads"] * d

    def n(*shape, s=1.0):
        return (rng.standard_normal(shape) * s).astype(np.float32)

    w = {"model.word_embeddings.weight": n(v, h), "lm_head.weight": n(v, h, s=3.0 / np.sqrt(h)),
         "model.norm.weight": 1.0 + n(h, s=0.1)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        w[f"{p}.input_layernorm.weight"] = 1.0 + n(h, s=0.1)
        w[f"{p}.post_attention_layernorm.weight"] = 1.0 + n(h, s=0.1)
        w[f"{p}.self_attn.q_norm.weight"] = 1.0 + n(d, s=0.1)
        w[f"{p}.self_attn.k_norm.weight"] = 1.0 + n(d, s=0.1)
        w[f"{p}.self_attn.q_proj.weight"] = n(nq, h, s=h ** -0.5)
        w[f"{p}.self_attn.k_proj.weight"] = n(nkv, h, s=h ** -0.5)
        w[f"{p}.self_attn.v_proj.weight"] = n(nkv, h, s=h ** -0.5)
        w[f"{p}.self_attn.o_proj.weight"] = n(h, nq, s=nq ** -0.5)
        w[f"{p}.mlp.gate.weight"] = n(e, h, s=2.0 * h ** -0.5)
        for j in range(e):
            q = f"{p}.mlp.experts.{j}"
            w[f"{q}.gate_proj.weight"] = n(inter, h, s=h ** -0.5)
            w[f"{q}.up_proj.weight"] = n(inter, h, s=h ** -0.5)
            w[f"{q}.down_proj.weight"] = n(h, inter, s=inter ** -0.5)
    return w


def _bf16(torch, t):
    return t.to(torch.bfloat16).to(t.dtype) if t.is_floating_point() else t


def install_bf16_stores(torch):
    """Round every kernel output the reference stores as bf16 on a GPU."""
    import maple_run.linear as lin
    import maple_run.model as mdl

    def rounding(fn, cache_args=()):
        def wrapped(*args, **kwargs):
            out = fn(*args, **kwargs)
            for i in cache_args:  # K/V caches written in place
                args[i].copy_(_bf16(torch, args[i]))
            if isinstance(out, tuple):
                return tuple(_bf16(torch, o) for o in out)
            return _bf16(torch, out)
        return wrapped

    for name in ("ternary_gemv", "ternary_expert_swiglu", "ternary_expert_gemv", "rtn4_gemv", "rtn4_embedding"):
        setattr(lin, name, rounding(getattr(lin, name)))
    for name in ("decode_gqa_attn", "add_rms_norm", "moe_reduce_add", "rms_norm"):
        setattr(mdl, name, rounding(getattr(mdl, name)))
    mdl.apply_qkv_decode = rounding(mdl.apply_qkv_decode, cache_args=(5, 6))


def main(root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(root) / "src"))
    import torch
    from safetensors.numpy import save_file
    from safetensors.torch import load_file

    torch.Tensor.is_cuda = property(lambda self: True)  # interpreter only
    from maple_run.convert import convert_checkpoint

    install_bf16_stores(torch)
    from maple_run.model import MapleForCausalLM

    rng = np.random.RandomState(SEED)
    with tempfile.TemporaryDirectory() as tmp:
        src, dst = Path(tmp) / "src", Path(tmp) / "packed"
        src.mkdir()
        (src / "config.json").write_text(json.dumps(TINY, indent=2))
        save_file(source_weights(TINY, rng), str(src / "model.safetensors"))
        convert_checkpoint(str(src), str(dst))
        if OUT_DIR.exists():
            shutil.rmtree(OUT_DIR)
        OUT_DIR.mkdir()
        for f in sorted(dst.iterdir()):
            if f.name == "config.json" or f.suffix == ".safetensors" or f.name.endswith(".index.json"):
                shutil.copy2(f, OUT_DIR / f.name)

    config = json.loads((OUT_DIR / "config.json").read_text())
    weights = {}
    for f in sorted(OUT_DIR.glob("*.safetensors")):
        weights.update(load_file(str(f)))
    # a bf16 model holds the router and RTN scales/biases in bf16
    # (model.py:719-748 _cast_side_tensors); the fp32 run keeps their values
    for key in weights:
        if key.endswith(MapleForCausalLM._BF16_SUFFIXES):
            weights[key] = _bf16(torch, weights[key])
    model = MapleForCausalLM.from_weight_dict(config, weights, device=torch.device("cpu"), dtype=torch.float32)
    model.rotary.ensure_length(4096)
    model.rotary.cos_table = _bf16(torch, model.rotary.cos_table)
    model.rotary.sin_table = _bf16(torch, model.rotary.sin_table)

    prompt = rng.randint(0, TINY["vocab_size"], size=PROMPT_LEN).astype(np.int64)
    total = PROMPT_LEN + N_NEW
    cache = model.make_cache(max_len=total, batch=1)
    logits_steps, ids = [], []
    nxt = None
    with torch.inference_mode():
        for i in range(total - 1):
            tok = int(prompt[i]) if i < PROMPT_LEN else nxt
            logits = model.forward(torch.tensor([[tok]]), cache=cache)[0, -1]
            logits_steps.append(logits.numpy().copy())
            nxt = int(logits.argmax())
            if i >= PROMPT_LEN - 1:
                ids.append(nxt)
        gen = model.generate(torch.from_numpy(prompt), max_tokens=N_NEW)[0, PROMPT_LEN:].numpy()
    logits_steps = np.stack(logits_steps)
    top2 = -np.sort(-logits_steps, axis=-1)[:, :2]
    np.savez_compressed(HERE / "tiny_greedy.npz", prompt=prompt, ids=np.asarray(ids, np.int64),
                        logits=logits_steps.astype(np.float32), generate_ids=gen.astype(np.int64))
    print("greedy ids", ids)
    print("generate()", gen.tolist())
    print("min top-1/top-2 logit margin", float((top2[:, 0] - top2[:, 1]).min()))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_tiny_model.py /path/to/maple-flash-dgx-spark")
    main(sys.argv[1])
