"""Whole-stack batch-1 decode in one persistent launch (``maple_decode_layers``).

Reference: the layer loop of model.py:848-886 at batch 1 / ``q_len`` 1 --
per layer ternary_gemv (RMSNorm->QKV), apply_qkv_decode, decode_gqa_attn,
ternary_gemv (O), add_rms_norm + router_topk, ternary_expert_swiglu and the
down GEMV + moe_reduce_add.  ``maple_decode_layers`` runs all of them for all
layers in one cooperative launch (one CTA per SM, grid barriers between the
six phases of a layer) and returns exactly the hidden row the operator-by-
operator path returns.

A :class:`FusedDecodePlan` holds what the launch needs for one (model, KV
cache) pair: a device array of per-layer weight/cache pointers and the
launch's own scratch (its first words are a grid barrier that persists across
launches, so the buffer is private to the plan).
"""

from __future__ import annotations

import os

import torch

from maple_flash_dgx_spark_b200._lib import BF16, F32, check, lib, ptr, stream_ptr

_DESC_WORDS = 17  # maple_decode_layer: 15 pointers + window + use_rope


def fused_decode_enabled() -> bool:
    """``MAPLE_FUSED_DECODE=1`` runs batch-1 decode steps as one persistent
    launch; otherwise (the default) the operator-by-operator path runs."""
    return os.environ.get("MAPLE_FUSED_DECODE", "0") == "1"


def _code(dtype: torch.dtype) -> int:
    return F32 if dtype == torch.float32 else BF16


class FusedDecodePlan:
    """Descriptor array and scratch of ``maple_decode_layers`` for one cache."""

    def __init__(self, model, cache):
        self.model_id = id(model)
        self.cache_id = id(cache)
        dev = model.device
        L = model.num_layers
        layers = model.layers
        self.keep: list[torch.Tensor] = []

        def held(t: torch.Tensor, dtype=None) -> torch.Tensor:
            t = t.reshape(-1) if t.dim() == 1 else t
            t = t.contiguous() if dtype is None else t.to(dtype).contiguous()
            self.keep.append(t)
            return t

        # One dtype per tensor family; a mix is widened to fp32 (exact for bf16).
        def family(ts):
            dts = {t.dtype for t in ts}
            return next(iter(dts)) if len(dts) == 1 else torch.float32

        # apply_qkv_decode uses the k_norm weight in the q_norm weight's dtype
        knorms = [ly.self_attn.k_norm.weight.reshape(-1).to(ly.self_attn.q_norm.weight.dtype) for ly in layers]
        norms = ([ly.input_layernorm.weight for ly in layers] + [ly.post_attention_layernorm.weight for ly in layers]
                 + [ly.self_attn.q_norm.weight for ly in layers] + knorms)
        self.norm_dtype = family(norms)
        alphas = []
        for ly in layers:
            alphas += [ly.self_attn.qkv_proj.row_alpha, ly.self_attn.o_proj.row_alpha, ly.mlp.up_gate.row_alpha,
                       ly.mlp.down.row_alpha]
        self.alpha_dtype = family(alphas)
        self.gate_dtype = family([ly.mlp.gate_weight for ly in layers])
        desc = torch.zeros(L, _DESC_WORDS, dtype=torch.int64)
        for i, ly in enumerate(layers):
            at, mlp = ly.self_attn, ly.mlp
            nd, ad, gd = self.norm_dtype, self.alpha_dtype, self.gate_dtype
            row = [
                ptr(held(at.qkv_proj.packed_weight)), ptr(held(at.qkv_proj.row_alpha.reshape(-1), ad)),
                ptr(held(at.o_proj.packed_weight)), ptr(held(at.o_proj.row_alpha.reshape(-1), ad)),
                ptr(held(ly.input_layernorm.weight.reshape(-1), nd)),
                ptr(held(ly.post_attention_layernorm.weight.reshape(-1), nd)),
                ptr(held(at.q_norm.weight.reshape(-1), nd)), ptr(held(knorms[i], nd)),
                ptr(held(mlp.gate_weight, gd)),
                ptr(held(mlp.up_gate.packed_weight)), ptr(held(mlp.up_gate.row_alpha, ad)),
                ptr(held(mlp.down.packed_weight)), ptr(held(mlp.down.row_alpha, ad)),
                ptr(cache.k[i]), ptr(cache.v[i]),
                int(at.sliding_window or 0), int(bool(at.use_rope)),
            ]
            desc[i] = torch.tensor(row, dtype=torch.int64)
        self.desc = desc.to(dev)
        k0 = cache.k[0]
        self.cache_sb, self.cache_sh = int(k0.stride(0)), int(k0.stride(1))
        for t in cache.k + cache.v:
            if t.stride() != k0.stride() or t.dtype != torch.bfloat16:
                raise ValueError("fused decode needs bf16 K/V caches of one layout.")
        nbytes = lib().maple_decode_layers_workspace_bytes(
            model.hidden_size, model.num_heads, model.num_kv_heads, model.head_dim, model.num_experts,
            model.top_k, model.moe_intermediate, cache.max_len, cache.split_len)
        if nbytes <= 0:
            raise ValueError("maple_decode_layers_workspace_bytes rejected the model/cache shape.")
        self.ws = torch.zeros(int(nbytes), dtype=torch.uint8, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    # byte offset of the trace region inside the workspace (after the fixed
    # scratch); mirrors step_layout() in csrc/decode_step.cu
    TRACE_BYTES = 1 << 20

    def enable_trace(self, on: bool = True) -> None:
        """Switch the per-barrier timestamps (and, when they fit, the per-phase
        clock64 checkpoints) on: sync word 2 of the workspace."""
        self.ws.view(torch.int32)[2] = 1 if on else 0
        self.ws[self.ws.numel() - self.TRACE_BYTES:].zero_()

    def read_marks(self, model) -> torch.Tensor:
        """Per-phase checkpoints of the last traced launch, ``[n_layers, 6, 8,
        grid]`` clock64 values (0 = not reached); present when ``n_layers *
        grid * 480`` bytes fit the trace region."""
        grid = torch.cuda.get_device_properties(self.ws.device).multi_processor_count
        L = model.num_layers
        off = self.ws.numel() - self.TRACE_BYTES + L * 6 * 2 * grid * 8
        n = L * 6 * 8 * grid
        return self.ws[off:off + n * 8].view(torch.int64).reshape(L, 6, 8, grid).cpu()

    def read_trace(self, model) -> torch.Tensor:
        """Barrier timestamps of the last launch, ``[n_barriers, 2, grid]`` ns
        (arrival, release); ``n_barriers = 6 * n_layers``."""
        grid = torch.cuda.get_device_properties(self.ws.device).multi_processor_count
        nb = 6 * model.num_layers
        off = self.ws.numel() - self.TRACE_BYTES
        raw = self.ws[off:off + nb * 2 * grid * 8].view(torch.int64)
        return raw.reshape(nb, 2, grid).cpu()

    def matches(self, model, cache) -> bool:
        return self.model_id == id(model) and self.cache_id == id(cache)

    def run(self, model, cache, hidden: torch.Tensor, seqlen: torch.Tensor, row_map: torch.Tensor | None) -> None:
        """Run every layer on ``hidden`` ([1, H] bf16, updated in place)."""
        rot = model.rotary
        rotary_dim = rot.rotary_dim
        cos, sin = rot.cos_table, rot.sin_table
        rm = None if row_map is None else row_map.reshape(-1)
        check(lib().maple_decode_layers(
            ptr(self.desc), model.num_layers, ptr(hidden), ptr(seqlen), ptr(rm), ptr(cos), ptr(sin), _code(cos.dtype),
            cos.stride(0), cos.shape[0], model.hidden_size, model.num_heads, model.num_kv_heads, model.head_dim,
            rotary_dim, model.num_experts, model.top_k, model.moe_intermediate, cache.batch, cache.max_len,
            self.cache_sb, self.cache_sh, cache.split_len, _code(self.alpha_dtype), _code(self.norm_dtype),
            _code(self.gate_dtype), float(model.rms_eps), float(model.head_dim ** -0.5), ptr(self.ws),
            self.ws.numel(), ptr(self.err), stream_ptr(hidden.device)), "decode_layers")


def fused_decode_supported(model, cache) -> bool:
    """Shapes ``maple_decode_layers`` accepts (the rest decode per operator)."""
    if model.dtype != torch.bfloat16 or not model.layers:
        return False
    if model.head_dim not in (64, 128) or model.num_heads % model.num_kv_heads:
        return False
    if model.num_heads // model.num_kv_heads > 8 or not 0 < model.top_k <= 8 or model.num_experts > 256:
        return False
    H, qd, inter = model.hidden_size, model.num_heads * model.head_dim, model.moe_intermediate
    if H % 64 or qd % 64 or inter % 64 or H > 8192 or qd > 8192 or (inter // 16 + 15) // 16 > 8:
        return False
    if cache.split_len not in (32, 64, 128):
        return False
    rot = model.rotary
    if rot.rotary_dim % 2 or rot.cos_table is None or rot.cos_table.stride(1) != 1:
        return False
    for ly in model.layers:
        if not hasattr(ly.mlp, "fused_add_norm") or not getattr(ly.self_attn, "qkv_proj", None):
            return False
    return all(t.dtype == torch.bfloat16 for t in cache.k[:1])


def phase_report(layers: int = 48, prompt_len: int = 512, seed: int = 1) -> str:
    """Per-phase timing of one whole-step launch on configs[2]-shaped layers
    (hidden 2048, 32/4 heads of 128, 64 experts top-8, intermediate 1024; a
    4096-token vocabulary, since the head is not part of the launch), read
    from the grid barriers' timestamps: for each phase the median over layers
    of its work (first release of the previous barrier to the last CTA's
    arrival), of the barrier itself (last arrival to last release) and of the
    previous barrier's release spread."""
    import statistics

    from maple_flash_dgx_spark_b200.kernels import argmax
    from maple_flash_dgx_spark_b200.model import MapleForCausalLM
    from maple_flash_dgx_spark_b200.synth import synthetic_config, synthetic_tokens, synthetic_weights

    os.environ["MAPLE_FUSED_DECODE"] = "1"
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = synthetic_config(num_layers=layers, vocab=4096)
    model = MapleForCausalLM.from_weight_dict(cfg, synthetic_weights(cfg, seed, dev), device=dev)
    cache = model.make_cache(max_len=prompt_len + 16)
    with torch.inference_mode():
        logits = model.forward(synthetic_tokens(seed, prompt_len, cfg["vocab_size"], dev).reshape(1, -1), cache=cache)
        tok = argmax(logits[:, -1, :]).reshape(1, 1)
        for _ in range(4):
            tok = argmax(model.forward(tok, cache=cache)[:, -1, :]).reshape(1, 1)
        plan = cache._fused_plan
        plan.enable_trace(True)
        model.forward(tok, cache=cache)
        torch.cuda.synchronize(dev)
        tr = plan.read_trace(model).double()
        plan.enable_trace(False)
    names = ["qkv", "attention", "o", "router", "swiglu", "down"]
    arr, rel = tr[:, 0, :], tr[:, 1, :]
    work = {n: [] for n in names}
    wait = {n: [] for n in names}
    spread = {n: [] for n in names}
    for b in range(1, tr.shape[0]):
        n = names[b % 6]
        work[n].append((arr[b].max() - rel[b - 1].min()).item() / 1000)
        wait[n].append((rel[b].max() - arr[b].max()).item() / 1000)
        spread[n].append((rel[b - 1].max() - rel[b - 1].min()).item() / 1000)
    lines = ["phase      work us  barrier us  release spread us (medians over layers)"]
    for n in names:
        lines.append(f"{n:10s} {statistics.median(work[n]):7.2f}  {statistics.median(wait[n]):10.2f}  "
                     f"{statistics.median(spread[n]):17.2f}")
    total = (rel[-1].max() - arr[0].min()).item() / 1000
    lines.append(f"first arrival -> last release: {total:.1f} us over {tr.shape[0]} barriers "
                 f"({total / layers:.2f} us per layer)")
    return "\n".join(lines)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="Phase timing of the whole-step decode launch (needs a GPU).")
    ap.add_argument("--layers", type=int, default=48)
    print(phase_report(ap.parse_args().layers))
