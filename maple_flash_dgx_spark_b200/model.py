"""Packed ternary MoE decoder on the sm_100a operators.

Reference: model.py:64-920 (MapleRotaryEmbedding, KVCache, MapleAttention,
MapleSparseMoeBlock, MapleDecoderLayer, MapleForCausalLM).  The class names,
constructor arguments, cache API and the forward signature are the
reference's, so generate/serve code written against it runs unchanged.

One difference of mechanism, not of interface: a prompt (``q_len > 1``) is run
as ``q_len`` decode rows in one forward -- row i writes K/V at position
``past + i`` of the same cache row (through ``row_map``) and attends to
``[0, past + i]`` -- so prefill uses exactly the decode kernels' arithmetic and
a prompt prefilled at once equals the same tokens fed one by one.
"""

from __future__ import annotations

import json
from contextlib import contextmanager
from pathlib import Path

import torch

from maple_flash_dgx_spark_b200.kernels import (
    GROUPED_MIN_TOKENS,
    add_rms_norm,
    add_rms_norm_router_topk,
    apply_qkv_decode,
    attn_split_len,
    decode_gqa_attn,
    decode_gqa_attn_qk,
    moe_plan,
    rms_norm,
    router_topk,
)
from maple_flash_dgx_spark_b200.linear import (
    DenseEmbedding,
    PackedRTN4Embedding,
    PackedRTN4Linear,
    PackedTernaryExperts,
    PackedTernaryLinear,
)

MLP_CLAMP = 7.0


# The fused QK-norm/RoPE/attention launch pays off where a row's splits all
# fit one thread-block cluster (the attention runs as one cluster per row and
# kv head); with more splits every split CTA would redo the q heads' norm and
# RoPE, and the separate QK launch is faster (batch 64 x 8192 positions: 1373
# against 1113 tok/s).
_QK_FUSED_MAX_SPLITS = 16


def _fused_qk_attention() -> bool:
    """``MAPLE_FUSED_QK_ATTN=0`` keeps QK-norm/RoPE/K-V store as its own launch."""
    import os

    return os.environ.get("MAPLE_FUSED_QK_ATTN", "1") != "0"


def _tc_attention() -> bool:
    """``MAPLE_TC_ATTN=0`` keeps long-context decode attention on the
    canonical CUDA-core kernel (bit-exact with the CPU oracle)."""
    import os

    return os.environ.get("MAPLE_TC_ATTN", "1") != "0"
HEAD_GROUP_SIZE = 64


class MapleRMSNorm:
    def __init__(self, weight: torch.Tensor, eps: float = 1e-6):
        self.weight = weight
        self.eps = eps

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return rms_norm(hidden_states, self.weight, self.eps)


class MapleRotaryEmbedding:
    """RoPE tables (reference model.py:64-113): inv_freq = theta^(-2i/rot),
    cos/sin of t * inv_freq duplicated over both halves, computed in fp32 with
    torch on the CPU and held on the device in the model dtype.  The decode
    kernel reads row ``clamp(seqlen[b])`` of the table itself."""

    def __init__(self, head_dim: int, partial_rotary_factor: float, theta: float, device, dtype=torch.bfloat16):
        self.rotary_dim = int(head_dim * partial_rotary_factor)
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, self.rotary_dim, 2, dtype=torch.float32) / self.rotary_dim))
        self.device = device
        self.dtype = dtype
        self.cos_table: torch.Tensor | None = None
        self.sin_table: torch.Tensor | None = None
        self.max_cached = 0
        self.ensure_length(4096)

    @staticmethod
    def tables(inv_freq: torch.Tensor, n: int):
        t = torch.arange(n, dtype=torch.float32)
        freqs = torch.outer(t, inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos(), emb.sin()

    def ensure_length(self, n: int) -> None:
        if n <= self.max_cached:
            return
        n = max(int(n), 64)
        cos, sin = self.tables(self.inv_freq, n)
        self.cos_table = cos.to(self.dtype).to(self.device)
        self.sin_table = sin.to(self.dtype).to(self.device)
        self.max_cached = n


class KVCache:
    """Preallocated K/V, ``[B, n_kv, T, D]`` per layer; decode writes in place at
    ``seqlen`` (reference model.py:116-310, same API).  ``split_len`` is the
    attention split length (a graph constant of the cache)."""

    def __init__(self, layer_types, window, *, n_kv, head_dim, max_len, batch, dtype, device, n_heads=None):
        self.layer_types = layer_types
        self.window = window
        self.max_len = max_len
        n = len(layer_types)
        self.k = [torch.zeros(batch, n_kv, max_len, head_dim, dtype=dtype, device=device) for _ in range(n)]
        self.v = [torch.zeros(batch, n_kv, max_len, head_dim, dtype=dtype, device=device) for _ in range(n)]
        self.batch = batch
        self.seqlen = torch.zeros(batch, dtype=torch.int64, device=device)
        self.seen = [0] * batch
        self.slot: int | None = None
        self.row_of = list(range(batch))
        self.row_map = torch.arange(batch, dtype=torch.int32, device=device)
        self.remap = False
        self.split_len = attn_split_len(max_len, batch, n_kv)
        # Decode attention on the tensor pipe (the reference's bf16 dots) where
        # the canonical CUDA-core kernel is instruction-bound: caches with more
        # positions than one thread-block cluster of splits covers.
        self.attn_tc = (dtype == torch.bfloat16 and head_dim in (64, 128) and
                        -(-max_len // self.split_len) > _QK_FUSED_MAX_SPLITS and _tc_attention())

    @contextmanager
    def prefill_slot(self, row: int):
        if not 0 <= row < self.batch:
            raise ValueError(f"slot {row} outside cache batch {self.batch}.")
        prev = self.slot
        self.slot = row
        try:
            yield self
        finally:
            self.slot = prev

    def slot_rows(self) -> slice:
        return slice(None) if self.slot is None else slice(self.slot, self.slot + 1)

    def rows(self) -> slice:
        if self.slot is None:
            if self.row_of != list(range(self.batch)):
                raise RuntimeError("The whole-batch cache path needs the identity row map; "
                                   "run permuted slots through the fused decode path.")
            return slice(None)
        row = self.row_of[self.slot]
        return slice(row, row + 1)

    def swap_slots(self, i: int, j: int) -> None:
        if i == j:
            return
        if not self.remap:
            raise RuntimeError("swap_slots needs cache.remap: without the map the kernels read cache row == slot, "
                               "and a swap would silently read the wrong sequence's K/V.")
        self.row_of[i], self.row_of[j] = self.row_of[j], self.row_of[i]
        self.row_map[i], self.row_map[j] = self.row_map[j].clone(), self.row_map[i].clone()
        self.seen[i], self.seen[j] = self.seen[j], self.seen[i]
        si = self.seqlen[i].clone()
        self.seqlen[i] = self.seqlen[j]
        self.seqlen[j] = si

    def reset_slot(self, slot: int) -> None:
        self.seen[slot] = 0
        self.seqlen[slot] = 0

    def reset_identity(self) -> None:
        self.remap = False
        self.slot = None
        self.row_of = list(range(self.batch))
        self.row_map.copy_(torch.arange(self.batch, device=self.row_map.device, dtype=self.row_map.dtype))
        for b in range(self.batch):
            self.reset_slot(b)

    def past(self) -> int:
        if self.slot is not None:
            return self.seen[self.slot]
        first = self.seen[0]
        if any(n != first for n in self.seen):
            raise RuntimeError(f"Ragged cache lengths {self.seen} need a prefill slot; prefill one sequence at a time.")
        return first

    def advance(self, n: int, width: int | None = None) -> None:
        if self.slot is not None:
            self.seen[self.slot] += n
            self.seqlen[self.slot] = self.seen[self.slot]
            return
        w = self.batch if width is None else width
        for b in range(w):
            self.seen[b] += n
        self.seqlen[:w].add_(n)

    def advance_host(self, n: int, width: int) -> None:
        for b in range(width):
            self.seen[b] += n

    def snapshot(self) -> dict:
        return {"seqlen": self.seqlen.clone(), "seen": list(self.seen), "k": [t.clone() for t in self.k],
                "v": [t.clone() for t in self.v]}

    def restore(self, snap: dict) -> None:
        self.seqlen.copy_(snap["seqlen"])
        self.seen = list(snap["seen"])
        for dst, src in zip(self.k, snap["k"], strict=True):
            dst.copy_(src)
        for dst, src in zip(self.v, snap["v"], strict=True):
            dst.copy_(src)


class MapleAttention:
    """Decode attention of one layer (reference model.py:320-414): fused
    RMSNorm->QKV GEMV, QK-norm/RoPE/KV-store, split-K GQA, O GEMV.
    ``marks`` (optional, an expert_parallel.PhaseMarks) records the phase
    boundaries after the QKV projection and after the attention."""

    marks = None

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            self.marks.mark(name)

    def __init__(self, qkv, o_proj, q_norm, k_norm, *, num_heads, num_kv_heads, head_dim, sliding_window,
                 use_qk_norm, use_rope, layer_idx):
        if not use_qk_norm:
            raise ValueError("the decode path requires QK RMSNorm (reference decode_attn.py:392-393).")
        self.qkv_proj = qkv
        self.o_proj = o_proj
        self.q_norm = q_norm
        self.k_norm = k_norm
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.scale = head_dim ** -0.5
        self.sliding_window = sliding_window
        self.use_rope = use_rope
        self.layer_idx = layer_idx

    def __call__(self, hidden, seqlen, row_map, rotary, cache, *, rms_weight, rms_eps, kv_final=False):
        rows = hidden.shape[0]
        qkv = self.qkv_proj(hidden, rms_weight=rms_weight, rms_eps=rms_eps)
        self._mark("qkv")
        k_cache, v_cache = cache.k[self.layer_idx], cache.v[self.layer_idx]
        if row_map is None:
            k_cache, v_cache = k_cache[:rows], v_cache[:rows]
        splits = -(-int(k_cache.shape[2]) // int(cache.split_len))
        if kv_final and _fused_qk_attention() and splits <= _QK_FUSED_MAX_SPLITS:
            # decode rows: QK-norm + RoPE + K/V store inside the attention launch
            attn = decode_gqa_attn_qk(qkv, self.q_norm.weight, self.k_norm.weight, rotary.cos_table,
                                      rotary.sin_table, k_cache, v_cache, seqlen, row_map=row_map,
                                      num_heads=self.num_heads, num_kv_heads=self.num_kv_heads,
                                      head_dim=self.head_dim, rotary_dim=rotary.rotary_dim, use_rope=self.use_rope,
                                      eps=self.q_norm.eps, scale=self.scale, window=self.sliding_window,
                                      split_len=cache.split_len)
            self._mark("attention")
            return self.o_proj(attn.reshape(rows, -1))
        q = apply_qkv_decode(qkv, self.q_norm.weight, self.k_norm.weight, rotary.cos_table, rotary.sin_table,
                             k_cache, v_cache, seqlen, row_map=row_map, num_heads=self.num_heads,
                             num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                             rotary_dim=rotary.rotary_dim, use_rope=self.use_rope, use_qk_norm=True,
                             eps=self.q_norm.eps, rope_table=True)
        attn = decode_gqa_attn(q, k_cache, v_cache, seqlen, row_map=row_map, scale=self.scale,
                               window=self.sliding_window, split_len=cache.split_len, kv_final=kv_final,
                               tensor_cores=getattr(cache, "attn_tc", False))
        self._mark("attention")
        return self.o_proj(attn.reshape(rows, -1))


class MapleSparseMoeBlock:
    """Router top-k + fused expert SwiGLU + fused down/combine/residual
    (reference model.py:448-474)."""

    def __init__(self, gate_weight, up_gate: PackedTernaryExperts, down: PackedTernaryExperts, top_k: int,
                 moe_intermediate: int):
        self.gate_weight = gate_weight
        self.up_gate = up_gate
        self.down = down
        self.top_k = top_k
        self.moe_intermediate = moe_intermediate

    def fused_add_norm(self, hidden, attn_out, norm: "MapleRMSNorm"):
        """The decoder layer's post-attention add + RMSNorm fused into the
        router launch; returns the layer output."""
        residual, normed, idx, wt = add_rms_norm_router_topk(hidden, attn_out, norm.weight, norm.eps,
                                                             self.gate_weight, self.top_k)
        return self._experts(normed, idx, wt, residual)

    def __call__(self, hidden_states, residual=None):
        idx, wt = router_topk(hidden_states, self.gate_weight, self.top_k)
        return self._experts(hidden_states, idx, wt, residual)

    def _experts(self, hidden_states, idx, wt, residual):
        tokens = hidden_states.numel() // hidden_states.shape[-1]
        # from a few tokens on, sort the slots by expert once and run each
        # selected expert's weights once over all of its tokens
        plan = moe_plan(idx, self.gate_weight.shape[0]) if tokens >= GROUPED_MIN_TOKENS else None
        h = self.up_gate.swiglu(hidden_states, idx, plan=plan)
        return self.down.down_reduce(h, idx, wt, residual=residual, plan=plan)


class MapleDecoderLayer:
    def __init__(self, self_attn, mlp, input_layernorm, post_attention_layernorm):
        self.self_attn = self_attn
        self.mlp = mlp
        self.input_layernorm = input_layernorm
        self.post_attention_layernorm = post_attention_layernorm

    def __call__(self, hidden, seqlen, row_map, rotary, cache, kv_final=False):
        attn_out = self.self_attn(hidden, seqlen, row_map, rotary, cache, rms_weight=self.input_layernorm.weight,
                                  rms_eps=self.input_layernorm.eps, kv_final=kv_final)
        if hasattr(self.mlp, "fused_add_norm"):
            return self.mlp.fused_add_norm(hidden, attn_out, self.post_attention_layernorm)
        hidden, mlp_in = add_rms_norm(hidden, attn_out, self.post_attention_layernorm.weight,
                                      self.post_attention_layernorm.eps)
        return self.mlp(mlp_in, residual=hidden)


def _require_packed_format(config: dict) -> None:
    meta = config.get("maple_run") or {}
    if meta.get("format") != "packed-ternary-v1":
        raise ValueError("Checkpoint is not maple-run packed-ternary-v1. Convert with `maple-run convert` rather "
                         "than loading the Hugging Face bf16 dump.")


def _as_uint32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint32 else t.view(torch.uint32)


def _cat_rows(tensors, dim):
    """Concatenate packed uint32 tensors (through an int32 view)."""
    return torch.cat([_as_uint32(t).view(torch.int32) for t in tensors], dim=dim).view(torch.uint32)


def packed_decode_bytes(config: dict, side_bytes: int = 2, alpha_bytes: int = 2, norm_bytes: int = 4,
                        *, flash_head: bool = False) -> dict[str, int]:
    """HBM bytes of weights read per decode token (reference model.py:562-628,
    with the element sizes of the tensors actually held)."""
    L = int(config["num_hidden_layers"])
    H = int(config["hidden_size"])
    n_q, n_kv, D = int(config["num_attention_heads"]), int(config["num_key_value_heads"]), int(config["head_dim"])
    E, k, I, V = (int(config["num_experts"]), int(config["num_experts_per_tok"]), int(config["moe_intermediate_size"]),
                  int(config["vocab_size"]))
    rtn = (config.get("maple_run") or {}).get("rtn_4bit", {})
    group = int(rtn.get("group_size", HEAD_GROUP_SIZE))
    symmetric = rtn.get("mode") == "symmetric"
    qkv_n = (n_q + 2 * n_kv) * D
    attn_codes = L * (qkv_n * H + H * n_q * D) // 4
    attn_alpha = L * (qkv_n + H) * alpha_bytes
    router = L * E * H * side_bytes
    expert_codes = L * k * (2 * I * H + H * I) // 4
    expert_alpha = L * k * (2 * I + H) * alpha_bytes
    meta = config.get("flash_head") or (config.get("maple_run") or {}).get("flash_head")
    if flash_head and meta:
        head_rows = int(meta["n_clusters"]) + int(meta.get("n_probes", 512)) * int(meta["cluster_size"]) + len(
            meta.get("force_tokens") or [])
    else:
        head_rows = V
    head_codes = head_rows * H // 2
    head_scales = head_rows * (H // group) * side_bytes * (1 if symmetric else 2)
    norms = L * (2 * H + 2 * D) * norm_bytes + H * norm_bytes
    emb_row = H * 2
    packed = attn_codes + attn_alpha + router + expert_codes + expert_alpha + head_codes + head_scales + norms + emb_row
    return {"packed_weight_bytes": packed, "attn_bytes": attn_codes + attn_alpha, "router_bytes": router,
            "expert_bytes": expert_codes + expert_alpha, "head_bytes": head_codes + head_scales}


def kv_bytes_per_token(config: dict, context: int, dtype_bytes: int = 2) -> int:
    """K+V bytes one decode token reads at ``context`` cached positions."""
    return (int(config["num_hidden_layers"]) * int(config["num_key_value_heads"]) * int(config["head_dim"]) * 2 *
            dtype_bytes * context)


class MapleForCausalLM:
    """Reference model.py:631-920."""

    def __init__(self, config: dict, *, device: torch.device, dtype: torch.dtype = torch.bfloat16):
        self.config = config
        self.device = device
        self.dtype = dtype
        self.hidden_size = int(config["hidden_size"])
        self.vocab_size = int(config["vocab_size"])
        self.num_layers = int(config["num_hidden_layers"])
        self.num_heads = int(config["num_attention_heads"])
        self.num_kv_heads = int(config["num_key_value_heads"])
        self.head_dim = int(config["head_dim"])
        self.num_experts = int(config["num_experts"])
        self.top_k = int(config["num_experts_per_tok"])
        self.moe_intermediate = int(config["moe_intermediate_size"])
        self.rms_eps = float(config.get("rms_norm_eps", 1e-6))
        self.sliding_window = int(config.get("sliding_window", 512))
        self.layer_types = list(config["layer_types"])
        self.use_qk_norm = bool(config.get("use_qk_norm", True))
        self.nope_on_global = bool(config.get("nope_on_global_attention", True))
        self.eos_token_id = config.get("eos_token_id")
        self.bos_token_id = config.get("bos_token_id")
        self.word_embeddings = None
        self.layers: list[MapleDecoderLayer] = []
        self.norm = None
        self.lm_head = None
        self.lm_head_flash = None
        self.rotary = MapleRotaryEmbedding(self.head_dim, float(config.get("partial_rotary_factor", 0.5)),
                                           float(config.get("rope_theta", 10000)), device, dtype)

    # ------------------------------------------------------------ loading --
    @classmethod
    def from_packed(cls, model_dir: str, *, device="cuda", dtype=torch.bfloat16, use_flash_head: bool = False):
        """Load a packed-ternary-v1 directory (reference model.py:664-706)."""
        from safetensors.torch import load_file

        model_dir = Path(model_dir).expanduser()
        config = json.loads((model_dir / "config.json").read_text())
        _require_packed_format(config)
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("MapleForCausalLM packed decode requires CUDA.")
        index_path = model_dir / "model.safetensors.index.json"
        if index_path.exists():
            shards = sorted(set(json.loads(index_path.read_text())["weight_map"].values()))
        else:
            shards = sorted(p.name for p in model_dir.glob("*.safetensors"))
        weights: dict[str, torch.Tensor] = {}
        for name in shards:
            if not use_flash_head and name == "model-flashhead.safetensors":
                continue
            weights.update(load_file(str(model_dir / name), device=str(device)))
        return cls.from_weight_dict(config, weights, device=device, dtype=dtype, use_flash_head=use_flash_head)

    @classmethod
    def from_weight_dict(cls, config: dict, weights: dict, *, device="cuda", dtype=torch.bfloat16,
                         use_flash_head: bool = False):
        _require_packed_format(config)
        device = torch.device(device)
        model = cls(config, device=device, dtype=dtype)
        model._load_weights(dict(weights), use_flash_head=use_flash_head)
        return model

    _BF16_SUFFIXES = (".mlp.gate.weight", ".scales", ".biases")

    def _cast_side_tensors(self, weights):
        """Router and RTN scales/biases held in the model dtype (reference model.py:730-748)."""
        for key in list(weights):
            if weights[key].dtype == torch.float32 and key.endswith(self._BF16_SUFFIXES):
                weights[key] = weights[key].to(self.dtype)

    def _load_weights(self, weights, *, use_flash_head: bool = False):
        self._cast_side_tensors(weights)
        rtn = (self.config.get("maple_run") or {}).get("rtn_4bit", {})
        group = int(rtn.get("group_size", HEAD_GROUP_SIZE))
        emb = weights.pop("model.word_embeddings.weight")
        if emb.dtype in (torch.uint32, torch.int32) and "model.word_embeddings.scales" in weights:
            self.word_embeddings = PackedRTN4Embedding(_as_uint32(emb), weights.pop("model.word_embeddings.scales"),
                                                       weights.pop("model.word_embeddings.biases", None), group)
        else:
            self.word_embeddings = DenseEmbedding(emb.to(self.dtype))
        self.lm_head = PackedRTN4Linear(_as_uint32(weights.pop("lm_head.weight")), weights.pop("lm_head.scales"),
                                        weights.pop("lm_head.biases", None), group_size=group)
        if use_flash_head:
            from maple_flash_dgx_spark_b200.flash_head import build_flash_head

            self.lm_head_flash = build_flash_head(config=self.config, lm_head=self.lm_head, weights=weights,
                                                  device=self.device, dtype=self.dtype)
        else:
            for key in [k for k in weights if k.startswith("lm_head_flash.")]:
                weights.pop(key)
        self.norm = MapleRMSNorm(weights.pop("model.norm.weight"), self.rms_eps)
        layers = []
        for i in range(self.num_layers):
            p = f"model.layers.{i}"
            layer_type = self.layer_types[i]
            use_rope = not (self.nope_on_global and layer_type == "full_attention")
            sliding = self.sliding_window if layer_type == "sliding_attention" else None
            qkv_w = _cat_rows([weights.pop(f"{p}.self_attn.{n}_proj.weight") for n in "qkv"], 0)
            qkv_a = torch.cat([weights.pop(f"{p}.self_attn.{n}_proj.row_alpha") for n in "qkv"], 0)
            up_w = _cat_rows([weights.pop(f"{p}.mlp.switch_mlp.up_proj.weight"),
                              weights.pop(f"{p}.mlp.switch_mlp.gate_proj.weight")], 1)
            up_a = torch.cat([weights.pop(f"{p}.mlp.switch_mlp.up_proj.row_alpha"),
                              weights.pop(f"{p}.mlp.switch_mlp.gate_proj.row_alpha")], 1)
            attn = MapleAttention(
                PackedTernaryLinear(qkv_w, qkv_a),
                PackedTernaryLinear(_as_uint32(weights.pop(f"{p}.self_attn.o_proj.weight")),
                                    weights.pop(f"{p}.self_attn.o_proj.row_alpha")),
                MapleRMSNorm(weights.pop(f"{p}.self_attn.q_norm.weight"), self.rms_eps),
                MapleRMSNorm(weights.pop(f"{p}.self_attn.k_norm.weight"), self.rms_eps),
                num_heads=self.num_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                sliding_window=sliding, use_qk_norm=self.use_qk_norm, use_rope=use_rope, layer_idx=i)
            mlp = MapleSparseMoeBlock(
                weights.pop(f"{p}.mlp.gate.weight"), PackedTernaryExperts(up_w, up_a),
                PackedTernaryExperts(_as_uint32(weights.pop(f"{p}.mlp.switch_mlp.down_proj.weight")),
                                     weights.pop(f"{p}.mlp.switch_mlp.down_proj.row_alpha")),
                top_k=self.top_k, moe_intermediate=self.moe_intermediate)
            layers.append(MapleDecoderLayer(
                attn, mlp, MapleRMSNorm(weights.pop(f"{p}.input_layernorm.weight"), self.rms_eps),
                MapleRMSNorm(weights.pop(f"{p}.post_attention_layernorm.weight"), self.rms_eps)))
        self.layers = layers

    # ------------------------------------------------------------ running --
    def make_cache(self, max_len: int = 2048, batch: int = 1) -> KVCache:
        self.rotary.ensure_length(max_len)
        return KVCache(self.layer_types, self.sliding_window, n_kv=self.num_kv_heads, head_dim=self.head_dim,
                       max_len=max_len, batch=batch, dtype=self.dtype, device=self.device, n_heads=self.num_heads)

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        h = self.word_embeddings(ids)
        return h if h.dtype == self.dtype else h.to(self.dtype)

    def forward(self, input_ids: torch.Tensor, cache: KVCache | None = None, *, logits_to_keep: int = 1):
        """Logits ``[B, keep, V]`` (reference model.py:848-886)."""
        if input_ids.dim() == 1:
            input_ids = input_ids.unsqueeze(0)
        bsz, seq_len = input_ids.shape
        if cache is None:
            cache = self.make_cache(max_len=seq_len, batch=bsz)
        if seq_len == 1:
            rows = bsz
            seqlen = cache.seqlen[cache.slot_rows()][:bsz]
            if cache.slot is not None:
                row_map = cache.row_map[cache.slot:cache.slot + 1]
            elif cache.remap:
                row_map = cache.row_map[:bsz]
            else:
                row_map = None
        else:
            if bsz != 1:
                raise RuntimeError("prefill one sequence at a time (cache.prefill_slot); batched rows decode only.")
            past = cache.past()
            if past + seq_len > cache.max_len:
                raise RuntimeError(f"KV cache overflow: need {past + seq_len} slots, max_len={cache.max_len}.")
            rows = seq_len
            seqlen = torch.arange(past, past + seq_len, device=self.device, dtype=torch.int64)
            row = cache.rows().start or 0
            row_map = torch.full((seq_len,), row, device=self.device, dtype=torch.int32)
        self.rotary.ensure_length(cache.max_len)
        hidden = self.embed(input_ids.reshape(rows))
        for layer in self.layers:
            hidden = layer(hidden, seqlen, row_map, self.rotary, cache, kv_final=seq_len == 1)
        cache.advance(seq_len, bsz)
        keep = hidden if seq_len == 1 else hidden[-logits_to_keep:] if logits_to_keep else hidden
        normed = self.norm(keep)
        if self.lm_head_flash is not None and bsz == 1 and seq_len == 1:
            return self.lm_head_flash(normed.reshape(1, 1, -1))
        return self.lm_head(normed).reshape(bsz, -1, self.vocab_size)

    __call__ = forward

    @torch.inference_mode()
    def generate(self, input_ids, max_tokens: int = 128):
        """Greedy decode (reference model.py:888-913)."""
        from maple_flash_dgx_spark_b200.kernels import argmax

        if not torch.is_tensor(input_ids):
            input_ids = torch.tensor(input_ids, device=self.device, dtype=torch.long)
        input_ids = input_ids.to(device=self.device, dtype=torch.long)
        if input_ids.dim() == 1:
            input_ids = input_ids.unsqueeze(0)
        prompt_len = int(input_ids.shape[-1])
        cache = self.make_cache(max_len=prompt_len + max(int(max_tokens), 1))
        logits = self.forward(input_ids, cache=cache, logits_to_keep=1)
        out = [input_ids]
        for _ in range(max_tokens):
            next_id = argmax(logits[:, -1, :]).reshape(1, 1)
            out.append(next_id)
            if self.eos_token_id is not None and int(next_id[0, 0]) == int(self.eos_token_id):
                break
            logits = self.forward(next_id, cache=cache, logits_to_keep=1)
        return torch.cat(out, dim=-1)

    def decode_traffic(self) -> dict[str, int]:
        return packed_decode_bytes(self.config, flash_head=self.lm_head_flash is not None)
