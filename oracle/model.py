"""CPU oracle of one decode step of the packed ternary MoE model -- TEST
INFRASTRUCTURE ONLY (checker / CPU baseline, never the product).

Restates reference model.py:320-506 (MapleAttention decode branch,
MapleSparseMoeBlock, MapleDecoderLayer) and :848-886 (forward) with the
oracle's operators, including the reference's rounding points: bf16 between
operators, fp32 inside them.  Prompts are fed one token at a time (the
reference's decode path); the CUDA engine's batched prefill must reproduce it.

Weights are regenerated here from the synthetic generator's definition
(``orc_synth_*`` in oracle.c), independently of the CUDA library.
"""

from __future__ import annotations

import ctypes
import time

import numpy as np

import oracle as O

# Stream ids of the synthetic generator (same definition as the engine's).
S_EMB, S_NORM, S_HEAD, S_PROMPT = 1, 2, 3, 50
L_IN_LN, L_POST_LN, L_Q_NORM, L_K_NORM = 0, 1, 2, 3
L_Q, L_QA, L_K, L_KA, L_V, L_VA, L_O, L_OA = 4, 5, 6, 7, 8, 9, 10, 11
L_ROUTER, L_UP, L_UPA, L_GATE, L_GATEA, L_DOWN, L_DOWNA = 12, 13, 14, 15, 16, 17, 18
L_KCACHE, L_VCACHE = 19, 20


def _stream(layer, kind):
    return 1000 + 64 * layer + kind


def _sigs():
    L = O.lib()
    u64, i64, dbl, flt, i = ctypes.c_uint64, ctypes.c_int64, ctypes.c_double, ctypes.c_float, ctypes.c_int
    u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
    f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
    i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
    L.orc_synth_ternary.argtypes = [u64, u64, i64, u32p]
    L.orc_synth_normal.argtypes = [u64, u64, i64, dbl, flt, i, i, f32p]
    L.orc_synth_rtn4_sym.argtypes = [u64, u64, i64, i64, i64, dbl, u32p, f32p]
    L.orc_synth_tokens.argtypes = [u64, u64, i64, i64, i64p]
    for f in (L.orc_synth_ternary, L.orc_synth_normal, L.orc_synth_rtn4_sym, L.orc_synth_tokens):
        f.restype = None
    return L


def synth_ternary(seed, stream, shape):
    out = np.empty(shape, np.uint32)
    _sigs().orc_synth_ternary(seed, stream, out.size, out)
    return out


def synth_normal(seed, stream, shape, scale, offset=0.0, use_abs=False, bf16=True):
    out = np.empty(shape, np.float32)
    _sigs().orc_synth_normal(seed, stream, out.size, float(scale), float(offset), int(use_abs), int(bf16), out)
    return out


def synth_rtn4_sym(seed, stream, rows, k, group, scale):
    codes = np.empty((rows, k // 8), np.uint32)
    scales = np.empty((rows, k // group), np.float32)
    _sigs().orc_synth_rtn4_sym(seed, stream, rows, k, group, float(scale), codes, scales)
    return codes, scales


def synth_tokens(seed, n, vocab, stream=S_PROMPT):
    out = np.empty(n, np.int64)
    _sigs().orc_synth_tokens(seed, stream, n, vocab, out)
    return out


def rope_tables(head_dim, partial, theta, n):
    """Reference model.py:67-92 (fp32, torch on the CPU), rounded to bf16."""
    import torch

    rot = int(head_dim * partial)
    inv_freq = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    t = torch.arange(n, dtype=torch.float32)
    emb = torch.cat((torch.outer(t, inv_freq),) * 2, dim=-1)
    cos = emb.cos().to(torch.bfloat16).float().numpy()
    sin = emb.sin().to(torch.bfloat16).float().numpy()
    return np.ascontiguousarray(cos), np.ascontiguousarray(sin)


class OracleModel:
    """Synthetic model of ``config`` (the engine's synthetic_config) held on the host."""

    def _setup(self, config: dict, max_len: int, split_len: int) -> None:
        c = config
        self.c = c
        self.L, self.H, self.V = c["num_hidden_layers"], c["hidden_size"], c["vocab_size"]
        self.Hq, self.Hkv, self.D = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        self.E, self.topk, self.I = c["num_experts"], c["num_experts_per_tok"], c["moe_intermediate_size"]
        self.eps = float(c["rms_norm_eps"])
        self.group = c["maple_run"]["rtn_4bit"]["group_size"]
        self.T, self.P = max_len, split_len
        self.scale = np.float32(self.D ** -0.5)
        self.cos, self.sin = rope_tables(self.D, float(c.get("partial_rotary_factor", 0.5)), float(c["rope_theta"]),
                                         max(self.T, 64))
        self.emb_rtn = None
        self.head_biases = None
        self.pos = 0

    def _layer_attention(self, i: int) -> dict:
        """Per-layer attention knobs (reference model.py:800-812): RoPE off on
        global layers when ``nope_on_global_attention``; sliding layers attend
        to the last ``sliding_window`` positions."""
        c = self.c
        kind = list(c["layer_types"])[i]
        nope = bool(c.get("nope_on_global_attention", True)) and kind == "full_attention"
        window = int(c.get("sliding_window", 512)) if kind == "sliding_attention" else 0
        return {"use_rope": not nope, "window": window,
                "kc": np.zeros((1, self.Hkv, self.T, self.D), np.float32),
                "vc": np.zeros((1, self.Hkv, self.T, self.D), np.float32)}

    def __init__(self, config: dict, seed: int, max_len: int, split_len: int):
        self._setup(config, max_len, split_len)
        H, D, E, I = self.H, self.D, self.E, self.I
        self.emb = synth_normal(seed, S_EMB, (self.V, H), 0.02)
        self.head_codes, self.head_scales = synth_rtn4_sym(seed, S_HEAD, self.V, H, self.group, 0.02)
        self.final_norm = synth_normal(seed, S_NORM, (H,), 0.02, 1.0, bf16=False)
        self.layers = []
        for i in range(self.L):
            s = lambda kind: _stream(i, kind)  # noqa: E731
            lay = {
                "in_ln": synth_normal(seed, s(L_IN_LN), (H,), 0.02, 1.0, bf16=False),
                "post_ln": synth_normal(seed, s(L_POST_LN), (H,), 0.02, 1.0, bf16=False),
                "q_norm": synth_normal(seed, s(L_Q_NORM), (D,), 0.02, 1.0, bf16=False),
                "k_norm": synth_normal(seed, s(L_K_NORM), (D,), 0.02, 1.0, bf16=False),
                "router": synth_normal(seed, s(L_ROUTER), (E, H), 0.02),
            }
            qkv = [synth_ternary(seed, s(L_Q), (self.Hq * D, H // 16)),
                   synth_ternary(seed, s(L_K), (self.Hkv * D, H // 16)),
                   synth_ternary(seed, s(L_V), (self.Hkv * D, H // 16))]
            qkv_a = [synth_normal(seed, s(L_QA), (self.Hq * D,), 0.02, 1e-3, True),
                     synth_normal(seed, s(L_KA), (self.Hkv * D,), 0.02, 1e-3, True),
                     synth_normal(seed, s(L_VA), (self.Hkv * D,), 0.02, 1e-3, True)]
            lay["qkv"] = np.ascontiguousarray(np.concatenate(qkv, 0))
            lay["qkv_a"] = np.ascontiguousarray(np.concatenate(qkv_a, 0))
            lay["o"] = synth_ternary(seed, s(L_O), (H, self.Hq * D // 16))
            lay["o_a"] = synth_normal(seed, s(L_OA), (H,), 0.02, 1e-3, True)
            up = synth_ternary(seed, s(L_UP), (E, I, H // 16))
            gate = synth_ternary(seed, s(L_GATE), (E, I, H // 16))
            lay["ug"] = np.ascontiguousarray(np.concatenate([up, gate], 1))
            lay["ug_a"] = np.ascontiguousarray(np.concatenate(
                [synth_normal(seed, s(L_UPA), (E, I), 0.02, 1e-3, True),
                 synth_normal(seed, s(L_GATEA), (E, I), 0.02, 1e-3, True)], 1))
            lay["down"] = synth_ternary(seed, s(L_DOWN), (E, H, I // 16))
            lay["down_a"] = synth_normal(seed, s(L_DOWNA), (E, H), 0.02, 1e-3, True)
            lay.update(self._layer_attention(i))
            self.layers.append(lay)

    @classmethod
    def from_weights(cls, config: dict, weights: dict, max_len: int, split_len: int) -> "OracleModel":
        """A converted packed-ternary-v1 checkpoint (tensor names of the
        reference's convert.py:180-303), as the reference loader holds it
        (model.py:719-832): router and RTN scales/biases in bf16, row_alpha
        and norm weights in fp32, QKV rows and [up; gate] rows concatenated."""
        m = cls.__new__(cls)
        m._setup(config, max_len, split_len)
        w = {k: np.asarray(v) for k, v in weights.items()}
        f32 = lambda k: np.ascontiguousarray(w[k], np.float32)  # noqa: E731
        b16 = lambda k: O.round_bf16(f32(k))  # noqa: E731
        u32 = lambda k: np.ascontiguousarray(w[k]).view(np.uint32)  # noqa: E731
        if "model.word_embeddings.scales" in w:
            m.emb = None
            m.emb_rtn = (u32("model.word_embeddings.weight"), b16("model.word_embeddings.scales"),
                         b16("model.word_embeddings.biases") if "model.word_embeddings.biases" in w else None)
        else:
            m.emb = b16("model.word_embeddings.weight")
        m.head_codes, m.head_scales = u32("lm_head.weight"), b16("lm_head.scales")
        m.head_biases = b16("lm_head.biases") if "lm_head.biases" in w else None
        m.final_norm = f32("model.norm.weight")
        m.layers = []
        for i in range(m.L):
            p = f"model.layers.{i}"
            lay = {
                "in_ln": f32(f"{p}.input_layernorm.weight"),
                "post_ln": f32(f"{p}.post_attention_layernorm.weight"),
                "q_norm": f32(f"{p}.self_attn.q_norm.weight"),
                "k_norm": f32(f"{p}.self_attn.k_norm.weight"),
                "router": b16(f"{p}.mlp.gate.weight"),
                "qkv": np.ascontiguousarray(np.concatenate([u32(f"{p}.self_attn.{n}_proj.weight") for n in "qkv"])),
                "qkv_a": np.concatenate([f32(f"{p}.self_attn.{n}_proj.row_alpha") for n in "qkv"]),
                "o": u32(f"{p}.self_attn.o_proj.weight"),
                "o_a": f32(f"{p}.self_attn.o_proj.row_alpha"),
                "ug": np.ascontiguousarray(np.concatenate([u32(f"{p}.mlp.switch_mlp.up_proj.weight"),
                                                           u32(f"{p}.mlp.switch_mlp.gate_proj.weight")], 1)),
                "ug_a": np.ascontiguousarray(np.concatenate([f32(f"{p}.mlp.switch_mlp.up_proj.row_alpha"),
                                                             f32(f"{p}.mlp.switch_mlp.gate_proj.row_alpha")], 1)),
                "down": u32(f"{p}.mlp.switch_mlp.down_proj.weight"),
                "down_a": f32(f"{p}.mlp.switch_mlp.down_proj.row_alpha"),
            }
            lay.update(m._layer_attention(i))
            m.layers.append(lay)
        return m

    def fill_cache(self, seed: int, length: int) -> None:
        """Random cached context: positions [0, length) of K/V bf16 N(0, 1)."""
        for i, lay in enumerate(self.layers):
            for kind, key in ((L_KCACHE, "kc"), (L_VCACHE, "vc")):
                lay[key][:, :, :length] = synth_normal(seed, _stream(i, kind), (1, self.Hkv, length, self.D), 1.0)
        self.pos = length

    def step(self, token: int, want_logits: bool = False):
        """One decode step at position ``self.pos``; returns the greedy next id
        (and the bf16 logits when asked)."""
        pos = np.array([self.pos], np.int64)
        cs_row = min(self.pos, self.cos.shape[0] - 1)
        cos, sin = self.cos[cs_row:cs_row + 1], self.sin[cs_row:cs_row + 1]
        if self.emb_rtn is not None:
            codes, sc, bi = self.emb_rtn
            h = O.rtn4_embedding(np.array([token]), codes, sc, bi, self.group)
        else:
            h = self.emb[token:token + 1]
        for lay in self.layers:
            qkv = O.ternary_gemv(h, lay["qkv"], lay["qkv_a"], lay["in_ln"], self.eps)
            q = O.apply_qkv_decode(qkv, lay["q_norm"], lay["k_norm"], cos, sin, lay["kc"], lay["vc"], pos,
                                   num_heads=self.Hq, num_kv_heads=self.Hkv, head_dim=self.D,
                                   use_rope=lay["use_rope"], eps=self.eps)
            attn = O.decode_gqa(q, lay["kc"], lay["vc"], pos, scale=self.scale, window=lay["window"],
                                split_len=self.P)
            o = O.ternary_gemv(attn.reshape(1, -1), lay["o"], lay["o_a"])
            res, normed = O.add_rms_norm(h, o, lay["post_ln"], self.eps)
            idx, wt = O.router_topk(normed, lay["router"], self.topk)
            hs = O.expert_swiglu(normed, lay["ug"], lay["ug_a"], idx)
            h = O.expert_down_reduce(hs, lay["down"], lay["down_a"], idx, wt, res, mode=0)
        self.pos += 1
        normed = O.rms_norm(h, self.final_norm, self.eps)
        logits = O.rtn4_gemv(normed, self.head_codes, self.head_scales, self.head_biases, self.group)
        nxt = int(O.argmax(logits)[0])
        return (nxt, logits[0]) if want_logits else nxt

    def greedy(self, prompt, n_new: int, log_every: int = 0):
        """Feed ``prompt`` token by token, then decode ``n_new`` greedy ids."""
        t0 = time.time()
        nxt = None
        for i, tok in enumerate(prompt):
            nxt = self.step(int(tok))
            if log_every and (i + 1) % log_every == 0:
                print(f"  oracle prefill {i + 1}/{len(prompt)} ({time.time() - t0:.0f}s)", flush=True)
        out = []
        for i in range(n_new):
            out.append(nxt)
            if i + 1 < n_new:
                nxt = self.step(nxt)
        return out
