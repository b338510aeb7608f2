"""Seeded test cases shared by the golden-vector generator and the tests.

``inputs()`` regenerates a case's inputs with numpy's frozen ``RandomState``
stream (so fixtures store outputs only); ``run_reference(torch)`` runs the
reference's own code on them (see make_golden.py).  Activations, caches and
scales are drawn as bf16-representable fp32 values, so the same numbers are
what the CUDA path reads from its bf16 tensors; the reference runs in fp32
(its IEEE paths), the precision where the Triton interpreter is exact.

Every ``kind`` names the reference entry point it pins (paths relative to
``src/maple_run/`` of the reference):

* ``ternary_gemv``    kernels/ternary_gemv.py:261-388
* ``router``          kernels/router.py:141-217
* ``norms``           kernels/fused_norm.py:105-202 (rms_norm, add_rms_norm, moe_reduce_add)
* ``experts``         kernels/ternary_expert.py:125-234, :403-556
* ``attention``       kernels/decode_attn.py:362-592 (apply_qkv_decode + decode_gqa_attn)
* ``rtn4``            kernels/rtn4.py:285-415 (rtn4_gemv), :514-611 (rtn4_indexed_gemv)
* ``sampler``         kernels/sampler.py:106-206 (fused_sample, fused_sample_batched)
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


def pack2(codes: np.ndarray) -> np.ndarray:
    *lead, k = codes.shape
    c = codes.astype(np.uint64).reshape(*lead, k // 16, 16)
    return np.bitwise_or.reduce(c << np.arange(0, 32, 2, dtype=np.uint64), axis=-1).astype(np.uint32)


def pack4(codes: np.ndarray) -> np.ndarray:
    *lead, k = codes.shape
    c = codes.astype(np.uint64).reshape(*lead, k // 8, 8)
    return np.bitwise_or.reduce(c << np.arange(0, 32, 4, dtype=np.uint64), axis=-1).astype(np.uint32)


def ternary_codes(rs: np.random.RandomState, shape) -> np.ndarray:
    """Codes t+1 with P(t=0)=0.4, P(t=-1)=P(t=+1)=0.3."""
    u = rs.random_sample(shape)
    t = np.where(u < 0.4, 0, np.where(u < 0.7, -1, 1))
    return (t + 1).astype(np.uint32)


def _alpha(rs, shape, scale=0.02):
    return bf16_round((np.abs(rs.standard_normal(shape) * scale) + 1e-3).astype(np.float32))


def _normal(rs, shape, scale=1.0, offset=0.0):
    return bf16_round((offset + scale * rs.standard_normal(shape)).astype(np.float32))


def _u32(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a).astype(np.int64)).to(torch.uint32)


def rope_rows(positions, rotary_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin rows of the reference rotary table (model.py:64-113: inv_freq =
    theta^(-2i/rot), angles duplicated over both halves, fp32) at the given
    positions, rounded to bf16 as the model holds them."""
    i = np.arange(0, rotary_dim, 2, dtype=np.float32)
    inv = (1.0 / (np.float32(theta) ** (i / np.float32(rotary_dim)))).astype(np.float32)
    ang = np.asarray(positions, np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([ang, ang], axis=-1).astype(np.float32)
    return bf16_round(np.cos(emb)), bf16_round(np.sin(emb))


@dataclass
class GemvCase:
    seed: int
    batch: int
    n: int
    k: int
    rms: bool
    bf16_inputs: bool = False
    kind: str = "ternary_gemv"
    extra: dict = field(default_factory=dict)

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        codes = ternary_codes(rs, (self.n, self.k))
        alpha = (np.abs(rs.standard_normal(self.n) * 0.02) + 1e-3).astype(np.float32)
        x = rs.standard_normal((self.batch, self.k)).astype(np.float32)
        w = (1.0 + 0.02 * rs.standard_normal(self.k)).astype(np.float32) if self.rms else None
        if self.bf16_inputs:
            alpha, x = bf16_round(alpha), bf16_round(x)
        return dict(packed=pack2(codes), alpha=alpha, x=x, rms_weight=w)

    def run_reference(self, torch):
        from maple_run.kernels.ternary_gemv import ternary_gemv

        d = self.inputs()
        packed = torch.from_numpy(d["packed"].astype(np.int64)).to(torch.uint32)
        y = ternary_gemv(
            torch.from_numpy(d["x"]),
            packed,
            torch.from_numpy(d["alpha"]),
            rms_weight=None if d["rms_weight"] is None else torch.from_numpy(d["rms_weight"]),
            rms_eps=1e-6,
        )
        return {"y": y.numpy()}


@dataclass
class RouterCase:
    """x [T, K] ~ N(0,1), gate [E, K] ~ N(0, 0.02) in bf16 values.  ``ties``
    copies gate rows so some experts score exactly alike (repeated argmax
    must then take the lower index first)."""

    seed: int
    tokens: int
    k: int = 2048
    n_exp: int = 64
    top_k: int = 8
    ties: bool = False
    kind: str = "router"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        x = _normal(rs, (self.tokens, self.k))
        gate = _normal(rs, (self.n_exp, self.k), 0.02)
        if self.ties:
            # expert 9 duplicates 5, 40 duplicates 3, and 17 = 30 = 61
            gate[9], gate[40] = gate[5], gate[3]
            gate[30], gate[61] = gate[17], gate[17]
            # make the duplicated experts score high for every token
            for e in (5, 9, 3, 40, 17, 30, 61):
                gate[e] = bf16_round(gate[e] + 0.02 * np.sign(x.sum(0)) * 0.25)
        return dict(x=x, gate=gate)

    def run_reference(self, torch):
        from maple_run.kernels.router import router_topk

        d = self.inputs()
        idx, wt = router_topk(torch.from_numpy(d["x"]), torch.from_numpy(d["gate"]), self.top_k)
        return {"idx": idx.numpy(), "wt": wt.numpy()}


@dataclass
class NormCase:
    """rms_norm, add_rms_norm and moe_reduce_add on bf16-valued rows."""

    seed: int
    rows: int
    n: int = 2048
    top_k: int = 8
    kind: str = "norms"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        x = _normal(rs, (self.rows, self.n))
        y = _normal(rs, (self.rows, self.n), 0.5)
        w = (1.0 + 0.02 * rs.standard_normal(self.n)).astype(np.float32)
        slots = _normal(rs, (self.rows, self.top_k, self.n), 0.3)
        p = np.abs(rs.standard_normal((self.rows, self.top_k))).astype(np.float32) + 0.05
        wt = (p / p.sum(-1, keepdims=True)).astype(np.float32)
        return dict(x=x, y=y, w=w, slots=slots, wt=wt)

    def run_reference(self, torch):
        from maple_run.kernels.fused_norm import add_rms_norm, moe_reduce_add, rms_norm

        d = {k: torch.from_numpy(v) for k, v in self.inputs().items()}
        rn = rms_norm(d["x"], d["w"], 1e-6)
        res, nrm = add_rms_norm(d["x"], d["y"], d["w"], 1e-6)
        red = moe_reduce_add(d["slots"], d["wt"], residual=d["x"])
        red0 = moe_reduce_add(d["slots"], d["wt"])
        return {"rms": rn.numpy(), "residual": res.numpy(), "normed": nrm.numpy(), "reduce": red.numpy(),
                "reduce_nores": red0.numpy()}


@dataclass
class ExpertCase:
    """Expert SwiGLU (rows [up; gate]), down projection per slot, the fused
    down + weighted sum + residual, on ``tokens`` tokens routed to ``top_k``
    distinct experts each.  ``alpha_scale`` large enough drives the SwiGLU
    clamps (|up| <= 7, gate <= 7)."""

    seed: int
    tokens: int
    k: int = 2048
    n_exp: int = 8
    inter: int = 256
    top_k: int = 4
    alpha_scale: float = 0.02
    kind: str = "experts"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        x = _normal(rs, (self.tokens, self.k))
        ug = pack2(ternary_codes(rs, (self.n_exp, 2 * self.inter, self.k)))
        ug_a = _alpha(rs, (self.n_exp, 2 * self.inter), self.alpha_scale)
        down = pack2(ternary_codes(rs, (self.n_exp, self.k, self.inter)))
        down_a = _alpha(rs, (self.n_exp, self.k))
        ids = np.stack([rs.permutation(self.n_exp)[: self.top_k] for _ in range(self.tokens)]).astype(np.int32)
        p = np.abs(rs.standard_normal((self.tokens, self.top_k))).astype(np.float32) + 0.05
        wt = (p / p.sum(-1, keepdims=True)).astype(np.float32)
        h_in = _normal(rs, (self.tokens, self.top_k, self.inter), 0.5)
        residual = _normal(rs, (self.tokens, self.k))
        return dict(x=x, ug=ug, ug_a=ug_a, down=down, down_a=down_a, ids=ids, wt=wt, h_in=h_in, residual=residual)

    def run_reference(self, torch):
        from maple_run.kernels.ternary_expert import (
            ternary_expert_down_sum,
            ternary_expert_gemv,
            ternary_expert_swiglu,
        )

        d = self.inputs()
        t = {k: (_u32(torch, v) if v.dtype == np.uint32 else torch.from_numpy(v)) for k, v in d.items()}
        h = ternary_expert_swiglu(t["x"], t["ug"], t["ug_a"], t["ids"])
        y = ternary_expert_gemv(t["h_in"], t["down"], t["down_a"], t["ids"])
        out = ternary_expert_down_sum(t["h_in"], t["down"], t["down_a"], t["ids"], t["wt"], residual=t["residual"])
        return {"h": h.numpy(), "down": y.numpy(), "down_sum": out.numpy()}


@dataclass
class AttentionCase:
    """apply_qkv_decode (QK RMSNorm, RoPE on the first ``rotary_dim`` dims,
    K/V store at ``seqlen``) followed by decode_gqa_attn, on fp32 caches
    holding bf16 values, rows at ragged lengths (the reference's own ragged
    set, tests/test_fused_decode.py:245-291), optionally through a row map
    and a sliding window."""

    seed: int
    lengths: tuple
    max_len: int = 1024
    hq: int = 8
    hkv: int = 2
    d: int = 128
    rotary_dim: int = 128
    use_rope: bool = True
    window: int = 0
    row_map: tuple | None = None
    theta: float = 1e6
    kind: str = "attention"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        B = len(self.lengths)
        Bc = B if self.row_map is None else max(self.row_map) + 1
        qkv = _normal(rs, (B, (self.hq + 2 * self.hkv) * self.d))
        qw = (1.0 + 0.02 * rs.standard_normal(self.d)).astype(np.float32)
        kw = (1.0 + 0.02 * rs.standard_normal(self.d)).astype(np.float32)
        kc = _normal(rs, (Bc, self.hkv, self.max_len, self.d))
        vc = _normal(rs, (Bc, self.hkv, self.max_len, self.d))
        seqlen = np.asarray(self.lengths, np.int64) - 1
        cos, sin = rope_rows(seqlen, self.rotary_dim, self.theta)
        rm = None if self.row_map is None else np.asarray(self.row_map, np.int32)
        return dict(qkv=qkv, qw=qw, kw=kw, kc=kc, vc=vc, seqlen=seqlen, cos=cos, sin=sin, row_map=rm)

    def run_reference(self, torch):
        from maple_run.kernels.decode_attn import apply_qkv_decode, decode_gqa_attn

        d = self.inputs()
        kc, vc = torch.from_numpy(d["kc"].copy()), torch.from_numpy(d["vc"].copy())
        seqlen = torch.from_numpy(d["seqlen"])
        rm = None if d["row_map"] is None else torch.from_numpy(d["row_map"])
        q = apply_qkv_decode(torch.from_numpy(d["qkv"]), torch.from_numpy(d["qw"]), torch.from_numpy(d["kw"]),
                             torch.from_numpy(d["cos"]), torch.from_numpy(d["sin"]), kc, vc, seqlen, row_map=rm,
                             num_heads=self.hq, num_kv_heads=self.hkv, head_dim=self.d, rotary_dim=self.rotary_dim,
                             use_rope=self.use_rope, use_qk_norm=True, eps=1e-6)
        out = decode_gqa_attn(q, kc, vc, seqlen, row_map=rm, scale=self.d ** -0.5,
                              window=self.window or None)
        rows = np.arange(len(self.lengths)) if d["row_map"] is None else d["row_map"]
        pos = d["seqlen"]
        k_new = kc.numpy()[rows, :, pos, :]
        v_new = vc.numpy()[rows, :, pos, :]
        return {"q": q.numpy()[:, :, 0, :], "k_new": k_new, "v_new": v_new, "out": out.numpy()[:, :, 0, :]}


@dataclass
class Rtn4Case:
    """4-bit RTN GEMV/GEMM (rtn4_gemv) and, with ``n_clusters``, the FlashHead
    cluster-indexed GEMV (rtn4_indexed_gemv).  ``symmetric`` is the configs'
    g128 symmetric head expressed to the reference kernel as bias = -8*s."""

    seed: int
    batch: int
    n: int = 512
    k: int = 2048
    group: int = 128
    symmetric: bool = True
    n_clusters: int = 0
    cluster_size: int = 32
    n_probes: int = 0
    kind: str = "rtn4"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        rows = self.n_clusters * self.cluster_size if self.n_clusters else self.n
        codes = rs.randint(0, 16, size=(rows, self.k)).astype(np.uint32)
        ng = self.k // self.group
        s = _alpha(rs, (rows, ng), 0.004)
        b = bf16_round(-8.0 * s) if self.symmetric else _normal(rs, (rows, ng), 0.03)
        x = _normal(rs, (self.batch, self.k))
        cids = (np.sort(rs.permutation(self.n_clusters)[: self.n_probes]).astype(np.int64)
                if self.n_clusters else None)
        return dict(packed=pack4(codes), s=s, b=b, x=x, cids=cids)

    def run_reference(self, torch):
        from maple_run.kernels.rtn4 import rtn4_gemv, rtn4_indexed_gemv

        d = self.inputs()
        x, s, b = torch.from_numpy(d["x"]), torch.from_numpy(d["s"]), torch.from_numpy(d["b"])
        if not self.n_clusters:
            return {"y": rtn4_gemv(x, _u32(torch, d["packed"]), s, b, self.group).numpy()}
        C, S = self.n_clusters, self.cluster_size
        packed = _u32(torch, d["packed"].reshape(C, S, -1))
        y = rtn4_indexed_gemv(x, packed, s.reshape(C, S, -1), b.reshape(C, S, -1), torch.from_numpy(d["cids"]),
                              self.group)
        return {"y": y.numpy()}


@dataclass
class SamplerCase:
    """fused_sample / fused_sample_batched at fixed uniforms (the reference
    test's CDF-inversion check, tests/test_fused_sampler.py:26-48)."""

    seed: int
    batch: int
    vocab: int
    temperature: float
    top_p: float
    top_k: int
    uniforms: tuple = (0.0, 0.25, 0.5, 0.75, 0.999)
    kind: str = "sampler"

    def inputs(self):
        rs = np.random.RandomState(self.seed)
        logits = (rs.standard_normal((self.batch, self.vocab)) * 3.0).astype(np.float32)
        return dict(logits=logits, u=np.asarray(self.uniforms, np.float32))

    def run_reference(self, torch):
        from maple_run.kernels.sampler import fused_sample, fused_sample_batched

        d = self.inputs()
        logits = torch.from_numpy(d["logits"])
        kw = dict(temperature=self.temperature, top_p=self.top_p, top_k=self.top_k)
        single = np.array([[int(fused_sample(logits[b], torch.tensor(float(u)), **kw)) for u in d["u"]]
                           for b in range(self.batch)], np.int64)
        batched = np.stack([fused_sample_batched(logits, torch.full((self.batch,), float(u)), **kw).numpy()
                            for u in d["u"]], axis=1)
        return {"single": single, "batched": batched}


_RAGGED = (1, 63, 64, 65, 300, 511, 1000)

CASES = {
    "gemv_small": GemvCase(seed=10, batch=1, n=64, k=256, rms=False),
    "gemv_rms": GemvCase(seed=11, batch=1, n=96, k=512, rms=True),
    "gemv_batch": GemvCase(seed=12, batch=3, n=48, k=128, rms=True),
    "gemv_cfg0": GemvCase(seed=0, batch=1, n=4096, k=2048, rms=False, bf16_inputs=True),
    "router_b1": RouterCase(seed=20, tokens=1),
    "router_b5": RouterCase(seed=21, tokens=5),
    "router_ties": RouterCase(seed=22, tokens=3, ties=True),
    "norms": NormCase(seed=30, rows=3),
    "experts_b1": ExpertCase(seed=40, tokens=1),
    "experts_b3": ExpertCase(seed=41, tokens=3, top_k=3),
    "experts_clamp": ExpertCase(seed=42, tokens=2, alpha_scale=0.4),
    "attn_ragged": AttentionCase(seed=50, lengths=_RAGGED),
    "attn_partial_rope": AttentionCase(seed=51, lengths=(5, 130, 700), rotary_dim=64, theta=1e4),
    "attn_nope_window": AttentionCase(seed=52, lengths=(3, 40, 300), use_rope=False, window=32, max_len=512),
    "attn_row_map": AttentionCase(seed=53, lengths=(17, 200, 90), row_map=(2, 0, 1), max_len=256),
    "rtn4_b1_sym": Rtn4Case(seed=60, batch=1),
    "rtn4_b3_sym": Rtn4Case(seed=61, batch=3),
    "rtn4_b1_affine64": Rtn4Case(seed=62, batch=1, group=64, symmetric=False),
    "rtn4_indexed": Rtn4Case(seed=63, batch=1, n_clusters=24, n_probes=6),
    "sampler_k20": SamplerCase(seed=70, batch=3, vocab=9000, temperature=0.8, top_p=0.95, top_k=20),
    "sampler_k64_p1": SamplerCase(seed=71, batch=2, vocab=5000, temperature=1.0, top_p=1.0, top_k=64),
    "sampler_k2": SamplerCase(seed=72, batch=2, vocab=4096, temperature=0.7, top_p=0.95, top_k=2),
}
