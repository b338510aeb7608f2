"""CPU oracle for the maple-b200 decode path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as the checker (or the timed CPU
baseline); the product path never does.

It restates the reference (cloud-000/maple-flash-dgx-spark, paths relative to
``src/maple_run/``) on the CPU:

* NumPy restatements of the packing format (``pack.py``), bit-exact;
* a C library (``oracle.c``, built by ``oracle/build.py``) for the arithmetic
  operators, following the reference's rounding points and the canonical
  numerics of the CUDA kernels so that GPU results compare bit for bit.

Parity pins: ``tests/test_oracle_pins.py`` checks these functions against the
reference's own known-answer tests (restated) and against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's code in
this container (Triton interpreter, fp32).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# ----------------------------------------------------------------- packing --
# Reference: pack.py:18-21 (16 two-bit codes per uint32, 8 four-bit codes, LSB first)
_SHIFTS_2 = np.arange(0, 32, 2, dtype=np.uint64)
_SHIFTS_4 = np.arange(0, 32, 4, dtype=np.uint64)
DEFAULT_THRESHOLD_SCALE = 0.7          # pack.py:13
TERNARY_GROUP = 128                    # pack.py:14
HEAD_GROUP_SIZE = 64                   # pack.py:15


def pack_2bit(codes: np.ndarray) -> np.ndarray:
    """Reference pack.py:23-38. Last axis K (multiple of 16) -> K/16 uint32."""
    *lead, k = codes.shape
    if k % 16:
        raise ValueError(f"2-bit packing requires the last axis to be a multiple of 16; got {k}.")
    c = codes.astype(np.uint64).reshape(*lead, k // 16, 16)
    # the shifted fields are summed in 64 bits and narrowed (codes > 3 carry)
    return np.sum(c << _SHIFTS_2, axis=-1, dtype=np.uint64).astype(np.uint32)


def unpack_2bit(packed: np.ndarray) -> np.ndarray:
    """Reference pack.py:41-45."""
    p = packed.astype(np.uint64)
    codes = (p[..., None] >> _SHIFTS_2) & np.uint64(3)
    return codes.reshape(*packed.shape[:-1], packed.shape[-1] * 16).astype(np.uint32)


def pack_4bit(codes: np.ndarray) -> np.ndarray:
    """Reference pack.py:48-57."""
    *lead, k = codes.shape
    if k % 8:
        raise ValueError(f"4-bit packing requires the last axis to be a multiple of 8; got {k}.")
    c = codes.astype(np.uint64).reshape(*lead, k // 8, 8)
    return np.sum(c << _SHIFTS_4, axis=-1, dtype=np.uint64).astype(np.uint32)


def unpack_4bit(packed: np.ndarray) -> np.ndarray:
    """Reference pack.py:60-64."""
    p = packed.astype(np.uint64)
    codes = (p[..., None] >> _SHIFTS_4) & np.uint64(0xF)
    return codes.reshape(*packed.shape[:-1], packed.shape[-1] * 8).astype(np.uint32)


def ternarize(weight: np.ndarray, threshold_scale: float = DEFAULT_THRESHOLD_SCALE):
    """Reference pack.py:120-149: threshold 0.7*mean|w| per row, alpha = mean|w|
    of the survivors (fp32 math, alpha cast to the weight dtype), codes t+1."""
    if weight.shape[-1] % TERNARY_GROUP:
        raise ValueError(
            f"Ternary conversion requires the reduction dim to be a multiple of {TERNARY_GROUP}; "
            f"got {weight.shape[-1]}.")
    w = weight.astype(np.float32)
    aw = np.abs(w)
    thr = np.float32(threshold_scale) * np.mean(aw, axis=-1, keepdims=True, dtype=np.float32)
    mask = (aw > thr).astype(np.float32)
    num = np.sum(aw * mask, axis=-1, keepdims=True, dtype=np.float32)
    den = np.maximum(np.sum(mask, axis=-1, keepdims=True, dtype=np.float32), np.float32(1))
    alpha = (num / den).astype(weight.dtype)[..., 0]
    ternary = np.sign(w) * mask
    return pack_2bit((ternary + 1).astype(np.uint32)), alpha


def quantize_rtn(weight: np.ndarray, group_size: int = HEAD_GROUP_SIZE):
    """Reference pack.py:67-100: affine 4-bit RTN, dequant = code*scale + bias."""
    k = weight.shape[-1]
    if k % group_size:
        raise ValueError(f"RTN conversion requires the last axis to be a multiple of {group_size}; got {k}.")
    w = weight.astype(np.float32)
    lead = w.shape[:-1]
    g = w.reshape(*lead, k // group_size, group_size)
    wmin = g.min(axis=-1, keepdims=True)
    wmax = g.max(axis=-1, keepdims=True)
    scale = (wmax - wmin) / np.float32(15)
    zero = scale == 0
    safe = np.where(zero, np.float32(1), scale)
    q = np.clip(np.rint((g - wmin) / safe), 0, 15)
    q = np.where(zero, 0, q)
    return (pack_4bit(q.reshape(*lead, k).astype(np.uint32)), scale[..., 0].astype(np.float32),
            wmin[..., 0].astype(np.float32))


def dequantize_rtn(packed, scales, biases, group_size: int = HEAD_GROUP_SIZE):
    """Reference pack.py:103-117."""
    codes = unpack_4bit(packed).astype(np.float32)
    k = codes.shape[-1]
    g = codes.reshape(*codes.shape[:-1], k // group_size, group_size)
    return (g * scales[..., None] + biases[..., None]).reshape(codes.shape)


# ------------------------------------------------------------------- bf16 --
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern, round-to-nearest-even, NaN -> 0x7FC0."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), r)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


# ------------------------------------------------------------- C library --
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_flt = ctypes.c_float

_SIGS = {
    "orc_exp": (_flt, [_flt]),
    "orc_r128_sum": (_flt, [_f32p, _i64]),
    "orc_r128_sumsq": (_flt, [_f32p, _i64]),
    "orc_r128_dot": (_flt, [_f32p, _f32p, _i64]),
    "orc_ternary_gemv": (None, [_f32p, _i64, _i64, _u32p, _i64, _f32p, _vp, _flt, _int, _f32p]),
    "orc_rms_norm": (None, [_f32p, _i64, _i64, _f32p, _flt, _int, _f32p]),
    "orc_add_rms_norm": (None, [_f32p, _f32p, _i64, _i64, _f32p, _flt, _int, _f32p, _f32p]),
    "orc_router_topk": (None, [_f32p, _i64, _i64, _f32p, _i64, _i64, _i32p, _f32p]),
    "orc_expert_gemv": (None, [_f32p, _i64, _i32p, _i64, _i64, _u32p, _i64, _i64, _f32p, _int, _f32p]),
    "orc_expert_swiglu": (None, [_f32p, _i64, _i64, _i64, _u32p, _i64, _i64, _f32p, _i32p, _int, _f32p]),
    "orc_expert_down_reduce": (None, [_f32p, _i64, _i64, _i64, _i32p, _f32p, _u32p, _i64, _i64, _f32p, _vp,
                                      _int, _int, _f32p]),
    "orc_moe_reduce_add": (None, [_f32p, _f32p, _vp, _i64, _i64, _i64, _int, _f32p]),
    "orc_apply_qkv_decode": (None, [_f32p, _i64, _f32p, _f32p, _f32p, _f32p, _i64, _f32p, _f32p, _f32p, _i64,
                                    _i64, _i64p, _vp, _i64, _i64, _i64, _int, _flt, _int]),
    "orc_decode_gqa": (None, [_f32p, _i64, _i64, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64p, _vp, _flt, _i64,
                              _i64, _int, _f32p]),
    "orc_rtn4_gemv": (None, [_f32p, _i64, _i64, _u32p, _i64, _f32p, _vp, _i64, _vp, _int, _f32p]),
    "orc_argmax": (None, [_f32p, _i64, _i64, _i64p]),
    "orc_fused_sample": (None, [_f32p, _i64, _i64, _f32p, _flt, _flt, _i64, _i64p]),
    "orc_rtn4_embedding": (None, [_i64p, _i64, _u32p, _f32p, _vp, _i64, _i64, _i64, _int, _f32p]),
    "orc_km_dots": (None, [_f32p, _i64, _f32p, _i64, _i64, _f32p]),
    "orc_km_normalize": (None, [_f32p, _i64, _i64]),
    "orc_km_update": (None, [_f32p, _i64, _i64, _i32p, _i64, _f32p]),
    "orc_km_objective": (ctypes.c_double, [_f32p, _i64, _i64, _i32p, _f32p]),
}


def lib():
    global _lib
    if _lib is None:
        from oracle.build import build

        L = ctypes.CDLL(str(build()))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _opt(a, dtype=np.float32):
    if a is None:
        return None, None
    arr = np.ascontiguousarray(a, dtype=dtype)
    return arr, arr.ctypes.data_as(ctypes.c_void_p)


def mexp(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    f = lib().orc_exp
    return np.array([f(float(v)) for v in x.reshape(-1)], dtype=np.float32).reshape(x.shape)


def ternary_gemv(x, packed, alpha, rms_weight=None, eps: float = 1e-6, out_bf16: bool = True):
    """Oracle of kernels/ternary_gemv.py:261 ternary_gemv (inputs as fp32 values)."""
    x = _f32(x)
    lead, k = x.shape[:-1], x.shape[-1]
    x2 = x.reshape(-1, k)
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    n = packed.shape[0]
    if packed.shape[1] * 16 != k:
        raise ValueError("x last dim != packed K")
    w, wp = _opt(None if rms_weight is None else np.asarray(rms_weight).reshape(-1))
    y = np.empty((x2.shape[0], n), dtype=np.float32)
    lib().orc_ternary_gemv(x2, x2.shape[0], k, packed, n, _f32(alpha).reshape(-1), wp, float(eps),
                           int(out_bf16), y)
    return y.reshape(*lead, n)


def rms_norm(x, w, eps=1e-6, out_bf16=True):
    x = _f32(x)
    n = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_rms_norm(x.reshape(-1, n), x.size // n, n, _f32(w).reshape(-1), float(eps), int(out_bf16), y)
    return y


def add_rms_norm(x, y, w, eps=1e-6, out_bf16=True):
    x, y = _f32(x), _f32(y)
    n = x.shape[-1]
    res, nrm = np.empty_like(x), np.empty_like(x)
    lib().orc_add_rms_norm(x, y, x.size // n, n, _f32(w).reshape(-1), float(eps), int(out_bf16), res, nrm)
    return res, nrm


def router_topk(x, gate, top_k):
    x, gate = _f32(x), _f32(gate)
    k = x.shape[-1]
    T = x.size // k
    E = gate.shape[0]
    idx = np.empty((T, top_k), np.int32)
    wt = np.empty((T, top_k), np.float32)
    lib().orc_router_topk(x, T, k, gate, E, top_k, idx, wt)
    return idx.reshape(*x.shape[:-1], top_k), wt.reshape(*x.shape[:-1], top_k)


def expert_gemv(x, packed, alpha, ids, x_rows_per_token=1, out_bf16=True):
    x = _f32(x)
    ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
    packed = np.ascontiguousarray(packed, np.uint32)
    E, N, nw = packed.shape
    y = np.empty((ids.size, N), np.float32)
    lib().orc_expert_gemv(x, x_rows_per_token, ids, ids.size, nw * 16, packed, E, N, _f32(alpha), int(out_bf16), y)
    return y


def expert_swiglu(x, packed, alpha, ids, out_bf16=True):
    x = _f32(x)
    ids = np.ascontiguousarray(ids, np.int32)
    T, topk = ids.shape
    packed = np.ascontiguousarray(packed, np.uint32)
    E, rows, nw = packed.shape
    h = np.empty((T, topk, rows // 2), np.float32)
    lib().orc_expert_swiglu(x, T, topk, nw * 16, packed, E, rows // 2, _f32(alpha), ids, int(out_bf16), h)
    return h


def expert_down_reduce(h, packed, alpha, ids, wt, residual=None, mode=0, out_bf16=True):
    h = _f32(h)
    ids = np.ascontiguousarray(ids, np.int32)
    T, topk = ids.shape
    packed = np.ascontiguousarray(packed, np.uint32)
    E, N, nw = packed.shape
    r, rp = _opt(residual)
    out = np.empty((T, N), np.float32)
    lib().orc_expert_down_reduce(h, T, topk, nw * 16, ids, _f32(wt), packed, E, N, _f32(alpha), rp, int(mode),
                                 int(out_bf16), out)
    return out


def moe_reduce_add(x, w, residual=None, out_bf16=True):
    x = _f32(x)
    T, topk, N = x.shape
    r, rp = _opt(residual)
    y = np.empty((T, N), np.float32)
    lib().orc_moe_reduce_add(x, _f32(w), rp, T, topk, N, int(out_bf16), y)
    return y


def apply_qkv_decode(qkv, q_w, k_w, cos, sin, k_cache, v_cache, seqlen, row_map=None, *, num_heads, num_kv_heads,
                     head_dim, use_rope=True, eps=1e-6, out_bf16=True):
    """Returns q [B, H, D]; k_cache/v_cache (fp32 arrays [Bc, Hkv, T, D]) are updated in place."""
    qkv = _f32(qkv)
    B = qkv.shape[0]
    cos, sin = _f32(cos).reshape(B, -1), _f32(sin).reshape(B, -1)
    R = cos.shape[1]
    assert k_cache.dtype == np.float32 and k_cache.flags.c_contiguous
    Bc, Hkv, T, D = k_cache.shape
    q = np.empty((B, num_heads, head_dim), np.float32)
    rm, rmp = _opt(row_map, np.int32)
    lib().orc_apply_qkv_decode(qkv, B, _f32(q_w), _f32(k_w), cos, sin, R, q, k_cache, v_cache, Bc, T,
                               np.ascontiguousarray(seqlen, np.int64), rmp, num_heads, num_kv_heads, head_dim,
                               int(use_rope), float(eps), int(out_bf16))
    return q


def decode_gqa(q, k_cache, v_cache, seqlen, row_map=None, *, scale, window=0, split_len=64, out_bf16=True):
    q = _f32(q)
    B, Hq, D = q.shape
    Bc, Hkv, T, _ = k_cache.shape
    out = np.empty_like(q)
    rm, rmp = _opt(row_map, np.int32)
    lib().orc_decode_gqa(q, B, Hq, _f32(k_cache), _f32(v_cache), Bc, Hkv, T, D,
                         np.ascontiguousarray(seqlen, np.int64), rmp, float(scale), int(window or 0),
                         int(split_len), int(out_bf16), out)
    return out


def rtn4_gemv(x, packed, scales, biases=None, group_size=HEAD_GROUP_SIZE, row_index=None, out_bf16=True):
    x = _f32(x)
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    packed = np.ascontiguousarray(packed, np.uint32).reshape(-1, k // 8)
    scales = _f32(scales).reshape(packed.shape[0], -1)
    b, bp = _opt(None if biases is None else np.asarray(biases).reshape(packed.shape[0], -1))
    ri, rip = _opt(row_index, np.int64)
    n = packed.shape[0] if row_index is None else ri.size
    y = np.empty((x2.shape[0], n), np.float32)
    lib().orc_rtn4_gemv(x2, x2.shape[0], k, packed, n, scales, bp, int(group_size), rip, int(out_bf16), y)
    return y.reshape(*x.shape[:-1], n)


def order_keys(x):
    """float32 -> uint32 keys in the float order, NaN above everything."""
    x = _f32(x)
    u = x.view(np.uint32).astype(np.uint64)
    key = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return np.where(np.isnan(x), np.uint64(0xFFFFFFFF), key)


def topk_select(scores, k):
    """Indices of the k largest scores (ties -> lowest index), ascending; the
    canonical form of flash_head.py:343 torch.topk as a set."""
    keys = order_keys(np.asarray(scores).reshape(-1)).astype(np.int64)
    order = np.lexsort((np.arange(keys.size), -keys))
    return np.sort(order[:k]).astype(np.int32)


def flash_head(hidden, *, centroids_weight, centroids_scales, centroids_biases, centroid_group, token_map,
               head_weight, head_scales, head_biases, group_size, force_ids, force_weight, force_scales,
               force_biases, n_probes, vocab_size):
    """Reference flash_head.py:330-369 (FlashHead.__call__): logits [V] with
    -inf outside the probed clusters' tokens and the forced tokens."""
    hv = _f32(hidden).reshape(-1, _f32(hidden).shape[-1])[-1:]
    scores = rtn4_gemv(hv, centroids_weight, centroids_scales, centroids_biases, centroid_group)[0]
    cids = topk_select(scores, n_probes)
    n_clusters, cs = token_map.shape
    rows = (cids.astype(np.int64)[:, None] * cs + np.arange(cs)).reshape(-1)
    nw = head_weight.shape[-1]
    hb = None if head_biases is None else np.asarray(head_biases).reshape(n_clusters * cs, -1)
    probe = rtn4_gemv(hv, np.asarray(head_weight).reshape(-1, nw), np.asarray(head_scales).reshape(n_clusters * cs, -1),
                      hb, group_size, row_index=rows)[0]
    full = np.full(vocab_size, -np.inf, np.float32)
    full[np.asarray(token_map)[cids].reshape(-1)] = probe
    if len(force_ids):
        full[np.asarray(force_ids)] = rtn4_gemv(hv, force_weight, force_scales, force_biases, group_size)[0]
    return full, cids


def argmax(logits):
    logits = _f32(logits)
    V = logits.shape[-1]
    B = logits.size // V
    out = np.empty(B, np.int64)
    lib().orc_argmax(logits.reshape(B, V), B, V, out)
    return out


def fused_sample(logits, uniform, *, temperature, top_p, top_k):
    logits = _f32(logits)
    V = logits.shape[-1]
    B = logits.size // V
    out = np.empty(B, np.int64)
    lib().orc_fused_sample(logits.reshape(B, V), B, V, _f32(uniform).reshape(-1), float(temperature),
                           float(top_p), int(top_k), out)
    return out


def rtn4_embedding(ids, packed, scales, biases=None, group_size=HEAD_GROUP_SIZE, out_bf16=True):
    ids = np.ascontiguousarray(ids, np.int64).reshape(-1)
    packed = np.ascontiguousarray(packed, np.uint32)
    V, nw = packed.shape
    b, bp = _opt(biases)
    out = np.empty((ids.size, nw * 8), np.float32)
    lib().orc_rtn4_embedding(ids, ids.size, packed, _f32(scales), bp, V, nw * 8, int(group_size),
                             int(out_bf16), out)
    return out
