"""Checkpoint packing on the GPU: 2-/4-bit code packing, ternarize, RTN-4.

Reference: pack.py:23-149 (NumPy on the CPU).  Same function names, argument
meaning and results (bit for bit: the kernels reproduce NumPy's float32
pairwise summation order for the ternarize means); inputs and outputs are CUDA
tensors.  Unpacked codes are returned as uint8 (the reference returns the same
values as uint32).
"""

from __future__ import annotations

import torch

from maple_flash_dgx_spark_b200._lib import check, dtype_code, lib, ptr, require_cuda, stream_ptr

DEFAULT_THRESHOLD_SCALE = 0.7
GROUP_SIZE = 128
HEAD_GROUP_SIZE = 64
HEAD_BITS = 4


def _pack(codes: torch.Tensor, bits: int, op: str) -> torch.Tensor:
    require_cuda(op, codes)
    per = 32 // bits
    *lead, k = codes.shape
    if k % per:
        raise ValueError(f"{bits}-bit packing requires the last axis to be a multiple of {per}; got {k}.")
    c = codes.to(torch.uint8).contiguous()
    out = torch.empty(*lead, k // per, dtype=torch.uint32, device=codes.device)
    check(lib().maple_pack_codes(ptr(c), c.numel(), bits, ptr(out), stream_ptr(codes.device)), op)
    return out


def _unpack(packed: torch.Tensor, bits: int, op: str) -> torch.Tensor:
    require_cuda(op, packed)
    p = packed.contiguous()
    if p.dtype != torch.uint32:
        p = p.view(torch.uint32)
    per = 32 // bits
    out = torch.empty(*p.shape[:-1], p.shape[-1] * per, dtype=torch.uint8, device=p.device)
    check(lib().maple_unpack_codes(ptr(p), p.numel(), bits, ptr(out), stream_ptr(p.device)), op)
    return out


def pack_2bit(codes: torch.Tensor) -> torch.Tensor:
    """16 two-bit codes per uint32, LSB first (reference pack.py:23-38)."""
    return _pack(codes, 2, "pack_2bit")


def unpack_2bit(packed: torch.Tensor) -> torch.Tensor:
    return _unpack(packed, 2, "unpack_2bit")


def pack_4bit(codes: torch.Tensor) -> torch.Tensor:
    """8 four-bit codes per uint32, LSB first (reference pack.py:48-57)."""
    return _pack(codes, 4, "pack_4bit")


def unpack_4bit(packed: torch.Tensor) -> torch.Tensor:
    return _unpack(packed, 4, "unpack_4bit")


def ternarize(weight: torch.Tensor, threshold_scale: float = DEFAULT_THRESHOLD_SCALE):
    """Row-wise ternary pack of ``[..., N, K]`` weights (reference
    pack.py:120-149): threshold ``threshold_scale * mean|w|``, alpha = mean of
    the surviving ``|w|`` in the weight dtype, codes ``sign(w)*mask + 1``.
    Returns ``(packed uint32 [..., N, K/16], row_alpha [..., N])``."""
    op = "ternarize"
    require_cuda(op, weight)
    k = weight.shape[-1]
    if k % GROUP_SIZE:
        raise ValueError(f"Ternary conversion requires the reduction dim to be a multiple of {GROUP_SIZE}; got {k}.")
    w = weight.contiguous()
    rows = w.numel() // k
    packed = torch.empty(*w.shape[:-1], k // 16, dtype=torch.uint32, device=w.device)
    alpha = torch.empty(w.shape[:-1], dtype=w.dtype, device=w.device)
    check(lib().maple_ternarize(ptr(w), dtype_code(w, op), rows, k, float(threshold_scale), ptr(packed), ptr(alpha),
                                dtype_code(alpha, op), stream_ptr(w.device)), op)
    return packed, alpha


def quantize_rtn(weight: torch.Tensor, group_size: int = HEAD_GROUP_SIZE, bits: int = HEAD_BITS):
    """Affine 4-bit round-to-nearest along the last axis (reference
    pack.py:67-100).  Returns ``(packed uint32, scales fp32, biases fp32)``."""
    op = "quantize_rtn"
    if bits != HEAD_BITS:
        raise ValueError(f"Only {HEAD_BITS}-bit RTN is implemented; got {bits}.")
    require_cuda(op, weight)
    k = weight.shape[-1]
    if k % group_size:
        raise ValueError(f"RTN conversion requires the last axis to be a multiple of {group_size}; got {k}.")
    w = weight.contiguous()
    rows = w.numel() // k
    lead = w.shape[:-1]
    packed = torch.empty(*lead, k // 8, dtype=torch.uint32, device=w.device)
    scales = torch.empty(*lead, k // group_size, dtype=torch.float32, device=w.device)
    biases = torch.empty_like(scales)
    check(lib().maple_quantize_rtn(ptr(w), dtype_code(w, op), rows, k, group_size, ptr(packed), ptr(scales),
                                   ptr(biases), stream_ptr(w.device)), op)
    return packed, scales, biases


def dequantize_rtn(packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                   group_size: int = HEAD_GROUP_SIZE, bits: int = HEAD_BITS) -> torch.Tensor:
    """Inverse of :func:`quantize_rtn` (reference pack.py:103-117), fp32."""
    op = "dequantize_rtn"
    if bits != HEAD_BITS:
        raise ValueError(f"Only {HEAD_BITS}-bit RTN is implemented; got {bits}.")
    require_cuda(op, packed, scales, biases)
    p = packed.contiguous()
    if p.dtype != torch.uint32:
        p = p.view(torch.uint32)
    k = p.shape[-1] * 8
    rows = p.numel() // p.shape[-1]
    s = scales.float().contiguous()
    b = biases.float().contiguous()
    out = torch.empty(*p.shape[:-1], k, dtype=torch.float32, device=p.device)
    check(lib().maple_dequantize_rtn(ptr(p), ptr(s), ptr(b), rows, k, group_size, ptr(out), stream_ptr(p.device)), op)
    return out
