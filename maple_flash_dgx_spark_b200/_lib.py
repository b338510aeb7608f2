"""ctypes binding of ``libmaple_b200.so`` (C ABI in ``include/maple_b200.h``).

There is no CPU fallback: if the library is missing, or the tensors are not on
a CUDA device, every operator raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libmaple_b200.so"

F32, BF16 = 0, 1
_DTYPE = {torch.float32: F32, torch.bfloat16: BF16}

# maple_status -> exception type (reference wrappers raise ValueError for
# shapes, TypeError for dtypes, RuntimeError for device problems).
_ERRORS = {
    1: (ValueError, "invalid shape or size"),
    2: (TypeError, "unsupported dtype"),
    3: (ValueError, "index out of bounds"),
    4: (RuntimeError, "bounded device wait timed out"),
    5: (RuntimeError, "CUDA launch failed"),
    6: (ValueError, "workspace missing or too small"),
    7: (ValueError, "pointer or stride not 16-byte aligned"),
    8: (ValueError, "request exceeds the library's fixed scratch"),
}

_lib = None
_lock = threading.Lock()

i32, i64, f32, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/maple_b200.h
_SIGS: dict[str, tuple] = {
    "maple_ternary_gemv_workspace_bytes": (i64, [i64, i64, i64]),
    "maple_ternary_gemv": (i32, [vp, i32, i64, i64, i64, vp, i64, vp, i32, vp, i32, f32, vp, i64, vp, i64, vp]),
    "maple_ternary_gemv_noalloc": (i32, [vp, i32, i64, i64, i64, vp, i64, vp, i32, vp, i32, f32, vp, i64, vp]),
    "maple_topk_select": (i32, [vp, i32, i64, i64, vp, vp]),
    "maple_flash_scatter": (i32, [vp, i32, vp, i64, i64, vp, i64, vp, vp, i64, vp, i64, vp, vp]),
    "maple_pack_codes": (i32, [vp, i64, i32, vp, vp]),
    "maple_unpack_codes": (i32, [vp, i64, i32, vp, vp]),
    "maple_ternarize": (i32, [vp, i32, i64, i64, f32, vp, vp, i32, vp]),
    "maple_quantize_rtn": (i32, [vp, i32, i64, i64, i64, vp, vp, vp, vp]),
    "maple_dequantize_rtn": (i32, [vp, vp, vp, i64, i64, i64, vp, vp]),
    "maple_fxa_frag_bytes": (i64, [i64, i64]),
    "maple_fxa_meta_bytes": (i64, [i64]),
    "maple_fxa_encode": (i32, [vp, i32, i64, i64, i64, vp, i32, f32, vp, vp, vp]),
    "maple_ternary_gemm": (i32, [vp, vp, i64, i64, vp, i64, vp, i32, i32, vp, i32, i64, vp, vp]),
    "maple_moe_plan": (i32, [vp, i64, i64, vp, vp, vp]),
    "maple_moe_plan_range": (i32, [vp, i64, i64, i64, i64, vp, vp, vp]),
    "maple_ep_combine": (i32, [vp, i32, i64, i64, i64, i64, vp, vp, i64, vp, vp, vp]),
    "maple_p2p_dispatch_bytes": (i64, [i64, i64, i64, i32, i64]),
    "maple_p2p_combine_bytes": (i64, [i64, i64, i64, i32]),
    "maple_p2p_dispatch": (i32, [vp, i32, i32, i64, vp, i32, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp, vp]),
    "maple_p2p_combine": (i32, [vp, i32, i32, i64, vp, i32, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp, vp, vp,
                                vp]),
    "maple_km_assign_workspace_bytes": (i64, [i64, i64]),
    "maple_km_assign": (i32, [vp, i64, i64, vp, i64, vp, vp, vp, i64, vp]),
    "maple_km_dots": (i32, [vp, vp, i64, i64, vp, i64, vp, vp]),
    "maple_km_reassign": (i32, [vp, vp, i64, i64, vp, i64, vp, vp, vp]),
    "maple_km_update": (i32, [vp, i64, vp, vp, i64, vp, vp]),
    "maple_km_objective_blocks": (i64, [i64]),
    "maple_km_objective": (i32, [vp, i64, i64, vp, vp, vp, vp]),
    "maple_km_normalize": (i32, [vp, i64, i64, vp]),
    "maple_ternary_grouped_gemm": (i32, [vp, vp, i64, i64, vp, i64, i64, vp, i32, vp, vp, i64, i64, i32, i32, vp,
                                         i32, i64, vp, vp]),
    "maple_ternary_grouped_gemm_tc_workspace_bytes": (i64, [i64, i64]),
    "maple_ternary_grouped_gemm_tc": (i32, [vp, i32, i64, i64, i64, vp, i64, i64, vp, i32, vp, vp, i64, i64, i32,
                                            vp, i32, f32, vp, i32, i64, vp, i64, vp, vp]),
    "maple_ternary_expert_gemv_workspace_bytes": (i64, [i64, i64, i64]),
    "maple_ternary_expert_gemv": (i32, [vp, i32, i64, i64, vp, i64, i64, vp, i64, i64, vp, i32, vp, i64, vp,
                                        i64, vp]),
    "maple_ternary_expert_swiglu_workspace_bytes": (i64, [i64, i64, i64]),
    "maple_ternary_expert_swiglu": (i32, [vp, i32, i64, vp, i64, i64, i64, vp, i64, i64, vp, i32, vp, i64, vp,
                                          i64, vp, vp]),
    "maple_ternary_expert_down_reduce": (i32, [vp, i32, i64, i64, vp, vp, i64, i64, i64, vp, i64, i64, vp, i32,
                                               vp, i64, vp, i64, vp, vp]),
    "maple_ternary_expert_down_sum": (i32, [vp, i32, i64, i64, vp, vp, i64, i64, i64, vp, i64, i64, vp, i32,
                                            vp, i64, vp, i64, vp, vp]),
    "maple_moe_reduce_add": (i32, [vp, i32, i64, i64, vp, i64, i64, i64, vp, i64, vp, i64, vp]),
    "maple_router_topk_workspace_bytes": (i64, [i64, i64]),
    "maple_router_topk": (i32, [vp, i32, i64, i64, i64, vp, i32, i64, i64, vp, vp, vp, i64, vp]),
    "maple_add_norm_router_topk": (i32, [vp, vp, i32, i64, i64, i64, vp, i32, f32, vp, i32, i64, i64, vp, vp, vp, vp,
                                         vp, i64, vp]),
    "maple_rms_norm": (i32, [vp, i32, i64, i64, i64, vp, i32, f32, vp, i64, vp]),
    "maple_add_rms_norm": (i32, [vp, vp, i32, i64, i64, i64, i64, vp, i32, f32, vp, i64, vp, i64, vp]),
    "maple_apply_qkv_decode": (i32, [vp, i32, i64, i64, vp, vp, i32, vp, vp, i32, i64, i64, vp, i64, i64, vp, vp,
                                     i64, i64, i64, i64, vp, vp, i64, i64, i64, i64, i32, f32, vp, vp]),
    "maple_decode_gqa_workspace_bytes": (i64, [i64, i64, i64, i64, i64]),
    "maple_decode_gqa_attn": (i32, [vp, i32, i64, i64, i64, i64, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp,
                                    f32, i64, i64, i32, vp, i64, i64, vp, i64, vp, vp]),
    "maple_decode_gqa_attn_qk": (i32, [vp, i32, i64, i64, vp, vp, i32, vp, vp, i32, i64, i64, i64, i32, f32, i64,
                                       vp, vp, i64, i64, i64, i64, i64, i64, vp, vp, f32, i64, i64, vp, i64, i64, vp,
                                       i64, vp, vp]),
    "maple_decode_gqa_attn_tc_workspace_bytes": (i64, [i64, i64, i64, i64]),
    "maple_decode_gqa_attn_tc": (i32, [vp, i32, i64, i64, i64, i64, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp,
                                       f32, i64, vp, i64, i64, vp, i64, vp, vp]),
    "maple_rtn4_gemv": (i32, [vp, i32, i64, i64, i64, vp, i64, vp, vp, i32, i64, vp, i64, vp]),
    "maple_rtn4_frag_bytes": (i64, [i64, i64]),
    "maple_row_uniform": (i32, [vp, i64, vp, vp, vp]),
    "maple_rtn4_gemm": (i32, [vp, i32, i64, i64, i64, vp, i64, vp, vp, i32, i64, vp, i64, vp, i64, vp, vp]),
    "maple_rtn4_indexed_gemv": (i32, [vp, i32, i64, i64, i64, vp, i64, i64, vp, vp, i32, i64, vp, i64, vp, i64,
                                      vp]),
    "maple_argmax_workspace_bytes": (i64, [i64, i64]),
    "maple_argmax": (i32, [vp, i32, i64, i64, i64, vp, vp, i64, vp]),
    "maple_fused_sample_workspace_bytes": (i64, [i64, i64, i64]),
    "maple_fused_sample": (i32, [vp, i32, i64, i64, i64, vp, f32, f32, i64, vp, vp, i64, vp]),
    "maple_embedding": (i32, [vp, i64, vp, i32, i64, i64, vp, i32, i64, vp, vp]),
    "maple_rtn4_embedding": (i32, [vp, i64, vp, vp, vp, i32, i64, i64, i64, vp, i32, i64, vp, vp]),
    "maple_synth_ternary": (i32, [ctypes.c_uint64, ctypes.c_uint64, i64, vp, vp]),
    "maple_synth_normal": (i32, [ctypes.c_uint64, ctypes.c_uint64, i64, ctypes.c_double, f32, i32, i32, vp, vp]),
    "maple_synth_rtn4_sym": (i32, [ctypes.c_uint64, ctypes.c_uint64, i64, i64, i64, ctypes.c_double, vp, vp, vp]),
    "maple_synth_tokens": (i32, [ctypes.c_uint64, ctypes.c_uint64, i64, i64, vp, vp]),
}


def lib() -> ctypes.CDLL:
    """Load the CUDA library (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python -m maple_flash_dgx_spark_b200.build` "
                        "(there is no CPU fallback)."
                    )
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, op: str) -> None:
    if status != 0:
        exc, what = _ERRORS.get(status, (RuntimeError, f"status {status}"))
        raise exc(f"{op}: {what} (maple status {status})")


def dtype_code(t: torch.Tensor, op: str) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise TypeError(f"{op}: dtype {t.dtype} is not supported (float32 or bfloat16).") from None


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(op: str, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{op} requires CUDA tensors (packed weights stay on the GPU).")


class Workspace:
    """Zero-initialised device scratch shared by sequential launches on one
    stream.  Kernels that use it leave it zeroed again, so one buffer serves
    every call (and every replay of a captured graph)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if nbytes > self.buf.numel():
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "maple workspace must grow during CUDA graph capture; run the step once "
                    "eagerly before capturing."
                )
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel(), 1 << 20), dtype=torch.uint8,
                                   device=self.device)
        return self.buf


_workspaces: dict[int, Workspace] = {}


def workspace(device: torch.device) -> Workspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = _workspaces[idx] = Workspace(torch.device("cuda", idx))
    return ws


_errors: dict[int, torch.Tensor] = {}


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word that kernels OR flags into (1: a bounded
    wait timed out, 2: an index or position was out of range).  Allocated
    outside inference mode, so it can be cleared in place from either mode."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    e = _errors.get(idx)
    if e is None:
        with torch.inference_mode(False):
            e = _errors[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
    return e


def take_device_errors(device: torch.device) -> int:
    """Read (synchronising) and clear the device error word."""
    e = error_word(device)
    v = int(e.item())
    if v:
        e.zero_()
    return v


_DEVICE_FLAGS = {1: "a bounded device wait gave up", 2: "an index or position was out of range"}


def raise_device_errors(device: torch.device, where: str) -> None:
    """Read and clear the device error word; raise if a kernel flagged
    anything since the last read.  The drivers call this at their existing
    synchronisation points (end of a generate call, every serve step, every
    expert-parallel step), so a give-up or a clamped index never passes
    silently as wrong tokens."""
    v = take_device_errors(device)
    if v:
        what = ", ".join(msg for bit, msg in _DEVICE_FLAGS.items() if v & bit) or f"flags {v:#x}"
        raise RuntimeError(f"{where}: device error word {v:#x} ({what}); results of this call are not valid.")
