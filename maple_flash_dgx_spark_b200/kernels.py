"""Reference-named operator surface, backed by the sm_100a C ABI.

Each function keeps the name, argument meaning, output allocation and error
types of its counterpart in the reference (cloud-000/maple-flash-dgx-spark,
``src/maple_run/kernels/*.py``), so model code written against the reference
runs unchanged.  All arithmetic happens in ``libmaple_b200.so``.
"""

from __future__ import annotations

import torch

from maple_flash_dgx_spark_b200 import _lib
from maple_flash_dgx_spark_b200._lib import check, dtype_code, lib, ptr, require_cuda, stream_ptr

_CODES_PER_WORD = 16


def ternary_gemv(
    x: torch.Tensor,
    packed_weight: torch.Tensor,
    row_alpha: torch.Tensor,
    *,
    rms_weight: torch.Tensor | None = None,
    rms_eps: float = 1e-6,
    packed_kn: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode GEMV ``y = x @ W`` with ``W`` kept as packed uint32 codes.

    Reference: kernels/ternary_gemv.py:261-388.  ``x`` is ``[K]`` or ``[..., K]``;
    ``packed_weight`` is uint32 ``[N, K/16]`` (``[K/16, N]`` with ``packed_kn``);
    ``row_alpha`` is ``[N]``; ``rms_weight`` folds an input RMSNorm into the GEMV.
    Returns ``[..., N]`` in ``x.dtype``.
    """
    op = "ternary_gemv"
    require_cuda(op, x, packed_weight, row_alpha, rms_weight)
    if packed_weight.dtype != torch.uint32:
        raise TypeError(
            f"packed_weight must be uint32 codes, got {packed_weight.dtype}; "
            "refusing to run a dense-weight path."
        )
    if packed_weight.ndim != 2:
        raise ValueError(
            f"packed_weight must be 2-D [N, K/16] or [K/16, N]; got shape "
            f"{tuple(packed_weight.shape)}."
        )
    if packed_kn:
        packed_weight = packed_weight.t()
    packed_weight = packed_weight.contiguous()
    n_out, nwords = packed_weight.shape
    k_in = nwords * _CODES_PER_WORD
    alpha = row_alpha.reshape(-1)
    if alpha.numel() != n_out:
        raise ValueError(f"row_alpha has {alpha.numel()} elements, expected one per output row ({n_out}).")
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    if k_in % 64:
        raise ValueError(f"K={k_in} must be a multiple of 64 for the sm_100a GEMV.")
    xd = dtype_code(x, op)
    leading = x.shape[:-1]
    batch = int(x.numel() // k_in) if k_in else 0
    x_mat = x.reshape(batch, k_in)
    if x_mat.stride(-1) != 1:
        x_mat = x_mat.contiguous()
    alpha = alpha.contiguous()
    rms = None
    if rms_weight is not None:
        rms = rms_weight.reshape(-1).contiguous()
        if rms.numel() != k_in:
            raise ValueError(f"rms_weight has {rms.numel()} elements, expected {k_in}.")
    y = out if out is not None else torch.empty(batch, n_out, device=x.device, dtype=x.dtype)
    L = lib()
    if (use_tc_dense(batch, k_in, n_out) and packed_weight.data_ptr() % 256 == 0 and
            (y.dim() == 1 or y.stride(-1) == 1)):
        _grouped_tc(op, x_mat, 1, packed_weight.reshape(1, n_out, nwords), alpha.reshape(1, n_out),
                    _dense_plan(batch, x.device), False, y.reshape(batch, n_out), rms=rms, rms_eps=rms_eps)
        return y.reshape(*leading, n_out)
    if batch >= GEMM_MIN_ROWS and k_in <= 4096:
        frag, meta = fxa_encode(x_mat, rms, rms_eps)
        check(L.maple_ternary_gemm(ptr(frag), ptr(meta), batch, k_in, ptr(packed_weight), n_out, ptr(alpha),
                                   dtype_code(alpha, op), int(rms is not None), ptr(y), dtype_code(y, op),
                                   y.stride(0) if y.dim() > 1 else n_out, ptr(_err(x.device)),
                                   stream_ptr(x.device)), op)
        return y.reshape(*leading, n_out)
    nbytes = L.maple_ternary_gemv_workspace_bytes(batch, n_out, k_in)
    ws = _lib.workspace(x.device).get(nbytes) if nbytes else None
    st = L.maple_ternary_gemv(
        ptr(x_mat), xd, batch, k_in, x_mat.stride(0), ptr(packed_weight), n_out, ptr(alpha),
        dtype_code(alpha, op), ptr(rms), dtype_code(rms, op) if rms is not None else 0,
        float(rms_eps), ptr(y), y.stride(0) if y.dim() > 1 else n_out, ptr(ws),
        ws.numel() if ws is not None else 0, stream_ptr(x.device),
    )
    check(st, op)
    return y.reshape(*leading, n_out)


def _u32(t: torch.Tensor, op: str) -> torch.Tensor:
    if t.dtype != torch.uint32:
        raise TypeError(f"{op}: packed_weight must be uint32 codes, got {t.dtype}; refusing to run a dense-weight path.")
    return t


def _ws(device: torch.device, nbytes: int) -> torch.Tensor | None:
    return _lib.workspace(device).get(nbytes) if nbytes > 0 else None


def _err(device: torch.device) -> torch.Tensor:
    return _lib.error_word(device)


def _expert_nk(packed_weight: torch.Tensor, packed_kn: bool, op: str) -> torch.Tensor:
    if packed_weight.ndim != 3:
        raise ValueError(f"{op}: packed_weight must be 3-D [E, N, K/16]; got shape {tuple(packed_weight.shape)}.")
    _u32(packed_weight, op)
    if packed_kn:
        packed_weight = packed_weight.transpose(1, 2)
    return packed_weight.contiguous()


# Row counts from which the batched kernels (weights read once per batch) take
# over from the per-row GEMV launches.
GEMM_MIN_ROWS = 4
GROUPED_MIN_TOKENS = 4
HEAD_GEMM_MIN_ROWS = 2


def fxa_encode(x2d: torch.Tensor, rms_weight: torch.Tensor | None = None, eps: float = 1e-6):
    """FXA digits of each row of ``x2d`` ``[R, K]`` (optionally RMS-normalised
    by ``rms_weight``) for the batched GEMMs: returns ``(frag, meta)`` uint8
    buffers of ``maple_fxa_frag_bytes`` / ``maple_fxa_meta_bytes``."""
    op = "fxa_encode"
    require_cuda(op, x2d, rms_weight)
    rows, k_in = x2d.shape
    if x2d.stride(-1) != 1 or (x2d.stride(0) * x2d.element_size()) % 16 or x2d.data_ptr() % 16:
        x2d = x2d.contiguous()
    L = lib()
    frag = torch.empty(L.maple_fxa_frag_bytes(rows, k_in), dtype=torch.uint8, device=x2d.device)
    meta = torch.empty(L.maple_fxa_meta_bytes(rows), dtype=torch.uint8, device=x2d.device)
    check(L.maple_fxa_encode(ptr(x2d), dtype_code(x2d, op), rows, k_in, x2d.stride(0), ptr(rms_weight),
                             dtype_code(rms_weight, op) if rms_weight is not None else 0, float(eps), ptr(frag),
                             ptr(meta), stream_ptr(x2d.device)), op)
    return frag, meta


class MoePlan:
    """(token, slot) pairs of a routing decision sorted by expert on the device
    (``offsets [E+1]`` int32, ``slots`` uint32), shared by the grouped up|gate
    and down GEMMs of one MoE layer."""

    def __init__(self, offsets: torch.Tensor, slots: torch.Tensor, n_experts: int, n_slots: int,
                 total_experts: int | None = None):
        self.offsets = offsets
        self.slots = slots
        self.n_experts = n_experts
        self.n_slots = n_slots
        self.total_experts = n_experts if total_experts is None else total_experts


def moe_plan(expert_ids: torch.Tensor, n_experts: int, *, e_first: int = 0, n_local: int | None = None) -> MoePlan:
    """Sort the routed slots by expert.  With ``e_first`` / ``n_local`` only the
    experts ``[e_first, e_first + n_local)`` (one rank's share under expert
    parallelism) are listed, indexed locally."""
    op = "moe_plan"
    require_cuda(op, expert_ids)
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    n = ids.numel()
    n_local = n_experts if n_local is None else int(n_local)
    offsets = torch.empty(n_local + 1, dtype=torch.int32, device=ids.device)
    slots = torch.empty(max(n, 1), dtype=torch.int32, device=ids.device)
    check(lib().maple_moe_plan_range(ptr(ids), n, n_experts, int(e_first), n_local, ptr(offsets), ptr(slots),
                                     stream_ptr(ids.device)), op)
    return MoePlan(offsets, slots, n_local, n, total_experts=n_experts)


def ep_combine(recv: torch.Tensor, expert_ids: torch.Tensor, topk_weight: torch.Tensor, n_experts: int,
               residual: torch.Tensor | None = None) -> torch.Tensor:
    """Expert-parallel weighted top-k sum: ``recv [world, tokens*topk, N]`` holds
    every rank's expert rows for this rank's tokens; the row of the rank that
    owns each slot's expert enters ``moe_reduce_add``'s sum.  Returns
    ``[tokens, N]``."""
    op = "ep_combine"
    require_cuda(op, recv, expert_ids, topk_weight, residual)
    world, rows, n = recv.shape
    tokens, topk = expert_ids.shape
    if rows != tokens * topk:
        raise ValueError(f"recv rows {rows} != tokens*topk {tokens * topk}.")
    r = recv.contiguous()
    ids = expert_ids.to(torch.int32).contiguous()
    w = topk_weight.float().contiguous()
    res = residual.reshape(tokens, n).contiguous() if residual is not None else None
    y = torch.empty(tokens, n, device=recv.device, dtype=recv.dtype)
    check(lib().maple_ep_combine(ptr(r), dtype_code(r, op), world, tokens, topk, n, ptr(ids), ptr(w), n_experts,
                                 ptr(res), ptr(y), stream_ptr(recv.device)), op)
    return y


TC_GEMM_MIN_SLOTS = 16


def _tc_gemm_enabled() -> bool:
    """``MAPLE_TC_GEMM=0`` keeps every grouped expert GEMM on mma.sync."""
    import os

    return os.environ.get("MAPLE_TC_GEMM", "1") != "0"


def use_tc_grouped(plan: "MoePlan", k_in: int) -> bool:
    """The tcgen05 grouped GEMM pays off once the experts average at least
    TC_GEMM_MIN_SLOTS routed slots (prompt prefill, large batches): its MMA
    tile is 64 slots wide.  Both paths give identical results."""
    return (_tc_gemm_enabled() and k_in % 128 == 0 and
            plan.n_slots >= TC_GEMM_MIN_SLOTS * max(plan.total_experts, 1))


def _grouped_tc(op, x_rows, per, w, alpha, plan, swiglu, y, rms=None, rms_eps=1e-6):
    E, rows, nwords = w.shape
    k_in = nwords * _CODES_PER_WORD
    if x_rows.stride(-1) != 1 or (x_rows.stride(0) * x_rows.element_size()) % 16 or x_rows.data_ptr() % 16:
        x_rows = x_rows.contiguous()
    L = lib()
    ws = torch.empty(L.maple_ternary_grouped_gemm_tc_workspace_bytes(plan.n_slots, k_in), dtype=torch.uint8,
                     device=x_rows.device)
    check(L.maple_ternary_grouped_gemm_tc(
        ptr(x_rows), dtype_code(x_rows, op), x_rows.shape[0], k_in, x_rows.stride(0), ptr(w), E, rows, ptr(alpha),
        dtype_code(alpha, op), ptr(plan.offsets), ptr(plan.slots), plan.n_slots, per, int(swiglu), ptr(rms),
        dtype_code(rms, op) if rms is not None else 0, float(rms_eps), ptr(y), dtype_code(y, op), y.stride(0),
        ptr(ws), ws.numel(), ptr(_err(x_rows.device)), stream_ptr(x_rows.device)), op)
    return y


# Dense batched GEMMs move to the tcgen05 kernel (as one expert whose plan
# lists every row) where it measured faster than mma.sync: at least 64 rows
# and at least 4096 output rows, so that its 128-row tiles cover the SMs
# (QKV N=5120: 27.3 -> 20.0 us at 64 rows, 168 -> 125 us at 512; the O
# projection, N=2048, stays on mma.sync: 23 vs 29 us at 64 rows, 159 vs 197
# at 512).  Both paths give identical results.
TC_DENSE_MIN_ROWS, TC_DENSE_MIN_OUT = 64, 4096
_dense_plans: dict = {}


def use_tc_dense(batch: int, k_in: int, n_out: int) -> bool:
    import os

    if os.environ.get("MAPLE_TC_DENSE", "1") == "0" or not _tc_gemm_enabled():
        return False
    if k_in % 128 or k_in > 8192:
        return False
    return batch >= TC_DENSE_MIN_ROWS and n_out >= TC_DENSE_MIN_OUT


def _dense_plan(batch: int, device: torch.device) -> "MoePlan":
    key = (batch, device.index)
    plan = _dense_plans.get(key)
    if plan is None:
        offsets = torch.tensor([0, batch], dtype=torch.int32, device=device)
        slots = torch.arange(batch, dtype=torch.int32, device=device)
        plan = _dense_plans[key] = MoePlan(offsets, slots, 1, batch, total_experts=1)
    return plan


def _grouped(op, x_rows, per, w, alpha, plan, swiglu, out_rows, n_out, dtype, out=None, tc=None):
    """Grouped expert GEMM: input row of slot s is ``s // per``.  ``tc``
    forces (True) or forbids (False) the tcgen05 path; by default it runs
    where the experts average enough routed slots."""
    E, rows, nwords = w.shape
    k_in = nwords * _CODES_PER_WORD
    if tc is None:
        tc = use_tc_grouped(plan, k_in)
    if tc:
        y = out if out is not None else torch.empty(out_rows, n_out, device=x_rows.device, dtype=dtype)
        return _grouped_tc(op, x_rows, per, w, alpha, plan, swiglu, y)
    frag, meta = fxa_encode(x_rows)
    y = out if out is not None else torch.empty(out_rows, n_out, device=x_rows.device, dtype=dtype)
    check(lib().maple_ternary_grouped_gemm(
        ptr(frag), ptr(meta), x_rows.shape[0], k_in, ptr(w), E, rows, ptr(alpha), dtype_code(alpha, op),
        ptr(plan.offsets), ptr(plan.slots), plan.n_slots, per, int(swiglu), 1, ptr(y), dtype_code(y, op), n_out,
        ptr(_err(x_rows.device)), stream_ptr(x_rows.device)), op)
    return y


def ternary_expert_gemv(x, packed_weight, row_alpha, expert_ids, *, packed_kn: bool = False,
                        plan: MoePlan | None = None):
    """Indexed GEMV over stacked experts.  Reference kernels/ternary_expert.py:125-234.

    ``x`` is one row per token (``x.shape[:-1] == expert_ids.shape[:-1]``) or one
    row per slot (``x.shape[:-1] == expert_ids.shape``).  Returns
    ``expert_ids.shape + (N,)`` in ``x.dtype``."""
    op = "ternary_expert_gemv"
    if not x.is_cuda or not packed_weight.is_cuda or not row_alpha.is_cuda:
        raise RuntimeError(f"{op} requires CUDA tensors.")
    if not expert_ids.is_cuda:
        raise RuntimeError("expert_ids must be a CUDA tensor (no GPU->CPU routing).")
    w = _expert_nk(packed_weight, packed_kn, op)
    E, N, nwords = w.shape
    k_in = nwords * _CODES_PER_WORD
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    if tuple(row_alpha.shape) != (E, N):
        raise ValueError(f"row_alpha shape {tuple(row_alpha.shape)} != {(E, N)}.")
    id_shape = tuple(expert_ids.shape)
    if tuple(x.shape[:-1]) == id_shape:
        per = 1
    elif tuple(x.shape[:-1]) == id_shape[:-1]:
        per = id_shape[-1]
    else:
        raise ValueError(f"x shape {tuple(x.shape)} incompatible with expert_ids {id_shape}.")
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    slots = ids.numel()
    xm = x.reshape(-1, k_in).contiguous()
    alpha = row_alpha.contiguous()
    if k_in <= 4096 and (plan is not None or slots // max(id_shape[-1] if id_shape else 1, 1) >= GROUPED_MIN_TOKENS):
        dtype_code(x, op)
        plan = plan if plan is not None else moe_plan(ids, E)
        y = _grouped(op, xm, per, w, alpha, plan, False, slots, N, x.dtype)
        return y.reshape(*id_shape, N)
    y = torch.empty(slots, N, device=x.device, dtype=x.dtype)
    L = lib()
    ws = _ws(x.device, L.maple_ternary_expert_gemv_workspace_bytes(slots, N, k_in))
    check(L.maple_ternary_expert_gemv(
        ptr(xm), dtype_code(x, op), xm.stride(0), per, ptr(ids), slots, k_in, ptr(w), E, N, ptr(alpha),
        dtype_code(alpha, op), ptr(y), N, ptr(ws), ws.numel() if ws is not None else 0, stream_ptr(x.device)), op)
    return y.reshape(*id_shape, N)


def ternary_expert_swiglu(x, packed_weight, row_alpha, expert_ids, *, packed_kn: bool = False,
                          plan: MoePlan | None = None):
    """Fused up|gate GEMV + clamp + SiLU.  Reference kernels/ternary_expert.py:403-468.
    Returns ``[..., topk, I]`` with ``I = packed rows / 2``."""
    op = "ternary_expert_swiglu"
    if not x.is_cuda or not packed_weight.is_cuda or not expert_ids.is_cuda:
        raise RuntimeError(f"{op} requires CUDA tensors.")
    if packed_weight.ndim != 3 or packed_weight.dtype != torch.uint32:
        raise ValueError("packed_weight must be uint32 [E, 2N, K/16] or [E, K/16, 2N].")
    w = _expert_nk(packed_weight, packed_kn, op)
    E, rows, nwords = w.shape
    if rows % 2:
        raise ValueError(f"packed up_gate rows must be even, got {rows}.")
    inter = rows // 2
    k_in = nwords * _CODES_PER_WORD
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    if tuple(row_alpha.shape) != (E, rows):
        raise ValueError(f"row_alpha shape {tuple(row_alpha.shape)} != {(E, rows)}.")
    id_shape = tuple(expert_ids.shape)
    if tuple(x.shape[:-1]) != id_shape[:-1]:
        raise ValueError(f"x shape {tuple(x.shape)} incompatible with expert_ids {id_shape}.")
    topk = id_shape[-1]
    xm = x.reshape(-1, k_in).contiguous()
    tokens = xm.shape[0]
    ids = expert_ids.reshape(-1).to(torch.int32).contiguous()
    alpha = row_alpha.contiguous()
    if k_in <= 4096 and (plan is not None or tokens >= GROUPED_MIN_TOKENS):
        dtype_code(x, op)
        plan = plan if plan is not None else moe_plan(ids, E)
        y = _grouped(op, xm, topk, w, alpha, plan, True, tokens * topk, inter, x.dtype)
        return y.reshape(*id_shape, inter)
    y = torch.empty(tokens * topk, inter, device=x.device, dtype=x.dtype)
    L = lib()
    ws = _ws(x.device, L.maple_ternary_expert_swiglu_workspace_bytes(tokens * topk, inter, k_in))
    check(L.maple_ternary_expert_swiglu(
        ptr(xm), dtype_code(x, op), xm.stride(0), ptr(ids), tokens, topk, k_in, ptr(w), E, inter, ptr(alpha),
        dtype_code(alpha, op), ptr(y), inter, ptr(ws), ws.numel() if ws is not None else 0,
        ptr(_err(x.device)), stream_ptr(x.device)), op)
    return y.reshape(*id_shape, inter)


def _down(x, packed_weight, row_alpha, expert_ids, topk_weight, residual, packed_kn, fn, op):
    if not x.is_cuda or not packed_weight.is_cuda or not expert_ids.is_cuda:
        raise RuntimeError(f"{op} requires CUDA tensors.")
    w = _expert_nk(packed_weight, packed_kn, op)
    E, N, nwords = w.shape
    k_in = nwords * _CODES_PER_WORD
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    if tuple(row_alpha.shape) != (E, N):
        raise ValueError(f"row_alpha shape {tuple(row_alpha.shape)} != {(E, N)}.")
    if expert_ids.shape != topk_weight.shape or tuple(x.shape[:-1]) != tuple(expert_ids.shape):
        raise ValueError("x / expert_ids / topk_weight leading dims must match.")
    topk = int(expert_ids.shape[-1])
    tokens = int(expert_ids.numel() // topk)
    xm = x.reshape(tokens, topk, k_in).contiguous()
    ids = expert_ids.reshape(tokens, topk).to(torch.int32).contiguous()
    wts = topk_weight.reshape(tokens, topk).float().contiguous()
    alpha = row_alpha.contiguous()
    res = None
    if residual is not None:
        res = residual.reshape(tokens, N).contiguous()
    y = torch.empty(tokens, N, device=x.device, dtype=x.dtype)
    check(fn(ptr(xm), dtype_code(x, op), topk * k_in, k_in, ptr(ids), ptr(wts), tokens, topk, k_in, ptr(w), E, N,
             ptr(alpha), dtype_code(alpha, op), ptr(res), N, ptr(y), N, ptr(_err(x.device)), stream_ptr(x.device)),
          op)
    return y.reshape(*expert_ids.shape[:-1], N)


def ternary_expert_down_sum(x, packed_weight, row_alpha, expert_ids, topk_weight, residual=None, *,
                            packed_kn: bool = False):
    """Down GEMV, weighted top-k sum, optional residual.  Reference
    kernels/ternary_expert.py:471-556 (no rounding of per-slot outputs)."""
    return _down(x, packed_weight, row_alpha, expert_ids, topk_weight, residual, packed_kn,
                 lib().maple_ternary_expert_down_sum, "ternary_expert_down_sum")


def ternary_expert_down_reduce(x, packed_weight, row_alpha, expert_ids, topk_weight, residual=None, *,
                               packed_kn: bool = False, plan: MoePlan | None = None):
    """The reference model's down + combine (model.py:471-473: ternary_expert_gemv
    with per-slot outputs in ``x.dtype``, then moe_reduce_add): one launch for a
    few tokens; from GROUPED_MIN_TOKENS tokens (or with a ``plan``) the grouped
    GEMM (each expert's weights read once) followed by moe_reduce_add, with the
    same rounding."""
    tokens = int(expert_ids.numel() // max(int(expert_ids.shape[-1]), 1)) if expert_ids.ndim else 0
    if plan is not None or tokens >= GROUPED_MIN_TOKENS:
        y = ternary_expert_gemv(x, packed_weight, row_alpha, expert_ids, packed_kn=packed_kn, plan=plan)
        return moe_reduce_add(y, topk_weight, residual)
    return _down(x, packed_weight, row_alpha, expert_ids, topk_weight, residual, packed_kn,
                 lib().maple_ternary_expert_down_reduce, "ternary_expert_down_reduce")


def moe_reduce_add(expert_out, topk_weight, residual=None):
    """``y = (expert_out * topk_weight).sum(topk) [+ residual]``.  Reference kernels/fused_norm.py:164-202."""
    op = "moe_reduce_add"
    require_cuda(op, expert_out, topk_weight, residual)
    if expert_out.ndim < 2:
        raise ValueError("expert_out must be [..., topk, N].")
    topk, n = int(expert_out.shape[-2]), int(expert_out.shape[-1])
    if tuple(topk_weight.shape) != tuple(expert_out.shape[:-1]):
        raise ValueError("topk_weight must match expert_out without the last dim.")
    tokens = int(expert_out.numel() // (topk * n))
    x = expert_out.reshape(tokens, topk, n).contiguous()
    w = topk_weight.reshape(tokens, topk).float().contiguous()
    res = residual.reshape(tokens, n).contiguous() if residual is not None else None
    y = torch.empty(tokens, n, device=x.device, dtype=x.dtype)
    check(lib().maple_moe_reduce_add(ptr(x), dtype_code(x, op), topk * n, n, ptr(w), tokens, topk, n, ptr(res), n,
                                     ptr(y), n, stream_ptr(x.device)), op)
    return y.reshape(*expert_out.shape[:-2], n)


def router_topk(x, gate_weight, top_k):
    """Router logits -> softmax -> top-k -> renormalised weights.  Reference
    kernels/router.py:141-217.  Returns ``(idx int32 [..., k], weight fp32 [..., k])``."""
    op = "router_topk"
    if not x.is_cuda or not gate_weight.is_cuda:
        raise RuntimeError("router_topk requires CUDA tensors.")
    if gate_weight.ndim != 2:
        raise ValueError(f"gate_weight must be 2-D [E, K], got {tuple(gate_weight.shape)}.")
    n_exp, k_in = gate_weight.shape
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != router K ({k_in}).")
    if top_k > n_exp:
        raise ValueError(f"top_k={top_k} exceeds {n_exp} experts.")
    leading = x.shape[:-1]
    xm = x.reshape(-1, k_in).contiguous()
    tokens = xm.shape[0]
    g = gate_weight.contiguous()
    idx = torch.empty(tokens, top_k, device=x.device, dtype=torch.int32)
    wt = torch.empty(tokens, top_k, device=x.device, dtype=torch.float32)
    L = lib()
    ws = _ws(x.device, L.maple_router_topk_workspace_bytes(tokens, n_exp))
    check(L.maple_router_topk(ptr(xm), dtype_code(x, op), k_in, tokens, k_in, ptr(g), dtype_code(g, op), n_exp,
                              top_k, ptr(idx), ptr(wt), ptr(ws), ws.numel(), stream_ptr(x.device)), op)
    return idx.reshape(*leading, top_k), wt.reshape(*leading, top_k)


def add_rms_norm_router_topk(x, y, norm_weight, eps: float, gate_weight, top_k):
    """``add_rms_norm`` followed by ``router_topk`` in one launch: returns
    ``(x + y, rms_norm(x + y) * w, idx, weight)`` with both operators' exact
    results (reference model.py:498-506 runs them in sequence)."""
    op = "add_rms_norm_router_topk"
    require_cuda(op, x, y, norm_weight, gate_weight)
    if x.shape != y.shape or x.dtype != y.dtype:
        raise ValueError("x and y must have the same shape and dtype.")
    n_exp, k_in = gate_weight.shape
    if x.shape[-1] != k_in or norm_weight.numel() != k_in:
        raise ValueError(f"hidden size mismatch: x {tuple(x.shape)}, norm {norm_weight.numel()}, gate {k_in}.")
    if top_k > n_exp:
        raise ValueError(f"top_k={top_k} exceeds {n_exp} experts.")
    leading = x.shape[:-1]
    xm = x.reshape(-1, k_in).contiguous()
    ym = y.reshape(-1, k_in).contiguous()
    tokens = xm.shape[0]
    w = norm_weight.reshape(-1).contiguous()
    g = gate_weight.contiguous()
    res = torch.empty_like(xm)
    normed = torch.empty_like(xm)
    idx = torch.empty(tokens, top_k, device=x.device, dtype=torch.int32)
    wt = torch.empty(tokens, top_k, device=x.device, dtype=torch.float32)
    L = lib()
    ws = _ws(x.device, L.maple_router_topk_workspace_bytes(tokens, n_exp))
    check(L.maple_add_norm_router_topk(ptr(xm), ptr(ym), dtype_code(x, op), k_in, tokens, k_in, ptr(w),
                                       dtype_code(w, op), float(eps), ptr(g), dtype_code(g, op), n_exp, top_k,
                                       ptr(res), ptr(normed), ptr(idx), ptr(wt), ptr(ws), ws.numel(),
                                       stream_ptr(x.device)), op)
    return (res.reshape(x.shape), normed.reshape(x.shape), idx.reshape(*leading, top_k),
            wt.reshape(*leading, top_k))


def rms_norm(x, weight, eps: float = 1e-6):
    """RMSNorm over the last dim (fp32 math, output ``x.dtype``).  Reference kernels/fused_norm.py:105-125."""
    op = "rms_norm"
    if not x.is_cuda:
        raise RuntimeError("rms_norm requires CUDA tensors.")
    n = int(x.shape[-1])
    rows = int(x.numel() // n)
    xm = x.reshape(rows, n).contiguous()
    w = weight.reshape(-1).contiguous()
    if w.numel() != n:
        raise ValueError(f"rms_norm weight has {w.numel()} elements, expected {n}.")
    y = torch.empty_like(xm)
    check(lib().maple_rms_norm(ptr(xm), dtype_code(x, op), rows, n, n, ptr(w), dtype_code(w, op), float(eps),
                               ptr(y), n, stream_ptr(x.device)), op)
    return y.reshape(x.shape)


def add_rms_norm(x, y, weight, eps: float = 1e-6):
    """``residual = x + y`` and ``norm = rms_norm(residual)`` in one launch.  Reference kernels/fused_norm.py:128-161."""
    op = "add_rms_norm"
    if not x.is_cuda or not y.is_cuda:
        raise RuntimeError("add_rms_norm requires CUDA tensors.")
    if x.shape != y.shape:
        raise ValueError(f"add_rms_norm shape mismatch {tuple(x.shape)} vs {tuple(y.shape)}.")
    n = int(x.shape[-1])
    rows = int(x.numel() // n)
    xm = x.reshape(rows, n).contiguous()
    ym = y.reshape(rows, n).contiguous().to(x.dtype)
    w = weight.reshape(-1).contiguous()
    if w.numel() != n:
        raise ValueError(f"add_rms_norm weight has {w.numel()} elements, expected {n}.")
    residual = torch.empty_like(xm)
    normed = torch.empty_like(xm)
    check(lib().maple_add_rms_norm(ptr(xm), ptr(ym), dtype_code(x, op), rows, n, n, n, ptr(w), dtype_code(w, op),
                                   float(eps), ptr(residual), n, ptr(normed), n, stream_ptr(x.device)), op)
    return residual.reshape(x.shape), normed.reshape(x.shape)


def apply_qkv_decode(qkv, q_weight, k_weight, cos, sin, k_cache, v_cache, seqlen, *, row_map=None, num_heads,
                     num_kv_heads, head_dim, rotary_dim, use_rope, use_qk_norm, eps, rope_table: bool = False,
                     q_out=None):
    """QK RMSNorm + RoPE + K/V store at ``seqlen``.  Reference kernels/decode_attn.py:362-439.
    Returns Q ``[B, H, 1, D]``.  With ``rope_table`` the ``cos``/``sin``
    arguments are whole ``[T, rotary_dim]`` tables read at ``clamp(seqlen[b])``
    inside the kernel (no per-step gather)."""
    op = "apply_qkv_decode"
    if qkv.ndim != 2:
        raise ValueError(f"apply_qkv_decode expects [B, qkv], got {tuple(qkv.shape)}.")
    if not use_qk_norm:
        raise ValueError("apply_qkv_decode requires QK RMSNorm.")
    require_cuda(op, qkv, k_cache, v_cache, seqlen)
    bsz = qkv.shape[0]
    if row_map is None and (k_cache.shape[0] != bsz or v_cache.shape[0] != bsz):
        raise ValueError(f"KV cache batch {k_cache.shape[0]} != qkv batch {bsz}.")
    if seqlen.numel() != bsz:
        raise ValueError(f"seqlen has {seqlen.numel()} entries, expected {bsz}.")
    if qkv.stride(1) != 1:
        raise ValueError("apply_qkv_decode needs a row-contiguous qkv.")
    if k_cache.stride(3) != 1 or k_cache.stride(2) != head_dim or k_cache.stride() != v_cache.stride():
        raise ValueError("KV caches must be [B, n_kv, T, D] with contiguous (T, D).")
    if k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype:
        raise TypeError("KV cache dtype must match qkv dtype.")
    if q_out is None:
        q_out = torch.empty(bsz, num_heads, 1, head_dim, device=qkv.device, dtype=qkv.dtype)
    rot = max(int(rotary_dim), 0) if use_rope else 0
    table_len = int(cos.shape[0]) if (use_rope and rope_table) else 0
    cos2 = (cos if rope_table else cos.reshape(bsz, -1)) if use_rope else None
    sin2 = (sin if rope_table else sin.reshape(bsz, -1)) if use_rope else None
    if use_rope and (cos2.stride(1) != 1 or sin2.stride(1) != 1 or cos2.stride(0) != sin2.stride(0)):
        cos2, sin2 = cos2.contiguous(), sin2.contiguous()
    sl = seqlen.reshape(-1).to(torch.int64)
    rm = row_map.reshape(-1).to(torch.int32) if row_map is not None else None
    qw = q_weight.reshape(-1).contiguous()
    kw = k_weight.reshape(-1).contiguous().to(qw.dtype)
    check(lib().maple_apply_qkv_decode(
        ptr(qkv), dtype_code(qkv, op), bsz, qkv.stride(0), ptr(qw), ptr(kw), dtype_code(qw, op), ptr(cos2), ptr(sin2),
        dtype_code(cos2, op) if cos2 is not None else 0, cos2.stride(0) if cos2 is not None else 0, table_len,
        ptr(q_out),
        q_out.stride(0), q_out.stride(1), ptr(k_cache), ptr(v_cache), k_cache.shape[0], k_cache.stride(0),
        k_cache.stride(1), k_cache.shape[2], ptr(sl), ptr(rm), num_heads, num_kv_heads, head_dim, rot,
        int(bool(use_rope)), float(eps), ptr(_err(qkv.device)), stream_ptr(qkv.device)), op)
    return q_out


_BLOCK_T = 64
_MAX_SPLITS = 8


def gqa_splits(max_len: int, window: int | None) -> int:
    """Reference kernels/decode_attn.py:446-467 (split count of the reference's
    grid); kept for API compatibility.  The sm_100a kernel splits by length,
    see :func:`attn_split_len`."""
    span = max_len if window is None else min(max_len, window)
    tiles = max(1, -(-span // _BLOCK_T))
    if tiles <= 8:
        return 1
    splits = 1
    while splits < min(_MAX_SPLITS, tiles):
        splits *= 2
    return splits


def attn_split_len(max_len: int, batch: int = 1, num_kv_heads: int = 4) -> int:
    """Positions per attention split (32, 64 or 128), a CUDA-graph constant
    fixed with the cache and part of the canonical arithmetic.  Contexts up to
    1024 use 64 (at most 16 splits, merged inside one thread-block cluster);
    longer ones the largest split whose grid still covers ~2 waves of 148 SMs."""
    if max_len <= 1024:
        return 64
    for p in (128, 64):
        if batch * num_kv_heads * -(-max_len // p) >= 296:
            return p
    return 32


def decode_gqa_attn(q, k_cache, v_cache, seqlen, *, row_map=None, scale: float, window: int | None,
                    workspace=None, split_len: int | None = None, kv_final: bool = False,
                    tensor_cores: bool = False):
    """GQA attention for ``q_len=1``.  Reference kernels/decode_attn.py:470-592.
    ``q`` is ``[B, H, 1, D]``, caches ``[B, n_kv, T, D]``; ``seqlen[b]`` is the
    index just written.  ``workspace`` may be a byte tensor from
    :func:`attn_workspace` (a reference-style tuple is accepted and ignored).
    ``kv_final`` promises K/V before ``seqlen[b]`` was written before the
    previous launch (decode rows), so those rows can load early.

    ``tensor_cores`` (bf16 caches, head_dim 64/128): the reference kernel's
    own arithmetic -- bf16 q.K^T and P.V dots with fp32 accumulation, P
    rounded to bf16 -- on the tensor pipe (``maple_decode_gqa_attn_tc``), for
    long contexts and large batches where the CUDA-core path is
    instruction-bound.  Its sums are in the tensor pipe's order, so it agrees
    with the canonical fp32 path to the attention tolerance, not bit for bit."""
    op = "decode_gqa_attn"
    if q.ndim != 4 or q.shape[2] != 1:
        raise ValueError(f"decode_gqa_attn expects q [B, H, 1, D], got {tuple(q.shape)}.")
    require_cuda(op, q, k_cache, v_cache, seqlen)
    bsz, n_q, _, head_dim = q.shape
    if row_map is None and (k_cache.shape[0] != bsz or v_cache.shape[0] != bsz):
        raise ValueError(f"KV cache batch {k_cache.shape[0]} != q batch {bsz}.")
    if seqlen.numel() != bsz:
        raise ValueError(f"seqlen has {seqlen.numel()} entries, expected {bsz}.")
    n_kv, max_len = k_cache.shape[1], k_cache.shape[2]
    if n_q % n_kv != 0:
        raise ValueError(f"n_q={n_q} not divisible by n_kv={n_kv}.")
    if k_cache.stride(3) != 1 or k_cache.stride(2) != head_dim or k_cache.stride() != v_cache.stride():
        raise ValueError("KV caches must be [B, n_kv, T, D] with contiguous (T, D).")
    out = torch.empty_like(q)
    q3, o3 = q[:, :, 0, :], out[:, :, 0, :]
    L = lib()
    if tensor_cores:
        if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
            raise TypeError("tensor-core decode attention needs bf16 q and caches.")
        nbytes = L.maple_decode_gqa_attn_tc_workspace_bytes(bsz, n_q, head_dim, max_len)
        ws = workspace if isinstance(workspace, torch.Tensor) and workspace.numel() >= nbytes else _ws(q.device, nbytes)
        sl = seqlen.reshape(-1).to(torch.int64)
        rm = row_map.reshape(-1).to(torch.int32) if row_map is not None else None
        check(L.maple_decode_gqa_attn_tc(
            ptr(q3), dtype_code(q, op), bsz, n_q, q3.stride(0), q3.stride(1), ptr(k_cache), ptr(v_cache),
            k_cache.shape[0], n_kv, k_cache.stride(0), k_cache.stride(1), max_len, head_dim, ptr(sl), ptr(rm),
            float(scale), int(window or 0), ptr(o3), o3.stride(0), o3.stride(1), ptr(ws),
            ws.numel() if ws is not None else 0, ptr(_err(q.device)), stream_ptr(q.device)), op)
        return out
    P = split_len or attn_split_len(max_len, bsz, n_kv)
    nbytes = L.maple_decode_gqa_workspace_bytes(bsz, n_q, head_dim, max_len, P) if -(-max_len // P) > 16 else 0
    ws = workspace if isinstance(workspace, torch.Tensor) and workspace.numel() >= nbytes else _ws(q.device, nbytes)
    sl = seqlen.reshape(-1).to(torch.int64)
    rm = row_map.reshape(-1).to(torch.int32) if row_map is not None else None
    check(L.maple_decode_gqa_attn(
        ptr(q3), dtype_code(q, op), bsz, n_q, q3.stride(0), q3.stride(1), ptr(k_cache), ptr(v_cache), k_cache.shape[0],
        n_kv, k_cache.stride(0), k_cache.stride(1), max_len, head_dim, ptr(sl), ptr(rm), float(scale),
        int(window or 0), P, int(bool(kv_final)), ptr(o3), o3.stride(0), o3.stride(1), ptr(ws),
        ws.numel() if ws is not None else 0, ptr(_err(q.device)),
        stream_ptr(q.device)), op)
    return out


def decode_gqa_attn_qk(qkv, q_weight, k_weight, cos, sin, k_cache, v_cache, seqlen, *, row_map=None, num_heads,
                       num_kv_heads, head_dim, rotary_dim, use_rope, eps, scale: float, window: int | None,
                       split_len: int | None = None):
    """:func:`apply_qkv_decode` (RoPE tables read at ``clamp(seqlen[b])``)
    followed by :func:`decode_gqa_attn` with ``kv_final`` in one launch: the
    decode branch of reference model.py:368-414 over kernels/decode_attn.py
    :362-439 and :470-592.  Every K/V position before ``seqlen[b]`` must be
    final (decode rows, not a prompt's rows).  Returns ``[B, H, 1, D]``; the
    new K/V rows are written to the caches as apply_qkv_decode writes them."""
    op = "decode_gqa_attn_qk"
    if qkv.ndim != 2 or qkv.stride(1) != 1:
        raise ValueError(f"decode_gqa_attn_qk expects a row-contiguous [B, qkv], got {tuple(qkv.shape)}.")
    require_cuda(op, qkv, k_cache, v_cache, seqlen)
    bsz = qkv.shape[0]
    if row_map is None and (k_cache.shape[0] != bsz or v_cache.shape[0] != bsz):
        raise ValueError(f"KV cache batch {k_cache.shape[0]} != qkv batch {bsz}.")
    if seqlen.numel() != bsz:
        raise ValueError(f"seqlen has {seqlen.numel()} entries, expected {bsz}.")
    if k_cache.stride(3) != 1 or k_cache.stride(2) != head_dim or k_cache.stride() != v_cache.stride():
        raise ValueError("KV caches must be [B, n_kv, T, D] with contiguous (T, D).")
    if k_cache.dtype != qkv.dtype or v_cache.dtype != qkv.dtype:
        raise TypeError("KV cache dtype must match qkv dtype.")
    if num_heads % num_kv_heads:
        raise ValueError(f"n_q={num_heads} not divisible by n_kv={num_kv_heads}.")
    n_kv, max_len = k_cache.shape[1], k_cache.shape[2]
    P = split_len or attn_split_len(max_len, bsz, n_kv)
    out = torch.empty(bsz, num_heads, 1, head_dim, device=qkv.device, dtype=qkv.dtype)
    o3 = out[:, :, 0, :]
    L = lib()
    nbytes = L.maple_decode_gqa_workspace_bytes(bsz, num_heads, head_dim, max_len, P) if -(-max_len // P) > 16 else 0
    ws = _ws(qkv.device, nbytes)
    sl = seqlen.reshape(-1).to(torch.int64)
    rm = row_map.reshape(-1).to(torch.int32) if row_map is not None else None
    qw = q_weight.reshape(-1).contiguous()
    kw = k_weight.reshape(-1).contiguous().to(qw.dtype)
    rot = max(int(rotary_dim), 0) if use_rope else 0
    if use_rope and (cos.stride(1) != 1 or sin.stride(1) != 1 or cos.stride(0) != sin.stride(0)):
        cos, sin = cos.contiguous(), sin.contiguous()
    check(L.maple_decode_gqa_attn_qk(
        ptr(qkv), dtype_code(qkv, op), bsz, qkv.stride(0), ptr(qw), ptr(kw), dtype_code(qw, op),
        ptr(cos) if use_rope else None, ptr(sin) if use_rope else None, dtype_code(cos, op) if use_rope else 0,
        cos.stride(0) if use_rope else 0, int(cos.shape[0]) if use_rope else 0, rot, int(bool(use_rope)), float(eps),
        num_heads, ptr(k_cache), ptr(v_cache), k_cache.shape[0], n_kv, k_cache.stride(0), k_cache.stride(1), max_len,
        head_dim, ptr(sl), ptr(rm), float(scale), int(window or 0), P, ptr(o3), o3.stride(0), o3.stride(1), ptr(ws),
        ws.numel() if ws is not None else 0, ptr(_err(qkv.device)), stream_ptr(qkv.device)), op)
    return out


def _rtn4_common(x, packed_weight, scales, biases, op):
    require_cuda(op, x, packed_weight, scales, biases)
    _u32(packed_weight, op)
    if biases is not None and biases.dtype != scales.dtype:
        biases = biases.to(scales.dtype)
    return biases


def rtn4_gemv(x, packed_weight, scales, biases, group_size: int = 64, *, packed_kn: bool = False):
    """Decode GEMV with a 4-bit RTN weight (``code*scale + bias``).  Reference
    kernels/rtn4.py:285-415.  ``biases=None`` means symmetric (bias = -8*scale)."""
    op = "rtn4_gemv"
    if packed_weight.dtype != torch.uint32:
        raise TypeError(f"packed_weight must be uint32 codes, got {packed_weight.dtype}; "
                        "refusing to run a dense-weight path.")
    if packed_weight.ndim != 2:
        raise ValueError(f"packed_weight must be 2-D [N, K/8] or [K/8, N]; got shape {tuple(packed_weight.shape)}.")
    if not x.is_cuda or not packed_weight.is_cuda:
        raise RuntimeError("rtn4_gemv requires CUDA tensors.")
    biases = _rtn4_common(x, packed_weight, scales, biases, op)
    if packed_kn:
        packed_weight, scales = packed_weight.t(), scales.t()
        biases = biases.t() if biases is not None else None
    w = packed_weight.contiguous()
    n_out, nwords = w.shape
    n_groups = nwords * 8 // group_size
    if tuple(scales.shape) != (n_out, n_groups) or (biases is not None and tuple(biases.shape) != (n_out, n_groups)):
        raise ValueError(f"scales/biases expected {(n_out, n_groups)}, got {tuple(scales.shape)} and "
                         f"{None if biases is None else tuple(biases.shape)}.")
    k_in = nwords * 8
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    leading = x.shape[:-1]
    xm = x.reshape(-1, k_in).contiguous()
    batch = xm.shape[0]
    s = scales.contiguous()
    b = biases.contiguous() if biases is not None else None
    y = torch.empty(batch, n_out, device=x.device, dtype=x.dtype)
    L = lib()
    if batch >= HEAD_GEMM_MIN_ROWS and k_in <= 4096:
        # rows encoded once, the head streamed once per chunk of 16 rows
        scratch = torch.empty(L.maple_rtn4_frag_bytes(batch, k_in), dtype=torch.uint8, device=x.device)
        check(L.maple_rtn4_gemm(ptr(xm), dtype_code(x, op), batch, k_in, k_in, ptr(w), n_out, ptr(s), ptr(b),
                                dtype_code(s, op), group_size, ptr(y), n_out, ptr(scratch), scratch.numel(),
                                ptr(_err(x.device)), stream_ptr(x.device)), op)
        return y.reshape(*leading, n_out)
    check(L.maple_rtn4_gemv(ptr(xm), dtype_code(x, op), batch, k_in, k_in, ptr(w), n_out, ptr(s), ptr(b),
                            dtype_code(s, op), group_size, ptr(y), n_out, stream_ptr(x.device)), op)
    return y.reshape(*leading, n_out)


def rtn4_indexed_gemv(x, packed_weight, scales, biases, cluster_ids, group_size: int = 64):
    """GEMV over FlashHead clusters ``head[cluster_ids[n // C], n % C]``.
    Reference kernels/rtn4.py:514-611.  Output ``[..., n_probes * C]``."""
    op = "rtn4_indexed_gemv"
    if packed_weight.dtype != torch.uint32:
        raise TypeError(f"packed_weight must be uint32 codes, got {packed_weight.dtype}; "
                        "refusing to run a dense-weight path.")
    if packed_weight.ndim != 3:
        raise ValueError(f"packed_weight must be 3-D [n_clusters, cluster_size, nwords]; got shape "
                         f"{tuple(packed_weight.shape)}.")
    if not x.is_cuda or not packed_weight.is_cuda:
        raise RuntimeError("rtn4_indexed_gemv requires CUDA tensors.")
    if cluster_ids.ndim != 1:
        raise ValueError(f"cluster_ids must be 1-D [n_probes]; got shape {tuple(cluster_ids.shape)}.")
    biases = _rtn4_common(x, packed_weight, scales, biases, op)
    n_clusters, csize, nwords = packed_weight.shape
    n_groups = nwords * 8 // group_size
    expect = (n_clusters, csize, n_groups)
    if tuple(scales.shape) != expect or (biases is not None and tuple(biases.shape) != expect):
        raise ValueError(f"scales/biases expected {expect}.")
    k_in = nwords * 8
    if x.shape[-1] != k_in:
        raise ValueError(f"x last dim {x.shape[-1]} != packed K ({k_in}).")
    leading = x.shape[:-1]
    xm = x.reshape(-1, k_in).contiguous()
    batch = xm.shape[0]
    n_probes = int(cluster_ids.shape[0])
    ids = cluster_ids.to(torch.int32).contiguous()
    w, s = packed_weight.contiguous(), scales.contiguous()
    b = biases.contiguous() if biases is not None else None
    n_out = n_probes * csize
    y = torch.empty(batch, n_out, device=x.device, dtype=x.dtype)
    check(lib().maple_rtn4_indexed_gemv(ptr(xm), dtype_code(x, op), batch, k_in, k_in, ptr(w), n_clusters, csize,
                                        ptr(s), ptr(b), dtype_code(s, op), group_size, ptr(ids), n_probes, ptr(y),
                                        n_out, stream_ptr(x.device)), op)
    return y.reshape(*leading, n_out)


def rtn4_embedding(input_ids, packed_weight, scales, biases, group_size: int = 64, out_dtype=torch.float32):
    """Gather packed rows and dequantise them (fp32, as the reference).  Reference kernels/rtn4.py:27-47."""
    op = "rtn4_embedding"
    if packed_weight.dtype != torch.uint32:
        raise TypeError(f"packed_weight must be uint32 codes, got {packed_weight.dtype}.")
    require_cuda(op, input_ids, packed_weight, scales, biases)
    V, nwords = packed_weight.shape
    H = nwords * 8
    ids = input_ids.reshape(-1).to(torch.int64).contiguous()
    s = scales.contiguous()
    b = biases.contiguous().to(s.dtype) if biases is not None else None
    out = torch.empty(ids.numel(), H, device=ids.device, dtype=out_dtype)
    check(lib().maple_rtn4_embedding(ptr(ids), ids.numel(), ptr(packed_weight), ptr(s), ptr(b), dtype_code(s, op), V,
                                     H, group_size, ptr(out), dtype_code(out, op), H, ptr(_err(ids.device)),
                                     stream_ptr(ids.device)), op)
    return out.reshape(*input_ids.shape, H)


def embedding(input_ids, table, out_dtype=None):
    """Plain embedding gather (the configs' bf16 table)."""
    op = "embedding"
    require_cuda(op, input_ids, table)
    V, H = table.shape
    ids = input_ids.reshape(-1).to(torch.int64).contiguous()
    out = torch.empty(ids.numel(), H, device=ids.device, dtype=out_dtype or table.dtype)
    check(lib().maple_embedding(ptr(ids), ids.numel(), ptr(table), dtype_code(table, op), V, H, ptr(out),
                                dtype_code(out, op), H, ptr(_err(ids.device)), stream_ptr(ids.device)), op)
    return out.reshape(*input_ids.shape, H)


def argmax(logits, out=None):
    """Greedy token: first index of the max over the last dim (int64).  Reference generate.py:147-148."""
    op = "argmax"
    require_cuda(op, logits)
    V = int(logits.shape[-1])
    lm = logits.reshape(-1, V)
    if lm.stride(1) != 1:
        lm = lm.contiguous()
    B = lm.shape[0]
    o = out if out is not None else torch.empty(B, device=logits.device, dtype=torch.int64)
    L = lib()
    ws = _ws(logits.device, L.maple_argmax_workspace_bytes(B, V))
    check(L.maple_argmax(ptr(lm), dtype_code(logits, op), B, V, lm.stride(0), ptr(o), ptr(ws),
                         ws.numel() if ws is not None else 0, stream_ptr(logits.device)), op)
    return o.reshape(logits.shape[:-1])


MAX_TOP_K = 64


def _sample(logits2d, uniform, temperature, top_p, top_k, workspace, out):
    op = "fused_sample"
    if not 0 < top_k <= MAX_TOP_K:
        raise ValueError(f"fused_sample needs 0 < top_k <= {MAX_TOP_K}, got {top_k}.")
    if temperature <= 0:
        raise ValueError("fused_sample needs temperature > 0 (greedy is argmax).")
    B, V = logits2d.shape
    if logits2d.stride(1) != 1:
        logits2d = logits2d.contiguous()
    u = uniform.reshape(-1).float().contiguous()
    if u.numel() != B:
        raise ValueError(f"uniform has {u.numel()} draws, expected {B}.")
    L = lib()
    nbytes = L.maple_fused_sample_workspace_bytes(B, V, top_k)
    ws = workspace if isinstance(workspace, torch.Tensor) and workspace.numel() >= nbytes else _ws(logits2d.device, nbytes)
    check(L.maple_fused_sample(ptr(logits2d), dtype_code(logits2d, op), B, V, logits2d.stride(0), ptr(u),
                               float(temperature), float(top_p), top_k, ptr(out), ptr(ws), ws.numel(),
                               stream_ptr(logits2d.device)), op)
    return out


def fused_sample(logits, uniform, *, temperature: float, top_p: float, top_k: int, workspace=None):
    """Sample one token id from 1-D ``logits`` with a caller uniform in [0, 1).
    Reference kernels/sampler.py:106-149.  Returns a 0-D int64 CUDA tensor."""
    if logits.ndim != 1:
        raise ValueError(f"fused_sample expects 1-D logits, got {tuple(logits.shape)}.")
    require_cuda("fused_sample", logits, uniform)
    out = torch.empty(1, device=logits.device, dtype=torch.int64)
    ws = workspace[0] if isinstance(workspace, tuple) else workspace
    return _sample(logits.reshape(1, -1), uniform, temperature, top_p, top_k, ws, out).reshape(())


def fused_sample_batched(logits, uniform, *, temperature: float, top_p: float, top_k: int, workspace=None):
    """One id per row of ``logits [B, V]``; ``uniform`` is ``[B]``.  Reference kernels/sampler.py:152-206."""
    if logits.ndim != 2:
        raise ValueError(f"fused_sample_batched expects [B, vocab], got {tuple(logits.shape)}.")
    require_cuda("fused_sample_batched", logits, uniform)
    out = torch.empty(logits.shape[0], device=logits.device, dtype=torch.int64)
    ws = workspace[0] if isinstance(workspace, tuple) else workspace
    return _sample(logits, uniform, temperature, top_p, top_k, ws, out)


class RowUniform:
    """Per-sequence uniforms for the fused sampler: row b draws
    splitmix64(seed_b, step) with the step counter kept on the device, so the
    draw can live inside a captured decode graph."""

    def __init__(self, seeds, device):
        self.seeds = torch.as_tensor(list(seeds), dtype=torch.int64).to(device).view(torch.uint64) \
            if not isinstance(seeds, torch.Tensor) else seeds.to(device=device, dtype=torch.int64).view(torch.uint64)
        self.counter = torch.zeros(1, dtype=torch.int64, device=device)
        self.out = torch.empty(self.seeds.numel(), dtype=torch.float32, device=device)

    def __call__(self) -> torch.Tensor:
        check(lib().maple_row_uniform(ptr(self.seeds), self.seeds.numel(), ptr(self.counter), ptr(self.out),
                                      stream_ptr(self.out.device)), "row_uniform")
        return self.out


def sampler_workspace(vocab: int, top_k: int, device):
    """Preallocated sampler scratch (zeroed; the kernel leaves it reusable).  Reference kernels/sampler.py:209."""
    return batched_sampler_workspace(vocab, top_k, 1, device)


def batched_sampler_workspace(vocab: int, top_k: int, batch: int, device):
    """Sampler scratch for up to ``batch`` rows.  Reference kernels/sampler.py:219."""
    n = lib().maple_fused_sample_workspace_bytes(batch, vocab, top_k)
    return (torch.zeros(n, dtype=torch.uint8, device=device),)
