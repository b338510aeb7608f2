"""Packed linear layers: hold codes + scales and call the sm_100a operators.

Reference: linear.py:16-111 (PackedTernaryLinear, PackedTernaryExperts,
PackedRTN4Linear, PackedRTN4Embedding).  The reference passes every output
through ``eggroll.perturb.add_adapter_delta``, a no-op unless an EGGROLL
adapter is attached; adapters are outside this engine's scope, so the hook is
not called.
"""

from __future__ import annotations

from maple_flash_dgx_spark_b200.kernels import (
    embedding,
    rtn4_embedding,
    rtn4_gemv,
    ternary_expert_down_reduce,
    ternary_expert_down_sum,
    ternary_expert_gemv,
    ternary_expert_swiglu,
    ternary_gemv,
)

HEAD_GROUP_SIZE = 64


class PackedTernaryLinear:
    """Codes stay in the checkpoint's ``[N, K/16]`` order (reference linear.py:16-41)."""

    def __init__(self, packed_weight, row_alpha):
        self.packed_weight = packed_weight.contiguous()
        self.row_alpha = row_alpha.contiguous()

    def forward(self, x, rms_weight=None, rms_eps: float = 1e-6):
        return ternary_gemv(x, self.packed_weight, self.row_alpha, rms_weight=rms_weight, rms_eps=rms_eps)

    __call__ = forward


class PackedTernaryExperts:
    """Stacked experts ``[E, N, K/16]``; one launch over the selected ids (reference linear.py:44-69)."""

    def __init__(self, packed_weight, row_alpha):
        self.packed_weight = packed_weight.contiguous()
        self.row_alpha = row_alpha.contiguous()

    def forward(self, x, expert_ids, plan=None):
        return ternary_expert_gemv(x, self.packed_weight, self.row_alpha, expert_ids, plan=plan)

    def swiglu(self, x, expert_ids, plan=None):
        return ternary_expert_swiglu(x, self.packed_weight, self.row_alpha, expert_ids, plan=plan)

    def down_sum(self, x, expert_ids, topk_weight, residual=None):
        return ternary_expert_down_sum(x, self.packed_weight, self.row_alpha, expert_ids, topk_weight,
                                       residual=residual)

    def down_reduce(self, x, expert_ids, topk_weight, residual=None, plan=None):
        """Down projection + the model's weighted combine + residual (the
        rounding of ``forward`` followed by ``moe_reduce_add``)."""
        return ternary_expert_down_reduce(x, self.packed_weight, self.row_alpha, expert_ids, topk_weight,
                                          residual=residual, plan=plan)

    __call__ = forward


class PackedRTN4Linear:
    """4-bit head ``[N, K/8]`` (reference linear.py:72-92).  ``biases=None``
    means a symmetric head (bias = -8 * scale)."""

    def __init__(self, packed_weight, scales, biases, group_size: int = HEAD_GROUP_SIZE):
        self.packed_weight = packed_weight.contiguous()
        self.scales = scales.contiguous()
        self.biases = None if biases is None else biases.contiguous()
        self.group_size = group_size

    def forward(self, x):
        return rtn4_gemv(x, self.packed_weight, self.scales, self.biases, group_size=self.group_size)

    __call__ = forward


class PackedRTN4Embedding:
    """Reference linear.py:95-111: gather + dequant of the selected rows (fp32 out)."""

    def __init__(self, packed_weight, scales, biases, group_size: int = HEAD_GROUP_SIZE):
        self.packed_weight = packed_weight
        self.scales = scales
        self.biases = biases
        self.group_size = group_size

    def forward(self, input_ids):
        return rtn4_embedding(input_ids, self.packed_weight, self.scales, self.biases, group_size=self.group_size)

    __call__ = forward


class DenseEmbedding:
    """Plain ``[V, H]`` table (the benchmark configs' bf16 embedding)."""

    def __init__(self, weight):
        self.weight = weight.contiguous()

    def forward(self, input_ids):
        return embedding(input_ids, self.weight)

    __call__ = forward
