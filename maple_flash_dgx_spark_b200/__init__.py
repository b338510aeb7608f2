"""maple-b200: B200-native (sm_100a) decode engine for packed 2-bit ternary MoE LMs.

A drop-in for the decode path of cloud-000/maple-flash-dgx-spark (``maple-run``):
the same operator names and signatures (``kernels``), packed linear wrappers
(``linear``), model / KV cache (``model``) and generate loop (``generate``),
with every kernel hand-written CUDA for sm_100a behind the C ABI declared in
``include/maple_b200.h``.
"""

from __future__ import annotations

__version__ = "0.1.0"
