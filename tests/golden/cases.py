"""Seeded test cases shared by the golden-vector generator and the tests.

``inputs()`` regenerates a case's inputs with numpy's frozen ``RandomState``
stream (so fixtures store outputs only); ``run_reference(torch)`` runs the
reference's own code on them (see make_golden.py).
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


def ternary_codes(rs: np.random.RandomState, shape) -> np.ndarray:
    """Codes t+1 with P(t=0)=0.4, P(t=-1)=P(t=+1)=0.3."""
    u = rs.random_sample(shape)
    t = np.where(u < 0.4, 0, np.where(u < 0.7, -1, 1))
    return (t + 1).astype(np.uint32)


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


CASES = {
    "gemv_small": GemvCase(seed=10, batch=1, n=64, k=256, rms=False),
    "gemv_rms": GemvCase(seed=11, batch=1, n=96, k=512, rms=True),
    "gemv_batch": GemvCase(seed=12, batch=3, n=48, k=128, rms=True),
    "gemv_cfg0": GemvCase(seed=0, batch=1, n=4096, k=2048, rms=False, bf16_inputs=True),
}
