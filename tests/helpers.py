"""Shared test helpers: seeded bf16-valued inputs and device transfer."""

from __future__ import annotations

import numpy as np

import oracle
from tests.golden.cases import pack2, ternary_codes


def rng(seed):
    return np.random.RandomState(seed)


def bf(a):
    return oracle.round_bf16(np.asarray(a, dtype=np.float32))


def randn_bf(rs, *shape, scale=1.0):
    return bf(rs.standard_normal(shape).astype(np.float32) * scale)


def tern_packed(rs, *shape):
    return pack2(ternary_codes(rs, shape))


def alpha_bf(rs, *shape):
    return bf(np.abs(rs.standard_normal(shape) * 0.02) + 1e-3)


def to_dev(a, dev, dtype=None):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(dev).view(torch.uint32)
    t = torch.from_numpy(a).to(dev)
    return t.to(dtype) if dtype is not None else t


def to_np(t):
    import torch

    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.detach().cpu().numpy()
