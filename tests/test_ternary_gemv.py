"""sm_100a ternary GEMV vs the CPU oracle: bit-exact (GPU)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden.cases import CASES, GemvCase, bf16_round, pack2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(case: GemvCase, dev, x_dtype):
    from maple_flash_dgx_spark_b200.kernels import ternary_gemv

    d = case.inputs()
    x = d["x"] if x_dtype == torch.float32 else bf16_round(d["x"])
    xt = torch.from_numpy(x).to(dev, x_dtype)
    packed = torch.from_numpy(d["packed"].view(np.int32)).to(dev).view(torch.uint32)
    alpha = torch.from_numpy(d["alpha"]).to(dev)
    w = None if d["rms_weight"] is None else torch.from_numpy(d["rms_weight"]).to(dev)
    y = ternary_gemv(xt, packed, alpha, rms_weight=w, rms_eps=1e-6)
    y_or = oracle.ternary_gemv(x, d["packed"], d["alpha"], d["rms_weight"], 1e-6,
                               out_bf16=x_dtype == torch.bfloat16)
    return y.float().cpu().numpy(), y_or


@pytest.mark.parametrize("x_dtype", ["f32", "bf16"])
@pytest.mark.parametrize(
    "case",
    [
        *[c for c in CASES.values() if c.kind == "ternary_gemv"],
        GemvCase(seed=21, batch=1, n=5120, k=2048, rms=True),     # cfg1 QKV (fused RMSNorm)
        GemvCase(seed=22, batch=1, n=2048, k=4096, rms=False),    # cfg1 O proj
        GemvCase(seed=23, batch=2, n=2048, k=1024, rms=False),    # expert down shape
        GemvCase(seed=24, batch=1, n=37, k=64, rms=True),         # ragged N, tiny K
        GemvCase(seed=25, batch=5, n=300, k=1472, rms=True),      # partial K iteration
    ],
    ids=lambda c: f"b{c.batch}n{c.n}k{c.k}{'r' if c.rms else ''}" if isinstance(c, GemvCase) else c,
)
def test_gemv_bit_exact_vs_oracle(cuda, case, x_dtype):
    dt = torch.float32 if x_dtype == "f32" else torch.bfloat16
    y, y_or = _run(case, cuda, dt)
    np.testing.assert_array_equal(y, y_or)


def test_gemv_lsb_first_known_codes(cuda):
    """Reference tests/test_ternary_gemv.py:115-132: code 2 -> +alpha, 0 -> -alpha."""
    from maple_flash_dgx_spark_b200.kernels import ternary_gemv

    codes = np.ones((2, 128), dtype=np.uint32)
    codes[0, 0] = 2
    codes[1, 1] = 0
    packed = torch.from_numpy(pack2(codes).view(np.int32)).to(cuda).view(torch.uint32)
    alpha = torch.tensor([0.5, 1.25], device=cuda)
    x = torch.arange(128, dtype=torch.float32, device=cuda)
    y = ternary_gemv(x, packed, alpha)
    assert y.shape == (2,)
    torch.testing.assert_close(y, torch.tensor([0.0, -1.25], device=cuda), rtol=0, atol=0)


def test_gemv_vs_dequantized_linear(cuda):
    """Within the reference's own tolerance of dequantized F.linear (1e-4 fp32)."""
    from maple_flash_dgx_spark_b200.kernels import ternary_gemv

    rng = np.random.default_rng(1)
    w = rng.standard_normal((512, 2048)).astype(np.float32)
    packed, alpha = oracle.ternarize(w)
    x = torch.from_numpy(rng.standard_normal((4, 2048)).astype(np.float32)).to(cuda)
    pt = torch.from_numpy(packed.view(np.int32)).to(cuda).view(torch.uint32)
    at = torch.from_numpy(alpha).to(cuda)
    y = ternary_gemv(x, pt, at)
    w_hat = torch.from_numpy((oracle.unpack_2bit(packed).astype(np.float32) - 1) * alpha[:, None]).to(cuda)
    torch.testing.assert_close(y, x @ w_hat.T, rtol=1e-4, atol=1e-4)


def test_gemv_errors(cuda):
    from maple_flash_dgx_spark_b200.kernels import ternary_gemv

    x = torch.randn(1, 128, device=cuda)
    p = torch.zeros(4, 8, dtype=torch.int32, device=cuda)
    a = torch.ones(4, device=cuda)
    with pytest.raises(TypeError, match="dense-weight"):
        ternary_gemv(x, p, a)
    with pytest.raises(ValueError):
        ternary_gemv(x, p.view(torch.uint32)[:, :4], a)
    with pytest.raises(RuntimeError):
        ternary_gemv(x.cpu(), p.view(torch.uint32), a)


def test_gemv_repeated_calls_reuse_workspace(cuda):
    """Split-K tickets are reset by the kernel, so back-to-back calls agree."""
    case = GemvCase(seed=31, batch=1, n=5120, k=2048, rms=True)
    y1, y_or = _run(case, cuda, torch.bfloat16)
    y2, _ = _run(case, cuda, torch.bfloat16)
    np.testing.assert_array_equal(y1, y_or)
    np.testing.assert_array_equal(y2, y_or)
