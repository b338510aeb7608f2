"""The no-allocation ternary GEMV entry point (GPU).

maple_ternary_gemv_noalloc serves callers that cannot allocate device memory
(a host binding the library through a thin FFI with only its input and output
buffers, or a serving loop whose memory is all reserved): its split-K scratch
is a fixed array inside the library instead of a caller workspace.  It must
return exactly what maple_ternary_gemv returns, call after call, since every
call reuses the same array.  This file is collected last on purpose.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import alpha_bf, randn_bf, rng, tern_packed, to_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16 = 1


def _inputs(dev, batch, n, k, rms, seed):
    rs = rng(seed)
    x = to_dev(randn_bf(rs, batch, k), dev, torch.bfloat16)
    codes = to_dev(tern_packed(rs, n, k), dev)
    alpha = to_dev(alpha_bf(rs, n), dev, torch.bfloat16)
    w = to_dev((1 + 0.02 * rs.standard_normal(k)).astype(np.float32), dev) if rms else None
    return x, codes, alpha, w


def _with_workspace(L, x, codes, alpha, w, batch, n, k, stream):
    y = torch.empty(batch, n, dtype=torch.bfloat16, device=x.device)
    nbytes = L.maple_ternary_gemv_workspace_bytes(batch, n, k)
    ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    rc = L.maple_ternary_gemv(x.data_ptr(), BF16, batch, k, k, codes.data_ptr(), n, alpha.data_ptr(), BF16,
                              None if w is None else w.data_ptr(), 0, 1e-6, y.data_ptr(), n, ws.data_ptr(),
                              ws.numel(), stream)
    assert rc == 0
    return y


def _no_alloc(L, x, codes, alpha, w, batch, n, k, stream):
    y = torch.full((batch, n), float("nan"), dtype=torch.bfloat16, device=x.device)
    rc = L.maple_ternary_gemv_noalloc(x.data_ptr(), BF16, batch, k, k, codes.data_ptr(), n, alpha.data_ptr(), BF16,
                                      None if w is None else w.data_ptr(), 0, 1e-6, y.data_ptr(), n, stream)
    return rc, y


# k=2048: one K split (no scratch); 4096: two; 6144: three; 8192: four splits,
# whose last-arriving CTA sums the partials of the others through the scratch
@pytest.mark.parametrize("batch,n,k,rms", [(1, 2048, 4096, False), (3, 1000, 4096, True), (2, 512, 2048, True),
                                           (1, 1024, 6144, False), (1, 1024, 6144, True), (2, 512, 8192, True),
                                           (2, 512, 8192, False)])
def test_no_alloc_equals_workspace_entry_point(cuda, batch, n, k, rms):
    from maple_flash_dgx_spark_b200._lib import lib

    L = lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    x, codes, alpha, w = _inputs(cuda, batch, n, k, rms, seed=batch * 1000 + n)
    want = _with_workspace(L, x, codes, alpha, w, batch, n, k, stream)
    for _ in range(2):  # the shared scratch must come back clean for the next call
        rc, got = _no_alloc(L, x, codes, alpha, w, batch, n, k, stream)
        torch.cuda.synchronize(cuda)
        assert rc == 0
        torch.testing.assert_close(got, want, rtol=0, atol=0)


def test_no_alloc_rejects_requests_beyond_its_scratch(cuda):
    from maple_flash_dgx_spark_b200._lib import lib

    L = lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    batch, n, k = 64, 2048, 4096  # 64 * 2 splits * 2048 rows * 16 B = 4 MiB > 2 MiB - 16 KiB
    x, codes, alpha, w = _inputs(cuda, batch, n, k, False, seed=9)
    rc, _ = _no_alloc(L, x, codes, alpha, w, batch, n, k, stream)
    assert rc == 8  # MAPLE_ERR_SCRATCH_LIMIT, nothing launched
