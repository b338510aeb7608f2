"""Device-side failure reporting (GPU, no fault).

Every wait inside the library's kernels is bounded: a wait that gives up sets
bit 1 of the device error word and the kernel returns, so the context stays
usable and the host learns of it at its next check
(``_lib.raise_device_errors``).  Here a peer-flag wait is made to run out on
one GPU: the expert-parallel dispatch is told there are two ranks, and the
second "peer" buffer is an ordinary local buffer that no rank ever signals
through.  Nothing faults or hangs: the wait gives up after about a second.
"""

from __future__ import annotations

import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_peer_flag_wait_gives_up_and_is_reported(cuda):
    from maple_flash_dgx_spark_b200 import _lib

    L = _lib.lib()
    T, H, k = 4, 512, 2
    code = _lib.dtype_code(torch.empty(0, dtype=torch.bfloat16), "t")
    total = L.maple_p2p_dispatch_bytes(2, T, H, code, k)
    mine = torch.zeros(total, dtype=torch.uint8, device=cuda)
    silent_peer = torch.zeros(total, dtype=torch.uint8, device=cuda)  # nobody sends to us from here
    bases = (ctypes.c_void_p * 2)(mine.data_ptr(), silent_peer.data_ptr())
    x = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    ids = torch.randint(0, 8, (T, k), dtype=torch.int32, device=cuda)
    rows = torch.zeros(2 * T, H, dtype=torch.bfloat16, device=cuda)
    ids_all = torch.zeros(2 * T, k, dtype=torch.int32, device=cuda)
    state = torch.zeros(2, dtype=torch.int32, device=cuda)  # seq, ticket
    err = _lib.error_word(cuda)
    _lib.take_device_errors(cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rc = L.maple_p2p_dispatch(bases, 2, 0, 0, x.data_ptr(), code, H, T, H, ids.data_ptr(), k, rows.data_ptr(),
                              ids_all.data_ptr(), state.data_ptr(), state.data_ptr() + 4, err.data_ptr(), stream)
    assert rc == 0
    torch.cuda.synchronize(cuda)  # returns: the polls for the silent rank's words are bounded
    # this rank's own rows and ids still arrived through its own area
    assert torch.equal(rows[:T], x) and torch.equal(ids_all[:T], ids)
    with pytest.raises(RuntimeError, match="bounded device wait gave up"):
        _lib.raise_device_errors(cuda, "p2p dispatch with a silent peer")
    assert _lib.take_device_errors(cuda) == 0  # read and cleared
    assert int(state[0]) == 1 and int(state[1]) == 0  # the call still completed its bookkeeping
    x = torch.arange(16, device=cuda, dtype=torch.float32)
    assert float(x.sum()) == 120.0  # the context is intact
