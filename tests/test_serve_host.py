"""Host-side request logic of the continuous-batching worker (CPU)."""

from __future__ import annotations

import pytest


def test_resolve_max_tokens():
    """Reference generate.py:31-38: -1 = the rest of the context; caps clip to it."""
    from maple_flash_dgx_spark_b200.generate import resolve_max_tokens

    assert resolve_max_tokens(-1, 4, 16) == 12
    assert resolve_max_tokens(64000, 4, 16) == 12
    assert resolve_max_tokens(5, 4, 16) == 5
    assert resolve_max_tokens(0, 4, 16) == 0
    assert resolve_max_tokens(8, 20, 16) == 0
    with pytest.raises(ValueError):
        resolve_max_tokens(-2, 4, 16)


def test_engine_defaults_and_sampling_records():
    from maple_flash_dgx_spark_b200.serve import DEFAULT_MAX_BATCH, DEFAULT_MAX_LEN, Sampling, ServerDefaults

    d = ServerDefaults()
    assert (d.max_batch, d.max_len) == (DEFAULT_MAX_BATCH, DEFAULT_MAX_LEN)
    s = Sampling(temperature=0.0, top_p=1.0, top_k=1, max_tokens=4, seed=None)
    with pytest.raises(Exception):
        s.top_k = 2  # frozen, as the reference's record
