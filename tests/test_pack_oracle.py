"""The oracle's packing restatement and FlashHead top-k rule, pinned against
the reference's own pack.py outputs (tests/golden/reference_pack.npz, made by
tests/golden/make_pack_golden.py).  CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from tests.golden.make_pack_golden import RTN, TERNARIZE, rtn_input, ternarize_input

GOLD = np.load(Path(__file__).parent / "golden" / "reference_pack.npz")


@pytest.mark.parametrize("seed,n,k", TERNARIZE)
def test_oracle_ternarize_equals_reference(seed, n, k):
    packed, alpha = oracle.ternarize(ternarize_input(seed, n, k))
    np.testing.assert_array_equal(packed, GOLD[f"tern_{seed}_packed"])
    np.testing.assert_array_equal(alpha, GOLD[f"tern_{seed}_alpha"])


@pytest.mark.parametrize("seed,n,k,g", RTN)
def test_oracle_rtn_equals_reference(seed, n, k, g):
    packed, scales, biases = oracle.quantize_rtn(rtn_input(seed, n, k), group_size=g)
    np.testing.assert_array_equal(packed, GOLD[f"rtn_{seed}_packed"])
    np.testing.assert_array_equal(scales, GOLD[f"rtn_{seed}_scales"])
    np.testing.assert_array_equal(biases, GOLD[f"rtn_{seed}_biases"])


def test_oracle_pack_overflowing_codes_equal_reference():
    np.testing.assert_array_equal(oracle.pack_2bit(GOLD["pack_overflow_codes"]), GOLD["pack_overflow_words"])


def test_topk_select_rule():
    rs = np.random.RandomState(0)
    for n, k in [(4748, 512), (100, 100), (37, 1), (64, 63)]:
        x = np.round(rs.standard_normal(n) * 4).astype(np.float32)  # many ties
        x[rs.randint(0, n)] = np.nan
        sel = oracle.topk_select(x, k)
        key = np.where(np.isnan(x), np.inf, x)
        # brute force: sort by (value desc, index asc)
        want = sorted(range(n), key=lambda i: (-key[i], i))[:k]
        np.testing.assert_array_equal(sel, np.sort(want))
