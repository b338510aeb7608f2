"""The CUDA balanced spherical k-means (csrc/kmeans.cu, driven by
flash_head.balanced_spherical_kmeans) against the oracle restatement, which
tests/test_kmeans_oracle.py pins to the reference's own k-means: labels and
centroids bit for bit (GPU)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle.kmeans import balanced_kmeans, km_dots
from tests.golden.make_kmeans_golden import CASES, unit_rows

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).parent / "golden" / "kmeans_golden.npz")


def _gpu_kmeans(w, k, init, iters, cuda):
    from maple_flash_dgx_spark_b200.flash_head import balanced_spherical_kmeans

    cent, labels = balanced_spherical_kmeans(torch.from_numpy(w).to(cuda), k, n_iter=iters,
                                             init=torch.from_numpy(np.asarray(init)).to(cuda))
    return cent.cpu().numpy(), labels.cpu().numpy()


@pytest.mark.parametrize("name", sorted(CASES))
def test_kmeans_equals_oracle_and_reference(cuda, name):
    n, d, c, iters, dseed, _ = CASES[name]
    w = unit_rows(n, d, dseed)
    init = GOLD[f"{name}.init"]
    cent, labels = _gpu_kmeans(w, c, init, iters, cuda)
    o_cent, o_labels, _ = balanced_kmeans(w, c, init, iters)
    np.testing.assert_array_equal(labels, o_labels)
    np.testing.assert_array_equal(cent, o_cent)
    np.testing.assert_array_equal(labels, GOLD[f"{name}.labels"])  # the reference's own clustering


def test_kmeans_larger_case_equals_oracle(cuda):
    """16384 rows of 256 into 512 clusters of 32 (many evictions per
    iteration), random init rows."""
    w = unit_rows(16384, 256, 5)
    init = np.random.default_rng(6).permutation(16384)[:512]
    cent, labels = _gpu_kmeans(w, 512, init, 4, cuda)
    o_cent, o_labels, _ = balanced_kmeans(w, 512, init, 4)
    assert np.bincount(labels, minlength=512).tolist() == [32] * 512
    np.testing.assert_array_equal(labels, o_labels)
    np.testing.assert_array_equal(cent, o_cent)


def test_kmeans_similarities_are_the_oracle_dots(cuda):
    from maple_flash_dgx_spark_b200 import _lib

    rs = np.random.default_rng(8)
    w = unit_rows(300, 64, 9)
    cent = unit_rows(200, 64, 10)
    rows = rs.permutation(300)[:77].astype(np.int32)
    out = torch.empty(77, 200, dtype=torch.float32, device=cuda)
    wd, cd, rd = (torch.from_numpy(a).to(cuda) for a in (w, cent, rows))
    L = _lib.lib()
    _lib.check(L.maple_km_dots(wd.data_ptr(), rd.data_ptr(), 77, 64, cd.data_ptr(), 200, out.data_ptr(),
                               torch.cuda.current_stream(cuda).cuda_stream), "km_dots")
    np.testing.assert_array_equal(out.cpu().numpy(), km_dots(w[rows], cent))
