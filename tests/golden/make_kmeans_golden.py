"""Golden vectors for the FlashHead balanced spherical k-means, produced by the
reference's own function (src/maple_run/flash_head.py:30-110,
_balanced_spherical_kmeans) run on the CPU.

Usage (from the repository root, with the reference checkout available):
    python tests/golden/make_kmeans_golden.py /path/to/reference

Writes tests/golden/kmeans_golden.npz: for each case the initial centroid
rows (the reference's own torch.randperm draw on the CPU for the case's seed)
and the reference's returned labels and centroids; the unit rows are
regenerated from the case's data seed by unit_rows().
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

CASES = {
    # name: (rows, dim, clusters, iterations, data seed, k-means seed)
    "n2048_d64_c64": (2048, 64, 64, 8, 0, 0),
    "n4096_d128_c128": (4096, 128, 128, 6, 1, 42),
}


def unit_rows(n: int, d: int, seed: int) -> np.ndarray:
    w = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return (w / (np.linalg.norm(w, axis=1, keepdims=True) + 1e-8)).astype(np.float32)


def main(ref_root: str) -> None:
    import torch

    sys.path.insert(0, str(Path(ref_root) / "src"))
    spec = importlib.util.spec_from_file_location("ref_flash_head",
                                                  Path(ref_root) / "src" / "maple_run" / "flash_head.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    for name, (n, d, c, iters, dseed, kseed) in CASES.items():
        w = unit_rows(n, d, dseed)
        g = torch.Generator(device="cpu")
        g.manual_seed(int(kseed))
        init = torch.randperm(n, generator=g)[:c].numpy().astype(np.int64)  # the reference's first draw
        cent, labels = mod._balanced_spherical_kmeans(torch.from_numpy(w), c, n_iter=iters, seed=kseed)
        out[f"{name}.init"] = init
        out[f"{name}.labels"] = np.asarray(labels, np.int32)
        out[f"{name}.centroids"] = np.asarray(cent, np.float32)
    np.savez_compressed(Path(__file__).parent / "kmeans_golden.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_kmeans_golden.py <reference checkout>")
    main(sys.argv[1])
