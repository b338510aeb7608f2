"""Balanced spherical k-means restated for the FlashHead clustering.  TEST
INFRASTRUCTURE ONLY: the checker of the CUDA k-means
(maple_flash_dgx_spark_b200/csrc/kmeans.cu), never part of the product path.

Reference: src/maple_run/flash_head.py:30-110 (_balanced_spherical_kmeans):
per iteration, assign every row to its most similar centroid; for each
over-full cluster (ascending) keep its cluster_size most similar members and
evict the rest (in ascending row order); reassign the evicted rows one by one,
in that order, to their most similar cluster that is not yet full; recompute
the centroids as normalised member means; keep the iteration with the best
objective (mean similarity of each row to its centroid).

The arithmetic is the CUDA k-means' canonical one (oracle.c orc_km_*): every
similarity is one fp32 fmaf chain over k in order, so the eviction and
reassignment see exactly the assignment's values.  Ties: the lowest cluster
index wins an argmax; among equally similar members the lower row index is
kept.  The reference's fp32 matmuls sum in another order, so its labels can
differ from these where two similarities are within a rounding of each other.
"""

from __future__ import annotations

import numpy as np

from oracle import _f32, lib


def km_dots(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    out = np.empty((a.shape[0], b.shape[0]), np.float32)
    lib().orc_km_dots(a, a.shape[0], b, b.shape[0], a.shape[1], out)
    return out


def km_normalize(v: np.ndarray) -> np.ndarray:
    v = _f32(v).copy()
    lib().orc_km_normalize(v, v.shape[0], v.shape[1])
    return v


def km_update(w: np.ndarray, labels: np.ndarray, n_clusters: int) -> np.ndarray:
    w = _f32(w)
    cent = np.empty((n_clusters, w.shape[1]), np.float32)
    lib().orc_km_update(w, w.shape[0], w.shape[1], np.ascontiguousarray(labels, np.int32), n_clusters, cent)
    return cent


def km_objective(w: np.ndarray, labels: np.ndarray, cent: np.ndarray) -> float:
    w = _f32(w)
    return float(lib().orc_km_objective(w, w.shape[0], w.shape[1], np.ascontiguousarray(labels, np.int32),
                                        _f32(cent)))


def rebalance(sims: np.ndarray, labels: np.ndarray, cluster_size: int) -> np.ndarray:
    """The eviction and sequential reassignment of one iteration
    (flash_head.py:62-96) on the assignment's similarity matrix."""
    labels = labels.astype(np.int64).copy()
    K = sims.shape[1]
    counts = np.bincount(labels, minlength=K)
    over = np.where(counts > cluster_size)[0]
    if not len(over):
        return labels
    evict: list[int] = []
    for ci in over:
        members = np.where(labels == ci)[0]
        s = sims[members, ci]
        order = np.lexsort((members, -s))  # most similar first, lower row first on ties
        dumped = np.sort(members[order[cluster_size:]])
        labels[dumped] = -1
        evict.extend(dumped.tolist())
    recount = np.bincount(labels[labels >= 0], minlength=K)
    full = recount >= cluster_size
    for pt in evict:
        row = np.where(full, -np.inf, sims[pt])
        bc = int(np.argmax(row))
        if not np.isfinite(row[bc]):
            bc = int(np.argmax(recount < cluster_size))
        labels[pt] = bc
        recount[bc] += 1
        if recount[bc] >= cluster_size:
            full[bc] = True
    return labels


def balanced_kmeans(w: np.ndarray, n_clusters: int, init: np.ndarray, n_iter: int):
    """Returns (best centroids [K, D] fp32, best labels [N] int32, best objective)."""
    w = _f32(w)
    N = w.shape[0]
    cs = N // n_clusters
    cent = km_normalize(w[np.asarray(init, np.int64)])
    best = (-1.0, None, None)
    for _ in range(n_iter):
        sims = km_dots(w, cent)
        labels = sims.argmax(axis=1)
        labels = rebalance(sims, labels, cs)
        cent = km_update(w, labels, n_clusters)
        obj = km_objective(w, labels, cent)
        if obj > best[0]:
            best = (obj, cent.copy(), labels.astype(np.int32))
    return best[1], best[2], best[0]
