"""FlashHead: two-phase RTN-4 lm_head for batch-1 decode.

Reference: flash_head.py:282-369 (``FlashHead``), :372-463
(``build_flash_head``), :30-110 and :150-279 (clustering, offline: the
balanced spherical k-means runs on this package's CUDA kernels).

Phase one scores the cluster centroids (``rtn4_gemv``), picks the
``n_probes`` best clusters on the device (``maple_topk_select``: radix select,
ties to the lowest cluster index), phase two computes exact RTN-4 logits of
the probed clusters' rows (``rtn4_indexed_gemv`` over the cluster-permuted
head) and of the forced tokens, and scatters them into a ``-inf`` row of the
vocabulary (``maple_flash_scatter``).  Every step is a CUDA kernel of this
package; the buffers are allocated once, so the call is CUDA-graph safe.
"""

from __future__ import annotations

import torch

from maple_flash_dgx_spark_b200 import _lib
from maple_flash_dgx_spark_b200._lib import check, dtype_code, lib, ptr, stream_ptr
from maple_flash_dgx_spark_b200.kernels import rtn4_gemv, rtn4_indexed_gemv

DEFAULT_N_CLUSTERS = 4748
DEFAULT_N_PROBES = 512
DEFAULT_KMEANS_ITERS = 60
HEAD_GROUP_SIZE = 64


def topk_select(scores: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Indices (int32, ascending) of the ``k`` largest of a 1-D score vector;
    NaN ranks highest, ties at the k-th value go to the lowest indices."""
    op = "topk_select"
    _lib.require_cuda(op, scores)
    x = scores.reshape(-1)
    if x.stride(0) != 1:
        x = x.contiguous()
    out = out if out is not None else torch.empty(k, dtype=torch.int32, device=x.device)
    check(lib().maple_topk_select(ptr(x), dtype_code(x, op), x.numel(), int(k), ptr(out), stream_ptr(x.device)), op)
    return out


class FlashHead:
    """Reference flash_head.py:282-369, same constructor and call."""

    def __init__(self, *, centroids_weight, centroids_scales, centroids_biases, token_map, head_weight, head_scales,
                 head_biases, force_ids, force_weight, force_scales, force_biases, n_probes: int, vocab_size: int,
                 group_size: int = HEAD_GROUP_SIZE, dtype: torch.dtype, device: torch.device,
                 centroid_group_size: int = HEAD_GROUP_SIZE):
        self.centroids_weight = centroids_weight.contiguous()
        self.centroids_scales = centroids_scales.contiguous()
        self.centroids_biases = None if centroids_biases is None else centroids_biases.contiguous()
        self.token_map = token_map.to(torch.int32).contiguous()
        self.head_weight = head_weight.contiguous()
        self.head_scales = head_scales.contiguous()
        self.head_biases = None if head_biases is None else head_biases.contiguous()
        self.n_clusters, self.cluster_size, _ = self.head_weight.shape
        self.n_probes = min(int(n_probes), self.n_clusters)
        self.group_size = int(group_size)
        self.centroid_group_size = int(centroid_group_size)
        self.vocab_size = int(vocab_size)
        self.force_ids = force_ids.to(torch.int64).contiguous()
        self.force_weight = force_weight
        self.force_scales = force_scales
        self.force_biases = force_biases
        self.n_force = int(self.force_ids.numel())
        self._full = torch.empty(1, 1, self.vocab_size, device=device, dtype=dtype)
        self._cluster_ids = torch.empty(self.n_probes, device=device, dtype=torch.int32)

    def head_bytes(self) -> int:
        """HBM bytes one call reads (centroids, probed rows, forced rows, scales)."""
        def rows_bytes(w, s, b, n):
            per = w[0].numel() * 4 + s[0].numel() * s.element_size()
            if b is not None:
                per += b[0].numel() * b.element_size()
            return n * per
        c = rows_bytes(self.centroids_weight, self.centroids_scales, self.centroids_biases, self.n_clusters)
        hw = self.head_weight.reshape(-1, self.head_weight.shape[-1])
        hs = self.head_scales.reshape(-1, self.head_scales.shape[-1])
        hb = None if self.head_biases is None else self.head_biases.reshape(-1, self.head_biases.shape[-1])
        p = rows_bytes(hw, hs, hb, self.n_probes * self.cluster_size)
        f = 0 if not self.n_force else rows_bytes(self.force_weight, self.force_scales, self.force_biases,
                                                  self.n_force)
        return c + p + f

    def __call__(self, hidden):
        hv = hidden.reshape(-1, hidden.shape[-1])[-1:]
        scores = rtn4_gemv(hv, self.centroids_weight, self.centroids_scales, self.centroids_biases,
                           group_size=self.centroid_group_size)
        topk_select(scores, self.n_probes, out=self._cluster_ids)
        probe = rtn4_indexed_gemv(hv, self.head_weight, self.head_scales, self.head_biases, self._cluster_ids,
                                  group_size=self.group_size).reshape(-1)
        force = None
        if self.n_force:
            force = rtn4_gemv(hv, self.force_weight, self.force_scales, self.force_biases,
                              group_size=self.group_size).reshape(-1)
        op = "flash_head"
        check(lib().maple_flash_scatter(
            ptr(probe), dtype_code(probe, op), ptr(self._cluster_ids), self.n_probes, self.cluster_size,
            ptr(self.token_map), self.n_clusters, ptr(force), ptr(self.force_ids) if self.n_force else None,
            self.n_force, ptr(self._full), self.vocab_size, ptr(_lib.error_word(probe.device)),
            stream_ptr(probe.device)), op)
        return self._full


def build_flash_head(*, config: dict, lm_head, weights: dict, device, dtype) -> FlashHead:
    """Reference flash_head.py:372-463: permute the lm_head rows by the token
    map at load (or take the checkpoint's permuted copy)."""
    meta = config.get("flash_head") or (config.get("maple_run") or {}).get("flash_head")
    if not meta:
        raise ValueError("Checkpoint has no flash_head metadata; run --flash-head-only.")
    if not meta.get("scaled_centroids"):
        raise ValueError("FlashHead metadata predates scaled centroids; regenerate with "
                         "`maple-run convert --flash-head-only`.")
    n_clusters, cluster_size = int(meta["n_clusters"]), int(meta["cluster_size"])
    n_probes = int(meta.get("n_probes", DEFAULT_N_PROBES))
    group_size = int(meta.get("head_group_size", meta.get("group_size", HEAD_GROUP_SIZE)))
    centroid_group = int(meta.get("group_size", HEAD_GROUP_SIZE))
    token_map = weights.pop("lm_head_flash.token_map").to(device=device, dtype=torch.int32)
    if tuple(token_map.shape) != (n_clusters, cluster_size):
        raise ValueError(f"token_map shape {tuple(token_map.shape)} != {(n_clusters, cluster_size)} "
                         "from flash_head metadata.")
    order = token_map.reshape(-1).to(torch.int64)

    def u32(t):
        return t if t.dtype == torch.uint32 else t.view(torch.uint32)

    if "lm_head_flash.head.weight" in weights:
        head_w = u32(weights.pop("lm_head_flash.head.weight")).reshape(n_clusters, cluster_size, -1)
        head_s = weights.pop("lm_head_flash.head.scales").reshape(n_clusters, cluster_size, -1)
        hb = weights.pop("lm_head_flash.head.biases", None)
        head_b = None if hb is None else hb.reshape(n_clusters, cluster_size, -1)
    else:
        packed = u32(lm_head.packed_weight)
        head_w = packed.view(torch.int32).index_select(0, order).view(torch.uint32)
        head_w = head_w.reshape(n_clusters, cluster_size, -1).contiguous()
        head_s = lm_head.scales.index_select(0, order).reshape(n_clusters, cluster_size, -1).contiguous()
        head_b = None if lm_head.biases is None else lm_head.biases.index_select(0, order).reshape(
            n_clusters, cluster_size, -1).contiguous()
    cw = u32(weights.pop("lm_head_flash.centroids.weight"))
    cs = weights.pop("lm_head_flash.centroids.scales")
    cb = weights.pop("lm_head_flash.centroids.biases", None)
    weights.pop("lm_head_flash.cluster_scale", None)
    side = lm_head.scales.dtype
    cs = cs.to(device=device, dtype=side)
    cb = None if cb is None else cb.to(device=device, dtype=side)
    force = [int(t) for t in meta.get("force_tokens", []) if 0 <= int(t) < int(config["vocab_size"])]
    if force:
        force_ids = torch.tensor(force, device=device, dtype=torch.int64)
        force_w = u32(lm_head.packed_weight).view(torch.int32).index_select(0, force_ids).view(torch.uint32)
        force_w = force_w.contiguous()
        force_s = lm_head.scales.index_select(0, force_ids).contiguous()
        force_b = None if lm_head.biases is None else lm_head.biases.index_select(0, force_ids).contiguous()
    else:
        force_ids = torch.empty(0, device=device, dtype=torch.int64)
        force_w = force_s = force_b = None
    return FlashHead(centroids_weight=cw.to(device), centroids_scales=cs, centroids_biases=cb, token_map=token_map,
                     head_weight=head_w, head_scales=head_s, head_biases=head_b, force_ids=force_ids,
                     force_weight=force_w, force_scales=force_s, force_biases=force_b, n_probes=n_probes,
                     vocab_size=int(config["vocab_size"]), group_size=group_size, dtype=dtype, device=device,
                     centroid_group_size=centroid_group)


def balanced_spherical_kmeans(w_dir: torch.Tensor, n_clusters: int, n_iter: int = DEFAULT_KMEANS_ITERS,
                              seed: int = 42, init: torch.Tensor | None = None):
    """Balanced spherical k-means over L2-normalised rows ``[N, D]`` into
    equal-size clusters (reference flash_head.py:30-110, same steps and
    tie rules), on this package's CUDA kernels (``maple_km_*``): per
    iteration the assignment, the eviction of each over-full cluster's least
    similar members, their sequential reassignment to the most similar open
    cluster, the centroid update and the objective; the best iteration's
    centroids and labels are returned.  ``init``: the initial centroid rows
    (default: the reference's ``torch.randperm`` draw for ``seed`` on the
    rows' device).  Returns ``(centroids [K, D] fp32, labels [N] int32)``."""
    op = "balanced_spherical_kmeans"
    _lib.require_cuda(op, w_dir)
    w = w_dir.float().contiguous()
    N, D = w.shape
    K = int(n_clusters)
    if K <= 0 or N % K:
        raise ValueError(f"{K} clusters do not divide {N} rows.")
    if D % 16:
        raise ValueError(f"row length {D} must be a multiple of 16.")
    cs = N // K
    dev = w.device
    L = lib()
    st = stream_ptr(dev)
    if init is None:
        g = torch.Generator(device=dev)
        g.manual_seed(int(seed))
        init = torch.randperm(N, generator=g, device=dev)[:K]
    cent = w.index_select(0, init.to(device=dev, dtype=torch.int64)).contiguous()
    check(L.maple_km_normalize(ptr(cent), K, D, st), op)
    labels = torch.empty(N, dtype=torch.int32, device=dev)
    best = torch.empty(N, dtype=torch.float32, device=dev)
    ws = torch.empty(L.maple_km_assign_workspace_bytes(N, K), dtype=torch.uint8, device=dev)
    partial = torch.empty(L.maple_km_objective_blocks(N), dtype=torch.float64, device=dev)
    rows = torch.arange(N, device=dev)
    best_obj, best_c, best_l = -1.0, None, None
    for _ in range(int(n_iter)):
        check(L.maple_km_assign(ptr(w), N, D, ptr(cent), K, ptr(labels), ptr(best), ptr(ws), ws.numel(), st), op)
        lab = labels.long()
        over = torch.bincount(lab, minlength=K) > cs
        if bool(over.any()):
            # each over-full cluster keeps its cs most similar members (lower row on ties)
            cand = rows[over[lab]]
            cand = cand[torch.argsort(-best[cand], stable=True)]
            cand = cand[torch.argsort(lab[cand], stable=True)]
            cl = lab[cand]
            rank = torch.arange(cand.numel(), device=dev) - torch.searchsorted(cl, cl)
            dumped = cand[rank >= cs].sort().values
            evict = dumped[torch.argsort(lab[dumped], stable=True)]  # by cluster, then row
            lab[evict] = -1
            recount = torch.bincount(lab[lab >= 0], minlength=K).to(torch.int32)
            evict32 = evict.to(torch.int32).contiguous()
            sims = torch.empty(evict32.numel(), K, dtype=torch.float32, device=dev)
            check(L.maple_km_dots(ptr(w), ptr(evict32), evict32.numel(), D, ptr(cent), K, ptr(sims), st), op)
            labels = lab.to(torch.int32).contiguous()
            scratch = torch.empty(max(1, evict32.numel()), dtype=torch.int32, device=dev)
            check(L.maple_km_reassign(ptr(sims), ptr(evict32), evict32.numel(), K, ptr(recount), cs, ptr(labels),
                                      ptr(scratch), st), op)
            del sims
        members = torch.argsort(labels.long(), stable=True).to(torch.int32)
        offsets = torch.zeros(K + 1, dtype=torch.int32, device=dev)
        offsets[1:] = torch.cumsum(torch.bincount(labels.long(), minlength=K), 0)
        check(L.maple_km_update(ptr(w), D, ptr(members), ptr(offsets), K, ptr(cent), st), op)
        check(L.maple_km_objective(ptr(w), N, D, ptr(labels), ptr(cent), ptr(partial), st), op)
        total = 0.0
        for p_ in partial.cpu().tolist():  # block sums in order
            total += p_
        obj = total / N
        if obj > best_obj:
            best_obj, best_c, best_l = obj, cent.clone(), labels.clone()
    return best_c, best_l


def token_map_of(labels: torch.Tensor, n_clusters: int) -> torch.Tensor:
    """``[K, N/K]`` rows of each cluster in ascending order (reference
    flash_head.py:212-217; a short cluster repeats its first member)."""
    K = int(n_clusters)
    cs = labels.numel() // K
    counts = torch.bincount(labels.long(), minlength=K)
    order = torch.argsort(labels.long(), stable=True)
    if bool((counts == cs).all()):
        return order.reshape(K, cs).to(torch.int32)
    lab = labels.cpu().numpy()
    out = torch.zeros(K, cs, dtype=torch.int32)
    for c in range(K):
        members = [int(i) for i in (lab == c).nonzero()[0][:cs]]
        while len(members) < cs:
            members.append(members[0] if members else 0)
        out[c] = torch.tensor(members, dtype=torch.int32)
    return out.to(labels.device)


def cluster_head(w_dir: torch.Tensor, n_clusters: int, n_iter: int = DEFAULT_KMEANS_ITERS, seed: int = 42):
    """Cluster L2-normalised head rows ``[V, D]``: ``(centroids [C, D],
    token_map [C, V/C])`` by the balanced spherical k-means."""
    cent, labels = balanced_spherical_kmeans(w_dir, n_clusters, n_iter=n_iter, seed=seed)
    return cent, token_map_of(labels, n_clusters)


def attach_flash_head(config: dict, weights: dict, *, n_clusters: int = DEFAULT_N_CLUSTERS,
                      n_probes: int = DEFAULT_N_PROBES, force_tokens=(), seed: int = 42,
                      n_iter: int = DEFAULT_KMEANS_ITERS) -> dict:
    """Cluster the RTN-4 ``lm_head`` in ``weights`` and add the
    ``lm_head_flash.*`` tensors and ``flash_head`` metadata the way the
    reference converter does (flash_head.py:150-279): rows are dequantised and
    L2-normalised, clustered into equal-size clusters, and each centroid (unit
    cluster mean scaled by the largest member row norm, rounded to bf16) is
    RTN-4 quantised with group 64, affine.  Runs on the GPU holding the head.
    Returns the metadata."""
    from maple_flash_dgx_spark_b200.pack import dequantize_rtn, quantize_rtn

    rtn = (config.get("maple_run") or {}).get("rtn_4bit", {})
    group = int(rtn.get("group_size", HEAD_GROUP_SIZE))
    w = weights["lm_head.weight"]
    w = w if w.dtype == torch.uint32 else w.view(torch.uint32)
    scales = weights["lm_head.scales"].float()
    biases = weights.get("lm_head.biases")
    biases = scales * -8.0 if biases is None else biases.float()
    V = w.shape[0]
    if V % n_clusters:
        raise ValueError(f"clusters must divide the vocab size {V}; got {n_clusters}")
    if n_probes > n_clusters:
        raise ValueError(f"probes ({n_probes}) must not exceed clusters ({n_clusters})")
    W = dequantize_rtn(w, scales, biases, group_size=group)
    norms = W.norm(dim=1, keepdim=True) + 1e-8
    centroids, token_map = cluster_head(W / norms, n_clusters, n_iter=n_iter, seed=seed)
    del W
    centroids = centroids / (centroids.norm(dim=1, keepdim=True) + 1e-8)
    cluster_scale = norms[:, 0][token_map.long()].amax(dim=1)
    scaled = (centroids * cluster_scale[:, None]).to(torch.bfloat16).float()
    cw, cs, cb = quantize_rtn(scaled, group_size=HEAD_GROUP_SIZE)
    weights["lm_head_flash.centroids.weight"] = cw
    weights["lm_head_flash.centroids.scales"] = cs
    weights["lm_head_flash.centroids.biases"] = cb
    weights["lm_head_flash.token_map"] = token_map
    meta = {"n_clusters": int(n_clusters), "cluster_size": int(V // n_clusters), "n_probes": int(n_probes),
            "group_size": HEAD_GROUP_SIZE, "bits": 4, "head_group_size": group, "head_bits": 4,
            "scaled_centroids": True, "force_tokens": [int(t) for t in force_tokens]}
    config["flash_head"] = meta
    maple_run = dict(config.get("maple_run") or {})
    maple_run["flash_head"] = meta
    config["maple_run"] = maple_run
    return meta
