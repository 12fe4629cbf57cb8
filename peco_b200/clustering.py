"""Token clustering and cluster-pair selection on the sm_100a kernels.

Mirrors peco/clustering.py (same functions, signatures, validation and
return values) for CUDA tensors.  CPU tensors are rejected: this package has
no CPU implementation.

* ``fit_token_clusters`` -- bf16 input with ``tol=0`` (what the processor
  uses) runs every Lloyd iteration of both problems inside one library call;
  other inputs iterate the drop-in assign/recompute entry points exactly like
  the reference's CUDA branch (peco/clustering.py:59-88).
* ``select_cluster_connections`` -- one kernel (peco/clustering.py:154-186).
* ``gather_clustered_tokens`` / ``restore_sequence_order`` -- counting-sort
  argsort plus a vectorised row permutation (peco/clustering.py:92-136).
"""

from __future__ import annotations

import math

import torch

from . import _native, clustering_cuda


def _check_fit_args(x, n_clusters, max_iters, tol, chunk_size):
    if x.ndim != 3 or not x.is_floating_point():
        raise ValueError("x must be a floating tensor with shape [batch_heads, tokens, dims]")
    batch, tokens, dims = x.shape
    if min(batch, tokens, dims) <= 0:
        raise ValueError("x dimensions must be nonzero")
    if not isinstance(n_clusters, int) or not 1 <= n_clusters <= tokens:
        raise ValueError("n_clusters must be an integer in [1, tokens]")
    if not isinstance(max_iters, int) or max_iters < 1:
        raise ValueError("max_iters must be a positive integer")
    if tol < 0 or not math.isfinite(tol):
        raise ValueError("tol must be finite and nonnegative")
    if not isinstance(chunk_size, int) or chunk_size < 1:
        raise ValueError("chunk_size must be a positive integer")


def _initial_centers(x, n_clusters, init_centroids):
    batch, tokens, dims = x.shape
    if init_centroids is None:
        idx = torch.randint(tokens, (batch, n_clusters), device=x.device)
        return x.gather(1, idx[..., None].expand(-1, -1, dims)).float().contiguous()
    if init_centroids.shape != (batch, n_clusters, dims) or init_centroids.device != x.device:
        raise ValueError("init_centroids must match [batch_heads, n_clusters, dims] and x.device")
    return init_centroids.float().contiguous().clone()


class KmeansBuffers:
    """Device buffers of one fixed-iteration clustering (fused path)."""

    def __init__(self, bh, tokens, clusters, dims, device, centers=None):
        f32, i32 = torch.float32, torch.int32
        self.labels = torch.empty((bh, tokens), dtype=i32, device=device)
        if centers is None:
            centers = torch.empty((bh, clusters, dims), dtype=f32, device=device)
        elif centers.shape != (bh, clusters, dims) or centers.dtype != f32 or not centers.is_contiguous():
            raise ValueError("centers must be a contiguous fp32 [BH, C, D] tensor")
        self.centers = centers
        # ping-pong centres, the centres' bf16 tensor-core image, token norms
        # and, for long sequences, the label sort's per-segment scratch
        self.work = torch.empty((bh, int(_native.load().peco_kmeans_work_floats(clusters, dims, tokens))),
                                dtype=f32, device=device)
        self.norms = torch.empty((bh, clusters), dtype=f32, device=device)
        self.counts = torch.empty((bh, clusters), dtype=i32, device=device)
        self.offsets = torch.empty((bh, clusters + 1), dtype=i32, device=device)
        self.perm = torch.empty((bh, tokens), dtype=i32, device=device)

    def tensors(self):
        return (self.labels, self.centers, self.work, self.norms, self.counts, self.offsets, self.perm)


def kmeans_fit_pair(q_rows, q_head_rows, q_tokens, q_init, k_rows, k_head_rows, k_tokens, k_init, bh, dims,
                    iters, *, q_centers=None, k_centers=None):
    """Fixed-iteration k-means of two bf16 problems in one library call.

    ``*_rows`` are bf16 tensors whose head b starts at row b*head_rows (the
    video prefix of a [B,H,S,D] tensor qualifies without a copy).  ``k_rows``
    may be None.  ``q_centers``/``k_centers`` optionally name the fp32 output
    centres (they may be the init tensors themselves: the fit then updates
    the centroids in place).  Returns KmeansBuffers per problem.
    """
    lib = _native.load()
    dev = _native.require_cuda(q_rows, q_init)
    qb = KmeansBuffers(bh, q_tokens, q_init.shape[1], dims, dev, q_centers)
    kb = KmeansBuffers(bh, k_tokens, k_init.shape[1], dims, dev, k_centers) if k_rows is not None else None
    z = _native.P(0)

    def args(rows, head_rows, tokens, init, b):
        if b is None:
            return [z, 0, 0, 0, z, z, z, z, z, z, z, z]
        return [_native.ptr(rows), int(head_rows), int(tokens), int(init.shape[1]), _native.ptr(b.labels),
                _native.ptr(init), _native.ptr(b.centers), _native.ptr(b.work), _native.ptr(b.norms),
                _native.ptr(b.counts), _native.ptr(b.offsets), _native.ptr(b.perm)]

    keep = [q_rows, q_init, *qb.tensors()]
    if kb is not None:
        keep += [k_rows, k_init, *kb.tensors()]
    with torch.cuda.device(dev):
        status = lib.peco_kmeans_fit(*args(q_rows, q_head_rows, q_tokens, q_init, qb),
                                     *args(k_rows, k_head_rows, k_tokens, k_init, kb), int(bh), int(dims),
                                     int(iters), _native.stream_of(dev, *keep))
    _native.check(status, "peco_kmeans_fit")
    return qb, kb


@torch.no_grad()
def fit_token_clusters(x, n_clusters, max_iters=100, tol=1e-4, init_centroids=None, *, chunk_size=1024):
    """Run Euclidean Lloyd updates independently for each batch/head.

    Input features have shape [BH,N,D]; optional initial centers [BH,K,D].
    Returns labels [BH,N] int32, centers [BH,K,D] fp32, counts [BH,K] int32
    and the iteration count.  Each nonempty center is the mean of its returned
    token partition; an empty cluster keeps its previous center.  ``tol > 0``
    stops early on the maximum center displacement (one host sync per
    iteration, as in the reference).
    """
    _check_fit_args(x, n_clusters, max_iters, tol, chunk_size)
    _native.require_cuda(x)
    batch, tokens, dims = x.shape
    centers = _initial_centers(x, n_clusters, init_centroids)
    if x.dtype == torch.bfloat16 and tol == 0:
        xb = x.contiguous()
        qb, _ = kmeans_fit_pair(xb, tokens, tokens, centers, None, 0, 0, centers, batch, dims, max_iters)
        return qb.labels, qb.centers, qb.counts, max_iters
    # other dtypes, or early stopping: one assignment and one update per
    # iteration on the drop-in entry points, in fp32
    x32 = x.float().contiguous()
    dev = x32.device
    labels = torch.empty((batch, tokens), dtype=torch.int32, device=dev)
    counts = torch.empty((batch, n_clusters), dtype=torch.int32, device=dev)
    sums = torch.empty_like(centers)
    norms = torch.empty((batch, n_clusters), dtype=torch.float32, device=dev)
    rows = min(chunk_size, tokens)
    scratch = torch.empty((rows, n_clusters), dtype=torch.float32, device=dev)
    current, following = centers, torch.empty_like(centers)
    done = 0
    while done < max_iters:
        done += 1
        clustering_cuda.assign_tokens_to_centers(x32, current, labels, scratch, norms, rows)
        clustering_cuda.recompute_cluster_centers(x32, labels, current, sums, counts, following)
        # the largest centre displacement, checked on the host only when asked for
        settled = tol > 0 and float((following - current).norm(dim=-1).max()) <= tol
        current, following = following, current
        if settled:
            break
    return labels, current, counts, done


def _prepare_sequence_indices(tensor, labels, dim, sorted_indices):
    """Validate token reordering and return contiguous int32 indices [BH,N]."""
    if tensor.ndim != 4 or dim not in (2, -2):
        raise ValueError("permutation expects [batch, heads, tokens, dims] with dim=2")
    if tensor.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("permutation supports float16, bfloat16, and float32")
    batch, heads, tokens, _ = tensor.shape
    if min(tensor.shape) <= 0:
        raise ValueError("permutation tensor dimensions must be nonzero")
    if sorted_indices is None:
        if labels is None or labels.numel() != batch * heads * tokens or labels.device != tensor.device:
            raise ValueError("labels must contain one cluster ID per token on the same device")
        flat = labels.reshape(batch * heads, tokens).to(torch.int32)
        clusters = int(flat.max().item()) + 1  # counting-sort width (one host sync)
        if int(flat.min().item()) < 0:
            raise ValueError("labels must be nonnegative")
        sorted_indices, _, _ = clustering_cuda.sort_labels(flat, clusters)
    if sorted_indices.numel() != batch * heads * tokens or sorted_indices.device != tensor.device:
        raise ValueError("sorted_indices must contain one index per token on the same device")
    return sorted_indices.reshape(batch * heads, tokens).to(torch.int32).contiguous()


@torch.no_grad()
def gather_clustered_tokens(tensor, labels, dim=2, sorted_indices=None):
    """Pack [B,H,N,D] features into cluster order and return the gather indices.

    ``indices[bh, j]`` is the original token at packed position ``j``; pass
    them as ``sorted_indices`` to pack V with exactly the K ordering.
    """
    _native.require_cuda(tensor)
    indices = _prepare_sequence_indices(tensor, labels, dim, sorted_indices)
    return clustering_cuda.reorder_token_features(tensor, indices), indices


@torch.no_grad()
def restore_sequence_order(tensor, sorted_indices, dim=2):
    """Scatter packed features back to the original sequence using gather indices."""
    _native.require_cuda(tensor)
    indices = _prepare_sequence_indices(tensor, None, dim, sorted_indices)
    return clustering_cuda.reorder_token_features(tensor, indices, inverse=True)


@torch.no_grad()
def select_cluster_connections(query_centroids, key_centroids, q_cluster_sizes, k_cluster_sizes, p, min_kc_ratio=0):
    """Choose nonempty query/key cluster pairs from estimated attention mass.

    Centroids [B,H,C,D], sizes [B,H,C]; returns a boolean [B,H,CQ,CK] mask.
    For each query cluster keep the smallest descending-probability prefix
    reaching ``p``, at least ceil(min_kc_ratio * CK) clusters and always the
    most likely one; empty clusters never produce active pairs.
    """
    if not 0 <= p <= 1 or not 0 <= min_kc_ratio <= 1:
        raise ValueError("p and min_kc_ratio must be in [0, 1]")
    dev = _native.require_cuda(query_centroids, key_centroids, q_cluster_sizes, k_cluster_sizes)
    b, h, cq, d = query_centroids.shape
    ck = key_centroids.shape[-2]
    qc = query_centroids.float().reshape(b * h, cq, d).contiguous()
    kc = key_centroids.float().reshape(b * h, ck, d).contiguous()
    qs = q_cluster_sizes.to(torch.int32).reshape(b * h, cq).contiguous()
    ks = k_cluster_sizes.to(torch.int32).reshape(b * h, ck).contiguous()
    out = torch.empty((b, h, cq, ck), dtype=torch.bool, device=dev)
    minimum = math.ceil(min_kc_ratio * ck)
    lib = _native.load()
    with torch.cuda.device(dev):
        status = lib.peco_select_cluster_connections(
            _native.ptr(qc), _native.ptr(kc), _native.ptr(qs), _native.ptr(ks), _native.ptr(out), b * h, cq, ck, d,
            float(p), int(minimum), _native.P(0), _native.stream_of(dev, qc, kc, qs, ks, out))
    _native.check(status, "peco_select_cluster_connections")
    return out
