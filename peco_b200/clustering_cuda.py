"""Clustering entry points over libpeco_b200.so, with the reference's signatures.

Mirrors peco/clustering_cuda.py: ``build_cluster_library`` (:22-56),
``assign_tokens_to_centers`` (:93-108), ``recompute_cluster_centers``
(:111-125) and ``reorder_token_features`` (:128-146).  Same argument meaning,
same in-place outputs and the same RuntimeError on a failed launch; the work
runs on the sm_100a kernels of this package.
"""

from __future__ import annotations

import torch

from . import _native
from .build import build as _build


def build_cluster_library():
    """Build libpeco_b200.so when missing or stale and return its path."""
    return _build()


def _raise(status: int) -> None:
    if status:
        lib = _native.load()
        msg = lib.peco_cluster_error_message(int(status)).decode("utf-8", "replace")
        raise RuntimeError(f"CUDA clustering failed: {msg} (status {status})")


def assign_tokens_to_centers(x, centers, labels, scratch, center_norms, chunk_size):
    """Assign FP32 x [B,N,D] to centers [B,C,D], writing int32 labels [B,N].

    ``center_norms`` [B,C] receives ||c||^2.  ``scratch`` is accepted for
    signature compatibility and unused by the tensor-core path.
    """
    lib = _native.load()
    dev = _native.require_cuda(x, centers, labels, center_norms)
    batch, tokens, dims = x.shape
    clusters = centers.shape[1]
    with torch.cuda.device(dev):
        status = lib.peco_assign_tokens_to_centers(
            _native.ptr(x), _native.ptr(centers), _native.ptr(labels), _native.ptr(scratch),
            _native.ptr(center_norms), batch, tokens, dims, clusters, int(chunk_size),
            _native.stream_of(dev, x, centers, labels, scratch, center_norms))
    _raise(status)


def recompute_cluster_centers(x, labels, previous, sums, counts, means):
    """Write FP32 means [B,C,D] and int32 counts [B,C] for labels [B,N]; sums too.

    Empty clusters retain ``previous``.  Deterministic: each cluster sums its
    tokens in ascending token order.
    """
    lib = _native.load()
    dev = _native.require_cuda(x, labels, previous, sums, counts, means)
    batch, tokens, dims = x.shape
    with torch.cuda.device(dev):
        status = lib.peco_recompute_cluster_centers(
            _native.ptr(x), _native.ptr(labels), _native.ptr(previous), _native.ptr(sums), _native.ptr(counts),
            _native.ptr(means), batch, tokens, dims, previous.shape[1],
            _native.stream_of(dev, x, labels, previous, sums, counts, means))
    _raise(status)


def reorder_token_features(tensor, indices, inverse=False):
    """Reorder features [B,H,N,D] using original token IDs [B*H,N].

    Forward gathers original IDs into sorted order; inverse scatters sorted
    rows back to original order.  Indices must be a valid permutation.
    """
    lib = _native.load()
    tensor = tensor.contiguous()
    indices = indices.to(dtype=torch.int32).contiguous()
    dev = _native.require_cuda(tensor, indices)
    batch, heads, tokens, dims = tensor.shape
    result = torch.empty_like(tensor)
    with torch.cuda.device(dev):
        status = lib.peco_reorder_token_features(
            _native.ptr(tensor), _native.ptr(indices), _native.ptr(result), batch * heads, tokens, dims,
            tensor.element_size(), int(inverse), _native.stream_of(dev, tensor, indices, result))
    _raise(status)
    return result


def sort_labels(labels, clusters):
    """Stable argsort of int32 labels [R,N] with values in [0, clusters).

    Returns (indices int32 [R,N], counts int32 [R,C], offsets int32 [R,C+1]).
    """
    lib = _native.load()
    labels = labels.to(torch.int32).contiguous()
    dev = _native.require_cuda(labels)
    rows, tokens = labels.shape
    idx = torch.empty_like(labels)
    counts = torch.empty((rows, clusters), dtype=torch.int32, device=dev)
    offsets = torch.empty((rows, clusters + 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        status = lib.peco_sort_labels(_native.ptr(labels), _native.ptr(idx), _native.ptr(counts),
                                      _native.ptr(offsets), rows, tokens, clusters,
                                      _native.stream_of(dev, labels, idx, counts, offsets))
    _raise(status)
    return idx, counts, offsets
