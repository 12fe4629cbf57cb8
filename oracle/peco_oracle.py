"""CPU restatement of the PECO attention hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA library in ``peco_b200``.  Only the
tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  The product path never calls
it: ``peco_b200`` raises when its CUDA library is unavailable.

Every function restates one step of the reference (Tom-HKUST/PECO) in plain
torch-on-CPU / numpy float32 arithmetic and cites the reference file:line it
follows.  Parity pins: ``tests/golden/make_golden.py`` runs the reference's own
CPU functions (clustering, selection, quantization, text partition) in the
build container and stores their outputs as fixtures; ``tests/test_oracle.py``
checks this module against them bit for bit.  The reference has no CPU
sparse-attention implementation (``peco/attention_cuda.py:96-99`` rejects CPU
tensors); :func:`sparse_attention` follows the CUDA kernel's semantics
(``peco/kernels/sparse_attention.cu:55-190``) and is pinned on the GPU box
against that kernel compiled from the reference's own source (``oracle/Makefile``).
"""

from __future__ import annotations

import math

import numpy as np
import torch


# --------------------------------------------------------------------------
# k-means (peco/clustering.py:16-89, CPU branch :66-80)
# --------------------------------------------------------------------------

def assign_labels(x: torch.Tensor, centers: torch.Tensor, chunk: int = 1024) -> torch.Tensor:
    """Nearest-centre labels of fp32 ``x`` [BH,N,D] against ``centers`` [BH,C,D].

    Distance = ||c||^2 - 2 x.c (the token norm is dropped, clustering.py:69-73);
    argmin keeps the first (lowest) index on exact ties, like torch.argmin and
    kmeans.cu:32.  Chunking mirrors the reference's chunk loop (clustering.py:68).
    """
    x = x.float()
    centers = centers.float()
    bh, n, _ = x.shape
    norms = centers.square().sum(-1).unsqueeze(1)           # [BH,1,C]
    labels = torch.empty((bh, n), dtype=torch.int32)
    for s in range(0, n, chunk):
        d = -2 * torch.bmm(x[:, s:s + chunk], centers.transpose(1, 2))
        d += norms
        labels[:, s:s + chunk] = d.argmin(-1).to(torch.int32)
    return labels


def assignment_margin(x: torch.Tensor, centers: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Distance gap between the second-best centre and the chosen one, per token.

    Used by the tests to excuse label differences that sit on fp32 distance
    ties (labels bit-exact except at fp32 ties).
    """
    x = x.double()
    c = centers.double()
    d = c.square().sum(-1).unsqueeze(1) - 2 * torch.bmm(x, c.transpose(1, 2))
    best = d.gather(-1, labels.long().unsqueeze(-1)).squeeze(-1)
    d.scatter_(-1, labels.long().unsqueeze(-1), float("inf"))
    return d.min(-1).values - best


def update_centers(x: torch.Tensor, labels: torch.Tensor, previous: torch.Tensor):
    """Means of each cluster's tokens; an empty cluster keeps ``previous``.

    Sums accumulate in fp32 in ascending token order (the order torch's CPU
    scatter_add uses, clustering.py:77); mean = sum / count (clustering.py:79-80).
    Returns (means, counts, sums).
    """
    x = x.float()
    bh, n, dims = x.shape
    c = previous.shape[1]
    sums = torch.zeros((bh, c, dims), dtype=torch.float32)
    counts = torch.zeros((bh, c), dtype=torch.int32)
    lab = labels.long()
    sums.scatter_add_(1, lab[..., None].expand(-1, -1, dims), x)
    counts.scatter_add_(1, lab, torch.ones_like(labels))
    means = torch.where(counts[..., None] > 0, sums / counts[..., None].clamp_min(1), previous.float())
    return means, counts, sums


def fit_token_clusters(x: torch.Tensor, n_clusters: int, iters: int, init: torch.Tensor):
    """Fixed-iteration Lloyd k-means (clustering.py:16-89 with tol=0).

    Returns (labels [BH,N] int32, centers [BH,K,D] fp32, counts [BH,K] int32).
    Labels/counts come from the last assignment; centers are the means of that
    partition (the swap at clustering.py:86).
    """
    x = x.float()
    centers = init.float().clone()
    assert centers.shape[1] == n_clusters
    labels = counts = None
    for _ in range(iters):
        labels = assign_labels(x, centers)
        centers, counts, _ = update_centers(x, labels, centers)
    return labels, centers, counts


# --------------------------------------------------------------------------
# reorder (peco/clustering.py:92-136)
# --------------------------------------------------------------------------

def sort_indices(labels: torch.Tensor) -> torch.Tensor:
    """Stable argsort of labels per row -> int32 gather indices (clustering.py:105,108)."""
    return torch.argsort(labels.long(), dim=-1, stable=True).to(torch.int32)


def gather_rows(t: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """packed[bh, j] = t[bh, indices[bh, j]] for [B,H,N,D] t (clustering.py:121-123)."""
    b, h, n, d = t.shape
    return t.gather(2, indices.long().view(b, h, n, 1).expand(-1, -1, -1, d))


def scatter_rows(t: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """out[bh, indices[bh, j]] = t[bh, j] (clustering.py:133-136)."""
    b, h, n, d = t.shape
    out = torch.empty_like(t)
    out.scatter_(2, indices.long().view(b, h, n, 1).expand(-1, -1, -1, d), t)
    return out


# --------------------------------------------------------------------------
# cluster-pair selection (peco/clustering.py:139-186)
# --------------------------------------------------------------------------

def cluster_probabilities(qc: torch.Tensor, kc: torch.Tensor, k_sizes: torch.Tensor) -> torch.Tensor:
    """softmax(Cq.Ck^T / sqrt(D) + log(count_k)) over key clusters, fp32.

    Empty key clusters get -inf logits; an all-empty row yields zeros
    (clustering.py:146-151, scale at :167-168).
    """
    scores = torch.matmul(qc.float(), kc.float().transpose(-1, -2))
    scores *= qc.shape[-1] ** -0.5
    w = k_sizes.float().unsqueeze(-2)
    logits = scores + torch.where(w > 0, w.log(), torch.full_like(w, -math.inf))
    mx = logits.max(dim=-1, keepdim=True).values
    mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    mass = torch.exp(logits - mx)
    return mass / mass.sum(dim=-1, keepdim=True).clamp_min(torch.finfo(torch.float32).tiny)


def select_cluster_connections(qc, kc, q_sizes, k_sizes, p: float, min_kc_ratio: float = 0.0):
    """Boolean [B,H,CQ,CK] map of kept (query cluster, key cluster) pairs.

    Per query cluster: sort probabilities descending (stable), keep while the
    mass before a candidate is < p (all if p == 1), always the first, at least
    ceil(min_kc_ratio*CK); then AND with nonempty key and query clusters
    (clustering.py:165-186).
    """
    probs = cluster_probabilities(qc, kc, k_sizes)
    sp, si = probs.sort(dim=-1, descending=True, stable=True)
    before = sp.cumsum(-1) - sp
    keep = before < p
    if p == 1:
        keep.fill_(True)
    keep[..., 0] = True
    minimum = math.ceil(min_kc_ratio * kc.shape[-2])
    if minimum:
        keep[..., :minimum] = True
    out = torch.zeros_like(probs, dtype=torch.bool)
    out.scatter_(-1, si, keep)
    out &= k_sizes.unsqueeze(-2) > 0
    out &= q_sizes.unsqueeze(-1) > 0
    return out


def extend_text_partition(dmap, q_sizes, k_sizes, valid_text: int, text_length: int):
    """Append the valid-text and padding groups (peco/processor.py:68-84).

    Row -2 (valid text) sees every column but padding; every row but padding
    sees column -2; padding sees only itself.
    """
    b, h, cq, ck = dmap.shape
    out = torch.zeros((b, h, cq + 2, ck + 2), dtype=torch.bool)
    out[..., :cq, :ck] = dmap
    out[..., -2, :-1] = True
    out[..., :-1, -2] = True
    out[..., -1, -1] = True
    extra = torch.tensor([valid_text, text_length - valid_text], dtype=torch.int32).expand(b, h, 2)
    return (out, torch.cat((q_sizes.int(), extra), -1).contiguous(),
            torch.cat((k_sizes.int(), extra), -1).contiguous())


# --------------------------------------------------------------------------
# Base-Offset quantization (peco/quantization.py:96-150), numpy float32
# --------------------------------------------------------------------------

def quantize_base_offset(x: np.ndarray, labels: np.ndarray, centroids: np.ndarray, bits: int):
    """Per token over D: r = x - C[label]; low/high = min/max r;
    scale = (high-low)/(2^b-1) or 1 when not > 0; code = clamp(rint((r-low)/scale)).

    Each step is one IEEE float32 operation, exactly as torch evaluates
    quantization.py:111-118 (no fused multiply-add).  x is [BH,N,D] (any float
    dtype, widened to fp32), labels [BH,N], centroids [BH,K,D].
    Returns (codes uint8 [BH,N,D], low fp32 [BH,N,1], scale fp32 [BH,N,1]).
    """
    assert bits in (4, 8)
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(centroids, dtype=np.float32)
    lab = np.asarray(labels, dtype=np.int64)
    base = np.take_along_axis(c, lab[..., None], axis=1)                    # [BH,N,D]
    r = (x - base).astype(np.float32)
    low = r.min(axis=-1, keepdims=True)
    high = r.max(axis=-1, keepdims=True)
    levels = np.float32((1 << bits) - 1)
    raw = ((high - low).astype(np.float32) / levels).astype(np.float32)
    scale = np.where(raw > 0, raw, np.float32(1)).astype(np.float32)
    q = ((r - low).astype(np.float32) / scale).astype(np.float32)
    codes = np.clip(np.rint(q), 0, levels).astype(np.uint8)
    return codes, low.astype(np.float32), scale


def dequantize_base_offset(codes, low, scale, labels, centroids) -> np.ndarray:
    """x_hat = C[label] + (low + scale*code), fp32, mul then add (quantization.py:134-136)."""
    c = np.asarray(centroids, dtype=np.float32)
    base = np.take_along_axis(c, np.asarray(labels, dtype=np.int64)[..., None], axis=1)
    res = (low + (scale * codes.astype(np.float32)).astype(np.float32)).astype(np.float32)
    return (base + res).astype(np.float32)


def fake_quantize_base_offset(x: torch.Tensor, labels, centroids, bits: int) -> torch.Tensor:
    """Quantize/dequantize ``x`` ([B,H,N,D] or [BH,N,D]); bits=0 is identity (quantization.py:139-150).

    The fp32 reconstruction is rounded once to x.dtype (round-to-nearest-even).
    """
    if bits == 0:
        return x
    shape = x.shape
    n, d = shape[-2:]
    flat = x.reshape(-1, n, d).float().numpy()
    lab = labels.reshape(flat.shape[:2]).numpy()
    cen = centroids.float().numpy()
    codes, low, scale = quantize_base_offset(flat, lab, cen, bits)
    xhat = dequantize_base_offset(codes, low, scale, lab, cen)
    return torch.from_numpy(xhat).to(x.dtype).reshape(shape)


# --------------------------------------------------------------------------
# cluster-block-sparse attention (semantics of peco/kernels/sparse_attention.cu)
# --------------------------------------------------------------------------

def group_prefix(sizes: torch.Tensor, total: int) -> torch.Tensor:
    """Run starts of consecutive groups, clamped like make_work_map (sparse_attention.cu:25-31)."""
    out = torch.zeros(sizes.shape[-1] + 1, dtype=torch.int64)
    off = 0
    for c, s in enumerate(sizes.tolist()):
        s = max(0, min(int(s), total - off))
        off += s
        out[c + 1] = off
    return out


def sparse_attention(q, k, v, dmap, q_sizes, k_sizes) -> torch.Tensor:
    """O = softmax(Q K^T / sqrt(D), masked by map[group(i), group(j)]) V, fp32.

    Q [B,H,SQ,D], K/V [B,H,SK,D] in group-packed order, map [B,H,GQ,GK] bool,
    sizes [B,H,GQ] / [B,H,GK].  A row with no allowed key, or a row outside
    every query group, returns zero (sparse_attention.cu:183-187; rows beyond
    the sizes' sum are never written by the reference and are zeros here).
    Computed per query group over the gathered allowed keys, so memory stays
    proportional to the sparse work.
    """
    b, h, sq, d = q.shape
    sk = k.shape[2]
    out = torch.zeros((b, h, sq, d), dtype=torch.float32)
    scale = 1.0 / math.sqrt(d)
    for bi in range(b):
        for hi in range(h):
            qp = group_prefix(q_sizes[bi, hi], sq)
            kp = group_prefix(k_sizes[bi, hi], sk)
            m = dmap[bi, hi]
            qf = q[bi, hi].float()
            kf = k[bi, hi].float()
            vf = v[bi, hi].float()
            for g in range(m.shape[0]):
                q0, q1 = int(qp[g]), int(qp[g + 1])
                if q1 <= q0:
                    continue
                cols = [torch.arange(int(kp[c]), int(kp[c + 1])) for c in torch.nonzero(m[g]).flatten().tolist()
                        if kp[c + 1] > kp[c]]
                if not cols:
                    continue
                idx = torch.cat(cols)
                s = (qf[q0:q1] @ kf[idx].T) * scale
                out[bi, hi, q0:q1] = torch.softmax(s, dim=-1) @ vf[idx]
    return out


def sparse_attention_rows(q, k, v, dmap, q_sizes, k_sizes, rows) -> torch.Tensor:
    """:func:`sparse_attention` of one head evaluated only at packed query ``rows``.

    q [SQ,D], k/v [SK,D] in group-packed order, dmap [GQ,GK], sizes [GQ]/[GK],
    rows a 1-D index tensor.  Each row attends to the key runs of the groups
    its own group selects (sparse_attention.cu:55-190); rows of no group or
    with no allowed key are zero.  Cost is proportional to the sampled rows,
    which is what makes the 119k-token configuration checkable on a CPU.
    Returns fp32 [len(rows), D].
    """
    sq, d = q.shape
    sk = k.shape[0]
    qp = group_prefix(q_sizes, sq)
    kp = group_prefix(k_sizes, sk)
    group = torch.searchsorted(qp[1:], rows.long(), right=True)
    out = torch.zeros((rows.numel(), d), dtype=torch.float32)
    scale = 1.0 / math.sqrt(d)
    kf, vf = k.float(), v.float()
    for g in torch.unique(group).tolist():
        if g >= dmap.shape[0]:
            continue
        sel = (group == g).nonzero().flatten()
        cols = [torch.arange(int(kp[c]), int(kp[c + 1])) for c in torch.nonzero(dmap[g]).flatten().tolist()
                if kp[c + 1] > kp[c]]
        if not cols:
            continue
        idx = torch.cat(cols)
        s = (q[rows[sel].long()].float() @ kf[idx].T) * scale
        out[sel] = torch.softmax(s, dim=-1) @ vf[idx]
    return out


# --------------------------------------------------------------------------
# one PECO attention call (peco/processor.py:115-157, non-warmup branch)
# --------------------------------------------------------------------------

def peco_attention_call(q, k, v, *, text_length: int, valid_text: int, num_q_centroids: int,
                        num_k_centroids: int, iters: int, q_init, k_init, top_p: float,
                        min_kc_ratio: float, bits: int, return_state: bool = False):
    """Full hot path on CPU: k-means Q/K, selection, fake quant, reorder,
    sparse attention, inverse reorder.  q/k/v are [1,H,S,D] (any float dtype);
    the output has q's dtype.  ``q_init``/``k_init`` are fp32 [H,C,D] centroids.
    """
    b, h, s, d = q.shape
    nv = s - text_length
    qv, kv, vv = q[:, :, :nv], k[:, :, :nv], v[:, :, :nv]
    q_lab, q_cen, q_cnt = fit_token_clusters(qv.reshape(b * h, nv, d), num_q_centroids, iters, q_init)
    k_lab, k_cen, k_cnt = fit_token_clusters(kv.reshape(b * h, nv, d), num_k_centroids, iters, k_init)
    q_sizes, k_sizes = q_cnt.reshape(b, h, -1), k_cnt.reshape(b, h, -1)
    dmap = select_cluster_connections(q_cen.reshape(b, h, -1, d), k_cen.reshape(b, h, -1, d),
                                      q_sizes, k_sizes, top_p, min_kc_ratio)
    qv = fake_quantize_base_offset(qv, q_lab, q_cen, bits)
    kv = fake_quantize_base_offset(kv, k_lab, k_cen, bits)
    qi, ki = sort_indices(q_lab), sort_indices(k_lab)
    qv, kv, vv = gather_rows(qv, qi), gather_rows(kv, ki), gather_rows(vv, ki)
    qp = torch.cat((qv, q[:, :, nv:]), 2)
    kp = torch.cat((kv, k[:, :, nv:]), 2)
    vp = torch.cat((vv, v[:, :, nv:]), 2)
    emap, eqs, eks = extend_text_partition(dmap, q_sizes, k_sizes, valid_text, text_length)
    packed = sparse_attention(qp, kp, vp, emap, eqs, eks)
    text_idx = torch.arange(nv, s, dtype=torch.int32)
    idx = torch.cat((qi.reshape(b * h, nv), text_idx.expand(b * h, -1)), -1)
    out = scatter_rows(packed, idx).to(q.dtype)
    if return_state:
        return out, dict(q_labels=q_lab, k_labels=k_lab, q_centroids=q_cen, k_centroids=k_cen,
                         q_counts=q_cnt, k_counts=k_cnt, map=dmap, q_indices=qi, k_indices=ki)
    return out
