"""The reference's own CUDA kernels, built from its sources by oracle/Makefile.

TEST INFRASTRUCTURE ONLY (the GPU tests use it to pin the B200 kernels and the
CPU oracle against the reference kernels; bench.py may time it as the
reference's GPU path).  The call sequence restates the reference's Python
glue: ``sparse_attention`` follows peco/attention_cuda.py:84-145 (workspace
int32 BH*(CK+2+3*(ceil(SQ/16)+CQ))), the clustering calls follow
peco/clustering_cuda.py:93-146 and peco/clustering.py:59-88, and
``peco_attention_call`` follows peco/processor.py:130-157.
"""

from __future__ import annotations

import ctypes
import math
from pathlib import Path

import torch

REF_DIR = Path(__file__).resolve().parent / "_ref"
_LIBS = {}


def available() -> bool:
    return (REF_DIR / "libpeco_attention_ref.so").exists() and (REF_DIR / "libpeco_clustering_ref.so").exists()


def _lib(name):
    if name not in _LIBS:
        lib = ctypes.CDLL(str(REF_DIR / name))
        P, I = ctypes.c_void_p, ctypes.c_int
        if "attention" in name:
            lib.peco_sparse_attention.argtypes = [P] * 8 + [I] * 7 + [P]
            lib.peco_sparse_attention.restype = I
        else:
            lib.peco_assign_tokens_to_centers.argtypes = [P] * 5 + [I] * 5 + [P]
            lib.peco_recompute_cluster_centers.argtypes = [P] * 6 + [I] * 4 + [P]
            lib.peco_reorder_token_features.argtypes = [P] * 3 + [I] * 5 + [P]
            for f in ("peco_assign_tokens_to_centers", "peco_recompute_cluster_centers",
                      "peco_reorder_token_features"):
                getattr(lib, f).restype = I
        _LIBS[name] = lib
    return _LIBS[name]


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def sparse_attention(q, k, v, dmap, q_sizes, k_sizes):
    """The reference WMMA kernel on contiguous CUDA tensors (no size asserts)."""
    b, h, sq, d = q.shape
    sk = k.shape[2]
    cq, ck = q_sizes.shape[-1], k_sizes.shape[-1]
    cap = (sq + 15) // 16 + cq
    ws = torch.empty(b * h * (ck + 2 + 3 * cap), dtype=torch.int32, device=q.device)
    out = torch.empty_like(q)
    st = _lib("libpeco_attention_ref.so").peco_sparse_attention(
        _p(q), _p(k), _p(v), _p(dmap), _p(q_sizes), _p(k_sizes), _p(out), _p(ws), b * h, sq, sk, d, cq, ck,
        0 if q.dtype == torch.float16 else 1, _stream(q.device))
    if st:
        raise RuntimeError(f"reference sparse attention failed ({st})")
    return out


def fit_token_clusters(x, n_clusters, iters, init, chunk_size=1024):
    """Reference CUDA k-means loop (cuBLAS SGEMM + argmin, atomic update)."""
    lib = _lib("libpeco_clustering_ref.so")
    x = x.float().contiguous()
    bh, n, d = x.shape
    centers = init.float().contiguous().clone()
    labels = torch.empty((bh, n), dtype=torch.int32, device=x.device)
    counts = torch.empty((bh, n_clusters), dtype=torch.int32, device=x.device)
    sums = torch.empty_like(centers)
    means = torch.empty_like(centers)
    chunk = min(chunk_size, n)
    scratch = torch.empty((chunk, n_clusters), dtype=torch.float32, device=x.device)
    norms = torch.empty((bh, n_clusters), dtype=torch.float32, device=x.device)
    s = _stream(x.device)
    for _ in range(iters):
        st = lib.peco_assign_tokens_to_centers(_p(x), _p(centers), _p(labels), _p(scratch), _p(norms), bh, n, d,
                                               n_clusters, chunk, s)
        st = st or lib.peco_recompute_cluster_centers(_p(x), _p(labels), _p(centers), _p(sums), _p(counts),
                                                      _p(means), bh, n, d, n_clusters, s)
        if st:
            raise RuntimeError(f"reference clustering failed ({st})")
        centers, means = means, centers
    return labels, centers, counts


def reorder(t, idx, inverse=False):
    lib = _lib("libpeco_clustering_ref.so")
    t = t.contiguous()
    out = torch.empty_like(t)
    b, h, n, d = t.shape
    st = lib.peco_reorder_token_features(_p(t), _p(idx), _p(out), b * h, n, d, t.element_size(), int(inverse),
                                         _stream(t.device))
    if st:
        raise RuntimeError(f"reference reorder failed ({st})")
    return out


def peco_attention_call(q, k, v, *, text_length, valid_text, num_q_centroids, num_k_centroids, iters, q_init,
                        k_init, top_p, min_kc_ratio, bits):
    """The reference GPU path of one call: its CUDA kernels for k-means, reorder
    and attention, torch ops for selection / quantization / text partition
    exactly as the reference runs them (CUDA tensors)."""
    from . import peco_oracle as O
    b, h, s, d = q.shape
    nv = s - text_length
    qv, kv, vv = (t[:, :, :nv].contiguous() for t in (q, k, v))
    ql, qc, qn = fit_token_clusters(qv.reshape(b * h, nv, d), num_q_centroids, iters, q_init)
    kl, kc, kn = fit_token_clusters(kv.reshape(b * h, nv, d), num_k_centroids, iters, k_init)
    qs, ks = qn.reshape(b, h, -1), kn.reshape(b, h, -1)
    dmap = O.select_cluster_connections(qc.reshape(b, h, -1, d), kc.reshape(b, h, -1, d), qs, ks, top_p,
                                        min_kc_ratio)
    if bits:
        qv = _fake_quant_torch(qv, ql, qc, bits)
        kv = _fake_quant_torch(kv, kl, kc, bits)
    qi = torch.argsort(ql, dim=-1, stable=True).to(torch.int32).contiguous()
    ki = torch.argsort(kl, dim=-1, stable=True).to(torch.int32).contiguous()
    qv, kv, vv = reorder(qv, qi), reorder(kv, ki), reorder(vv, ki)
    qp = torch.cat((qv, q[:, :, nv:]), 2).contiguous()
    kp = torch.cat((kv, k[:, :, nv:]), 2).contiguous()
    vp = torch.cat((vv, v[:, :, nv:]), 2).contiguous()
    import torch.nn.functional as F
    m = F.pad(dmap, (0, 2, 0, 2), value=False)
    m[..., -2, :-1] = True
    m[..., :-1, -2] = True
    m[..., -1, -1] = True
    extra = torch.tensor([valid_text, text_length - valid_text], device=q.device, dtype=torch.int32).expand(b, h, 2)
    eqs = torch.cat((qs, extra), -1).to(torch.int32).contiguous()
    eks = torch.cat((ks, extra), -1).to(torch.int32).contiguous()
    out = sparse_attention(qp, kp, vp, m.contiguous(), eqs, eks)
    text_idx = torch.arange(nv, s, device=q.device, dtype=torch.int32)
    idx = torch.cat((qi.reshape(b * h, nv), text_idx.expand(b * h, -1)), -1).contiguous()
    return reorder(out, idx, inverse=True)


def _fake_quant_torch(x, labels, centroids, bits):
    """peco/quantization.py:96-150 in torch ops on the tensors' device."""
    n, d = x.shape[-2:]
    flat = x.reshape(-1, n, d)
    lab = labels.long()
    base = centroids.gather(1, lab.unsqueeze(-1).expand(-1, -1, d))
    r = flat.float() - base
    low = r.amin(-1, keepdim=True)
    high = r.amax(-1, keepdim=True)
    levels = (1 << bits) - 1
    raw = (high - low) / levels
    scale = torch.where(raw > 0, raw, torch.ones_like(raw))
    codes = ((r - low) / scale).round().clamp_(0, levels).to(torch.uint8)
    res = low + scale * codes.float()
    return (base + res).to(x.dtype).reshape(x.shape)
