"""Cluster-sparse attention over libpeco_b200.so, with the reference's signature.

Mirrors peco/attention_cuda.py:65-145: same validation (shapes, dtypes,
contiguity, int32 limits, inference only), same workspace size, same output
convention (a completely masked row returns zero).  The kernel is the
tcgen05/TMEM implementation in csrc/attention.cu.  Size checks that the
reference performs with device asserts (``torch._assert_async``, which trap
the context) are done with a host-side reduction when ``validate_sizes`` is
set, so a bad call raises instead of killing the CUDA context.
"""

from __future__ import annotations

import torch

from . import _native


def _validate(q, k, v, dynamic_map, q_sizes, k_sizes):
    tensors = (q, k, v, dynamic_map, q_sizes, k_sizes)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        raise TypeError("All sparse attention inputs must be torch tensors")
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape:
        raise ValueError("Expected Q [B,H,SQ,D] and equal-shaped K/V [B,H,SK,D]")
    batch, heads, sq, dim = q.shape
    if batch < 1 or heads < 1 or batch * heads > 65535:
        raise ValueError("B*H must be between 1 and 65535")
    if k.shape[:2] != q.shape[:2] or k.shape[-1] != dim:
        raise ValueError("Q and K/V batch, head, and feature dimensions must match")
    if dim not in (64, 128):
        raise ValueError("CUDA attention supports head dimensions 64 and 128")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("Q/K/V must share dtype torch.float16 or torch.bfloat16")
    if not q.is_cuda or any(t.device != q.device for t in tensors):
        raise ValueError("All sparse attention inputs must reside on the same CUDA device")
    if any(not t.is_contiguous() for t in tensors):
        raise ValueError("All sparse attention inputs must be contiguous")
    if q_sizes.ndim != 3 or k_sizes.ndim != 3 or q_sizes.shape[:2] != (batch, heads) or k_sizes.shape[:2] != (batch, heads):
        raise ValueError("Cluster sizes must have shape [B,H,C]")
    cq, ck = q_sizes.shape[-1], k_sizes.shape[-1]
    if cq < 1 or ck < 1 or dynamic_map.shape != (batch, heads, cq, ck):
        raise ValueError("Expected a nonempty cluster axis and dynamic_map [B,H,CQ,CK]")
    if dynamic_map.dtype != torch.bool or q_sizes.dtype != torch.int32 or k_sizes.dtype != torch.int32:
        raise TypeError("dynamic_map must be bool and cluster sizes must be int32")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise RuntimeError("PECO CUDA sparse attention supports inference only; use torch.no_grad()")
    return batch, heads, sq, dim, cq, ck


def sparse_attention(q, k, v, dynamic_map, q_sizes, k_sizes, *, validate_sizes: bool = True):
    """Return cluster-masked softmax(QK^T/sqrt(D))V.

    Inputs must be contiguous CUDA tensors: Q [B,H,SQ,D], K/V [B,H,SK,D],
    bool map [B,H,CQ,CK], and int32 sizes [B,H,CQ/CK].  Tokens must already be
    grouped in cluster order.  Empty clusters and completely masked rows are
    supported; a completely masked row returns zero.  ``validate_sizes``
    checks nonnegative counts with exact sums (a host synchronisation); set it
    to False when the caller guarantees them.
    """
    batch, heads, sq, dim, cq, ck = _validate(q, k, v, dynamic_map, q_sizes, k_sizes)
    sk = k.shape[-2]
    capacity = (sq + 15) // 16 + cq
    stride = ck + 2 + 3 * capacity
    if max(sq, sk, cq, ck, capacity, stride) > 2**31 - 1:
        raise ValueError("Sequence/cluster metadata exceeds the CUDA int32 indexing limit")
    with torch.cuda.device(q.device):
        if validate_sizes:
            bad = ((q_sizes < 0).any() | (k_sizes < 0).any() | (q_sizes.sum(-1) != sq).any()
                   | (k_sizes.sum(-1) != sk).any())
            if bool(bad):
                raise ValueError("cluster sizes must be nonnegative and sum to the sequence lengths")
        output = torch.empty_like(q)
        if sq == 0:
            return output
        workspace = torch.empty(batch * heads * stride, dtype=torch.int32, device=q.device)
        lib = _native.load()
        status = lib.peco_sparse_attention(
            _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(dynamic_map), _native.ptr(q_sizes),
            _native.ptr(k_sizes), _native.ptr(output), _native.ptr(workspace), batch * heads, sq, sk, dim, cq, ck,
            0 if q.dtype == torch.float16 else 1,
            _native.stream_of(q.device, q, k, v, dynamic_map, q_sizes, k_sizes, workspace, output))
        if status:
            msg = lib.peco_attention_error_string(int(status)).decode("utf-8", errors="replace")
            raise RuntimeError(f"PECO CUDA sparse attention launch failed: {msg} ({status})")
        return output


def plan_key_blocks(dynamic_map, q_sizes, k_sizes, sq, k, v):
    """Plan a fused attention call and pack row-major K/V [B,H,SK,D] into key
    blocks: returns (workspace, k_blocks, v_blocks) for
    ``peco_sparse_attention_restore``.  The same steps the drop-in
    ``sparse_attention`` takes internally, exposed for callers that keep the
    plan (and tests of the fused entry points)."""
    batch, heads, sk, dim = k.shape
    bh = batch * heads
    gq, gk = q_sizes.shape[-1], k_sizes.shape[-1]
    lib = _native.load()
    with torch.cuda.device(k.device):
        ws = torch.empty(bh * int(lib.peco_attention_workspace_stride(sq, sk, gq, gk)), dtype=torch.int32,
                         device=k.device)
        kb = torch.empty((bh, int(lib.peco_key_block_rows(sk, gk)), dim), dtype=k.dtype, device=k.device)
        vb = torch.empty_like(kb)
        stream = _native.stream_of(k.device, dynamic_map, q_sizes, k_sizes, k, v, ws, kb, vb)
        _native.check(lib.peco_attention_plan(_native.ptr(dynamic_map), _native.ptr(q_sizes), _native.ptr(k_sizes),
                                              _native.ptr(kb), _native.ptr(vb), _native.ptr(ws), bh, sq, sk, dim, gq,
                                              gk, stream), "peco_attention_plan")
        _native.check(lib.peco_pack_key_blocks(_native.ptr(k), _native.ptr(v), _native.ptr(kb), _native.ptr(vb),
                                               _native.ptr(ws), bh, sq, sk, dim, gq, gk, stream),
                      "peco_pack_key_blocks")
    return ws, kb, vb
