"""Sequence-to-head resharding for long-video PECO attention (Ulysses style).

Long sequences arrive sequence-sharded: rank r of P holds the tokens
[r*S/P, (r+1)*S/P) of every head, ``[B, H, S/P, D]``.  PECO's stages are
per head, so one exchange regroups the data as all tokens of H/P heads,
``[B, H/P, S, D]`` (rank r owns heads [r*H/P, (r+1)*H/P)).  The PECO call runs
on those heads with no further communication, and the inverse exchange
returns each rank's token shard of the output.

The exchange is one batch of point-to-point transfers per tensor
(``torch.distributed.batch_isend_irecv``: NCCL over NVLink on a B200 box,
gloo on the CPU in the tests).  Every transferred piece is one (batch, head)
row block of S/P x D elements, which is contiguous both where it is read and
where it lands, so the transfers read the caller's tensor and write the final
layout directly -- no packing copy before and no unpacking copy after.  Only
the rank's own piece moves by a local device copy.  K's and V's transfers can
stay in flight while the call clusters Q (and K), see
:func:`sequence_parallel_attention`.  No kernel reads another GPU's memory.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group):
    """Ranks in the group (1 when torch.distributed is not initialised)."""
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def _rank(group):
    return dist.get_rank(group)


def _peer(group, q):
    """Global rank of group rank q (P2P ops address global ranks)."""
    return q if group is None else dist.get_global_rank(group, q)


def _exchange(ops):
    """Start a batch of P2P ops; returns the works (empty when there are none)."""
    return dist.batch_isend_irecv(ops) if ops else []


def seq_to_heads_async(x: torch.Tensor, group=None):
    """Start resharding [B, H, S/P, D] -> [B, H/P, S, D]; returns ``(out, ready)``.

    ``out`` is the head shard's buffer; it holds the data once ``ready()`` has
    run on the stream that reads it (``ready`` makes that stream wait for the
    transfers).  ``x`` must stay unmodified until then."""
    p = _world(group)
    if p == 1:
        return x, (lambda: None)
    b, h, s_local, d = x.shape
    if h % p:
        raise ValueError(f"{h} heads do not split over {p} ranks")
    x = x.contiguous()
    r, hl = _rank(group), h // p
    out = torch.empty((b, hl, p * s_local, d), dtype=x.dtype, device=x.device)
    # out[bi, j, q*S/P:(q+1)*S/P] = rank q's tokens of head r*H/P + j
    pieces = out.view(b, hl, p, s_local, d)
    ops = []
    for q in range(p):
        if q == r:
            continue
        for bi in range(b):
            for j in range(hl):
                ops.append(dist.P2POp(dist.isend, x[bi, q * hl + j], _peer(group, q), group))
                ops.append(dist.P2POp(dist.irecv, pieces[bi, j, q], _peer(group, q), group))
    works = _exchange(ops)
    pieces[:, :, r].copy_(x[:, r * hl:(r + 1) * hl])

    def ready(x=x):  # holds the source until the transfers are done
        for w in works:
            w.wait()

    return out, ready


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, H, S/P, D] sequence shard -> [B, H/P, S, D] head shard (this rank's heads)."""
    out, ready = seq_to_heads_async(x, group)
    ready()
    return out


def heads_to_seq(o: torch.Tensor, group=None) -> torch.Tensor:
    """[B, H/P, S, D] head shard -> [B, H, S/P, D] sequence shard (inverse of seq_to_heads)."""
    p = _world(group)
    if p == 1:
        return o
    b, hl, s, d = o.shape
    if s % p:
        raise ValueError(f"{s} tokens do not split over {p} ranks")
    o = o.contiguous()
    r, sl = _rank(group), s // p
    out = torch.empty((b, p * hl, sl, d), dtype=o.dtype, device=o.device)
    # rank q receives its tokens of this rank's heads; this rank receives its
    # tokens of rank q's heads into heads [q*H/P, (q+1)*H/P)
    src = o.view(b, hl, p, sl, d)
    ops = []
    for q in range(p):
        if q == r:
            continue
        for bi in range(b):
            for j in range(hl):
                ops.append(dist.P2POp(dist.isend, src[bi, j, q], _peer(group, q), group))
                ops.append(dist.P2POp(dist.irecv, out[bi, q * hl + j], _peer(group, q), group))
    works = _exchange(ops)
    out[:, r * hl:(r + 1) * hl].copy_(src[:, :, r])
    for w in works:
        w.wait()
    return out


def sequence_parallel_attention(attention, query, key, value, group=None, *, overlap=False):
    """Run a per-head attention callable (e.g. ``PecoAttention.attention``) on
    sequence-sharded Q/K/V ``[B, H, S/P, D]`` and return the output in the same
    sharding: reshard to heads, attend locally, reshard back.

    With ``overlap`` the callable must accept ``key_ready=`` and
    ``value_ready=`` (as ``PecoAttention.attention`` does): Q's exchange
    completes first, K's and V's are still in flight when the call starts,
    and each is waited for on the stream where that tensor is first read --
    K after Q's clustering, V after both.  Pending transfers are always waited
    for, also when the callable raises, so no buffer is reused while a
    transfer still writes it."""
    q = seq_to_heads(query, group)
    if not overlap:
        return heads_to_seq(attention(q, seq_to_heads(key, group), seq_to_heads(value, group)), group)
    k, k_ready = seq_to_heads_async(key, group)
    v, v_ready = seq_to_heads_async(value, group)
    pending = {"k": k_ready, "v": v_ready}

    def once(name):
        def ready():
            fn = pending.pop(name, None)
            if fn is not None:
                fn()
        return ready

    try:
        o = attention(q, k, v, key_ready=once("k"), value_ready=once("v"))
    finally:
        for fn in list(pending.values()):
            fn()
        pending.clear()
    return heads_to_seq(o, group)
