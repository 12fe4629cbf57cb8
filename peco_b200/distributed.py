"""Sequence-to-head resharding for long-video PECO attention (Ulysses style).

Long sequences arrive sequence-sharded: rank r of P holds the tokens
[r*S/P, (r+1)*S/P) of every head, ``[B, H, S/P, D]``.  PECO's stages are
per head, so one exchange regroups the data as all tokens of H/P heads,
``[B, H/P, S, D]`` (rank r owns heads [r*H/P, (r+1)*H/P)).  The PECO call runs
on those heads with no further communication, and the inverse exchange
returns each rank's token shard of the output.

Every transferred piece is one (batch, head) row block of S/P x D elements,
contiguous both where it is read and where it lands, so no exchange packs or
unpacks.  Two transports:

* CUDA tensors in an NCCL group: the library's peer-memory exchange
  (``peco_exchange_put`` / ``peco_exchange_wait``): every rank's receive
  buffers and flags live in torch symmetric memory, a rank copies its pieces
  straight into the destinations' buffers with plain stores over NVLink and
  raises a flag; the receiving stream waits (bounded) on the flags.  One
  buffer per ``slot``: an exchange overwrites its slot's previous contents.
* anything else (gloo on the CPU in the tests, or a process without symmetric
  memory): one batch of point-to-point transfers
  (``torch.distributed.batch_isend_irecv``) of the same pieces.

K's and V's exchanges can stay in flight while the call clusters Q (and K),
see :func:`sequence_parallel_attention`.  No kernel reads another GPU's
memory; no load uses multicast.
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


# slots of the peer-memory transport (one receive buffer each)
SLOT_Q, SLOT_K, SLOT_V, SLOT_O = 0, 1, 2, 3
_PEER = {}
last_transport = None  # "peer-memory" or "p2p-ops": the transport of the latest exchange


class _PeerSlot:
    """One receive buffer and flag array in symmetric memory, with the device
    tables of every rank's mapped addresses and the piece list of one
    exchange layout."""

    def __init__(self, group, shape, dtype, device, pieces):
        import torch.distributed._symmetric_memory as symm
        self.world, self.rank = _world(group), _rank(group)
        self.buf = symm.empty(shape, dtype=dtype, device=device)
        self.flags = symm.empty(self.world, dtype=torch.int64, device=device)
        self.flags.zero_()
        hb, hf = symm.rendezvous(self.buf, group or dist.group.WORLD), symm.rendezvous(self.flags, group or dist.group.WORLD)
        self.buffers = torch.tensor(list(hb.buffer_ptrs), dtype=torch.int64, device=device)
        self.flag_ptrs = torch.tensor(list(hf.buffer_ptrs), dtype=torch.int64, device=device)
        self.done = torch.zeros(1, dtype=torch.int32, device=device)
        src, dst_rank, dst = zip(*pieces)
        self.src_off = torch.tensor(src, dtype=torch.int64, device=device)
        self.dst_rank = torch.tensor(dst_rank, dtype=torch.int32, device=device)
        self.dst_off = torch.tensor(dst, dtype=torch.int64, device=device)
        self.pieces = len(pieces)
        self.epoch = 0
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every flag array is zero before any rank writes into it


def _peer_ok(x, group):
    return x.is_cuda and _world(group) > 1 and dist.get_backend(group) == "nccl"


def _peer_slot(group, slot, shape, dtype, device, pieces):
    key = (id(group), slot, tuple(shape), dtype, device)
    ps = _PEER.get(key)
    if ps is None:
        ps = _PEER[key] = _PeerSlot(group, shape, dtype, device, pieces)
    return ps


def _peer_put(ps, x, piece_bytes):
    from . import _native
    lib = _native.load()
    ps.epoch += 1
    keep = [x, ps.buffers, ps.flag_ptrs, ps.done, ps.src_off, ps.dst_rank, ps.dst_off, ps.buf, ps.flags]
    stream = _native.stream_of(x.device, *keep)
    _native.check(lib.peco_exchange_put(_native.ptr(x), _native.ptr(ps.src_off), _native.ptr(ps.dst_rank),
                                        _native.ptr(ps.dst_off), int(piece_bytes), ps.pieces, _native.ptr(ps.buffers),
                                        _native.ptr(ps.flag_ptrs), 0, ps.rank, ps.world, ps.epoch,
                                        _native.ptr(ps.done), stream), "peco_exchange_put")
    epoch = ps.epoch

    def ready():
        st = lib.peco_exchange_wait(_native.ptr(ps.flags), ps.world, 0, epoch,
                                    _native.stream_of(x.device, ps.flags, ps.buf))
        _native.check(st, "peco_exchange_wait")

    return ready


def seq_to_heads_async(x: torch.Tensor, group=None, slot: int = SLOT_Q):
    """Start resharding [B, H, S/P, D] -> [B, H/P, S, D]; returns ``(out, ready)``.

    ``out`` is the head shard's buffer; it holds the data once ``ready()`` has
    run on the stream that reads it (``ready`` makes that stream wait for the
    transfers).  ``x`` must stay unmodified until then.  On the peer-memory
    transport ``out`` is ``slot``'s receive buffer, overwritten by the slot's
    next exchange."""
    global last_transport
    p = _world(group)
    if p == 1:
        return x, (lambda: None)
    b, h, s_local, d = x.shape
    if h % p:
        raise ValueError(f"{h} heads do not split over {p} ranks")
    x = x.contiguous()
    r, hl = _rank(group), h // p
    if _peer_ok(x, group):
        es = x.element_size()
        piece = s_local * d * es
        # piece (q, bi, j): x[bi, q*hl + j] -> rank q's out[bi, j, r*S/P:(r+1)*S/P]
        pieces = [(((bi * h + q * hl + j) * s_local) * d * es, q, ((bi * hl + j) * p * s_local + r * s_local) * d * es)
                  for q in range(p) for bi in range(b) for j in range(hl)]
        ps = _peer_slot(group, slot, (b, hl, p * s_local, d), x.dtype, x.device, pieces)
        last_transport = "peer-memory"
        return ps.buf, _peer_put(ps, x, piece)
    last_transport = "p2p-ops"
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


def seq_to_heads(x: torch.Tensor, group=None, slot: int = SLOT_Q) -> torch.Tensor:
    """[B, H, S/P, D] sequence shard -> [B, H/P, S, D] head shard (this rank's heads)."""
    out, ready = seq_to_heads_async(x, group, slot)
    ready()
    return out


def heads_to_seq(o: torch.Tensor, group=None, slot: int = SLOT_O) -> torch.Tensor:
    """[B, H/P, S, D] head shard -> [B, H, S/P, D] sequence shard (inverse of
    seq_to_heads).  Returns a tensor of its own (not a transport buffer)."""
    global last_transport
    p = _world(group)
    if p == 1:
        return o
    b, hl, s, d = o.shape
    if s % p:
        raise ValueError(f"{s} tokens do not split over {p} ranks")
    o = o.contiguous()
    r, sl = _rank(group), s // p
    if _peer_ok(o, group):
        es = o.element_size()
        h = hl * p
        # piece (q, bi, j): o[bi, j, q*S/P:(q+1)*S/P] -> rank q's out[bi, r*hl + j]
        pieces = [(((bi * hl + j) * s + q * sl) * d * es, q, ((bi * h + r * hl + j) * sl) * d * es)
                  for q in range(p) for bi in range(b) for j in range(hl)]
        ps = _peer_slot(group, slot, (b, h, sl, d), o.dtype, o.device, pieces)
        _peer_put(ps, o, sl * d * es)()
        last_transport = "peer-memory"
        return ps.buf.clone()
    last_transport = "p2p-ops"
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
    q = seq_to_heads(query, group, SLOT_Q)
    if not overlap:
        return heads_to_seq(attention(q, seq_to_heads(key, group, SLOT_K), seq_to_heads(value, group, SLOT_V)), group)
    k, k_ready = seq_to_heads_async(key, group, SLOT_K)
    v, v_ready = seq_to_heads_async(value, group, SLOT_V)
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
