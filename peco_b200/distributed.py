"""Sequence-to-head resharding for long-video PECO attention (Ulysses style).

Long sequences arrive sequence-sharded: rank r of P holds the tokens
[r*S/P, (r+1)*S/P) of every head, ``[B, H, S/P, D]``.  PECO's stages are
per head, so one all-to-all regroups the data as all tokens of H/P heads,
``[B, H/P, S, D]`` (rank r owns heads [r*H/P, (r+1)*H/P)).  The PECO call runs
on those heads with no further communication, and the inverse all-to-all
returns each rank's token shard of the output.

Both all-to-alls are ``torch.distributed.all_to_all_single`` on the default
(or given) process group -- NCCL over NVLink on a B200 box, gloo on the CPU
in the tests.  V's can stay in flight while the call clusters Q and K
(``overlap_value``).  No kernel reads another GPU's memory.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group):
    """Ranks in the group (1 when torch.distributed is not initialised)."""
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def seq_to_heads_async(x: torch.Tensor, group=None):
    """Start resharding [B, H, S/P, D] -> [B, H/P, S, D]; returns ``(out, ready)``.

    ``out`` is the head shard's buffer; it holds the data once ``ready()`` has
    run on the stream that reads it (``ready`` waits for the all-to-all and
    lays the received chunks out in token order)."""
    p = _world(group)
    if p == 1:
        return x, (lambda: None)
    b, h, s_local, d = x.shape
    if h % p:
        raise ValueError(f"{h} heads do not split over {p} ranks")
    # chunk q of the send buffer (heads [q*H/P, (q+1)*H/P) of every batch) goes to rank q
    send = x.reshape(b, p, h // p, s_local, d).transpose(0, 1).contiguous()
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=group, async_op=True)
    out = torch.empty((b, h // p, p * s_local, d), dtype=x.dtype, device=x.device)

    def ready(send=send):  # holds the send buffer until the transfer is done
        work.wait()
        # recv[q] = rank q's tokens of this rank's heads: concatenate in rank order
        out.view(b, h // p, p, s_local, d).copy_(recv.permute(1, 2, 0, 3, 4))

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
    b, h_local, s, d = o.shape
    if s % p:
        raise ValueError(f"{s} tokens do not split over {p} ranks")
    # chunk q = this rank's heads over rank q's tokens
    send = o.reshape(b, h_local, p, s // p, d).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[q] = rank q's heads over this rank's tokens: heads in rank order
    return recv.transpose(0, 1).reshape(b, p * h_local, s // p, d)


def sequence_parallel_attention(attention, query, key, value, group=None, *, overlap_value=False):
    """Run a per-head attention callable (e.g. ``PecoAttention.attention``) on
    sequence-sharded Q/K/V ``[B, H, S/P, D]`` and return the output in the same
    sharding: reshard to heads, attend locally, reshard back.

    With ``overlap_value`` the callable must accept ``value_ready=`` (as
    ``PecoAttention.attention`` does): V's all-to-all is then still in flight
    when the call starts and is waited for where V is first read."""
    q = seq_to_heads(query, group)
    k = seq_to_heads(key, group)
    if overlap_value:
        v, ready = seq_to_heads_async(value, group)
        o = attention(q, k, v, value_ready=ready)
    else:
        o = attention(q, k, seq_to_heads(value, group))
    return heads_to_seq(o, group)
