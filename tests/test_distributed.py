"""Multi-process (gloo, world size 2 and 4, CPU) checks of the Ulysses reshard.

The reshard must reproduce, on every rank, exactly the head slice of the full
tensor (and invert exactly); composed with a per-head attention it must equal
running that attention on the full sequence and slicing the tokens.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import peco_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full(seed, b, h, s, d):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((b, h, s, d), generator=g)


def _worker(rank, world, port, kind, out_q):
    import torch.distributed as dist

    from peco_b200 import distributed as pd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b, h, s, d = (2 if kind == "reshard" else 1), 4 * world, 24 * world, 16
        sl, hl = s // world, h // world
        x = _full(1, b, h, s, d)
        shard = x[:, :, rank * sl:(rank + 1) * sl].contiguous()
        if kind == "reshard":
            heads = pd.seq_to_heads(shard)
            ok = torch.equal(heads, x[:, rank * hl:(rank + 1) * hl])
            back = pd.heads_to_seq(heads)
            ok = ok and torch.equal(back, shard)
        else:
            # a per-head sparse attention over cluster groups of the full sequence
            k_full, v_full = _full(2, b, h, s, d), _full(3, b, h, s, d)
            qs = torch.tensor([[[s // 2, s - s // 2]] * h], dtype=torch.int32)
            dmap = torch.ones((1, h, 2, 2), dtype=torch.bool)
            dmap[0, :, 1, 0] = False

            def attend(q, k, v, key_ready=None, value_ready=None):
                if kind == "overlap":  # K's and V's transfers are in flight until their hooks run
                    key_ready()
                    value_ready()
                lo = rank * hl
                return O.sparse_attention(q, k, v, dmap[:, lo:lo + hl], qs[:, lo:lo + hl], qs[:, lo:lo + hl])

            def failing(q, k, v, key_ready=None, value_ready=None):
                raise RuntimeError("attention failed before reading K and V")

            ks, vs = (t[:, :, rank * sl:(rank + 1) * sl].contiguous() for t in (k_full, v_full))
            ok = True
            if kind == "overlap":
                # a callable that raises before its hooks: the transfers are still
                # waited for, and the next exchange on the group works
                try:
                    pd.sequence_parallel_attention(failing, shard, ks, vs, overlap=True)
                    ok = False
                except RuntimeError:
                    pass
            got = pd.sequence_parallel_attention(attend, shard, ks, vs, overlap=kind == "overlap")
            ref = O.sparse_attention(x, k_full, v_full, dmap, qs, qs)[:, :, rank * sl:(rank + 1) * sl]
            ok = ok and torch.allclose(got, ref, atol=1e-6, rtol=1e-5)
        out_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("kind", ["reshard", "attention", "overlap"])
def test_ulysses_reshard_multi_process(world, kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(results[r] for r in range(world)), results
