"""Transformer integration (peco/model.py) on a small HunyuanVideo-architecture model.

CPU: install_attention wires one processor per block and a context hook that
reads the text lengths from the right-padded mask (run with exact-attention
processors sharing that context, since the PECO processors need the GPU);
reset_state rewinds the state; bad masks raise.
GPU: steady-state PECO steps run through PecoAttention.__call__; with every
cluster pair kept and quantisation off they reproduce the dense baseline
(cosine >= 0.999 on the block outputs).
"""

import pytest
import torch

from peco_b200.hunyuan import HunyuanConfig, Pipe, build_transformer, use_dense_attention
from peco_b200.model import install_attention, reset_state
from peco_b200.processor import InferenceContext, PecoAttention, PecoConfig

TINY = HunyuanConfig(hidden=256, heads=2, head_dim=128, dual_blocks=2, single_blocks=2, text_dim=64, pooled_dim=32)


def _inputs(device, dtype, frames=2, size=8, text=16, valid=12, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, 16, frames, size, size, generator=g).to(device, dtype)
    txt = torch.randn(1, text, TINY.text_dim, generator=g).to(device, dtype)
    mask = torch.zeros(1, text, dtype=torch.bool)
    mask[0, :valid] = True
    pooled = torch.randn(1, TINY.pooled_dim, generator=g).to(device, dtype)
    return x, torch.tensor([500.0], device=device), txt, mask.to(device), pooled


def test_install_attention_context_and_reset():
    model = build_transformer(TINY, device="cpu", dtype=torch.float32)
    pipe = Pipe(model)
    cfg = PecoConfig(num_q_centroids=4, num_k_centroids=8, warmup_steps=100, zero_step_kmeans_init=False)
    ctx = install_attention(pipe, cfg)
    procs = model._peco_processors
    assert len(procs) == 4 and [p.layer_idx for p in procs] == [0, 1, 2, 3]
    assert all(isinstance(b.attn.processor, PecoAttention) for b in [*model.transformer_blocks, *model.single_transformer_blocks])
    # The PECO processors run on the GPU only; the pre-hook and the shared
    # context are host logic, exercised here with exact-attention processors
    # that read the installed context.
    use_dense_attention(model, ctx)
    x, t, txt, mask, pooled = _inputs("cpu", torch.float32)
    with torch.no_grad():
        y = model(x, t, txt, mask, pooled)
        model(x, t, txt, mask, pooled)
    assert ctx.step == 1 and ctx.text_length == 16 and ctx.valid_text_length == 12
    # the lengths the hook read give the same attention as stating them
    use_dense_attention(model, InferenceContext(step=0, text_length=16, valid_text_length=12))
    with torch.no_grad():
        ref = model(x, t, txt, mask, pooled)
    assert (y - ref).abs().max().item() < 1e-5
    reset_state(pipe)
    assert ctx.step == -1 and all(p.q_centroids is None for p in procs)
    # a second install replaces the hook (one step counter, not two)
    ctx2 = install_attention(pipe, cfg)
    use_dense_attention(model, ctx2)
    with torch.no_grad():
        model(x, t, txt, mask, pooled)
    assert ctx2.step == 0 and ctx.step == -1


def test_mask_must_be_right_padded_single_prompt():
    model = build_transformer(TINY, device="cpu", dtype=torch.float32)
    install_attention(Pipe(model), PecoConfig(warmup_steps=100, zero_step_kmeans_init=False))
    x, t, txt, mask, pooled = _inputs("cpu", torch.float32)
    bad = mask.clone()
    bad[0, 0] = False
    with pytest.raises(ValueError):
        model(x, t, txt, bad, pooled)
    with pytest.raises(ValueError):
        model(x.expand(2, -1, -1, -1, -1), t.expand(2), txt.expand(2, -1, -1), mask.expand(2, -1), pooled.expand(2, -1))


@pytest.mark.gpu
def test_peco_steps_match_dense_when_every_pair_is_kept():
    model = build_transformer(TINY, device="cuda", dtype=torch.bfloat16)
    pipe = Pipe(model)
    cfg = PecoConfig(num_q_centroids=8, num_k_centroids=16, top_p=1.0, min_kc_ratio=1.0, kmeans_iter_init=3,
                     kmeans_iter_step=2, warmup_steps=1, base_offset_bits=0)
    ctx = install_attention(pipe, cfg)
    x, t, txt, mask, pooled = _inputs("cuda", torch.bfloat16, frames=2, size=16)
    with torch.no_grad():
        model(x, t, txt, mask, pooled)          # step 0: dense warm-up, centroids initialised
        got = model(x, t, txt, mask, pooled)    # step 1: sparse PECO path, all pairs kept
    assert ctx.step == 1 and all(p.q_centroids is not None for p in model._peco_processors)
    use_dense_attention(model, InferenceContext(step=0, text_length=16, valid_text_length=12))
    with torch.no_grad():
        ref = model(x, t, txt, mask, pooled)
    g, r = got.float().flatten(), ref.float().flatten()
    assert torch.isfinite(g).all()
    cos = torch.nn.functional.cosine_similarity(g, r, dim=0).item()
    assert cos >= 0.999, cos


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tensor_parallel_worker(rank, world, port, out_q):
    import os

    import torch.distributed as dist

    from peco_b200.hunyuan import TensorParallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = HunyuanConfig(hidden=256, heads=4, head_dim=64, dual_blocks=2, single_blocks=2, text_dim=64,
                            pooled_dim=32, rope_axes=(16, 24, 24))
        full = build_transformer(cfg, device="cpu", dtype=torch.float32)
        part = build_transformer(cfg, device="cpu", dtype=torch.float32, tp=TensorParallel(rank, world))
        ctx = InferenceContext(step=0, text_length=16, valid_text_length=12)
        use_dense_attention(full, ctx)
        use_dense_attention(part, ctx)
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, 16, 2, 8, 8, generator=g)
        txt = torch.randn(1, 16, 64, generator=g)
        mask = torch.zeros(1, 16, dtype=torch.bool)
        mask[0, :12] = True
        pooled = torch.randn(1, 32, generator=g)
        t = torch.tensor([500.0])
        with torch.no_grad():
            want = full(x, t, txt, mask, pooled)
            got = part(x, t, txt, mask, pooled)
        heads = part.transformer_blocks[0].attn.heads
        out_q.put((rank, bool(torch.allclose(got, want, atol=1e-4, rtol=1e-4)) and heads == 4 // world))
    except Exception as e:  # report instead of leaving the other ranks waiting
        out_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_parallel_model_equals_unsharded(world):
    """Heads and MLP units sharded over gloo ranks (column slices in, row slices
    plus an all-reduce out) reproduce the unsharded model's output."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tensor_parallel_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(results[r] is True for r in range(world)), results
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.gpu
def test_step_graph_replays_the_eager_step():
    """A steady-state step captured whole (every layer's PECO call and the
    model's kernels) replays bit-identically to the eager step, and keeps
    chaining the centroids like eager steps do."""
    from peco_b200.graph import PecoStepGraph
    cfg = PecoConfig(num_q_centroids=8, num_k_centroids=16, top_p=0.5, min_kc_ratio=0.25, kmeans_iter_init=3,
                     kmeans_iter_step=2, warmup_steps=1, base_offset_bits=4)
    models = [build_transformer(TINY, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    ctxs = [install_attention(Pipe(m), cfg) for m in models]
    x, t, txt, mask, pooled = _inputs("cuda", torch.bfloat16, frames=2, size=16)
    with torch.no_grad():
        for m in models:
            torch.manual_seed(0)  # the first fit draws its initial centroids at random
            m(x, t, txt, mask, pooled)  # dense warm-up step, centroids initialised
            m(x, t, txt, mask, pooled)  # first sparse step
    graph = PecoStepGraph(models[1], x, t, txt, mask, pooled)
    for i in range(2):
        x2 = x + 0.01 * (i + 1)
        with torch.no_grad():
            want = models[0](x2, t, txt, mask, pooled)
        got = graph(x2, t, txt, mask, pooled)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        for p0, p1 in zip(models[0]._peco_processors, models[1]._peco_processors):
            assert torch.equal(p0.q_centroids, p1.q_centroids) and torch.equal(p0.k_centroids, p1.k_centroids)
    assert ctxs[1].step == 1  # the graph does not advance the eager step counter
