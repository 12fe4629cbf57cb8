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
