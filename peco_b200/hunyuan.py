"""A random-init HunyuanVideo-architecture transformer in plain PyTorch.

Stands in for the diffusers ``HunyuanVideoTransformer3DModel`` (absent here)
so that one full denoising step runs with PECO
attention installed through ``peco_b200.model.install_attention``, exactly
the way peco/model.py attaches it to the diffusers model.  Only the
architecture matters (weights are random, N(0, 0.02)):

* patch embedding: Conv3d, kernel = stride = (1, 2, 2), 16 latent channels;
* text: a linear projection of 4096-dim embeddings (the reference's token
  refiner is folded into it), pooled text and timestep form the modulation
  vector;
* ``transformer_blocks``: dual-stream blocks (separate video/text weights,
  joint attention, adaLN-zero modulation, GELU-tanh MLP);
* ``single_transformer_blocks``: single-stream blocks (one projection to
  Q/K/V and the MLP, parallel attention + MLP, one output projection);
* RMSNorm on Q and K per head, 3D rotary embedding on the video tokens
  (head dim split 16 / 56 / 56 over time / height / width);
* adaLN output norm and un-patchify back to the latent shape.

Head parallelism (``TensorParallel``): rank r of P owns attention heads
[r H/P, (r+1) H/P) and the matching 1/P of every MLP hidden layer.  Q/K/V
and the first MLP layers are column slices of the full weights; the output
projections (``to_out``, ``to_add_out``, the MLPs' second layers, the
single-stream ``proj_out``) are row slices whose partial products are summed
by one all-reduce each; embedders, modulation and the final layer are
replicated.  Every parameter is drawn from a generator seeded by its own
name, so a sharded model holds exactly the slices of the unsharded one.  The
PECO processor of a rank clusters and attends only its own heads: per-head
work needs no communication, as in the reference's per-(batch, head) kernels.

The attention modules expose the attributes the PECO processor reads
(``heads``, ``to_q``/``to_k``/``to_v``, ``norm_q``/``norm_k``,
``add_q_proj``... for the text stream, ``to_out``, ``to_add_out``) and call
their processor as ``processor(attn, hidden_states, encoder_hidden_states,
attention_mask, image_rotary_emb)`` (peco/processor.py:159-197).
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .processor import InferenceContext, PecoAttention, PecoConfig


@dataclass(frozen=True)
class HunyuanConfig:
    in_channels: int = 16
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    mlp_ratio: int = 4
    dual_blocks: int = 20
    single_blocks: int = 40
    text_dim: int = 4096
    pooled_dim: int = 768
    patch: tuple = (1, 2, 2)
    rope_axes: tuple = (16, 56, 56)
    rope_theta: float = 256.0


class TensorParallel:
    """Head-parallel placement: this process is ``rank`` of ``world`` in ``group``."""

    def __init__(self, rank: int = 0, world: int = 1, group=None):
        if world < 1 or not 0 <= rank < world:
            raise ValueError("rank must lie in [0, world)")
        self.rank, self.world, self.group = rank, world, group

    def span(self, full: int) -> tuple:
        """(start, stop) of this rank's equal share of ``full`` features."""
        if full % self.world:
            raise ValueError(f"{full} features do not split over {self.world} ranks")
        n = full // self.world
        return self.rank * n, (self.rank + 1) * n


SINGLE = TensorParallel()


def _shard(param, full_shape, rows=None, cols=None):
    """Record how ``param`` is cut from the full tensor: ``rows`` a (start,
    stop) range of dim 0, ``cols`` a list of ranges of dim 1, concatenated."""
    param.full_shape = tuple(full_shape)
    param.shard_rows = rows
    param.shard_cols = cols
    return param


def column_linear(dim_in, dim_out, tp: TensorParallel):
    """nn.Linear holding this rank's rows (output features) of a [dim_out, dim_in] layer."""
    a, b = tp.span(dim_out)
    layer = nn.Linear(dim_in, b - a)
    _shard(layer.weight, (dim_out, dim_in), rows=(a, b))
    _shard(layer.bias, (dim_out,), rows=(a, b))
    return layer


class RowParallelLinear(nn.Module):
    """y = sum over ranks of x_r W_r^T, plus the bias: each rank holds the
    weight columns of its input features (``cols``, ranges of the full input)
    and one all-reduce adds the partial products."""

    def __init__(self, dim_out, full_in, cols, tp: TensorParallel):
        super().__init__()
        local = sum(b - a for a, b in cols)
        self.tp = tp
        self.weight = _shard(nn.Parameter(torch.empty(dim_out, local)), (dim_out, full_in), cols=list(cols))
        self.bias = _shard(nn.Parameter(torch.empty(dim_out)), (dim_out,))
        # nn.Linear's default initialisation, with the unsharded fan-in
        bound = 1.0 / math.sqrt(full_in)
        with torch.no_grad():
            if self.weight.device.type != "meta":
                self.weight.uniform_(-bound, bound)
                self.bias.uniform_(-bound, bound)

    def forward(self, x):
        y = F.linear(x, self.weight)
        if self.tp.world > 1:
            dist.all_reduce(y, group=self.tp.group)
        return y + self.bias


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


def _ln(x):
    return F.layer_norm(x, x.shape[-1:], eps=1e-6)


class SDPAProcessor(PecoAttention):
    """Exact joint attention with torch SDPA (the dense baseline).

    On CUDA bf16 it is the PECO processor's entry (the fused projection-side
    kernel) with the attention itself replaced by full softmax attention over
    [0, valid) and [valid, S).  Elsewhere (CPU, fp32) the same math runs as
    plain torch: projections, the modules' norms, the rotation of the video
    rows, SDPA and the output projections."""

    def __init__(self, context: InferenceContext):
        super().__init__(0, PecoConfig(), context)

    def attention(self, query, key, value, value_ready=None, key_ready=None):
        s = query.shape[2]
        valid = s - self.context.text_length + self.context.valid_text_length
        out = torch.empty_like(query)
        for a, b in ((0, valid), (valid, s)):
            if a < b:
                out[:, :, a:b] = F.scaled_dot_product_attention(query[:, :, a:b], key[:, :, a:b], value[:, :, a:b])
        return out

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        if hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16:
            return super().__call__(attn, hidden_states, encoder_hidden_states, attention_mask, image_rotary_emb)
        return self._torch_call(attn, hidden_states, encoder_hidden_states, image_rotary_emb)

    def _torch_call(self, attn, video, text, rope):
        separate = attn.add_q_proj is not None
        n_text = 0 if text is None else text.shape[1]

        def heads_of(x, layers, norms):
            q, k, v = (layer(x).unflatten(-1, (attn.heads, -1)).transpose(1, 2) for layer in layers)
            return norms[0](q), norms[1](k), v

        q, k, v = heads_of(video, (attn.to_q, attn.to_k, attn.to_v), (attn.norm_q, attn.norm_k))
        if rope is not None:
            q, k = rotate_pairs(q, *rope), rotate_pairs(k, *rope)
        if n_text:
            layers = (attn.add_q_proj, attn.add_k_proj, attn.add_v_proj) if separate else (attn.to_q, attn.to_k, attn.to_v)
            norms = (attn.norm_added_q, attn.norm_added_k) if separate else (attn.norm_q, attn.norm_k)
            tq, tk, tv = heads_of(text, layers, norms)
            q, k, v = torch.cat((q, tq), 2), torch.cat((k, tk), 2), torch.cat((v, tv), 2)
        rows = self.attention(q, k, v).transpose(1, 2).flatten(2)
        video_out, text_out = rows[:, : video.shape[1]], rows[:, video.shape[1]:]
        if not n_text:
            return video_out, text
        if attn.to_out is not None:
            for layer in attn.to_out:
                video_out = layer(video_out)
        if attn.to_add_out is not None:
            text_out = attn.to_add_out(text_out)
        return video_out, text_out


def rotate_pairs(x, cos, sin):
    """Rotary embedding of [.., N, D] rows with (cos, sin) tables [N, D], pairs
    (2i, 2i+1) interleaved: (a, b) -> (a cos - b sin, b cos + a sin), each
    product and the sum in fp32, rounded once to x's dtype."""
    a, b = x.float().unflatten(-1, (-1, 2)).unbind(-1)
    turned = torch.stack((-b, a), -1).flatten(-2)
    return (x.float() * cos.to(x.device) + turned * sin.to(x.device)).to(x.dtype)


class Attention(nn.Module):
    """Projections and norms of one attention layer (this rank's heads); the math is the processor's."""

    def __init__(self, dim, heads, head_dim, joint_text: bool, pre_only: bool, tp: TensorParallel = SINGLE):
        super().__init__()
        inner = heads * head_dim
        lo, hi = tp.span(inner)
        self.heads = heads // tp.world
        self.to_q, self.to_k, self.to_v = (column_linear(dim, inner, tp) for _ in range(3))
        self.norm_q, self.norm_k = RMSNorm(head_dim), RMSNorm(head_dim)
        if joint_text:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = (column_linear(dim, inner, tp) for _ in range(3))
            self.norm_added_q, self.norm_added_k = RMSNorm(head_dim), RMSNorm(head_dim)
            self.to_add_out = RowParallelLinear(dim, inner, [(lo, hi)], tp)
        else:
            self.add_q_proj = self.add_k_proj = self.add_v_proj = None
            self.norm_added_q = self.norm_added_k = None
            self.to_add_out = None
        self.to_out = None if pre_only else nn.ModuleList([RowParallelLinear(dim, inner, [(lo, hi)], tp), nn.Identity()])
        self.processor = None

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        return self.processor(self, hidden_states, encoder_hidden_states, attention_mask, image_rotary_emb)


def _mlp(dim, ratio, tp: TensorParallel = SINGLE):
    hidden = dim * ratio
    return nn.Sequential(column_linear(dim, hidden, tp), nn.GELU(approximate="tanh"),
                         RowParallelLinear(dim, hidden, [tp.span(hidden)], tp))


class DualStreamBlock(nn.Module):
    def __init__(self, cfg: HunyuanConfig, tp: TensorParallel = SINGLE):
        super().__init__()
        d = cfg.hidden
        self.img_mod = nn.Linear(d, 6 * d)
        self.txt_mod = nn.Linear(d, 6 * d)
        self.attn = Attention(d, cfg.heads, cfg.head_dim, joint_text=True, pre_only=False, tp=tp)
        self.ff = _mlp(d, cfg.mlp_ratio, tp)
        self.ff_context = _mlp(d, cfg.mlp_ratio, tp)

    def forward(self, img, txt, temb, rope):
        e = F.silu(temb)
        i_shift, i_scale, i_gate, i_shift2, i_scale2, i_gate2 = self.img_mod(e)[:, None].chunk(6, dim=-1)
        t_shift, t_scale, t_gate, t_shift2, t_scale2, t_gate2 = self.txt_mod(e)[:, None].chunk(6, dim=-1)
        a_img, a_txt = self.attn(_ln(img) * (1 + i_scale) + i_shift, _ln(txt) * (1 + t_scale) + t_shift, None, rope)
        img = img + i_gate * a_img
        txt = txt + t_gate * a_txt
        img = img + i_gate2 * self.ff(_ln(img) * (1 + i_scale2) + i_shift2)
        txt = txt + t_gate2 * self.ff_context(_ln(txt) * (1 + t_scale2) + t_shift2)
        return img, txt


class SingleStreamBlock(nn.Module):
    def __init__(self, cfg: HunyuanConfig, tp: TensorParallel = SINGLE):
        super().__init__()
        d = cfg.hidden
        inner, hidden = cfg.heads * cfg.head_dim, cfg.mlp_ratio * d
        self.mod = nn.Linear(d, 3 * d)
        self.attn = Attention(d, cfg.heads, cfg.head_dim, joint_text=False, pre_only=True, tp=tp)
        self.proj_mlp = column_linear(d, hidden, tp)
        # input = [attention rows (inner) | MLP hidden (hidden)]: this rank's slice of each
        a, b = tp.span(inner)
        c, e = tp.span(hidden)
        self.proj_out = RowParallelLinear(d, inner + hidden, [(a, b), (inner + c, inner + e)], tp)

    def forward(self, img, txt, temb, rope):
        n_txt = txt.shape[1]
        x = torch.cat((img, txt), 1)
        shift, scale, gate = self.mod(F.silu(temb))[:, None].chunk(3, dim=-1)
        h = _ln(x) * (1 + scale) + shift
        mlp = F.gelu(self.proj_mlp(h), approximate="tanh")
        a_img, a_txt = self.attn(h[:, :-n_txt], h[:, -n_txt:], None, rope)
        x = x + gate * self.proj_out(torch.cat((torch.cat((a_img, a_txt), 1), mlp), -1))
        return x[:, :-n_txt], x[:, -n_txt:]


def _timestep_embedding(t, dim=256, max_period=10000.0):
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat((torch.cos(args), torch.sin(args)), -1)


def rope_3d(grid, axes, theta, device):
    """(cos, sin) tables [T*H*W, sum(axes)] for a (T, H, W) token grid, pairs
    interleaved (the real form diffusers' apply_rotary_emb takes)."""
    tables = []
    coords = torch.meshgrid(*(torch.arange(n, dtype=torch.float32) for n in grid), indexing="ij")
    for dim, pos in zip(axes, coords):
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        ang = pos.reshape(-1, 1) * inv[None]
        tables.append(ang.repeat_interleave(2, dim=-1))
    ang = torch.cat(tables, -1)
    return ang.cos().to(device), ang.sin().to(device)


class HunyuanVideoTransformer(nn.Module):
    def __init__(self, cfg: HunyuanConfig = HunyuanConfig(), tp: TensorParallel = SINGLE):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        d = cfg.hidden
        self.x_embedder = nn.Conv3d(cfg.in_channels, d, kernel_size=cfg.patch, stride=cfg.patch)
        self.context_embedder = nn.Linear(cfg.text_dim, d)
        self.time_in = nn.Sequential(nn.Linear(256, d), nn.SiLU(), nn.Linear(d, d))
        self.vector_in = nn.Sequential(nn.Linear(cfg.pooled_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.transformer_blocks = nn.ModuleList(DualStreamBlock(cfg, tp) for _ in range(cfg.dual_blocks))
        self.single_transformer_blocks = nn.ModuleList(SingleStreamBlock(cfg, tp) for _ in range(cfg.single_blocks))
        self.norm_out = nn.Linear(d, 2 * d)
        self.proj_out = nn.Linear(d, cfg.in_channels * math.prod(cfg.patch))

    @torch.no_grad()
    def init_random(self, std=0.02, seed=0):
        """Weights ~N(0, std) drawn on the parameters' device, biases 0, RMSNorm
        gains 1.  Each weight comes from a generator seeded by (seed, its name)
        and is drawn at its full unsharded shape, then cut to this rank's
        slice, so every placement holds slices of the same model."""
        dev = next(self.parameters()).device
        for name, p in self.named_parameters():
            if p.ndim > 1:
                g = torch.Generator(device=dev).manual_seed(seed * 1000003 + zlib.crc32(name.encode()))
                full = torch.randn(getattr(p, "full_shape", p.shape), generator=g, device=dev, dtype=torch.float32)
                rows, cols = getattr(p, "shard_rows", None), getattr(p, "shard_cols", None)
                if rows is not None:
                    full = full[rows[0]:rows[1]]
                if cols is not None:
                    full = torch.cat([full[:, a:b] for a, b in cols], 1)
                p.copy_(full.mul_(std))
            elif name.endswith("norm_q.weight") or name.endswith("norm_k.weight") or "norm_added" in name:
                p.fill_(1.0)
            else:
                p.zero_()
        return self


    def forward(self, hidden_states, timestep, encoder_hidden_states, encoder_attention_mask, pooled_projections):
        b, c, t, h, w = hidden_states.shape
        pt, ph, pw = self.cfg.patch
        grid = (t // pt, h // ph, w // pw)
        img = self.x_embedder(hidden_states).flatten(2).transpose(1, 2)
        txt = self.context_embedder(encoder_hidden_states)
        temb = self.time_in(_timestep_embedding(timestep).to(img.dtype)) + self.vector_in(pooled_projections)
        key = (grid, img.device)
        rope = self._rope.get(key) if hasattr(self, "_rope") else None
        if rope is None:  # built once per grid (host tables copied to the device)
            rope = rope_3d(grid, self.cfg.rope_axes, self.cfg.rope_theta, img.device)
            self._rope = {key: rope}
        for block in self.transformer_blocks:
            img, txt = block(img, txt, temb, rope)
        for block in self.single_transformer_blocks:
            img, txt = block(img, txt, temb, rope)
        scale, shift = self.norm_out(F.silu(temb))[:, None].chunk(2, dim=-1)
        out = self.proj_out(_ln(img) * (1 + scale) + shift)
        out = out.reshape(b, *grid, c, pt, ph, pw).permute(0, 4, 1, 5, 2, 6, 3, 7)
        return out.reshape(b, c, t, h, w)


def build_transformer(cfg: HunyuanConfig = HunyuanConfig(), device="cuda", dtype=torch.bfloat16, seed=0,
                      tp: TensorParallel = SINGLE):
    """Random-init model (this rank's shard under ``tp``) built straight on
    ``device`` (no default initialisation pass)."""
    if cfg.heads % tp.world or (cfg.hidden * cfg.mlp_ratio) % tp.world:
        raise ValueError(f"{cfg.heads} heads / {cfg.hidden * cfg.mlp_ratio} MLP units do not split over {tp.world} ranks")
    with torch.device("meta"):
        model = HunyuanVideoTransformer(cfg, tp)
    shard_info = {n: (getattr(p, "full_shape", None), getattr(p, "shard_rows", None), getattr(p, "shard_cols", None))
                  for n, p in model.named_parameters()}
    model = model.to_empty(device=device).to(dtype)
    for n, p in model.named_parameters():  # to_empty/to() make new parameters: keep the shard records
        full_shape, rows, cols = shard_info[n]
        if full_shape is not None:
            _shard(p, full_shape, rows, cols)
    return model.init_random(seed=seed).eval()


class Pipe:
    """The part of a diffusers pipeline ``install_attention`` uses."""

    def __init__(self, transformer):
        self.transformer = transformer


def use_dense_attention(transformer, context: InferenceContext):
    """Give every attention layer the exact SDPA processor (the dense baseline)."""
    for block in [*transformer.transformer_blocks, *transformer.single_transformer_blocks]:
        block.attn.set_processor(SDPAProcessor(context))
