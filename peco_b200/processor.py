"""PECO attention processor (drop-in for peco/processor.py) on the sm_100a kernels.

``PecoConfig``, ``InferenceContext``, ``dense_attention``,
``extend_text_partition`` and ``PecoAttention`` keep the reference's names,
fields, validation and state semantics (centroids cached per layer across
denoising steps, reset by ``reset``).  ``PecoAttention.attention`` runs the
whole sparse call through five library entry points on the caller's stream:

1. ``peco_kmeans_fit``      -- Q and K Lloyd iterations together, straight from
                               the bf16 video prefix (no fp32 copy);
2. ``peco_select_text_partition`` -- cluster-pair selection written directly
                               into the text-extended map and sizes;
3. ``peco_attention_plan``  -- work units, per-unit key-cluster lists and the
                               key-block layout of the packed K/V;
4. ``peco_quantize_gather`` -- Base-Offset fake quant + cluster reorder of Q/K,
                               reorder of V, text rows copied, one pass; K and
                               V land directly in key blocks;
5. ``peco_sparse_attention_restore`` -- tcgen05 sparse attention whose epilogue
                               writes rows back in the original token order.

No host synchronisation happens inside a call.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _native
from .clustering import kmeans_fit_pair, fit_token_clusters


@dataclass(frozen=True)
class PecoConfig:
    num_q_centroids: int = 100
    num_k_centroids: int = 500
    top_p: float = 0.9
    min_kc_ratio: float = 0.1
    kmeans_iter_init: int = 50
    kmeans_iter_step: int = 2
    warmup_steps: int = 2
    warmup_layers: int = 0
    zero_step_kmeans_init: bool = True
    base_offset_bits: int = 4

    def __post_init__(self):
        if min(self.num_q_centroids, self.num_k_centroids, self.kmeans_iter_init, self.kmeans_iter_step) < 1:
            raise ValueError("Cluster counts and KMeans iteration counts must be positive")
        if not 0 < self.top_p <= 1 or not 0 <= self.min_kc_ratio <= 1:
            raise ValueError("top_p must be in (0, 1], min_kc_ratio in [0, 1]")
        if self.base_offset_bits not in (0, 4, 8):
            raise ValueError("base_offset_bits must be 0, 4 or 8")
        if self.warmup_steps < 0 or self.warmup_layers < 0:
            raise ValueError("Warmup counts must be nonnegative")


@dataclass
class InferenceContext:
    """Shared by processors in one pipeline; filled once per transformer call."""

    step: int = -1
    text_length: int = 0
    valid_text_length: int = 0


def dense_attention(query, key, value, valid_length):
    """Warmup path: exact attention within [0, valid) and within [valid, S)
    (peco/processor.py:52-65).

    Runs on the tcgen05 attention kernel as a two-group partition whose map
    is the 2x2 identity -- each group attends only to itself -- built on the
    device, so the call never synchronises and can be captured in a CUDA
    graph.  Takes CUDA fp16/bf16 Q/K/V of one shape with D in {64, 128}; there
    is no CPU path."""
    from .attention_cuda import sparse_attention
    _native.require_cuda(query, key, value)
    if query.dtype not in (torch.float16, torch.bfloat16) or key.dtype != query.dtype or value.dtype != query.dtype:
        raise TypeError("dense_attention takes float16 or bfloat16 Q/K/V of one dtype")
    if key.shape != query.shape or value.shape != query.shape or query.shape[-1] not in (64, 128):
        raise ValueError("dense_attention takes Q/K/V of one shape [B, H, S, D] with D in {64, 128}")
    b, h, s, _ = query.shape
    if not 0 <= valid_length <= s:
        raise ValueError("valid_length must lie in [0, S]")
    sizes = torch.tensor([valid_length, s - valid_length], dtype=torch.int32).to(query.device, non_blocking=True)
    sizes = sizes.expand(b, h, 2).contiguous()
    groups = torch.eye(2, dtype=torch.bool, device=query.device).expand(b, h, 2, 2).contiguous()
    return sparse_attention(query.contiguous(), key.contiguous(), value.contiguous(), groups, sizes, sizes,
                            validate_sizes=False)


def extend_text_partition(dynamic_map, q_sizes, k_sizes, valid_text, text_length):
    """The video-cluster partition [B, H, CQ, CK] grown by two groups on each
    side (peco/processor.py:68-84): group CQ / CK is the valid text and group
    CQ+1 / CK+1 the text padding.  Video clusters and valid text attend to
    each other, padding attends only to padding.  Returns (map [B, H, CQ+2,
    CK+2], q sizes [B, H, CQ+2], k sizes [B, H, CK+2]), int32 sizes."""
    b, h, cq, ck = dynamic_map.shape
    grown = torch.zeros((b, h, cq + 2, ck + 2), dtype=torch.bool, device=dynamic_map.device)
    grown[..., :cq, :ck] = dynamic_map
    grown[..., : cq + 1, ck] = True  # every non-padding row sees the valid text
    grown[..., cq, : ck + 1] = True  # the valid text sees video and itself
    grown[..., cq + 1, ck + 1] = True
    text = torch.tensor([valid_text, text_length - valid_text], dtype=torch.int32).to(q_sizes.device,
                                                                                       non_blocking=True)

    def with_text(sizes):
        out = torch.empty((*sizes.shape[:-1], sizes.shape[-1] + 2), dtype=torch.int32, device=sizes.device)
        out[..., :-2] = sizes
        out[..., -2:] = text
        return out

    return grown, with_text(q_sizes), with_text(k_sizes)


def _first_tokens_init(x_video, clusters):
    """Random-token initial centroids, as the reference draws them (peco/clustering.py:47-49)."""
    bh, n, d = x_video.shape
    idx = torch.randint(n, (bh, clusters), device=x_video.device)
    return x_video.gather(1, idx[..., None].expand(-1, -1, d)).float().contiguous()


class PecoAttention:
    def __init__(self, layer_idx, config: PecoConfig, context: InferenceContext):
        self.layer_idx = layer_idx
        self.config = config
        self.context = context
        self.q_centroids = None
        self.k_centroids = None
        # Optional list; when set, each sparse call appends a dict of CUDA
        # events recorded on the current stream at the stage boundaries
        # (kmeans, select, quantize_gather, attention) for profiling.
        self.stage_events = None
        # When set, steady-state calls write the new fp32 centroids into the
        # cached centroid tensors instead of fresh ones (fixed addresses, as a
        # captured CUDA graph of the call needs; see peco_b200.graph).
        self.update_centroids_in_place = False

    def reset(self):
        self.q_centroids = self.k_centroids = None

    # -- clustering state ---------------------------------------------------
    def _update_cluster_state(self, query, key, key_ready=None):
        """Fit Q/K partitions, reusing this layer's centres after initialization.

        ``query``/``key`` are [1,H,N,D] views (possibly of a longer sequence).
        Returns the two KmeansBuffers (labels, counts, perm, ...) and updates
        the cached fp32 centroids [H,C,D].  With ``key_ready`` (K still
        arriving) Q is clustered first, then ``key_ready()`` runs, then K is
        clustered; otherwise both run in the same launches.
        """
        b, h, n, d = query.shape
        initializing = self.q_centroids is None
        iters = self.config.kmeans_iter_init if initializing else self.config.kmeans_iter_step
        if query.dtype != torch.bfloat16:
            # fp16/fp32 inputs: the reference's fp32 iteration on the drop-in entry points
            ql, qc, qn, _ = fit_token_clusters(query.reshape(b * h, n, d).contiguous(), self.config.num_q_centroids,
                                               max_iters=iters, tol=0, init_centroids=self.q_centroids)
            if key_ready is not None:
                key_ready()
            kl, kc, kn, _ = fit_token_clusters(key.reshape(b * h, n, d).contiguous(), self.config.num_k_centroids,
                                               max_iters=iters, tol=0, init_centroids=self.k_centroids)
            self.q_centroids, self.k_centroids = qc, kc
            return (ql, qn), (kl, kn)
        in_place = self.update_centroids_in_place and not initializing

        def rows_and_init(x, cached, clusters):
            rows, stride = _rows_view(x)
            init = cached if not initializing else _first_tokens_init(x.reshape(b * h, n, d), clusters)
            return rows, stride, init

        q_rows, q_stride, q_init = rows_and_init(query, self.q_centroids, self.config.num_q_centroids)
        if key_ready is None:
            k_rows, k_stride, k_init = rows_and_init(key, self.k_centroids, self.config.num_k_centroids)
            qb, kb = kmeans_fit_pair(q_rows, q_stride, n, q_init, k_rows, k_stride, n, k_init, b * h, d, iters,
                                     q_centers=q_init if in_place else None, k_centers=k_init if in_place else None)
        else:
            qb, _ = kmeans_fit_pair(q_rows, q_stride, n, q_init, None, 0, 0, q_init, b * h, d, iters,
                                    q_centers=q_init if in_place else None)
            key_ready()
            k_rows, k_stride, k_init = rows_and_init(key, self.k_centroids, self.config.num_k_centroids)
            kb, _ = kmeans_fit_pair(k_rows, k_stride, n, k_init, None, 0, 0, k_init, b * h, d, iters,
                                    q_centers=k_init if in_place else None)
        self.q_centroids, self.k_centroids = qb.centers, kb.centers
        return qb, kb

    # -- one call -----------------------------------------------------------
    def attention(self, query, key, value, value_ready=None, key_ready=None):
        """PECO attention of [1, H, S, D] Q/K/V (peco/processor.py:115-157).

        ``key_ready`` / ``value_ready``, if given, are called on the current
        stream before the first read of ``key`` / ``value``: a caller still
        delivering K or V (a reshard in flight) can hand over the buffers
        early and let the transfers overlap the clustering of Q (K) and of
        Q and K (V).  The caller stays responsible for waiting on a transfer
        when this method raises before calling its hook.
        """
        batch, heads, length, dim = query.shape
        if batch != 1:
            raise ValueError("This minimal HunyuanVideo entry supports one prompt per call")
        text_length = self.context.text_length
        video_length = length - text_length
        valid_text = self.context.valid_text_length
        if video_length <= 0 or not 0 <= valid_text <= text_length:
            raise ValueError("Invalid video/text lengths in transformer context")
        warmup = self.context.step < self.config.warmup_steps or self.layer_idx < self.config.warmup_layers
        if warmup:
            if self.config.zero_step_kmeans_init and self.layer_idx >= self.config.warmup_layers:
                self._update_cluster_state(query[:, :, :video_length], key[:, :, :video_length], key_ready)
            elif key_ready is not None:
                key_ready()
            if value_ready is not None:
                value_ready()
            return dense_attention(query, key, value, video_length + valid_text)
        if query.dtype != torch.bfloat16 or key.dtype != torch.bfloat16 or value.dtype != torch.bfloat16:
            raise TypeError("the fused PECO call takes bfloat16 Q/K/V (HunyuanVideo's attention dtype)")
        return self._sparse_call(query.contiguous(), key.contiguous(), value.contiguous(), video_length,
                                 text_length, valid_text, value_ready, key_ready)

    def _sparse_call(self, q, k, v, video, text_length, valid_text, value_ready=None, key_ready=None):
        _native.require_cuda(q, k, v)
        lib = _native.load()
        _, h, s, d = q.shape
        cq, ck = self.config.num_q_centroids, self.config.num_k_centroids
        if cq > video or ck > video:
            raise ValueError("more clusters than video tokens")
        ev = None
        if self.stage_events is not None:
            ev = {n: torch.cuda.Event(enable_timing=True)
                  for n in ("start", "kmeans", "select", "plan", "gather", "attention")}
            self.stage_events.append(ev)
            ev["start"].record()
        qb, kb = self._update_cluster_state(q[:, :, :video], k[:, :, :video], key_ready)
        if ev:
            ev["kmeans"].record()
        dev = q.device
        gq, gk = cq + 2, ck + 2
        emap = torch.empty((1, h, gq, gk), dtype=torch.bool, device=dev)
        qs_ext = torch.empty((1, h, gq), dtype=torch.int32, device=dev)
        ks_ext = torch.empty((1, h, gk), dtype=torch.int32, device=dev)
        minimum = math.ceil(self.config.min_kc_ratio * ck)
        logits = torch.empty((h, cq, ck), dtype=torch.float32, device=dev)  # the selection's scratch
        stream = _native.stream_of(dev, emap, qs_ext, ks_ext, logits)
        with torch.cuda.device(dev):
            st = lib.peco_select_text_partition(
                _native.ptr(self.q_centroids), _native.ptr(self.k_centroids), _native.ptr(qb.counts),
                _native.ptr(kb.counts), _native.ptr(emap), _native.ptr(qs_ext), _native.ptr(ks_ext), h, cq, ck, d,
                float(self.config.top_p), int(minimum), int(valid_text), int(text_length), _native.ptr(logits),
                stream)
            _native.check(st, "peco_select_text_partition")
            if ev:
                ev["select"].record()
            keep = getattr(self, "keep_partition", False)
            if keep:
                self.last_partition = (emap, qs_ext, ks_ext)
            # plan first: it zeroes the padding rows of the key blocks and maps
            # every packed key row to its block row for the gather
            stride = int(lib.peco_attention_workspace_stride(s, s, gq, gk))
            ws = torch.empty(h * stride, dtype=torch.int32, device=dev)
            kblocks = torch.empty((h, int(lib.peco_key_block_rows(s, gk)), d), dtype=k.dtype, device=dev)
            vblocks = torch.empty_like(kblocks)
            stream = _native.stream_of(dev, ws, kblocks, vblocks)
            st = lib.peco_attention_plan(_native.ptr(emap), _native.ptr(qs_ext), _native.ptr(ks_ext),
                                         _native.ptr(kblocks), _native.ptr(vblocks), _native.ptr(ws), h, s, s, d,
                                         gq, gk, stream)
            _native.check(st, "peco_attention_plan")
            if ev:
                ev["plan"].record()
            qp = torch.empty_like(q)
            if value_ready is not None:  # V is first read here
                value_ready()
            stream = _native.stream_of(dev, q, k, v, qp)
            st = lib.peco_quantize_gather(
                _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(qp), _native.ptr(kblocks),
                _native.ptr(vblocks), _native.ptr(qb.perm), _native.ptr(kb.perm), _native.ptr(qb.labels),
                _native.ptr(kb.labels), _native.ptr(self.q_centroids), _native.ptr(self.k_centroids), cq, ck, h, s,
                video, d, int(self.config.base_offset_bits), _native.ptr(ws), gq, gk, stream)
            _native.check(st, "peco_quantize_gather")
            if ev:
                ev["gather"].record()
            if keep:
                # the call's intermediate state, for inspection by tests and tools
                self.last_state = dict(q_labels=qb.labels, k_labels=kb.labels, q_perm=qb.perm, k_perm=kb.perm,
                                       q_counts=qb.counts, k_counts=kb.counts, q_packed=qp)
            out = torch.empty_like(q)
            stream = _native.stream_of(dev, out, qb.perm)
            st = lib.peco_sparse_attention_restore(
                _native.ptr(qp), _native.ptr(kblocks), _native.ptr(vblocks), _native.ptr(ws), _native.ptr(out), h, s,
                s, d, gq, gk, _native.ptr(qb.perm), video, stream)
            _native.check(st, "peco_sparse_attention_restore")
            if ev:
                ev["attention"].record()
        return out

    @torch.no_grad()
    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        """Attention-processor entry of one HunyuanVideo attention module
        (drop-in for peco/processor.py:159-197; ``attention_mask`` is unused
        there too: the text lengths come from the shared context).

        Each stream is projected with the module's own linear layers (video
        rows by ``to_q/to_k/to_v``; text rows by ``add_*_proj`` in a
        dual-stream module, by the same layers in a single-stream one).
        ``peco_prepare_qkv`` then writes the call's [1, H, S, D] Q/K/V in one
        pass: head split, the modules' RMSNorm (``norm_q/norm_k``, or
        ``norm_added_*`` for a dual-stream module's text), the rotary
        embedding of the video rows and the text rows appended after them.
        The attention output goes back through ``to_out`` (video) and
        ``to_add_out`` (text) where the module has them.
        """
        _native.require_cuda(hidden_states)
        n_text = 0 if encoder_hidden_states is None else encoder_hidden_states.shape[1]
        separate_text = attn.add_q_proj is not None  # dual-stream: text has its own weights
        heads = attn.heads
        video_proj = [layer(hidden_states) for layer in (attn.to_q, attn.to_k, attn.to_v)]
        text_layers = (attn.add_q_proj, attn.add_k_proj, attn.add_v_proj) if separate_text else \
            (attn.to_q, attn.to_k, attn.to_v)
        text_proj = [layer(encoder_hidden_states) for layer in text_layers] if n_text else [None] * 3
        b, n_video, inner = video_proj[0].shape
        if b != 1:
            raise ValueError("This minimal HunyuanVideo entry supports one prompt per call")
        if inner % heads or inner // heads not in (64, 128):
            raise ValueError("head dimension must be 64 or 128")
        if any(t is not None and (t.dtype != torch.bfloat16 or t.stride(-1) != 1) for t in video_proj + text_proj):
            raise TypeError("the fused PECO call takes bfloat16 projections (HunyuanVideo's attention dtype)")
        dims = inner // heads
        video_norms = (_rms_gain(attn.norm_q, dims), _rms_gain(attn.norm_k, dims))
        text_norms = (_rms_gain(attn.norm_added_q, dims), _rms_gain(attn.norm_added_k, dims)) if separate_text \
            else video_norms
        cos = sin = None
        if image_rotary_emb is not None:
            cos, sin = (t.to(device=hidden_states.device, dtype=torch.float32).reshape(n_video, dims).contiguous()
                        for t in image_rotary_emb)
        seq = n_video + n_text
        q, k, v = (torch.empty((1, heads, seq, dims), dtype=torch.bfloat16, device=hidden_states.device)
                   for _ in range(3))
        lib = _native.load()
        opt = (lambda t: _native.ptr(t) if t is not None else _native.P(0))
        keep = [t for t in (*video_proj, *text_proj, cos, sin, q, k, v) if t is not None] + \
            [g for g, _ in (*video_norms, *text_norms) if g is not None]
        dev = hidden_states.device
        with torch.cuda.device(dev):
            st = lib.peco_prepare_qkv(
                *[_native.ptr(t) for t in video_proj], video_proj[0].stride(1), n_video,
                *[opt(t) for t in text_proj], text_proj[0].stride(1) if n_text else 0, n_text,
                opt(video_norms[0][0]), opt(video_norms[1][0]), video_norms[0][1], opt(text_norms[0][0]),
                opt(text_norms[1][0]), text_norms[0][1], opt(cos), opt(sin), _native.ptr(q), _native.ptr(k),
                _native.ptr(v), heads, dims, _native.stream_of(dev, *keep))
        _native.check(st, "peco_prepare_qkv")
        out = self.attention(q, k, v)
        rows = out.transpose(1, 2).reshape(1, seq, inner)  # token-major, heads side by side
        video_out, text_out = rows[:, :n_video], rows[:, n_video:]
        if not n_text:
            return video_out, encoder_hidden_states
        if getattr(attn, "to_out", None) is not None:
            for layer in attn.to_out:
                video_out = layer(video_out)
        if getattr(attn, "to_add_out", None) is not None:
            text_out = attn.to_add_out(text_out)
        return video_out, text_out


def _rms_gain(norm, dims):
    """(fp32 gain [D], eps) of an RMSNorm module, (None, 0.0) without one.

    Any module with ``weight`` and ``eps`` attributes qualifies: the kernel
    computes x * rsqrt(mean(x^2) + eps) * weight in fp32, rounded once to
    bf16."""
    if norm is None:
        return None, 0.0
    weight, eps = getattr(norm, "weight", None), getattr(norm, "eps", None)
    if weight is None or eps is None or weight.numel() != dims:
        raise TypeError("query/key norms must be RMSNorm modules (per-head ``weight`` and ``eps``)")
    return weight.detach().float().contiguous(), float(eps)


def _rows_view(x):
    """(tensor, head_rows) for a [1,H,N,D] view of a contiguous [1,H,S,D] tensor:
    head h's rows start at row h*S of the underlying storage."""
    if x.stride(3) != 1 or x.stride(2) != x.shape[3]:
        x = x.contiguous()
    return x, x.stride(1) // x.shape[3]
