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
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

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
    """Warmup path: full attention over [0, valid) and [valid, S) separately
    (peco/processor.py:52-65).

    CUDA fp16/bf16 inputs with D in {64, 128} run on the tcgen05 attention
    kernel as a two-group partition -- groups [0, valid) and [valid, S), each
    attending only to itself -- which is exactly the reference's pair of
    varlen SDPA calls.  Other inputs take the reference's SDPA route."""
    if (query.is_cuda and query.dtype in (torch.float16, torch.bfloat16) and query.shape[-1] in (64, 128)
            and key.dtype == query.dtype and value.dtype == query.dtype and key.shape == query.shape
            and value.shape == query.shape):
        return _dense_attention_tc(query.contiguous(), key.contiguous(), value.contiguous(), valid_length)
    output = torch.empty_like(query)
    backend = SDPBackend.FLASH_ATTENTION if query.is_cuda else SDPBackend.MATH
    with sdpa_kernel(backend):
        for start, end in ((0, valid_length), (valid_length, query.shape[2])):
            if start < end:
                output[:, :, start:end] = F.scaled_dot_product_attention(
                    query[:, :, start:end].contiguous(), key[:, :, start:end].contiguous(),
                    value[:, :, start:end].contiguous(), dropout_p=0.0)
    return output


def _dense_attention_tc(query, key, value, valid_length):
    """Block-diagonal partition of the sequence into [0, valid) and [valid, S)
    on the sparse kernel (built on the device, so the call never synchronises
    and can be captured in a CUDA graph)."""
    from .attention_cuda import sparse_attention
    b, h, s, _ = query.shape
    if not 0 <= valid_length <= s:
        raise ValueError("valid_length must lie in [0, S]")
    sizes = torch.empty((b, h, 2), dtype=torch.int32, device=query.device)
    sizes[..., 0] = valid_length
    sizes[..., 1] = s - valid_length
    groups = torch.eye(2, dtype=torch.bool, device=query.device).expand(b, h, 2, 2).contiguous()
    return sparse_attention(query, key, value, groups, sizes, sizes, validate_sizes=False)


def extend_text_partition(dynamic_map, q_sizes, k_sizes, valid_text, text_length):
    """Append valid-text and padding groups to the video-cluster partition
    (peco/processor.py:68-84): valid text and video see each other, padding
    forms its own sequence."""
    dynamic_map = F.pad(dynamic_map, (0, 2, 0, 2), value=False)
    dynamic_map[..., -2, :-1] = True
    dynamic_map[..., :-1, -2] = True
    dynamic_map[..., -1, -1] = True
    extra = torch.tensor([valid_text, text_length - valid_text], dtype=torch.int32).to(q_sizes.device,
                                                                                          non_blocking=True)
    extra = extra.expand(*q_sizes.shape[:-1], 2)
    return (dynamic_map.contiguous(), torch.cat((q_sizes, extra), -1).to(torch.int32).contiguous(),
            torch.cat((k_sizes, extra), -1).to(torch.int32).contiguous())


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
        stream = _native.stream_of(dev, emap, qs_ext, ks_ext)
        with torch.cuda.device(dev):
            st = lib.peco_select_text_partition(
                _native.ptr(self.q_centroids), _native.ptr(self.k_centroids), _native.ptr(qb.counts),
                _native.ptr(kb.counts), _native.ptr(emap), _native.ptr(qs_ext), _native.ptr(ks_ext), h, cq, ck, d,
                float(self.config.top_p), int(minimum), int(valid_text), int(text_length), stream)
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
        """diffusers attention-processor entry (peco/processor.py:159-197)."""
        apply_rotary_emb = _rotary()
        text_length = 0 if encoder_hidden_states is None else encoder_hidden_states.shape[1]
        if attn.add_q_proj is None and text_length:
            hidden_states = torch.cat((hidden_states, encoder_hidden_states), 1)

        def split_heads(x):
            return x.unflatten(2, (attn.heads, -1)).transpose(1, 2)

        query, key, value = (split_heads(proj(hidden_states)) for proj in (attn.to_q, attn.to_k, attn.to_v))
        if attn.norm_q is not None:
            query = attn.norm_q(query)
        if attn.norm_k is not None:
            key = attn.norm_k(key)
        if image_rotary_emb is not None:
            if attn.add_q_proj is None and text_length:
                query = torch.cat((apply_rotary_emb(query[:, :, :-text_length], image_rotary_emb),
                                   query[:, :, -text_length:]), 2)
                key = torch.cat((apply_rotary_emb(key[:, :, :-text_length], image_rotary_emb),
                                 key[:, :, -text_length:]), 2)
            else:
                query, key = (apply_rotary_emb(x, image_rotary_emb) for x in (query, key))
        if attn.add_q_proj is not None and text_length:
            eq, ek, ev = (split_heads(proj(encoder_hidden_states))
                          for proj in (attn.add_q_proj, attn.add_k_proj, attn.add_v_proj))
            if attn.norm_added_q is not None:
                eq = attn.norm_added_q(eq)
            if attn.norm_added_k is not None:
                ek = attn.norm_added_k(ek)
            query, key, value = torch.cat((query, eq), 2), torch.cat((key, ek), 2), torch.cat((value, ev), 2)
        output = self.attention(query.contiguous(), key.contiguous(), value.contiguous())
        output = output.transpose(1, 2).flatten(2, 3).to(query.dtype)
        if not text_length:
            return output, encoder_hidden_states
        output, encoder_output = output[:, :-text_length], output[:, -text_length:]
        if getattr(attn, "to_out", None) is not None:
            output = attn.to_out[1](attn.to_out[0](output))
        if getattr(attn, "to_add_out", None) is not None:
            encoder_output = attn.to_add_out(encoder_output)
        return output, encoder_output


def _rows_view(x):
    """(tensor, head_rows) for a [1,H,N,D] view of a contiguous [1,H,S,D] tensor:
    head h's rows start at row h*S of the underlying storage."""
    if x.stride(3) != 1 or x.stride(2) != x.shape[3]:
        x = x.contiguous()
    return x, x.stride(1) // x.shape[3]


def _rotary():
    """diffusers' apply_rotary_emb when installed, else the same rotation
    (real cos/sin tables, pairs interleaved along the last dim)."""
    try:
        from diffusers.models.embeddings import apply_rotary_emb
        return apply_rotary_emb
    except Exception:  # diffusers is optional
        def apply_rotary_emb(x, freqs_cis):
            cos, sin = freqs_cis
            cos, sin = cos[None, None].to(x.device), sin[None, None].to(x.device)
            xr, xi = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
            rotated = torch.stack([-xi, xr], dim=-1).flatten(3)
            return (x.float() * cos + rotated.float() * sin).to(x.dtype)
        return apply_rotary_emb
