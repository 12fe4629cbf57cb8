"""Whole-call CUDA graph of a steady-state PECO attention call.

A steady-state ``PecoAttention.attention`` call (cached centroids, past the
warm-up steps) is a fixed sequence of library launches whose sizes depend
only on the shapes: k-means (prep, then assign/sort/update per Lloyd
iteration), selection, plan, quantise+gather and attention.  ``PecoCallGraph``
captures that sequence once and replays it, so a denoising loop pays one
graph launch per layer call instead of about thirty kernel launches and the
Python around them (the per-call launch overhead of the reference,
peco/processor.py:115-157).

Capture keeps the processor's semantics:

* Q/K/V are copied into static input buffers before each replay;
* the processor's centroids become fixed tensors that every replay reads as
  the k-means init and overwrites with the new centres
  (``update_centroids_in_place``), exactly as eager calls chain them;
* the output is a static tensor, overwritten by the next replay.

The graph holds stream-ordered allocations of the library (selection
logits) as graph memory nodes; everything else comes from the graph's
private torch pool.
"""

from __future__ import annotations

import torch


class PecoCallGraph:
    """Capture ``processor.attention(query, key, value)`` and replay it.

    ``processor`` must already hold centroids (one eager call ran, or they were
    preset) and its context must be past the warm-up steps; every replay then
    performs the same work as one eager steady-state call on the new inputs.
    The context's text lengths are frozen at capture.
    """

    def __init__(self, processor, query, key, value):
        cfg, ctx = processor.config, processor.context
        if processor.q_centroids is None or processor.k_centroids is None:
            raise ValueError("capture a steady-state call: the processor needs cached centroids")
        if ctx.step < cfg.warmup_steps or processor.layer_idx < cfg.warmup_layers:
            raise ValueError("the warm-up (dense) steps are not captured")
        if not query.is_cuda:
            raise ValueError("CUDA tensors required")
        self.processor = processor
        self.frozen = (ctx.text_length, ctx.valid_text_length)
        self.inputs = tuple(t.detach().contiguous().clone() for t in (query, key, value))
        # fixed centroid tensors: every replay reads and overwrites them
        processor.q_centroids = processor.q_centroids.float().contiguous().clone()
        processor.k_centroids = processor.k_centroids.float().contiguous().clone()
        processor.update_centroids_in_place = True
        self.graph = torch.cuda.CUDAGraph()
        events, processor.stage_events = processor.stage_events, None
        try:
            # nothing runs during capture, so the centroids are untouched
            with torch.cuda.graph(self.graph):
                self.output = processor.attention(*self.inputs)
        finally:
            processor.stage_events = events

    @property
    def centroids(self):
        """The (q, k) centroid tensors the graph reads and writes."""
        return self.processor.q_centroids, self.processor.k_centroids

    def set_centroids(self, q_centroids, k_centroids):
        """Copy new centroids into the graph's state (e.g. to rerun from a fixed init)."""
        qc, kc = self.centroids
        qc.copy_(q_centroids)
        kc.copy_(k_centroids)

    def __call__(self, query, key, value):
        ctx = self.processor.context
        if (ctx.text_length, ctx.valid_text_length) != self.frozen:
            raise ValueError("text lengths changed since capture; capture a new graph")
        for dst, src in zip(self.inputs, (query, key, value)):
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        self.graph.replay()
        return self.output


class PecoStepGraph:
    """One denoising step of a PECO-installed transformer, all layers in one
    CUDA graph: each replay launches every layer's attention call (its whole
    k-means, selection, quantise/gather and attention sequence) and the model's
    own kernels in between, so the step costs one graph launch instead of a
    few thousand kernel launches scheduled from Python.

    ``model`` is the transformer ``peco_b200.model.install_attention`` set up,
    past its warm-up steps with every processor's centroids cached (one eager
    step ran).  The context's step counter and text lengths are frozen at
    capture (its pre-hook, which reads the mask on the host, runs only
    eagerly); every processor's centroids become fixed tensors that each
    replay reads as the k-means init and overwrites, so replays chain like
    eager steps.  ``inputs`` are the forward's positional arguments (CUDA
    tensors); a replay copies new values into the captured ones.
    """

    def __init__(self, model, *inputs):
        processors = getattr(model, "_peco_processors", None)
        ctx = getattr(model, "_peco_context", None)
        if not processors or ctx is None:
            raise ValueError("install PECO attention on the model first (peco_b200.model.install_attention)")
        for p in processors:
            cfg = p.config
            if p.q_centroids is None or ctx.step < cfg.warmup_steps or p.layer_idx < cfg.warmup_layers:
                raise ValueError("capture a steady-state step: run one eager step past the warm-up first")
            p.q_centroids = p.q_centroids.float().contiguous().clone()
            p.k_centroids = p.k_centroids.float().contiguous().clone()
            p.update_centroids_in_place = True
        self.model = model
        self.frozen = (ctx.step, ctx.text_length, ctx.valid_text_length)
        self.inputs = tuple(t.detach().clone() if torch.is_tensor(t) else t for t in inputs)
        hook = getattr(model, "_peco_context_hook", None)
        if hook is not None:
            hook.remove()
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.no_grad(), torch.cuda.graph(self.graph):
                self.output = model(*self.inputs)
        finally:
            if hook is not None:  # put the eager step counter back
                from .model import _register_context_hook
                _register_context_hook(model, ctx)

    def __call__(self, *inputs):
        for dst, src in zip(self.inputs, inputs):
            if torch.is_tensor(dst) and src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        self.graph.replay()
        return self.output
