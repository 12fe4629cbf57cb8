"""Attach PECO attention to a transformer (the integration of peco/model.py).

``install_attention(pipe, config)``: every dual-stream block, then every
single-stream block of ``pipe.transformer`` gets its own ``PecoAttention``
(its layer index is that order), all sharing one ``InferenceContext``.  A
forward pre-hook on the transformer advances ``context.step`` once per
denoising call and reads the text lengths from ``encoder_attention_mask``,
which must hold one prompt with right padding (peco/model.py:10-39).
Installing again replaces the previous hook.

``reset_state(pipe)``: before a new video, rewind the step counter and drop
every processor's cached centroids (peco/model.py:42-46).

Any transformer works that exposes ``transformer_blocks`` and
``single_transformer_blocks`` (blocks with ``attn.set_processor``) and whose
``forward`` takes ``encoder_attention_mask``: the diffusers HunyuanVideo
transformer, or ``peco_b200.hunyuan.HunyuanVideoTransformer``.
"""

from __future__ import annotations

import inspect

import torch

from .processor import InferenceContext, PecoAttention, PecoConfig


def _text_lengths(text_mask: torch.Tensor) -> tuple[int, int]:
    """(text_length, valid_text_length) of a [1, T] right-padded mask."""
    if text_mask.shape[0] != 1:
        raise ValueError("Use one prompt per inference call")
    keep = text_mask[0].detach().to(device="cpu", dtype=torch.bool)
    valid = int(keep.sum())
    if not bool(keep[:valid].all()) or bool(keep[valid:].any()):
        raise ValueError("Hunyuan text attention mask must use right padding")
    return keep.numel(), valid


def install_attention(pipe, config: PecoConfig) -> InferenceContext:
    model = pipe.transformer
    old_hook = getattr(model, "_peco_context_hook", None)
    if old_hook is not None:
        old_hook.remove()
    context = InferenceContext()
    layers = [*model.transformer_blocks, *model.single_transformer_blocks]
    processors = []
    for index, block in enumerate(layers):
        processors.append(PecoAttention(index, config, context))
        block.attn.set_processor(processors[-1])
    model._peco_context = context
    model._peco_processors = processors
    _register_context_hook(model, context)
    return context


def _register_context_hook(model, context: InferenceContext) -> None:
    """Forward pre-hook: advance the step and read the text lengths from the mask."""
    bind = inspect.signature(model.forward).bind_partial

    def before_forward(_module, args, kwargs):
        text_length, valid = _text_lengths(bind(*args, **kwargs).arguments["encoder_attention_mask"])
        context.step += 1
        context.text_length = text_length
        context.valid_text_length = valid

    model._peco_context_hook = model.register_forward_pre_hook(before_forward, with_kwargs=True)


def reset_state(pipe) -> None:
    """Call before each new video, including repeated calls on one pipeline."""
    pipe.transformer._peco_context.step = -1
    for processor in pipe.transformer._peco_processors:
        processor.reset()
