"""Base-Offset PE quantization of Q/K on the sm_100a kernels.

Mirrors peco/quantization.py: the same ``BaseOffsetQuantized`` payload and
``quantize_base_offset`` / ``dequantize_base_offset`` /
``fake_quantize_base_offset`` functions with the same validation.  Each token
row (per batch/head) is encoded against its cluster centroid with one affine
min-max quantizer over the D channels:

    r = x - C[label];  low = min r;  scale = (max r - low) / (2^bits - 1) (1 if not > 0)
    code = clamp(round_half_even((r - low) / scale), 0, 2^bits - 1)
    x_hat = C[label] + (low + scale * code)

The kernels evaluate every step as one IEEE fp32 operation, so codes,
offsets, scales and reconstructions are bit-identical to the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native


@dataclass(frozen=True)
class BaseOffsetQuantized:
    """Quantized payload with flattened batch/head axes.

    ``centroids`` fp32 [BH,K,D], ``labels`` int64 [BH,N], ``codes`` uint8
    [BH,N,D], ``offset_min`` / ``scale`` fp32 [BH,N,1]; ``original_shape``
    restores [BH,N,D] or [B,H,N,D].
    """

    centroids: torch.Tensor
    labels: torch.Tensor
    codes: torch.Tensor
    offset_min: torch.Tensor
    scale: torch.Tensor
    original_dtype: torch.dtype
    original_shape: tuple
    bits: int

    def dequantize(self) -> torch.Tensor:
        return dequantize_base_offset(self)


def _check_bits(bits: int, *, bypass_ok: bool) -> None:
    """Accept 4 or 8 bits, and 0 (the identity) where a bypass is allowed.

    The error text is the reference's (peco/quantization.py:55-59) so callers
    see the same exception; a bool or any non-int type is refused."""
    choices = (0, 4, 8) if bypass_ok else (4, 8)
    if type(bits) is not int or bits not in choices:
        hint = "" if bypass_ok else "; use fake_quantize_base_offset(..., bits=0) to bypass"
        raise ValueError(f"bits must be one of {choices}{hint}")


def _flatten_inputs(x, labels, centroids):
    if x.ndim not in (3, 4):
        raise ValueError("x must have shape [BH,N,D] or [B,H,N,D]")
    if any(size == 0 for size in x.shape):
        raise ValueError("x dimensions must be nonempty")
    if not x.is_floating_point() or not centroids.is_floating_point():
        raise TypeError("x and centroids must have floating-point dtypes")
    if labels.dtype not in (torch.int32, torch.int64):
        raise TypeError("labels must have dtype int32 or int64")
    if x.device != labels.device or x.device != centroids.device:
        raise ValueError("x, labels and centroids must be on the same device")
    n, d = x.shape[-2:]
    flat = x.reshape(-1, n, d)
    if labels.shape != flat.shape[:2]:
        raise ValueError(f"labels must have shape {tuple(flat.shape[:2])}")
    if centroids.ndim != 3 or centroids.shape[0] != flat.shape[0] or centroids.shape[1] == 0 or centroids.shape[2] != d:
        raise ValueError(f"centroids must have shape [{flat.shape[0]},K,{d}] with K > 0")
    if x.dtype not in _native.DTYPE_CODE:
        raise TypeError("x must be float16, bfloat16 or float32")
    return flat.contiguous(), labels.to(torch.int32).contiguous(), centroids.float().contiguous()


def _call(mode, flat, lab32, cen, out, codes, low, scale, bits, dtype):
    lib = _native.load()
    dev = _native.require_cuda(flat, lab32, cen)
    bh, n, d = flat.shape
    with torch.cuda.device(dev):
        status = lib.peco_base_offset(int(mode), _native.ptr(flat), _native.ptr(lab32), _native.ptr(cen),
                                      _native.ptr(out), _native.ptr(codes), _native.ptr(low), _native.ptr(scale),
                                      bh, n, d, cen.shape[1], int(bits), _native.DTYPE_CODE[dtype],
                                      _native.stream_of(dev, flat, lab32, cen, out, codes, low, scale))
    _native.check(status, "peco_base_offset")


@torch.no_grad()
def quantize_base_offset(x, labels, centroids, bits: int = 4) -> BaseOffsetQuantized:
    """Encode Q or K using its assigned cluster's vector centroid (bits 4 or 8)."""
    _check_bits(bits, bypass_ok=False)
    flat, lab32, cen = _flatten_inputs(x, labels, centroids)
    bh, n, d = flat.shape
    codes = torch.empty((bh, n, d), dtype=torch.uint8, device=flat.device)
    low = torch.empty((bh, n, 1), dtype=torch.float32, device=flat.device)
    scale = torch.empty((bh, n, 1), dtype=torch.float32, device=flat.device)
    _call(1, flat, lab32, cen, None, codes, low, scale, bits, flat.dtype)
    return BaseOffsetQuantized(centroids=cen, labels=labels.to(torch.int64), codes=codes, offset_min=low,
                               scale=scale, original_dtype=x.dtype, original_shape=tuple(x.shape), bits=bits)


@torch.no_grad()
def dequantize_base_offset(encoded: BaseOffsetQuantized) -> torch.Tensor:
    """Reconstruct a quantized payload to the input shape and dtype."""
    cen = encoded.centroids.float().contiguous()
    lab32 = encoded.labels.to(torch.int32).contiguous()
    bh, n, d = encoded.codes.shape
    out = torch.empty((bh, n, d), dtype=encoded.original_dtype, device=cen.device)
    _call(2, out, lab32, cen, out, encoded.codes.contiguous(), encoded.offset_min.float().contiguous(),
          encoded.scale.float().contiguous(), encoded.bits, encoded.original_dtype)
    return out.reshape(encoded.original_shape)


@torch.no_grad()
def fake_quantize_base_offset(x, labels, centroids, bits: int = 4) -> torch.Tensor:
    """Quantize/dequantize Q or K in one pass; bits=0 returns ``x`` itself."""
    _check_bits(bits, bypass_ok=True)
    if bits == 0:
        return x
    flat, lab32, cen = _flatten_inputs(x, labels, centroids)
    out = torch.empty_like(flat)
    _call(0, flat, lab32, cen, out, None, None, None, bits, flat.dtype)
    return out.reshape(x.shape)
