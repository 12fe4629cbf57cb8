"""The processor's input stage on the GPU (peco_prepare_qkv) and the fused
processor entry built on it.

``peco_prepare_qkv`` is compared with a torch evaluation of the same
formulas -- the model's RMSNorm module (fp32 normalise and gain, rounded to
bf16) and the pair rotation of the video rows -- on strided projection
views.  Tolerance: equal except where the sum of squares, accumulated in a
different order, moves a value across a bf16 rounding boundary (one bf16 ulp,
on at most 0.1% of the elements).  The fused ``PecoAttention.__call__`` path
(with exact attention) is compared with the plain torch path of the same
module math: cosine >= 0.9999 on the block outputs.
"""

import pytest
import torch

from peco_b200 import _native
from peco_b200.hunyuan import RMSNorm, rotate_pairs, rope_3d

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ulp_close(got, ref):
    g, r = got.float(), ref.float()
    diff = (g - r).abs()
    ulp = r.abs().clamp_min(1e-30) * 2.0 ** -7
    bad = diff > ulp * 1.01
    assert not bad.any(), f"{int(bad.sum())} elements off by more than one bf16 ulp"
    assert (diff > 0).float().mean().item() <= 1e-3


@pytest.mark.parametrize("dims,axes", [(128, (16, 56, 56)), (64, (16, 24, 24))])
@pytest.mark.parametrize("separate_text,use_rope", [(True, True), (False, True), (True, False)])
def test_prepare_qkv_matches_module_math(dims, axes, separate_text, use_rope):
    g = torch.Generator(device=DEV).manual_seed(dims + 7 * separate_text + use_rope)
    heads, grid, n_text = 3, (2, 6, 10), 37
    n_video = grid[0] * grid[1] * grid[2]
    inner = heads * dims
    # projection outputs as strided column blocks of one [rows, 3 * inner] buffer
    vbuf = torch.randn((n_video, 3 * inner), generator=g, device=DEV).to(torch.bfloat16) * 3
    tbuf = torch.randn((n_text, 3 * inner), generator=g, device=DEV).to(torch.bfloat16) * 3
    vq, vk, vv = vbuf.split(inner, dim=1)
    tq, tk, tv = tbuf.split(inner, dim=1)
    norms = [RMSNorm(dims).to(DEV) for _ in range(4)]
    with torch.no_grad():
        for n in norms:
            n.weight.copy_(1 + 0.1 * torch.randn(dims, generator=g, device=DEV))
    if not separate_text:
        norms[2], norms[3] = norms[0], norms[1]
    cos, sin = rope_3d(grid, axes, 256.0, DEV) if use_rope else (None, None)
    q, k, v = (torch.empty((1, heads, n_video + n_text, dims), dtype=torch.bfloat16, device=DEV) for _ in range(3))
    weights = [n.weight.detach().float().contiguous() for n in norms]
    lib = _native.load()
    opt = (lambda t: _native.ptr(t) if t is not None else _native.P(0))
    keep = [vbuf, tbuf, q, k, v, *weights] + ([cos, sin] if use_rope else [])
    st = lib.peco_prepare_qkv(_native.ptr(vq), _native.ptr(vk), _native.ptr(vv), 3 * inner, n_video,
                              _native.ptr(tq), _native.ptr(tk), _native.ptr(tv), 3 * inner, n_text,
                              _native.ptr(weights[0]), _native.ptr(weights[1]), 1e-6, _native.ptr(weights[2]),
                              _native.ptr(weights[3]), 1e-6, opt(cos), opt(sin), _native.ptr(q), _native.ptr(k),
                              _native.ptr(v), heads, dims, _native.stream_of(vbuf.device, *keep))
    _native.check(st, "peco_prepare_qkv")
    torch.cuda.synchronize()

    def split(x):
        return x.reshape(1, -1, heads, dims).transpose(1, 2)

    with torch.no_grad():
        rq, rk = norms[0](split(vq)), norms[1](split(vk))
        if use_rope:
            rq, rk = rotate_pairs(rq, cos, sin), rotate_pairs(rk, cos, sin)
        rq = torch.cat((rq, norms[2](split(tq))), 2)
        rk = torch.cat((rk, norms[3](split(tk))), 2)
        rv = torch.cat((split(vv), split(tv)), 2)
    assert torch.equal(v, rv)
    _ulp_close(q, rq)
    _ulp_close(k, rk)
    assert _native.device_status(clear=True) == 0


def test_prepare_qkv_rejects_bad_arguments():
    lib = _native.load()
    x = torch.empty((4, 256), dtype=torch.bfloat16, device=DEV)
    z = _native.P(0)
    p = _native.ptr(x)
    stream = _native.stream_of(x.device, x)
    # unsupported head size, stride below a row, rotation tables given only in part
    assert lib.peco_prepare_qkv(p, p, p, 256, 4, z, z, z, 0, 0, z, z, 0.0, z, z, 0.0, z, z, p, p, p, 1, 96,
                                stream) != 0
    assert lib.peco_prepare_qkv(p, p, p, 128, 4, z, z, z, 0, 0, z, z, 0.0, z, z, 0.0, z, z, p, p, p, 2, 128,
                                stream) != 0
    assert lib.peco_prepare_qkv(p, p, p, 256, 4, z, z, z, 0, 0, z, z, 0.0, z, z, 0.0, p, z, p, p, p, 2, 128,
                                stream) != 0


@pytest.mark.parametrize("dual", [True, False])
def test_fused_processor_entry_matches_torch_path(dual):
    """SDPAProcessor runs the fused entry on CUDA bf16 and its torch path
    otherwise; both with exact attention, so they differ only by the input
    stage's rounding."""
    from peco_b200.hunyuan import Attention, SDPAProcessor
    from peco_b200.processor import InferenceContext
    torch.manual_seed(3)
    heads, dims, n_text, grid = 4, 128, 24, (2, 4, 6)
    attn = Attention(256, heads, dims, joint_text=dual, pre_only=not dual).to(DEV, torch.bfloat16)
    ctx = InferenceContext(step=5, text_length=n_text, valid_text_length=20)
    proc = SDPAProcessor(ctx)
    attn.set_processor(proc)
    n_video = grid[0] * grid[1] * grid[2]
    video = torch.randn((1, n_video, 256), device=DEV).to(torch.bfloat16)
    text = torch.randn((1, n_text, 256), device=DEV).to(torch.bfloat16)
    rope = rope_3d(grid, (16, 56, 56), 256.0, DEV)
    with torch.no_grad():
        fused = attn(video, text, None, rope)
        plain = proc._torch_call(attn, video, text, rope)
    for a, b in zip(fused, plain):
        assert a.shape == b.shape
        cos = torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()
        assert cos >= 0.9999, cos
