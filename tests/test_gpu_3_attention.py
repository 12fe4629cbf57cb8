"""GPU parity of the tcgen05 cluster-sparse attention.

Tolerance (the north-star bound for bf16 attention): cosine >= 0.999 and
max |err| <= 2e-2 against the fp32 oracle; rows with no allowed key must be
exactly zero.  Where the reference's own kernel (built from its source by
oracle/Makefile) is present, the B200 kernel is also compared with it.
"""

import math

import pytest
import torch

from oracle import peco_oracle as O
from oracle import ref_gpu
from peco_b200 import synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"
COS_MIN, ABS_MAX = 0.999, 2e-2


@pytest.fixture(autouse=True)
def _clean_status():
    from peco_b200 import _native
    _native.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert _native.device_status(clear=True) == 0


def assert_close_attention(got, ref, zero_rows=None):
    g, r = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(g).all()
    err = (g - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(g.flatten(), r.flatten(), dim=0).item()
    assert err <= ABS_MAX and cos >= COS_MIN, f"max err {err:.3g}, cosine {cos:.6f}"
    if zero_rows is not None and zero_rows.any():
        assert (g[zero_rows] == 0).all()


def random_problem(h, sq, sk, d, gq, gk, dtype, seed, density=0.4, empty_groups=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((1, h, sq, d), generator=g).to(dtype)
    k = torch.randn((1, h, sk, d), generator=g).to(dtype)
    v = torch.randn((1, h, sk, d), generator=g).to(dtype)

    def sizes(total, groups):
        cuts = torch.sort(torch.randint(0, total + 1, (h, groups - 1), generator=g), dim=-1).values
        z = torch.zeros((h, 1), dtype=torch.long)
        e = torch.full((h, 1), total, dtype=torch.long)
        s = torch.diff(torch.cat((z, cuts, e), -1), dim=-1)
        if empty_groups and groups > 2:
            s[:, 1] += s[:, 0]
            s[:, 0] = 0
        return s.int().unsqueeze(0)

    qs, ks = sizes(sq, gq), sizes(sk, gk)
    dmap = torch.rand((1, h, gq, gk), generator=g) < density
    dmap[0, :, -1] = False  # one query group with no key
    return q, k, v, dmap, qs, ks


def zero_rows_of(dmap, qs, ks):
    b, h, gq, gk = dmap.shape
    rows = []
    for hi in range(h):
        allowed = (dmap[0, hi] & (ks[0, hi] > 0).unsqueeze(0)).any(-1)
        rows.append(torch.repeat_interleave(~allowed, qs[0, hi].long()))
    return torch.stack(rows).unsqueeze(0)


@pytest.mark.parametrize("d", [128, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_random_groups(d, dtype):
    from peco_b200 import attention_cuda
    q, k, v, dmap, qs, ks = random_problem(3, 700, 650, d, 9, 13, dtype, seed=d)
    got = attention_cuda.sparse_attention(*(t.to(DEV) for t in (q, k, v, dmap, qs, ks)))
    ref = O.sparse_attention(q, k, v, dmap, qs, ks)
    assert_close_attention(got, ref, zero_rows_of(dmap, qs, ks))


def test_large_group_runs_and_single_keys():
    """A query group larger than 128 rows, one-key groups, adjacent runs merged."""
    from peco_b200 import attention_cuda
    h, sq, sk, d = 2, 600, 530, 128
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn((1, h, n, d), generator=g).bfloat16() for n in (sq, sk, sk))
    qs = torch.tensor([[[300, 1, 0, 299], [1, 599, 0, 0]]], dtype=torch.int32)
    ks = torch.tensor([[[1, 1, 500, 28], [7, 0, 523, 0]]], dtype=torch.int32)
    dmap = torch.tensor([[[[1, 1, 1, 0], [0, 1, 0, 0], [1, 1, 1, 1], [1, 0, 0, 1]],
                          [[0, 0, 1, 1], [1, 1, 1, 1], [1, 0, 0, 0], [0, 1, 0, 0]]]], dtype=torch.bool)
    got = attention_cuda.sparse_attention(*(t.to(DEV) for t in (q, k, v, dmap, qs, ks)))
    ref = O.sparse_attention(q, k, v, dmap, qs, ks)
    assert_close_attention(got, ref, zero_rows_of(dmap, qs, ks))


def test_dense_map_equals_full_attention():
    from peco_b200 import attention_cuda
    h, s, d = 2, 520, 128
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn((1, h, s, d), generator=g).bfloat16() for _ in range(3))
    qs = torch.tensor([[[200, 320], [520, 0]]], dtype=torch.int32)
    ks = torch.tensor([[[100, 420], [260, 260]]], dtype=torch.int32)
    dmap = torch.ones((1, h, 2, 2), dtype=torch.bool)
    got = attention_cuda.sparse_attention(*(t.to(DEV) for t in (q, k, v, dmap, qs, ks)))
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert_close_attention(got, ref)


def key_block_image(x, sizes, sk):
    """Restatement of the key-block layout: row-major x [H,SK,D] (16-bit) ->
    [H, blocks * 8, D] in block image order, and the blocks each head uses.
    Cluster c (extent clamped to SK) starts block gp[c]; block b holds D/64
    panels of 8 rows x 128 bytes and the 16-byte chunk c of row i sits at
    chunk c ^ i; padding rows are zero (blocks past the used ones are left
    unwritten by the kernels)."""
    h, _, d = x.shape
    gk = sizes.shape[-1]
    blocks = (sk + 7) // 8 + gk
    i = torch.arange(8).view(8, 1)
    dd = torch.arange(d).view(1, d)
    off = ((dd // 64) * 1024 + i * 128 + (((dd % 64) // 8) ^ i) * 16 + (dd % 8) * 2) // 2  # [8, D] element slots
    img = torch.zeros((h, blocks, 8 * d), dtype=x.dtype)
    used = []
    for hh in range(h):
        ends = torch.cumsum(sizes[hh].clamp_min(0).long(), 0).clamp_max(sk)
        starts = torch.cat((torch.zeros(1, dtype=torch.long), ends[:-1]))
        nb = (ends - starts + 7) // 8
        gp = torch.cat((torch.zeros(1, dtype=torch.long), torch.cumsum(nb, 0)[:-1]))
        for c in range(gk):
            for r in range(int(ends[c] - starts[c])):
                b, ii = divmod(int(gp[c]) * 8 + r, 8)
                img[hh, b, off[ii]] = x[hh, int(starts[c]) + r]
        used.append(int(nb.sum()))
    return img.view(h, blocks * 8, d), used


def test_key_blocks_match_layout_restatement():
    """Plan + pack of row-major K/V reproduce the key-block image bit for bit."""
    from peco_b200 import attention_cuda
    for d, seed in ((128, 5), (64, 6)):
        q, k, v, dmap, qs, ks = random_problem(2, 300, 290, d, 5, 9, torch.bfloat16, seed=seed)
        ks[0, 1, 3] += 40  # sizes that overrun SK are clamped like the reference's work map
        args = [t.to(DEV).contiguous() for t in (dmap, qs, ks, k, v)]
        ws, kb, vb = attention_cuda.plan_key_blocks(args[0], args[1], args[2], 300, args[3], args[4])
        for got, x in ((kb, k), (vb, v)):
            ref, used = key_block_image(x[0], ks[0], 290)
            for hh, n in enumerate(used):
                assert torch.equal(got[hh, :8 * n].cpu().view(torch.int16), ref[hh, :8 * n].view(torch.int16))


def _pipeline_inputs(w, seed, heads):
    """Packed Q/K/V, text-extended map and sizes of a real PECO call (oracle)."""
    q, k, v = synthetic.make_inputs(w, seed=seed, heads=heads)
    nv, d = w.video_tokens, w.dims
    qv, kv = q[:, :, :nv].reshape(heads, nv, d), k[:, :, :nv].reshape(heads, nv, d)
    ql, qc, qn = O.fit_token_clusters(qv, w.q_clusters, w.iters, synthetic.init_centroids(qv, w.q_clusters, w.init))
    kl, kc, kn = O.fit_token_clusters(kv, w.k_clusters, w.iters, synthetic.init_centroids(kv, w.k_clusters, w.init))
    qs, ks = qn.reshape(1, heads, -1), kn.reshape(1, heads, -1)
    dmap = O.select_cluster_connections(qc.reshape(1, heads, -1, d), kc.reshape(1, heads, -1, d), qs, ks, w.top_p,
                                        w.min_kc_ratio)
    qi, ki = O.sort_indices(ql), O.sort_indices(kl)
    qp = torch.cat((O.gather_rows(q[:, :, :nv], qi), q[:, :, nv:]), 2).contiguous()
    kp = torch.cat((O.gather_rows(k[:, :, :nv], ki), k[:, :, nv:]), 2).contiguous()
    vp = torch.cat((O.gather_rows(v[:, :, :nv], ki), v[:, :, nv:]), 2).contiguous()
    em, eqs, eks = O.extend_text_partition(dmap, qs, ks, w.valid_text, w.text_length)
    return qp, kp, vp, em, eqs, eks, qi


def test_headline_layer_two_heads():
    """Two heads of the HV-480 layer with the real cluster map and text groups."""
    from peco_b200 import attention_cuda
    w = synthetic.workload("hv480", valid_text=200)
    qp, kp, vp, em, eqs, eks, _ = _pipeline_inputs(w, seed=0, heads=2)
    got = attention_cuda.sparse_attention(*(t.to(DEV) for t in (qp, kp, vp, em, eqs, eks)))
    ref = O.sparse_attention(qp, kp, vp, em, eqs, eks)
    assert_close_attention(got, ref, zero_rows_of(em, eqs, eks))
    if ref_gpu.available():
        rk = ref_gpu.sparse_attention(*(t.to(DEV) for t in (qp, kp, vp, em, eqs, eks)))
        assert_close_attention(rk, ref)          # pins the oracle to the reference kernel
        assert_close_attention(got, rk.float())  # and ours to it directly


def test_restore_epilogue_scatters_rows():
    from peco_b200 import _native, attention_cuda
    w = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24, q_clusters=16,
                           k_clusters=32, top_k=8)
    qp, kp, vp, em, eqs, eks, qi = _pipeline_inputs(w, seed=4, heads=2)
    args = [t.to(DEV).contiguous() for t in (qp, kp, vp, em, eqs, eks)]
    packed_out = attention_cuda.sparse_attention(*args)
    h, s, d = 2, w.seq, w.dims
    nv = w.video_tokens
    out = torch.empty_like(args[0])
    lib = _native.load()
    gq, gk = em.shape[-2], em.shape[-1]
    ws, kb, vb = attention_cuda.plan_key_blocks(args[3], args[4], args[5], s, args[1], args[2])
    perm = qi.to(DEV).contiguous()
    keep = [args[0], kb, vb, ws, out, perm]
    st = lib.peco_sparse_attention_restore(_native.ptr(args[0]), _native.ptr(kb), _native.ptr(vb), _native.ptr(ws),
                                           _native.ptr(out), h, s, s, d, gq, gk, _native.ptr(perm), nv,
                                           _native.stream_of(args[0].device, *keep))
    _native.check(st, "peco_sparse_attention_restore")
    text_idx = torch.arange(nv, s, dtype=torch.int32)
    idx = torch.cat((qi, text_idx.expand(h, -1)), -1)
    assert torch.equal(out.cpu(), O.scatter_rows(packed_out.cpu(), idx))


def test_reference_kernel_pins_oracle_on_random_groups():
    if not ref_gpu.available():
        pytest.skip("oracle/_ref not built")
    q, k, v, dmap, qs, ks = random_problem(2, 300, 280, 128, 6, 7, torch.bfloat16, seed=77)
    rk = ref_gpu.sparse_attention(*(t.to(DEV).contiguous() for t in (q, k, v, dmap, qs, ks)))
    ref = O.sparse_attention(q, k, v, dmap, qs, ks)
    assert_close_attention(rk, ref)
