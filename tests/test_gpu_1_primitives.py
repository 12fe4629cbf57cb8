"""GPU parity of the memory-bound kernels against the oracle and the reference fixtures.

Bit-exact: reorder/restore, stable label sort, Base-Offset codes/offsets/scales
and reconstructions, the fused quantize+gather pass.  Selection maps agree
except where the reference's own probabilities tie within fp32 rounding.
"""

import numpy as np
import pytest
import torch

from oracle import peco_oracle as O
from peco_b200 import synthetic

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_status():
    from peco_b200 import _native
    _native.device_status(clear=True)
    yield
    torch.cuda.synchronize()
    assert _native.device_status(clear=True) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dims", [128, 64, 36])
def test_reorder_round_trip_bit_exact(dtype, dims):
    from peco_b200 import clustering_cuda
    g = torch.Generator().manual_seed(dims)
    b, h, n = 1, 3, 777
    x = torch.randn((b, h, n, dims), generator=g).to(dtype)
    idx = torch.stack([torch.randperm(n, generator=g) for _ in range(b * h)]).to(torch.int32)
    fwd = clustering_cuda.reorder_token_features(x.to(DEV), idx.to(DEV))
    assert torch.equal(fwd.cpu(), O.gather_rows(x, idx))
    inv = clustering_cuda.reorder_token_features(fwd, idx.to(DEV), inverse=True)
    assert torch.equal(inv.cpu(), x)


@pytest.mark.parametrize("tokens,clusters", [(1350, 32), (6750, 256), (5000, 2048), (31, 1), (100, 100)])
def test_stable_sort_matches_argsort(tokens, clusters):
    from peco_b200 import clustering_cuda
    g = torch.Generator().manual_seed(tokens)
    lab = torch.randint(clusters, (3, tokens), generator=g, dtype=torch.int32)
    lab[1] = lab[1] // max(1, clusters // 4)  # runs of equal labels and empty clusters
    idx, counts, offsets = clustering_cuda.sort_labels(lab.to(DEV), clusters)
    assert torch.equal(idx.cpu(), O.sort_indices(lab))
    ref_counts = torch.stack([torch.bincount(r.long(), minlength=clusters) for r in lab]).int()
    assert torch.equal(counts.cpu(), ref_counts)
    assert torch.equal(offsets.cpu()[:, 1:], ref_counts.cumsum(-1).int())


def test_gather_and_restore_api_bit_exact(golden):
    from peco_b200 import clustering
    gd = golden("small_bf16")
    raw = torch.from_numpy(gd["inputs"]).view(torch.bfloat16)
    q = raw[0:1]
    nv = 432
    qv = q[:, :, :nv].contiguous()
    labels = torch.from_numpy(gd["q_labels"])
    packed, idx = clustering.gather_clustered_tokens(qv.to(DEV), labels.to(DEV))
    np.testing.assert_array_equal(idx.cpu().numpy(), gd["q_indices"])
    assert torch.equal(packed.cpu(), O.gather_rows(qv, idx.cpu()))
    assert torch.equal(clustering.restore_sequence_order(packed, idx).cpu(), qv)


def _golden_small(golden):
    gd = golden("small_bf16")
    raw = torch.from_numpy(gd["inputs"]).view(torch.bfloat16)
    return gd, raw[0:1], raw[1:2], raw[2:3]


def test_base_offset_matches_reference_fixture(golden):
    from peco_b200 import quantization
    gd, q, _, _ = _golden_small(golden)
    nv = 432
    qv = q[:, :, :nv].contiguous().to(DEV)
    lab = torch.from_numpy(gd["q_labels"]).to(DEV)
    cen = torch.from_numpy(gd["q_centroids"]).to(DEV)
    for bits in (4, 8):
        enc = quantization.quantize_base_offset(qv, lab, cen, bits)
        np.testing.assert_array_equal(enc.codes.cpu().numpy(), gd[f"q_codes{bits}"])
        np.testing.assert_array_equal(enc.offset_min.cpu().numpy(), gd[f"q_low{bits}"])
        np.testing.assert_array_equal(enc.scale.cpu().numpy(), gd[f"q_scale{bits}"])
        ref = torch.from_numpy(gd[f"q_fake{bits}"]).view(torch.bfloat16)
        assert torch.equal(quantization.fake_quantize_base_offset(qv, lab, cen, bits).cpu(), ref)
        assert torch.equal(enc.dequantize().cpu(), ref)
    assert quantization.fake_quantize_base_offset(qv, lab, cen, 0) is qv


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_base_offset_other_dtypes_bit_exact(dtype):
    from peco_b200 import quantization
    g = torch.Generator().manual_seed(5)
    bh, n, d, k = 2, 300, 128, 7
    x = (torch.randn((bh, n, d), generator=g) * 3).to(dtype)
    lab = torch.randint(k, (bh, n), generator=g, dtype=torch.int32)
    cen = torch.randn((bh, k, d), generator=g)
    x[0, 5] = cen[0, lab[0, 5]].to(dtype)  # constant residual when exact in dtype
    ref = O.fake_quantize_base_offset(x, lab, cen, 4)
    got = quantization.fake_quantize_base_offset(x.to(DEV), lab.to(DEV), cen.to(DEV), 4).cpu()
    assert torch.equal(got.view(torch.int16 if dtype == torch.float16 else torch.int32),
                       ref.view(torch.int16 if dtype == torch.float16 else torch.int32))


def test_base_offset_edge_fixture(golden):
    from peco_b200 import quantization
    e = golden("edge")
    x = torch.from_numpy(e["x"]).to(DEV)
    lab = torch.from_numpy(e["labels"]).to(DEV)
    cen = torch.from_numpy(e["centroids"]).to(DEV)
    enc = quantization.quantize_base_offset(x, lab, cen, 4)
    np.testing.assert_array_equal(enc.codes.cpu().numpy(), e["codes"])
    np.testing.assert_array_equal(enc.offset_min.cpu().numpy(), e["low"])
    np.testing.assert_array_equal(enc.scale.cpu().numpy(), e["scale"])
    fq = quantization.fake_quantize_base_offset(x.to(torch.bfloat16), lab, cen, 4)
    np.testing.assert_array_equal(fq.cpu().view(torch.int16).numpy(), e["fake_bf16"])


@pytest.mark.parametrize("bits", [4, 8, 0])
def test_quantize_gather_bit_exact(bits):
    from peco_b200 import _native
    w = synthetic.workload("hv480", heads=3, grid=(2, 12, 18), text_length=32, valid_text=24, q_clusters=16,
                           k_clusters=32)
    q, k, v = synthetic.make_inputs(w, seed=11)
    h, s, d, nv = w.heads, w.seq, w.dims, w.video_tokens
    g = torch.Generator().manual_seed(2)
    ql = torch.randint(16, (h, nv), generator=g, dtype=torch.int32)
    kl = torch.randint(32, (h, nv), generator=g, dtype=torch.int32)
    qc = torch.randn((h, 16, d), generator=g)
    kc = torch.randn((h, 32, d), generator=g)
    qi, ki = O.sort_indices(ql), O.sort_indices(kl)
    ref_q = torch.cat((O.gather_rows(O.fake_quantize_base_offset(q[:, :, :nv], ql, qc, bits), qi), q[:, :, nv:]), 2)
    ref_k = torch.cat((O.gather_rows(O.fake_quantize_base_offset(k[:, :, :nv], kl, kc, bits), ki), k[:, :, nv:]), 2)
    ref_v = torch.cat((O.gather_rows(v[:, :, :nv], ki), v[:, :, nv:]), 2)
    Q, K, V = (t.to(DEV).contiguous() for t in (q, k, v))
    outs = [torch.empty_like(Q) for _ in range(3)]
    lib = _native.load()
    dev = Q.device
    args = [Q, K, V, *outs, qi.to(DEV), ki.to(DEV), ql.to(DEV), kl.to(DEV), qc.to(DEV), kc.to(DEV)]
    st = lib.peco_quantize_gather(*[_native.ptr(t) for t in args], 16, 32, h, s, nv, d, bits, None, 0, 0,
                                  _native.stream_of(dev, *args))
    _native.check(st, "peco_quantize_gather")
    assert torch.equal(outs[0].cpu(), ref_q)
    assert torch.equal(outs[1].cpu(), ref_k)
    assert torch.equal(outs[2].cpu(), ref_v)


def test_quantize_gather_writes_key_blocks():
    """With a plan, K/V land in key blocks: identical to packing the
    row-major result of the same pass."""
    from peco_b200 import _native, attention_cuda
    w = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24, q_clusters=16,
                           k_clusters=32)
    q, k, v = synthetic.make_inputs(w, seed=12)
    h, s, d, nv = w.heads, w.seq, w.dims, w.video_tokens
    g = torch.Generator().manual_seed(3)
    ql = torch.randint(16, (h, nv), generator=g, dtype=torch.int32)
    kl = torch.randint(32, (h, nv), generator=g, dtype=torch.int32)
    qc = torch.randn((h, 16, d), generator=g)
    kc = torch.randn((h, 32, d), generator=g)
    qi, ki = O.sort_indices(ql), O.sort_indices(kl)
    qs = torch.cat((torch.bincount(ql[0], minlength=16).view(1, 1, 16).expand(1, h, 16),
                    torch.tensor([24, 8]).view(1, 1, 2).expand(1, h, 2)), -1).int().contiguous()
    ks = torch.cat((torch.stack([torch.bincount(kl[i], minlength=32) for i in range(h)]).view(1, h, 32),
                    torch.tensor([24, 8]).view(1, 1, 2).expand(1, h, 2)), -1).int().contiguous()
    dmap = torch.rand((1, h, 18, 34), generator=g) < 0.5
    Q, K, V = (t.to(DEV).contiguous() for t in (q, k, v))
    lib = _native.load()
    dev = Q.device
    rows = [torch.empty_like(Q) for _ in range(3)]
    common = [qi.to(DEV), ki.to(DEV), ql.to(DEV), kl.to(DEV), qc.to(DEV), kc.to(DEV)]
    st = lib.peco_quantize_gather(*[_native.ptr(t) for t in [Q, K, V, *rows, *common]], 16, 32, h, s, nv, d, 4,
                                  None, 0, 0, _native.stream_of(dev, Q, K, V, *rows, *common))
    _native.check(st, "peco_quantize_gather")
    meta = [t.to(DEV).contiguous() for t in (dmap, qs, ks)]
    ws, kb_ref, vb_ref = attention_cuda.plan_key_blocks(*meta, s, rows[1], rows[2])
    qp = torch.empty_like(Q)
    kb, vb = torch.empty_like(kb_ref), torch.empty_like(vb_ref)
    st = lib.peco_attention_plan(*[_native.ptr(t) for t in (*meta, kb, vb, ws)], h, s, s, d, 18, 34,
                                 _native.stream_of(dev, *meta, kb, vb, ws))
    _native.check(st, "peco_attention_plan")
    st = lib.peco_quantize_gather(*[_native.ptr(t) for t in [Q, K, V, qp, kb, vb, *common]], 16, 32, h, s, nv, d, 4,
                                  _native.ptr(ws), 18, 34, _native.stream_of(dev, Q, K, V, qp, kb, vb, ws, *common))
    _native.check(st, "peco_quantize_gather")
    assert torch.equal(qp, rows[0])
    for hh in range(h):  # blocks past the ones a head uses are never written
        used = 8 * int(((ks[0, hh].long() + 7) // 8).sum())
        assert torch.equal(kb[hh, :used].view(torch.int16), kb_ref[hh, :used].view(torch.int16))
        assert torch.equal(vb[hh, :used].view(torch.int16), vb_ref[hh, :used].view(torch.int16))


def _select_ties_explain(qc, kc, qs, ks, p, ratio, got, ref):
    """Every differing map entry must sit on a near-tie of the reference's
    probabilities (relative gap < 1e-5 at the selection boundary)."""
    probs = O.cluster_probabilities(qc, kc, ks)
    diff = (got != ref).nonzero().tolist()
    for (b, h, i, j) in diff:
        row = probs[b, h, i]
        pj = row[j]
        close = ((row - pj).abs() <= 1e-5 * pj.abs().clamp_min(1e-30)).sum() > 1
        assert close, f"map differs at {(b, h, i, j)} without a tie"


@pytest.mark.parametrize("tag", ["map", "map_p09", "map_p1", "map_p0"])
def test_select_matches_reference_fixture(golden, tag):
    from peco_b200 import clustering
    w = synthetic.workload("cpu-plumbing")
    gd = golden("cpu_plumbing")
    params = {"map": (w.top_p, w.min_kc_ratio), "map_p09": (0.9, 0.1), "map_p1": (1.0, 0.0), "map_p0": (0.0, 0.0)}
    p, ratio = params[tag]
    qc = torch.from_numpy(gd["q_centroids"]).reshape(1, 2, -1, 128)
    kc = torch.from_numpy(gd["k_centroids"]).reshape(1, 2, -1, 128)
    qs = torch.from_numpy(gd["q_counts"]).reshape(1, 2, -1)
    ks = torch.from_numpy(gd["k_counts"]).reshape(1, 2, -1)
    got = clustering.select_cluster_connections(qc.to(DEV), kc.to(DEV), qs.to(DEV), ks.to(DEV), p, ratio).cpu()
    ref = torch.from_numpy(gd[tag])
    _select_ties_explain(qc, kc, qs, ks, p, ratio, got, ref)
    assert (got != ref).float().mean() < 1e-3


def test_select_text_partition_fused(golden):
    from peco_b200 import _native
    gd = golden("small_bf16")
    qc = torch.from_numpy(gd["q_centroids"]).to(DEV)
    kc = torch.from_numpy(gd["k_centroids"]).to(DEV)
    qs = torch.from_numpy(gd["q_counts"]).to(DEV)
    ks = torch.from_numpy(gd["k_counts"]).to(DEV)
    h, cq, ck = 2, 16, 32
    emap = torch.empty((1, h, cq + 2, ck + 2), dtype=torch.bool, device=DEV)
    eq = torch.empty((1, h, cq + 2), dtype=torch.int32, device=DEV)
    ek = torch.empty((1, h, ck + 2), dtype=torch.int32, device=DEV)
    lib = _native.load()
    args = [qc, kc, qs, ks, emap, eq, ek]
    logits = torch.empty((h, cq, ck), dtype=torch.float32, device=DEV)  # the caller's scratch
    st = lib.peco_select_text_partition(*[_native.ptr(t) for t in args], h, cq, ck, 128, 1e-9, 8, 24, 32,
                                        _native.ptr(logits), _native.stream_of(qc.device, *args, logits))
    _native.check(st, "peco_select_text_partition")
    assert torch.equal(emap.cpu(), torch.from_numpy(gd["ext_map"]))
    assert torch.equal(eq.cpu(), torch.from_numpy(gd["ext_q_sizes"]))
    assert torch.equal(ek.cpu(), torch.from_numpy(gd["ext_k_sizes"]))


def _units_by_rule(sizes, sq, split=1):
    """The planner's packing rule, sequentially: query groups in descending
    order; consecutive whole groups share a unit while their rows fit in 128
    and there are at most four (empty groups included, but a unit never starts
    with one); a group above 128 rows gets one unit per 128 rows, and with
    ``split`` > 1 the pieces of the first such group (at most four pieces)
    get ``split`` units each, one per key-range part.  Returns the (q_start,
    q_count, first group, groups, bounds, split word) records."""
    starts, counts, pre = [], [], 0
    for v in sizes:  # clamped extents
        v = max(0, v)
        s0, s1 = min(sq, pre), min(sq, pre + v)
        starts.append(s0)
        counts.append(s1 - s0)
        pre += v
    units, cur = [], []

    def flush():
        lo, ng = cur[-1], len(cur)
        bounds = 0xFFFFFF
        for m in range(1, ng):
            bounds = (bounds & ~(0xFF << (8 * (m - 1)))) | ((starts[lo + m] - starts[lo]) << (8 * (m - 1)))
        units.append((starts[lo], sum(counts[g] for g in cur), lo, ng, bounds, 0))
        cur.clear()

    first_big = True
    for q in range(len(sizes) - 1, -1, -1):
        n = counts[q]
        if n > 128:
            if cur:
                flush()
            pieces = (n + 127) // 128
            parts = split if first_big and split > 1 and pieces <= 4 else 1
            first_big = False
            for i in range(pieces):
                for p in range(parts):
                    word = (i << 16) | (p << 8) | parts if parts > 1 else 0
                    units.append((starts[q] + 128 * i, min(128, n - 128 * i), q, 1, 0xFFFFFF, word))
            continue
        if len(cur) == 4 or sum(counts[g] for g in cur) + n > 128:
            flush()
        if n == 0 and not cur:
            continue
        cur.append(q)
    if cur:
        flush()
    return units


@pytest.mark.parametrize("gq,gk,seed", [(18, 34, 0), (130, 258, 1), (130, 258, 2), (1026, 64, 3)])
def test_attention_plan_units_follow_the_packing_rule(gq, gk, seed):
    """The planner packs query groups into units in parallel (next-start
    pointers and pointer doubling); its unit records must be exactly the ones
    the sequential packing rule gives, for group sizes with empty groups,
    groups above 128 rows and sizes past the sequence end (clamped)."""
    from peco_b200 import _native
    g = torch.Generator().manual_seed(seed)
    h = 2
    kind = torch.randint(0, 4, (h, gq), generator=g)
    sizes = torch.where(kind == 0, torch.zeros((), dtype=torch.long),
                        torch.where(kind == 1, torch.randint(129, 400, (h, gq), generator=g),
                                    torch.randint(1, 90, (h, gq), generator=g)))
    sq = int(sizes.sum(-1).max()) - 50  # the last groups run past the end and are clamped
    ks = torch.randint(0, 40, (1, h, gk), generator=g).int()
    sk = int(ks.sum(-1).max())
    qs = sizes.view(1, h, gq).int()
    dmap = torch.rand((1, h, gq, gk), generator=g) < 0.3
    lib = _native.load()
    meta = [t.to(DEV).contiguous() for t in (dmap, qs, ks)]
    stride = int(lib.peco_attention_workspace_stride(sq, sk, gq, gk))
    ws = torch.zeros(h * stride, dtype=torch.int32, device=DEV)
    st = lib.peco_attention_plan(*[_native.ptr(t) for t in meta], None, None, _native.ptr(ws), h, sq, sk, 128, gq, gk,
                                 _native.stream_of(ws.device, *meta, ws))
    _native.check(st, "peco_attention_plan")
    ws = ws.view(h, stride).cpu()
    off_units = (4 + 2 * (gk + 1) + 3) & ~3  # header, then the key row and block prefixes
    for hh in range(h):
        want = _units_by_rule(sizes[hh].tolist(), sq, split=4 if h <= 4 and sk <= 32768 else 1)  # few heads, short keys
        n = int(ws[hh, 0])
        assert n == len(want)
        rec = ws[hh, off_units:off_units + 8 * n].view(n, 8)
        got = [(int(r[0]), int(r[1]), int(r[4]), int(r[5]), int(r[6]) & 0xFFFFFFFF, int(r[7])) for r in rec]
        assert got == want
