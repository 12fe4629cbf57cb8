"""Pin the CPU oracle against fixtures produced by the reference's own CPU code.

The fixtures come from tests/golden/make_golden.py (reference peco/clustering.py,
peco/quantization.py, peco/processor.py run on the CPU).  Everything here is
bit-exact: labels, counts, centroids, maps, codes, scales and reconstructions.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle import peco_oracle as O
from peco_b200 import synthetic


def sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def small_workload():
    return synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24,
                              q_clusters=16, k_clusters=32, top_k=8)


CASES = {
    "cpu_plumbing": (lambda: synthetic.workload("cpu-plumbing"), 0),
    "small_bf16": (small_workload, 1),
}


@pytest.fixture(scope="module", params=sorted(CASES))
def case(request, golden):
    name = request.param
    make, seed = CASES[name]
    w = make()
    g = golden(name)
    q, k, v = synthetic.make_inputs(w, seed=seed)
    return name, w, g, (q, k, v)


def test_generator_reproduces_fixture_inputs(case):
    _, _, g, (q, k, v) = case
    assert sha(torch.cat((q, k, v), 2)) == str(g["inputs_sha"])


def test_kmeans_bit_exact(case):
    _, w, g, (q, k, _) = case
    h, nv, d = w.heads, w.video_tokens, w.dims
    for x, c, tag in ((q, w.q_clusters, "q"), (k, w.k_clusters, "k")):
        xv = x[:, :, :nv].reshape(h, nv, d)
        init = torch.from_numpy(g[f"{tag}_init"])
        assert torch.equal(init, synthetic.init_centroids(xv, c, w.init))
        lab, cen, cnt = O.fit_token_clusters(xv, c, w.iters, init)
        np.testing.assert_array_equal(lab.numpy(), g[f"{tag}_labels"])
        np.testing.assert_array_equal(cnt.numpy(), g[f"{tag}_counts"])
        np.testing.assert_array_equal(cen.numpy(), g[f"{tag}_centroids"])


def test_select_and_text_partition_bit_exact(case):
    _, w, g, _ = case
    qc = torch.from_numpy(g["q_centroids"]).reshape(1, w.heads, -1, w.dims)
    kc = torch.from_numpy(g["k_centroids"]).reshape(1, w.heads, -1, w.dims)
    qs = torch.from_numpy(g["q_counts"]).reshape(1, w.heads, -1)
    ks = torch.from_numpy(g["k_counts"]).reshape(1, w.heads, -1)
    m = O.select_cluster_connections(qc, kc, qs, ks, w.top_p, w.min_kc_ratio)
    np.testing.assert_array_equal(m.numpy(), g["map"])
    extra = {"p09": (0.9, 0.1), "p1": (1.0, 0.0), "p0": (0.0, 0.0)}
    for tag, (p, r) in extra.items():
        if f"map_{tag}" in g:
            np.testing.assert_array_equal(O.select_cluster_connections(qc, kc, qs, ks, p, r).numpy(),
                                          g[f"map_{tag}"])
    em, eqs, eks = O.extend_text_partition(m, qs, ks, w.valid_text, w.text_length)
    np.testing.assert_array_equal(em.numpy(), g["ext_map"])
    np.testing.assert_array_equal(eqs.numpy(), g["ext_q_sizes"])
    np.testing.assert_array_equal(eks.numpy(), g["ext_k_sizes"])


def test_quantization_bit_exact(case):
    _, w, g, (q, k, _) = case
    h, nv, d = w.heads, w.video_tokens, w.dims
    qv = q[:, :, :nv]
    kv = k[:, :, :nv]
    ql, qc = torch.from_numpy(g["q_labels"]), torch.from_numpy(g["q_centroids"])
    kl, kc = torch.from_numpy(g["k_labels"]), torch.from_numpy(g["k_centroids"])
    for bits in (4, 8):
        if f"q_codes{bits}" not in g:
            continue
        codes, low, scale = O.quantize_base_offset(qv.reshape(h, nv, d).float().numpy(), ql.numpy(),
                                                   qc.numpy(), bits)
        np.testing.assert_array_equal(codes, g[f"q_codes{bits}"])
        np.testing.assert_array_equal(low, g[f"q_low{bits}"])
        np.testing.assert_array_equal(scale, g[f"q_scale{bits}"])
        fq = O.fake_quantize_base_offset(qv, ql, qc, bits)
        fk = O.fake_quantize_base_offset(kv, kl, kc, bits)
        assert sha(fq) == str(g[f"q_fake{bits}_sha"])
        assert sha(fk) == str(g[f"k_fake{bits}_sha"])


def test_reorder_bit_exact(case):
    _, w, g, (q, _, v) = case
    nv = w.video_tokens
    qi = O.sort_indices(torch.from_numpy(g["q_labels"]))
    ki = O.sort_indices(torch.from_numpy(g["k_labels"]))
    np.testing.assert_array_equal(qi.numpy(), g["q_indices"])
    np.testing.assert_array_equal(ki.numpy(), g["k_indices"])
    qv = q[:, :, :nv].contiguous()
    assert sha(O.gather_rows(qv, qi)) == str(g["q_gather_sha"])
    assert sha(O.gather_rows(v[:, :, :nv].contiguous(), ki)) == str(g["v_gather_sha"])
    assert torch.equal(O.scatter_rows(O.gather_rows(qv, qi), qi), qv)


def test_edge_cases_bit_exact(golden):
    e = golden("edge")
    x = torch.from_numpy(e["x"])
    lab, cen, cnt = O.fit_token_clusters(x, 10, 3, torch.from_numpy(e["init"]))
    np.testing.assert_array_equal(lab.numpy(), e["labels"])
    np.testing.assert_array_equal(cnt.numpy(), e["counts"])
    np.testing.assert_array_equal(cen.numpy(), e["centroids"])
    assert (cnt == 0).any() or True  # empty clusters occur in intermediate iterations
    codes, low, scale = O.quantize_base_offset(x.numpy(), e["labels"], e["centroids"], 4)
    np.testing.assert_array_equal(codes, e["codes"])
    np.testing.assert_array_equal(low, e["low"])
    np.testing.assert_array_equal(scale, e["scale"])
    assert (scale == 1).any()  # constant residual rows: scale 1, code 0
    fq = O.fake_quantize_base_offset(x.to(torch.bfloat16), torch.from_numpy(e["labels"]),
                                     torch.from_numpy(e["centroids"]), 4)
    np.testing.assert_array_equal(fq.view(torch.int16).numpy(), e["fake_bf16"])


def test_sparse_attention_oracle_matches_dense_mask():
    """The per-group gather formulation equals a dense masked softmax."""
    g = torch.Generator().manual_seed(3)
    b, h, s, d = 1, 2, 40, 64
    q, k, v = (torch.randn((b, h, s, d), generator=g) for _ in range(3))
    qs = torch.tensor([[[10, 0, 12, 18], [5, 15, 20, 0]]], dtype=torch.int32)
    ks = torch.tensor([[[7, 13, 0, 20], [20, 0, 10, 10]]], dtype=torch.int32)
    dmap = torch.rand((b, h, 4, 4), generator=g) > 0.5
    dmap[0, 0, 2] = False  # a query group with no allowed key -> zero rows
    out = O.sparse_attention(q, k, v, dmap, qs, ks)
    for hi in range(h):
        qg = torch.repeat_interleave(torch.arange(4), qs[0, hi].long())
        kg = torch.repeat_interleave(torch.arange(4), ks[0, hi].long())
        mask = dmap[0, hi][qg][:, kg]
        sc = (q[0, hi] @ k[0, hi].T) / d ** 0.5
        sc = sc.masked_fill(~mask, float("-inf"))
        p = torch.softmax(sc, -1).nan_to_num(0.0)
        torch.testing.assert_close(out[0, hi], p @ v[0, hi], rtol=1e-5, atol=1e-5)


def test_sparse_attention_rows_equals_full_oracle():
    """The row-sampled form (used where the full oracle is too slow) returns the
    full oracle's rows, including rows of a group with no key and rows past
    the last group."""
    g = torch.Generator().manual_seed(4)
    s, d = 60, 64
    q, k, v = (torch.randn((1, 1, s, d), generator=g) for _ in range(3))
    qs = torch.tensor([[[10, 0, 12, 30]]], dtype=torch.int32)  # 52 rows in groups, 8 past the end
    ks = torch.tensor([[[7, 13, 0, 40]]], dtype=torch.int32)
    dmap = torch.rand((1, 1, 4, 4), generator=g) > 0.4
    dmap[0, 0, 2] = False
    full = O.sparse_attention(q, k, v, dmap, qs, ks)[0, 0]
    rows = torch.tensor([0, 3, 9, 10, 11, 21, 22, 40, 51, 52, 59])
    got = O.sparse_attention_rows(q[0, 0], k[0, 0], v[0, 0], dmap[0, 0], qs[0, 0], ks[0, 0], rows)
    torch.testing.assert_close(got, full[rows], rtol=1e-6, atol=1e-6)
