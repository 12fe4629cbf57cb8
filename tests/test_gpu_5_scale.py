"""Parity at the sizes the benchmark times.

* The headline call with all 24 HV-480 heads in one launch sequence (the
  attention kernel claims units across every head, the k-means runs all 144
  centroid groups): heads 0, 11 and 23 are checked against the oracle.
* The long-video configuration (119,056 tokens, 1024 query / 2048 key
  clusters, top-64): the chunked-centroid k-means, the per-row selection
  kernel for more than 256 key clusters, the quantised packed rows and the
  attention over 1026 x 2050 groups, on two heads, with head 1 checked stage by
  stage.  The oracle evaluates the attention only at ~2,000 sampled rows
  (each through a gather of its selected key runs), which keeps the CPU side
  to seconds.

Tolerances: labels equal to the oracle's fp32 fit except at distance ties
(<= 0.1% of tokens), centres bit-equal when the labels are; selection maps
equal except at probability ties; packed quantised rows and permutations
bit-exact; attention cosine >= 0.999 and max |err| <= 2e-2.
"""

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


def make_processor(w, q, k):
    from peco_b200.processor import InferenceContext, PecoAttention, PecoConfig
    cfg = PecoConfig(num_q_centroids=w.q_clusters, num_k_centroids=w.k_clusters, top_p=w.top_p,
                     min_kc_ratio=w.min_kc_ratio, kmeans_iter_init=w.iters, kmeans_iter_step=w.iters,
                     warmup_steps=0, base_offset_bits=w.bits)
    ctx = InferenceContext(step=1, text_length=w.text_length, valid_text_length=w.valid_text)
    proc = PecoAttention(0, cfg, ctx)
    nv, d, h = w.video_tokens, w.dims, q.shape[1]
    proc.q_centroids = synthetic.init_centroids(q[:, :, :nv].reshape(h, nv, d), w.q_clusters, w.init).to(DEV)
    proc.k_centroids = synthetic.init_centroids(k[:, :, :nv].reshape(h, nv, d), w.k_clusters, w.init).to(DEV)
    proc.keep_partition = True
    return proc


def check(got, ref):
    g, r = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(g).all()
    err = (g - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(g.flatten(), r.flatten(), dim=0).item()
    assert err <= 2e-2 and cos >= 0.999, f"max err {err:.3g}, cosine {cos:.6f}"


def check_fit(got_labels, got_centers, x, clusters, iters, init):
    rl, rc, _ = O.fit_token_clusters(x, clusters, iters, init)
    mism = (got_labels != rl).float().mean().item()
    assert mism <= 1e-3, f"label mismatch {mism:.4%}"
    if mism == 0:
        assert torch.equal(got_centers, rc)
    return mism


def test_full_headline_call_sampled_heads_match_oracle():
    """All 24 heads of the benchmark's own input (seed 1000) in one call."""
    w = synthetic.workload("hv480")
    q, k, v = synthetic.make_inputs(w, seed=1000)
    proc = make_processor(w, q, k)
    qi, ki = proc.q_centroids.cpu(), proc.k_centroids.cpu()
    out = proc.attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    torch.cuda.synchronize()
    heads = [0, 11, 23]
    ref, state = O.peco_attention_call(q[:, heads], k[:, heads], v[:, heads], text_length=w.text_length,
                                       valid_text=w.valid_text, num_q_centroids=w.q_clusters,
                                       num_k_centroids=w.k_clusters, iters=w.iters, q_init=qi[heads],
                                       k_init=ki[heads], top_p=w.top_p, min_kc_ratio=w.min_kc_ratio, bits=w.bits,
                                       return_state=True)
    check(out[:, heads], ref)
    st = proc.last_state
    for name, cen in (("q", proc.q_centroids), ("k", proc.k_centroids)):
        got = st[f"{name}_labels"].cpu()[heads]
        mism = (got != state[f"{name}_labels"]).float().mean().item()
        assert mism <= 1e-3, f"{name} labels differ on {mism:.4%}"
        if mism == 0:
            assert torch.equal(cen.cpu()[heads], state[f"{name}_centroids"])
    emap = proc.last_partition[0].cpu()[0, heads, :w.q_clusters, :w.k_clusters]
    if torch.equal(st["q_labels"].cpu()[heads], state["q_labels"]) and \
            torch.equal(st["k_labels"].cpu()[heads], state["k_labels"]):
        assert torch.equal(emap, state["map"][0])


def test_long_config_two_heads_stage_by_stage():
    w = synthetic.workload("hv-long", heads=2)
    nv, d, s = w.video_tokens, w.dims, w.seq
    cq, ck = w.q_clusters, w.k_clusters
    q, k, v = synthetic.make_inputs(w, seed=11)
    proc = make_processor(w, q, k)
    qi, ki = proc.q_centroids.cpu(), proc.k_centroids.cpu()
    out = proc.attention(q.to(DEV), k.to(DEV), v.to(DEV)).cpu()
    torch.cuda.synchronize()
    st = proc.last_state
    emap, eqs, eks = (t.cpu() for t in proc.last_partition)
    assert emap.shape == (1, 2, cq + 2, ck + 2)
    h = 1
    qv, kv = q[0, h, :nv], k[0, h, :nv]
    q_lab, k_lab = st["q_labels"][h].cpu(), st["k_labels"][h].cpu()
    qc, kc = proc.q_centroids[h].cpu(), proc.k_centroids[h].cpu()
    q_cnt, k_cnt = st["q_counts"][h].cpu(), st["k_counts"][h].cpu()

    # k-means: the chunked-centroid assign (C > 256) against the fp32 Lloyd fit
    check_fit(q_lab[None], qc[None], qv[None], cq, w.iters, qi[h:h + 1])
    check_fit(k_lab[None], kc[None], kv[None], ck, w.iters, ki[h:h + 1])
    q_perm, k_perm = st["q_perm"][h].cpu(), st["k_perm"][h].cpu()
    assert torch.equal(q_perm, O.sort_indices(q_lab[None])[0])
    assert torch.equal(k_perm, O.sort_indices(k_lab[None])[0])
    assert torch.equal(q_cnt, torch.bincount(q_lab.long(), minlength=cq).int())
    assert torch.equal(k_cnt, torch.bincount(k_lab.long(), minlength=ck).int())

    # selection: the per-row kernel for more than 256 key clusters, on the call's own centres and counts
    ref_map = O.select_cluster_connections(qc[None, None], kc[None, None], q_cnt[None, None], k_cnt[None, None],
                                           w.top_p, w.min_kc_ratio)
    got_map = emap[:, h:h + 1, :cq, :ck]
    diff = (got_map != ref_map).nonzero().tolist()
    if diff:
        probs = O.cluster_probabilities(qc[None, None], kc[None, None], k_cnt[None, None])
        for (_, _, i, j) in diff:
            row = probs[0, 0, i]
            assert ((row - row[j]).abs() <= 1e-5 * row[j].abs().clamp_min(1e-30)).sum() > 1, (i, j)
    assert len(diff) <= 1e-3 * cq * ck
    assert int(got_map[0, 0].sum(-1).max()) <= w.top_k
    ext, eq_ref, ek_ref = O.extend_text_partition(got_map, q_cnt[None, None], k_cnt[None, None], w.valid_text,
                                                  w.text_length)
    assert torch.equal(emap[:, h:h + 1], ext)
    assert torch.equal(eqs[:, h:h + 1], eq_ref) and torch.equal(eks[:, h:h + 1], ek_ref)

    # Base-Offset codes and the reorder: the packed quantised Q rows bit-exact
    q_hat = O.fake_quantize_base_offset(qv[None], q_lab[None], qc[None], w.bits)[0]
    k_hat = O.fake_quantize_base_offset(kv[None], k_lab[None], kc[None], w.bits)[0]
    packed_q = torch.cat((q_hat[q_perm.long()], q[0, h, nv:]), 0)
    assert torch.equal(st["q_packed"][0, h].cpu(), packed_q)

    # attention at sampled rows: video rows from every part of the sequence plus text rows
    g = torch.Generator().manual_seed(3)
    rows = torch.cat((torch.randperm(nv, generator=g)[:1900], torch.arange(nv, s)[::3])).sort().values
    packed_k = torch.cat((k_hat[k_perm.long()], k[0, h, nv:]), 0)
    packed_v = torch.cat((v[0, h, :nv][k_perm.long()], v[0, h, nv:]), 0)
    ref_rows = O.sparse_attention_rows(packed_q, packed_k, packed_v, emap[0, h], eqs[0, h], eks[0, h], rows)
    orig = torch.where(rows < nv, q_perm.long()[rows.clamp_max(nv - 1)], rows)
    check(out[0, h, orig], ref_rows)
