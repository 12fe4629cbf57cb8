"""One full PECO attention call through the drop-in processor API vs the oracle.

The call (k-means Q/K -> selection -> Base-Offset quant -> reorder -> sparse
attention -> inverse reorder) is compared with the CPU oracle of
peco/processor.py:115-157 on the same seeded inputs and initial centroids.
Tolerance: cosine >= 0.999 and max |err| <= 2e-2 (bf16 output).
"""

import pytest
import torch

from oracle import peco_oracle as O
from oracle import ref_gpu
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
    return proc


def oracle_call(w, q, k, v, proc_init_q, proc_init_k):
    return O.peco_attention_call(q, k, v, text_length=w.text_length, valid_text=w.valid_text,
                                 num_q_centroids=w.q_clusters, num_k_centroids=w.k_clusters, iters=w.iters,
                                 q_init=proc_init_q, k_init=proc_init_k, top_p=w.top_p,
                                 min_kc_ratio=w.min_kc_ratio, bits=w.bits, return_state=True)


def check(got, ref):
    g, r = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(g).all()
    err = (g - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(g.flatten(), r.flatten(), dim=0).item()
    assert err <= 2e-2 and cos >= 0.999, f"max err {err:.3g}, cosine {cos:.6f}"


@pytest.mark.parametrize("bits", [4, 0])
def test_small_call_matches_oracle(bits):
    w = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24, q_clusters=16,
                           k_clusters=32, top_k=8, bits=bits)
    q, k, v = synthetic.make_inputs(w, seed=1)
    proc = make_processor(w, q, k)
    qi, ki = proc.q_centroids.cpu(), proc.k_centroids.cpu()
    out = proc.attention(q.to(DEV), k.to(DEV), v.to(DEV))
    ref, state = oracle_call(w, q, k, v, qi, ki)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert torch.equal(proc.q_centroids.cpu(), state["q_centroids"])
    assert torch.equal(proc.k_centroids.cpu(), state["k_centroids"])
    check(out, ref)


def test_headline_call_two_heads_matches_oracle_and_reference_gpu():
    w = synthetic.workload("hv480")
    q, k, v = synthetic.make_inputs(w, seed=0, heads=2)
    proc = make_processor(w, q, k)
    qi, ki = proc.q_centroids.cpu(), proc.k_centroids.cpu()
    out = proc.attention(q.to(DEV), k.to(DEV), v.to(DEV))
    ref, state = oracle_call(w, q, k, v, qi, ki)
    check(out, ref)
    if ref_gpu.available():
        rg = ref_gpu.peco_attention_call(q.to(DEV), k.to(DEV), v.to(DEV), text_length=w.text_length,
                                         valid_text=w.valid_text, num_q_centroids=w.q_clusters,
                                         num_k_centroids=w.k_clusters, iters=w.iters, q_init=qi.to(DEV),
                                         k_init=ki.to(DEV), top_p=w.top_p, min_kc_ratio=w.min_kc_ratio, bits=w.bits)
        check(rg, ref)


def test_config1_fp32_plumbing_through_fp32_path():
    """configs[0] is fp32: the processor clusters through the drop-in fp32 entry
    points; the attention itself needs 16-bit inputs, so compare the clustering."""
    from peco_b200 import clustering
    w = synthetic.workload("cpu-plumbing")
    q, _, _ = synthetic.make_inputs(w, seed=0)
    nv = w.video_tokens
    x = q[:, :, :nv].reshape(2, nv, 128).contiguous()
    init = synthetic.init_centroids(x, w.q_clusters, "first")
    lab, cen, cnt, _ = clustering.fit_token_clusters(x.to(DEV), w.q_clusters, max_iters=w.iters, tol=0,
                                                     init_centroids=init.to(DEV))
    rl, rc, rn = O.fit_token_clusters(x, w.q_clusters, w.iters, init)
    assert (lab.cpu() != rl).float().mean() <= 1e-3


def test_warmup_then_sparse_state_machine():
    """Warmup steps run dense attention and seed the centroids; the next step reuses them."""
    from peco_b200.processor import InferenceContext, PecoAttention, PecoConfig
    w = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=32, q_clusters=16,
                           k_clusters=32, top_k=8)
    q, k, v = (t.to(DEV) for t in synthetic.make_inputs(w, seed=2))
    cfg = PecoConfig(num_q_centroids=16, num_k_centroids=32, top_p=0.9, min_kc_ratio=0.1, kmeans_iter_init=4,
                     kmeans_iter_step=2, warmup_steps=1)
    ctx = InferenceContext(step=0, text_length=32, valid_text_length=32)
    proc = PecoAttention(0, cfg, ctx)
    dense = proc.attention(q, k, v)
    ref_dense = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())
    assert (dense.float() - ref_dense).abs().max() < 2e-2
    assert proc.q_centroids is not None and proc.q_centroids.shape == (2, 16, 128)
    ctx.step = 1
    cached = proc.q_centroids.clone()
    out = proc.attention(q, k, v)
    assert torch.isfinite(out.float()).all()
    # the step call refines the cached centres with kmeans_iter_step iterations
    nv = w.video_tokens
    _, ref_centers, _ = O.fit_token_clusters(q[0, :, :nv].float().cpu(), 16, 2, cached.cpu())
    assert (proc.q_centroids.cpu() - ref_centers).abs().max() < 1e-2
    proc.reset()
    assert proc.q_centroids is None


@pytest.mark.parametrize("dtype,dims,valid", [(torch.bfloat16, 128, 700), (torch.float16, 64, 1000),
                                              (torch.bfloat16, 128, 1000), (torch.bfloat16, 64, 0)])
def test_dense_warmup_attention_on_tc_kernel(dtype, dims, valid):
    """dense_attention (peco/processor.py:52-65) on the tcgen05 kernel vs an fp32
    torch restatement: softmax(QK^T/sqrt(D))V within [0,valid) and [valid,S)."""
    from peco_b200.processor import dense_attention
    g = torch.Generator().manual_seed(5)
    s = 1000
    q, k, v = (torch.randn((1, 3, s, dims), generator=g).to(dtype) for _ in range(3))
    got = dense_attention(q.to(DEV), k.to(DEV), v.to(DEV), valid)
    ref = torch.empty((1, 3, s, dims))
    for a, b in ((0, valid), (valid, s)):
        if a < b:
            ref[:, :, a:b] = torch.nn.functional.scaled_dot_product_attention(
                q[:, :, a:b].float(), k[:, :, a:b].float(), v[:, :, a:b].float())
    check(got, ref)


def test_graph_replay_matches_eager_calls():
    """Three steady-state calls replayed from one captured CUDA graph equal three
    eager calls bit for bit (outputs and the chained centroids)."""
    from peco_b200.graph import PecoCallGraph
    w = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24, q_clusters=16,
                           k_clusters=32, top_k=8, iters=2)
    inputs = [tuple(t.to(DEV) for t in synthetic.make_inputs(w, seed=10 + i)) for i in range(3)]
    eager = make_processor(w, *[t.cpu() for t in inputs[0][:2]])
    graphed = make_processor(w, *[t.cpu() for t in inputs[0][:2]])
    assert torch.equal(eager.q_centroids, graphed.q_centroids)
    g = PecoCallGraph(graphed, *inputs[0])
    for q, k, v in inputs:
        want = eager.attention(q, k, v)
        got = g(q, k, v)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert torch.equal(graphed.q_centroids, eager.q_centroids)
        assert torch.equal(graphed.k_centroids, eager.k_centroids)
