"""Generate golden fixtures by running the reference PECO package on the CPU.

Run in a container where the reference source tree is mounted (it does not
travel to GPU machines):

    PECO_REFERENCE=/path/to/PECO python tests/golden/make_golden.py

The reference's CPU branches are the ground truth here: k-means
(peco/clustering.py:66-80), cluster selection (:154-186), stable reorder
(:92-136), Base-Offset quantization (peco/quantization.py:96-150) and the text
partition (peco/processor.py:68-84).  Inputs come from
``peco_b200.synthetic`` with fixed seeds; each fixture stores them (or a hash
of them when large) together with the reference outputs.
"""

from __future__ import annotations

import hashlib
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from peco_b200 import synthetic  # noqa: E402


def _reference():
    root = os.environ.get("PECO_REFERENCE")
    if not root:
        raise SystemExit("set PECO_REFERENCE to the reference source tree")
    sys.path.insert(0, root)
    import peco.clustering as clustering  # noqa: WPS433
    import peco.processor as processor
    import peco.quantization as quantization
    return clustering, quantization, processor


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def run_case(name: str, w: synthetic.Workload, seed: int, store_inputs: bool, extra_maps=()):
    clustering, quantization, processor = _reference()
    torch.manual_seed(1234)
    q, k, v = synthetic.make_inputs(w, seed=seed)
    b, h, s, d = q.shape
    nv = w.video_tokens
    qv, kv, vv = q[:, :, :nv].contiguous(), k[:, :, :nv].contiguous(), v[:, :, :nv].contiguous()
    q0 = synthetic.init_centroids(qv.reshape(h, nv, d), w.q_clusters, w.init)
    k0 = synthetic.init_centroids(kv.reshape(h, nv, d), w.k_clusters, w.init)
    out = {}
    ql, qc, qn, _ = clustering.fit_token_clusters(qv.reshape(h, nv, d), w.q_clusters, max_iters=w.iters,
                                                  tol=0, init_centroids=q0)
    kl, kc, kn, _ = clustering.fit_token_clusters(kv.reshape(h, nv, d), w.k_clusters, max_iters=w.iters,
                                                  tol=0, init_centroids=k0)
    # one assignment step from the initial centres, isolated from the iteration
    ql1, _, _, _ = clustering.fit_token_clusters(qv.reshape(h, nv, d), w.q_clusters, max_iters=1, tol=0,
                                                 init_centroids=q0)
    qs, ks = qn.reshape(b, h, -1), kn.reshape(b, h, -1)
    dmap = clustering.select_cluster_connections(qc.reshape(b, h, -1, d), kc.reshape(b, h, -1, d), qs, ks,
                                                 w.top_p, w.min_kc_ratio)
    out.update(q_labels=ql.numpy(), q_centroids=qc.numpy(), q_counts=qn.numpy(),
               k_labels=kl.numpy(), k_centroids=kc.numpy(), k_counts=kn.numpy(),
               q_labels_iter1=ql1.numpy(), q_init=q0.numpy(), k_init=k0.numpy(), map=dmap.numpy())
    for tag, p, ratio in extra_maps:
        m = clustering.select_cluster_connections(qc.reshape(b, h, -1, d), kc.reshape(b, h, -1, d), qs, ks,
                                                  p, ratio)
        out[f"map_{tag}"] = m.numpy()
    bits_list = (4, 8) if w.bits else (4,)
    for bits in bits_list:
        enc = quantization.quantize_base_offset(qv, ql, qc, bits)
        out[f"q_codes{bits}"] = enc.codes.numpy()
        out[f"q_low{bits}"] = enc.offset_min.numpy()
        out[f"q_scale{bits}"] = enc.scale.numpy()
        fq = quantization.fake_quantize_base_offset(qv, ql, qc, bits)
        fk = quantization.fake_quantize_base_offset(kv, kl, kc, bits)
        if store_inputs:
            out[f"q_fake{bits}"] = fq.view(torch.int16 if fq.element_size() == 2 else torch.int32).numpy()
        out[f"q_fake{bits}_sha"] = np.array(sha(fq))
        out[f"k_fake{bits}_sha"] = np.array(sha(fk))
    qg, qi = clustering.gather_clustered_tokens(qv, ql, dim=2)
    kg, ki = clustering.gather_clustered_tokens(kv, kl, dim=2)
    vg, _ = clustering.gather_clustered_tokens(vv, kl, dim=2, sorted_indices=ki)
    out.update(q_indices=qi.numpy(), k_indices=ki.numpy(), q_gather_sha=np.array(sha(qg)),
               v_gather_sha=np.array(sha(vg)))
    restored = clustering.restore_sequence_order(qg, qi, dim=2)
    assert torch.equal(restored, qv)
    em, eqs, eks = processor.extend_text_partition(dmap, qs, ks, w.valid_text, w.text_length)
    out.update(ext_map=em.numpy(), ext_q_sizes=eqs.numpy(), ext_k_sizes=eks.numpy())
    out["inputs_sha"] = np.array(sha(torch.cat((q, k, v), 2)))
    if store_inputs:
        raw = torch.cat((q, k, v), 0)
        out["inputs"] = raw.view(torch.int16 if raw.element_size() == 2 else torch.int32).numpy()
    out["meta"] = np.array([seed, h, nv, w.text_length, w.valid_text, d, w.q_clusters, w.k_clusters,
                            w.iters, w.top_k, w.bits], dtype=np.int64)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, {k: getattr(v, "shape", None) for k, v in out.items()})


def run_edge_case():
    """Ties, empty clusters and constant residuals (kmeans.cu:32, clustering.py:27-28,
    quantization.py:17-18)."""
    clustering, quantization, _ = _reference()
    g = torch.Generator().manual_seed(7)
    d, n = 64, 96
    base = torch.randn((2, 6, d), generator=g)
    x = base[:, torch.arange(n) % 6] + 0.0  # only 6 distinct tokens per head
    x[:, 40:48] += 0.25 * torch.randn((2, 8, d), generator=g)
    x = x.to(torch.bfloat16).float()
    # 10 clusters > 6 distinct tokens -> some stay empty; duplicated initial
    # centres -> exact distance ties resolved to the lowest id
    init = torch.cat((x[:, :6], x[:, :4]), 1).contiguous()
    lab, cen, cnt, _ = clustering.fit_token_clusters(x, 10, max_iters=3, tol=0, init_centroids=init)
    enc = quantization.quantize_base_offset(x, lab, cen, 4)
    fq = quantization.fake_quantize_base_offset(x.to(torch.bfloat16), lab, cen, 4)
    np.savez_compressed(HERE / "edge.npz", x=x.numpy(), init=init.numpy(), labels=lab.numpy(),
                        centroids=cen.numpy(), counts=cnt.numpy(), codes=enc.codes.numpy(),
                        low=enc.offset_min.numpy(), scale=enc.scale.numpy(),
                        fake_bf16=fq.view(torch.int16).numpy())
    print("edge", lab.shape, cnt.tolist())


def main():
    run_case("cpu_plumbing", synthetic.workload("cpu-plumbing"), seed=0, store_inputs=False,
             extra_maps=(("p09", 0.9, 0.1), ("p1", 1.0, 0.0), ("p0", 0.0, 0.0)))
    small = synthetic.workload("hv480", heads=2, grid=(2, 12, 18), text_length=32, valid_text=24,
                               q_clusters=16, k_clusters=32, top_k=8)
    run_case("small_bf16", small, seed=1, store_inputs=True, extra_maps=(("p09", 0.9, 0.1),))
    run_edge_case()


if __name__ == "__main__":
    main()
