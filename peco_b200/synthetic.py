"""Seeded synthetic PECO attention workloads (the benchmark configurations).

The reference measures on real HunyuanVideo activations, which need model
weights and a network; these generators stand in for them with the shapes,
sizes and value distributions of the benchmark configurations:

* video Q and K are Gaussian mixtures (centres ~ N(0,1), per-token noise
  N(0, 0.3^2)), drawn independently for Q and K and for every head;
* ``mixture="iid"``: each token picks one of ``n_centres`` centres uniformly
  (config 1);
* ``mixture="blocks"``: the centre index is a coarse block map of the
  (frames, height, width) latent grid, so it varies smoothly in space and time
  (configs 2-4);
* text Q/K and all of V are N(0, 1).

Centroid initialisation: ``init="first"`` takes the first k video tokens
(config 1 as specified).  For the raster-ordered block mixtures the first k
tokens all lie in the first few blocks, so configs 2-4 take k tokens at a
fixed stride ``N // k`` instead (``init="strided"``), the same rule applied to
a view of the grid that visits every block.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    heads: int
    grid: tuple  # latent (frames, height, width); video tokens = product
    text_length: int
    valid_text: int
    dims: int
    q_clusters: int
    k_clusters: int
    iters: int
    top_k: int
    bits: int
    dtype: torch.dtype
    mixture: str = "blocks"
    n_centres: int = 32
    block: tuple = (1, 6, 9)
    init: str = "strided"
    noise: float = 0.3

    @property
    def video_tokens(self) -> int:
        t, h, w = self.grid
        return t * h * w

    @property
    def seq(self) -> int:
        return self.video_tokens + self.text_length

    @property
    def top_p(self) -> float:
        """Top-k expressed through the reference's knobs: a vanishing mass
        threshold keeps only the first sorted cluster, ``min_kc_ratio``
        forces exactly k (peco/clustering.py:173-181)."""
        return 1e-9

    @property
    def min_kc_ratio(self) -> float:
        return self.top_k / self.k_clusters


CONFIGS = {
    # CPU plumbing case
    "cpu-plumbing": Workload("cpu-plumbing", heads=2, grid=(1, 30, 45), text_length=64, valid_text=64,
                             dims=128, q_clusters=32, k_clusters=64, iters=3, top_k=16, bits=4,
                             dtype=torch.float32, mixture="iid", n_centres=32, init="first"),
    # HunyuanVideo 480x720x17 attention layer (the headline workload)
    "hv480": Workload("hv480", heads=24, grid=(5, 30, 45), text_length=256, valid_text=256,
                      dims=128, q_clusters=128, k_clusters=256, iters=5, top_k=32, bits=4,
                      dtype=torch.bfloat16),
    # configs[1]'s shape with Base-Offset PE off (top-k sweeps via replace())
    "hv480-nopq": Workload("hv480-nopq", heads=24, grid=(5, 30, 45), text_length=256, valid_text=256,
                           dims=128, q_clusters=128, k_clusters=256, iters=5, top_k=32, bits=0,
                           dtype=torch.bfloat16),
    # long video 720x1280x129
    "hv-long": Workload("hv-long", heads=24, grid=(33, 45, 80), text_length=256, valid_text=256,
                        dims=128, q_clusters=1024, k_clusters=2048, iters=5, top_k=64, bits=4,
                        dtype=torch.bfloat16),
}


def workload(name: str, **overrides) -> Workload:
    return replace(CONFIGS[name], **overrides)


def _block_ids(w: Workload) -> tuple:
    t, h, wd = w.grid
    bt, bh, bw = w.block
    nt, nh, nw = -(-t // bt), -(-h // bh), -(-wd // bw)
    ti = torch.arange(t).view(t, 1, 1) // bt
    hi = torch.arange(h).view(1, h, 1) // bh
    wi = torch.arange(wd).view(1, 1, wd) // bw
    ids = (ti * nh + hi) * nw + wi
    return ids.reshape(-1), nt * nh * nw


def _mixture(w: Workload, gen: torch.Generator, heads: int) -> torch.Tensor:
    n, d = w.video_tokens, w.dims
    dev = gen.device
    if w.mixture == "iid":
        centres = torch.randn((heads, w.n_centres, d), generator=gen, device=dev)
        comp = torch.randint(w.n_centres, (heads, n), generator=gen, device=dev)
    else:
        ids, nb = _block_ids(w)
        centres = torch.randn((heads, nb, d), generator=gen, device=dev)
        comp = ids.to(dev).unsqueeze(0).expand(heads, -1)
    base = centres.gather(1, comp.unsqueeze(-1).expand(-1, -1, d))
    return base + w.noise * torch.randn((heads, n, d), generator=gen, device=dev)


def make_inputs(w: Workload, seed: int = 0, heads: int | None = None, device="cpu", generate_on=None):
    """Return q, k, v [1,H,S,D] in ``w.dtype`` (video tokens first, then text).

    Generated on the CPU with a seeded torch.Generator so every machine gets
    the same bits, then moved to ``device``.  ``generate_on="cuda"`` draws the
    same distributions with a CUDA generator instead (fast for the 118k-token
    config; the bits then differ from the CPU stream).
    """
    heads = w.heads if heads is None else heads
    gen = torch.Generator(device=generate_on or "cpu").manual_seed(seed)
    t, d = w.text_length, w.dims
    qv = _mixture(w, gen, heads)
    kv = _mixture(w, gen, heads)
    dev = gen.device
    qt = torch.randn((heads, t, d), generator=gen, device=dev)
    kt = torch.randn((heads, t, d), generator=gen, device=dev)
    v = torch.randn((heads, w.seq, d), generator=gen, device=dev)
    q = torch.cat((qv, qt), 1).unsqueeze(0).to(w.dtype)
    k = torch.cat((kv, kt), 1).unsqueeze(0).to(w.dtype)
    v = v.unsqueeze(0).to(w.dtype)
    return q.to(device), k.to(device), v.to(device)


def init_centroids(x_video: torch.Tensor, k: int, rule: str) -> torch.Tensor:
    """fp32 [BH,k,D] initial centres from video tokens [BH,N,D]."""
    n = x_video.shape[1]
    if rule == "first":
        sel = x_video[:, :k]
    else:
        stride = max(1, n // k)
        sel = x_video[:, ::stride][:, :k]
    return sel.float().contiguous()
