"""GPU check of peco_recompute_cluster_centers_static, the centroid update
that allocates nothing (its sort scratch is a fixed per-device array).

Called through the C ABI and compared with the allocating entry point
peco_recompute_cluster_centers on the same inputs, twice in a row (the
second call reuses the scratch the first one left behind).  Tolerance:
bit-exact -- both run the same sort and update kernels.  Because a bug in
those shared kernels would pass that comparison, one case is also checked
against the CPU oracle's centroid update, and a problem that fills the fixed
scratch exactly is accepted and correct.
"""

import pytest
import torch

from oracle import peco_oracle as O
from peco_b200 import _native

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _problem(seed, batch, tokens, dims, clusters):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((batch, tokens, dims), generator=g)
    labels = torch.randint(0, clusters, (batch, tokens), generator=g, dtype=torch.int32)
    labels[labels == clusters - 1] = 0  # one empty cluster per row keeps its previous centre
    previous = torch.randn((batch, clusters, dims), generator=g)
    return [t.to(DEV).contiguous() for t in (x, labels, previous)]


def _outputs(batch, clusters, dims):
    return (torch.full((batch, clusters, dims), float("nan"), device=DEV),
            torch.full((batch, clusters), -1, dtype=torch.int32, device=DEV),
            torch.full((batch, clusters, dims), float("nan"), device=DEV))


def _call(fn, x, labels, previous, outs, batch, tokens, dims, clusters):
    sums, counts, means = outs
    stream = _native.stream_of(x.device, x, labels, previous, sums, counts, means)
    P = _native.ptr
    return fn(P(x), P(labels), P(previous), P(sums), P(counts), P(means), batch, tokens, dims, clusters, stream)


@pytest.mark.parametrize("batch,tokens,dims,clusters", [(3, 700, 128, 37), (24, 6750, 128, 256), (2, 513, 64, 16)])
def test_static_update_matches_allocating_update(batch, tokens, dims, clusters):
    lib = _native.load()
    x, labels, previous = _problem(batch * 1000 + tokens, batch, tokens, dims, clusters)
    ref = _outputs(batch, clusters, dims)
    _native.check(_call(lib.peco_recompute_cluster_centers, x, labels, previous, ref, batch, tokens, dims, clusters),
                  "peco_recompute_cluster_centers")
    for _ in range(2):
        got = _outputs(batch, clusters, dims)
        _native.check(_call(lib.peco_recompute_cluster_centers_static, x, labels, previous, got, batch, tokens, dims,
                            clusters), "peco_recompute_cluster_centers_static")
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert _native.device_status(clear=True) == 0
    if batch == 3:
        # independent of the shared kernels: the CPU restatement of the update
        means, counts, sums = O.update_centers(x.cpu(), labels.cpu(), previous.cpu())
        assert torch.equal(got[2].cpu(), means)
        assert torch.equal(got[1].cpu(), counts)
        assert torch.equal(got[0].cpu(), sums)


def test_static_update_accepts_a_problem_that_fills_its_scratch():
    lib = _native.load()
    cap = int(lib.peco_recompute_cluster_centers_static_capacity())
    batch, dims, clusters = 1, 64, 7
    tokens = cap - batch * (clusters + 1)  # batch*tokens + batch*(clusters+1) == cap
    g = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn((batch, tokens, dims), generator=g, device=DEV)
    labels = torch.randint(0, clusters, (batch, tokens), generator=g, device=DEV, dtype=torch.int32)
    previous = torch.randn((batch, clusters, dims), generator=g, device=DEV)
    ref, got = _outputs(batch, clusters, dims), _outputs(batch, clusters, dims)
    _native.check(_call(lib.peco_recompute_cluster_centers, x, labels, previous, ref, batch, tokens, dims, clusters),
                  "peco_recompute_cluster_centers")
    status = _call(lib.peco_recompute_cluster_centers_static, x, labels, previous, got, batch, tokens, dims, clusters)
    assert status == 0
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    assert int(got[1].sum()) == tokens
    assert _native.device_status(clear=True) == 0


def test_static_update_rejects_problems_beyond_its_scratch():
    lib = _native.load()
    cap = int(lib.peco_recompute_cluster_centers_static_capacity())
    assert cap == 1 << 21
    batch, dims, clusters = 2, 64, 8
    tokens = cap // batch  # batch*tokens + batch*(clusters+1) > cap
    x, labels, previous = (torch.empty(0, device=DEV) for _ in range(3))
    outs = (torch.empty(0, device=DEV),) * 3
    launches = lib.peco_launch_count()
    status = _call(lib.peco_recompute_cluster_centers_static, x, labels, previous, outs, batch, tokens, dims,
                   clusters)
    assert status == 20006
    assert b"fixed device scratch" in lib.peco_error_string(status)
    assert lib.peco_launch_count() == launches  # rejected before any launch
