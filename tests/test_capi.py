"""The C-ABI library builds, loads without a GPU and exports every declared symbol."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "peco_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(peco_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from peco_b200 import build
    path = build.build()
    return ctypes.CDLL(str(path))


def test_header_declares_the_reference_entry_points():
    names = declared_symbols()
    for ref in ("peco_assign_tokens_to_centers", "peco_recompute_cluster_centers", "peco_reorder_token_features",
                "peco_cluster_error_message", "peco_sparse_attention", "peco_attention_error_string"):
        assert ref in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_bindings_cover_the_header():
    from peco_b200 import _native
    assert set(declared_symbols()) <= set(_native._SIGNATURES), set(declared_symbols()) - set(_native._SIGNATURES)


def test_pure_host_functions(lib):
    from peco_b200 import _native
    l = _native.load()
    assert l.peco_library_version() == 1
    assert b"no error" in l.peco_error_string(0)
    assert b"workspace" in l.peco_error_string(20005)
    # plan workspace: header, two cluster prefixes, units (8 ints each; up to
    # 4 x 3 extra units from split key ranges), the key-row map, one int2 entry
    # per (unit, key cluster), the split-piece table and the split parts'
    # partial results (4 pieces x 4 parts x 128 rows x (128 + 2) floats); key
    # blocks: one 8-row block per started 8 rows plus one padding block per
    # cluster at most
    partials = 4 * 4 * 128 * (128 + 2)
    for sq, sk, gq, gk in ((11776, 11776, 130, 258), (119056, 119056, 1026, 2050), (64, 80, 64, 64), (1, 1, 1, 1)):
        units = (sq + 127) // 128 + gq + 4 * 3
        stride = l.peco_attention_workspace_stride(sq, sk, gq, gk)
        least = 4 + 2 * (gk + 1) + 8 * units + sk + 2 * units * gk + 8 + partials + 1
        assert stride % 4 == 0 and stride >= least
        assert stride <= least + 16
        assert l.peco_key_block_rows(sk, gk) == 8 * ((sk + 7) // 8 + gk)
    assert l.peco_attention_workspace_stride(1, 1, 0, 1) == -1


def test_product_path_refuses_cpu_tensors():
    import torch
    from peco_b200 import clustering, quantization, attention_cuda
    x = torch.zeros(2, 16, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        clustering.fit_token_clusters(x.bfloat16(), 4, max_iters=1, tol=0, init_centroids=x[:, :4].float())
    with pytest.raises(RuntimeError, match="CUDA"):
        quantization.fake_quantize_base_offset(x, torch.zeros(2, 16, dtype=torch.int32), x[:, :4], 4)
    q = torch.zeros(1, 2, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        attention_cuda.sparse_attention(q, q, q, torch.ones(1, 2, 1, 1, dtype=torch.bool),
                                        torch.full((1, 2, 1), 16, dtype=torch.int32),
                                        torch.full((1, 2, 1), 16, dtype=torch.int32))
