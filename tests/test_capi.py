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
    # the reference's workspace rule bounds ours
    for sq, gq, gk in ((7006, 130, 258), (119056, 1026, 2050), (64, 64, 64), (1, 1, 1)):
        ours = l.peco_attention_workspace_stride(sq, gq, gk)
        assert ours <= gk + 2 + 3 * ((sq + 15) // 16 + gq)


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
