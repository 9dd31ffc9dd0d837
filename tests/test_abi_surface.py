"""The C-ABI library and the torch extension load and expose the declared surface (CPU)."""
from __future__ import annotations

import re
from pathlib import Path

import pytest

from deepseekrpc_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "dsr_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dsr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.library()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version_is_reference_generation():
    assert _native.library().dsr_abi_version() == 2


def test_torch_extension_keeps_reference_op_names():
    import deepseekrpc_b200
    ext = deepseekrpc_b200.extension()
    for name in ("sparse_attention", "index_scores", "engram_decode", "scatter_slots", "abi_version"):
        assert hasattr(ext, name)
    assert ext.abi_version() == 2
    import deepseekrpc_cuda  # registered alias, as the reference's cuda_ops imports it
    assert deepseekrpc_cuda is ext


@pytest.mark.parametrize("call", [
    # heads beyond 64 are refused before any launch
    lambda n: n.dsr_index_scores(1, 1, 1, 1, 1, 1, 1, 1, 65, 8, 8, None),
    # width beyond 576
    lambda n: n.dsr_sparse_attention(1, 1, 1, 1, 1, 1, 1, 1, 1, 578, 1, 1, 1, 1.0, None),
    # non-finite scale
    lambda n: n.dsr_sparse_attention(1, 1, 1, 1, 1, 1, 1, 1, 1, 512, 1, 1, 1, float("nan"), None),
    # scatter rows beyond 4096
    lambda n: n.dsr_scatter_slots(1, 1, 1, 1, 1, 1, 4097, 512, 8, None),
    # engram rows beyond 1024
    lambda n: n.dsr_engram_decode(1, 1, 1, 1025, None),
    # top-k k beyond 8192
    lambda n: n.dsr_topk_select(1, None, 1, 1, None, 1, 1, 16, 8193, 0, 256, 1 << 20, None),
    # indexer heads not in {16,32,64}
    lambda n: n.dsr_indexer_decode(16, 16, 16, 1, 1, 1, 1, 1, 64, 1, 1, 48, None),
    # null pointers
    lambda n: n.dsr_append_kv_index(None, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, None, 1, 1, None),
    # peer exchange: no buffer table, more than 8 ranks, payload not in 16-byte units
    lambda n: n.dsr_p2p_allgather(16, 64, None, 0, 2, 64, 1, 16, None),
    lambda n: n.dsr_p2p_allgather(16, 64, 16, 0, 9, 64, 1, 16, None),
    lambda n: n.dsr_p2p_allgather(16, 24, 16, 0, 2, 32, 1, 16, None),
])
def test_host_side_validation_refuses_without_touching_a_device(call):
    lib = _native.library()
    assert call(lib) == _native.DSR_EINVAL
    assert _native.last_error()


def test_workspace_queries_are_pure_host_functions():
    lib = _native.library()
    assert lib.dsr_mla_workspace_bytes(1, 64, 2048) >= 17 * 64 * 512 * 4
    assert lib.dsr_decode_workspace_bytes(1, 131072, 64, 2048) >= 131072 * 4
