"""Host-side mirrors of the reference modules (cuda_ops, index_selection), on CPU:
argument validation, the error type, and merge_ranked against the reference's
own outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from deepseekrpc_b200 import cuda_ops
from deepseekrpc_b200.cuda_ops import ValidationError
from deepseekrpc_b200.index_selection import PagedIndexKeys, TiledIndexer, merge_ranked


def test_merge_ranked_matches_the_reference_outputs(golden):
    g = golden("merge_ranked")
    values = torch.from_numpy(g["values"])
    for name in "abc":
        scores, ids = torch.empty(0), torch.empty(0, dtype=torch.int64)
        start = 0
        for count in g[f"pieces_{name}"].tolist():
            scores, ids = merge_ranked(scores, ids, values[start:start + count],
                                       torch.arange(start, start + count), keep=13)
            start += count
        assert ids.tolist() == g[f"ids_{name}"].tolist()
        assert np.array_equal(scores.numpy(), g[f"scores_{name}"])
    nan_values = torch.from_numpy(g["nan_values"])
    _, ids = merge_ranked(torch.empty(0), torch.empty(0, dtype=torch.int64), nan_values,
                          torch.arange(len(nan_values)), keep=8)
    assert ids.tolist() == g["nan_ids"].tolist()


@pytest.mark.parametrize("kwargs", [dict(tile_rows=12), dict(tile_rows=4), dict(tile_rows=16384), dict(keep=0),
                                    dict(candidate_keep=9000), dict(tile_rows=True)])
def test_tiled_indexer_refuses_bad_parameters(kwargs):
    with pytest.raises(ValidationError):
        TiledIndexer(**kwargs)


def test_selection_refuses_host_tensors_and_mixed_modes():
    pool = PagedIndexKeys(torch.zeros((64, 128), dtype=torch.bfloat16), torch.zeros((1, 1), dtype=torch.int32))
    q, w = torch.zeros((1, 32, 128)), torch.zeros((1, 32))
    with pytest.raises(ValidationError):
        TiledIndexer().select(pool, q, w, [10])  # host tensors: no CPU fallback
    with pytest.raises(ValidationError):
        TiledIndexer().select(pool, q, w, [10], produce_candidates=True,
                              candidate_blocks=torch.zeros((1, 2048), dtype=torch.int32))


def test_cuda_ops_refuses_without_a_device_and_checks_scale():
    with pytest.raises(ValidationError):
        cuda_ops.sparse_attention(None, None, None, None, None, scale=float("nan"))
    if not torch.cuda.is_available():
        cuda_ops.extension.cache_clear()
        with pytest.raises(RuntimeError):
            cuda_ops.extension()
