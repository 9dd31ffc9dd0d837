"""TiledIndexer and cuda_ops mirrors on the B200, against the reference's own
known answers: the constructed-key tiled selection (its fixture) and the
candidate-restriction self-test lists."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from deepseekrpc_b200 import cuda_ops
from deepseekrpc_b200.cuda_ops import ValidationError
from deepseekrpc_b200.index_selection import PagedIndexKeys, TiledIndexer

pytestmark = pytest.mark.gpu


def constructed_pool(golden):
    """The fixture's 1025 constructed keys in a paged pool (blocks in reverse order)."""
    g = golden("tiled_select")
    keys = torch.from_numpy(g["keys_bits"].view(np.int16)).view(torch.bfloat16)
    blocks = (keys.shape[0] + 63) // 64
    pool = torch.zeros((blocks * 64, 128), dtype=torch.bfloat16)
    order = list(range(blocks))[::-1]  # logical block j lives in physical block blocks-1-j
    for j, pb in enumerate(order):
        chunk = keys[j * 64:(j + 1) * 64]
        pool[pb * 64:pb * 64 + len(chunk)] = chunk
    table = torch.tensor([order] * 3, dtype=torch.int32)
    return g, PagedIndexKeys(pool.cuda(), table.cuda())


def test_tiled_selection_matches_the_reference_fixture(cuda, golden):
    g, pool = constructed_pool(golden)
    q, w = torch.from_numpy(g["q"]).cuda(), torch.from_numpy(g["weights"]).cuda()
    selection = TiledIndexer(tile_rows=128).select(pool, q, w, g["visible"].tolist(), produce_candidates=True)
    assert np.array_equal(selection.topk.cpu().numpy(), g["expected"])
    # candidate blocks of the same scores, against the oracle's restatement
    assert selection.candidate_blocks.shape == (3, 2048)
    keys = g["keys_bits"].view(np.uint16)
    keys = oracle.bf16_bits_to_f32(keys)
    for row, n in enumerate(g["visible"].tolist()):
        scores = oracle.index_scores(g["q"][row:row + 1], keys[:n], g["weights"][row:row + 1],
                                     np.arange(n, dtype=np.int32)[None], np.array([n], np.int32))[0]
        assert np.array_equal(selection.candidate_blocks[row].cpu().numpy(), oracle.candidate_blocks(scores, n))


def test_candidate_restriction_matches_the_reference_self_test(cuda, golden):
    g, pool = constructed_pool(golden)
    q, w = torch.from_numpy(g["q"]).cuda(), torch.from_numpy(g["weights"]).cuda()
    lists = [[2, 30, 64], [0, 127, 128], [3, 14, 80]]
    candidates = torch.full((3, 2048), -1, dtype=torch.int32)
    for row in range(3):
        candidates[row, :3] = torch.tensor(lists[row], dtype=torch.int32)
    selected = TiledIndexer(tile_rows=128).select(pool, q, w, [513, 1025, 1025], candidate_blocks=candidates.cuda())
    for row, visible in enumerate([513, 1025, 1025]):
        expected = [p for block in lists[row] for p in range(block * 8, min(block * 8 + 8, visible))]
        assert selected.topk[row].cpu().tolist() == expected + [-1] * (512 - len(expected))


def test_stale_candidates_and_bad_ids_raise_validation_error(cuda, golden):
    g, pool = constructed_pool(golden)
    q, w = torch.from_numpy(g["q"]).cuda(), torch.from_numpy(g["weights"]).cuda()
    candidates = torch.full((3, 2048), -1, dtype=torch.int32)
    candidates[:, :2] = torch.tensor([5, 5], dtype=torch.int32)  # duplicated block
    with pytest.raises(ValidationError):
        TiledIndexer().select(pool, q, w, [513, 1025, 1025], candidate_blocks=candidates.cuda())
    keys = torch.zeros((16, 128), dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([[0, 99]], dtype=torch.int32, device="cuda")  # 99 is past the 16 keys
    with pytest.raises(ValidationError):
        cuda_ops.index_scores(torch.zeros((1, 32, 128), device="cuda"), keys, torch.zeros((1, 32), device="cuda"),
                              ids, torch.tensor([16], dtype=torch.int32, device="cuda"))
