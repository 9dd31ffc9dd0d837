"""Candidate-block mode of the indexer on the B200: block production from dense
scores and candidate-restricted selection, bit for bit against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import c_indexer, finish, host, status
from deepseekrpc_b200 import _native
from deepseekrpc_b200._native import call, ptr, stream_handle
from deepseekrpc_b200.workloads import make_decode_inputs, small_config

pytestmark = pytest.mark.gpu


def c_candidate_blocks(scores, visible, keep):
    rows, stride = scores.shape
    lib = _native.library()
    ws_bytes = lib.dsr_candidate_blocks_workspace_bytes(rows, stride, keep)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((rows, keep), dtype=torch.int32, device="cuda")
    err = status()
    call("dsr_candidate_blocks", ptr(scores), ptr(visible), rows, stride, keep, ptr(out), ptr(ws), ws_bytes,
         ptr(err), stream_handle())
    return out, finish(err)


def c_candidate_select(inp, blocks, k):
    rows, ncand = blocks.shape
    lib = _native.library()
    ws_bytes = lib.dsr_candidate_select_workspace_bytes(rows, ncand)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((rows, k), dtype=torch.int32, device="cuda")
    err = status()
    call("dsr_candidate_select", ptr(inp["idx_q"]), ptr(inp["idx_w"]), inp["idx_q"].shape[1], ptr(inp["index_pool"]),
         inp["index_pool"].shape[0] // 64, ptr(inp["block_table"]), inp["block_table"].shape[1],
         ptr(inp["visible"]), ptr(blocks), ncand, k, ptr(out), ptr(ws), ws_bytes, ptr(err), rows, stream_handle())
    return out, finish(err)


def test_candidate_blocks_from_dense_scores(cuda):
    cfg = small_config("cfg3", batch=3, seed=41)
    inp, lengths = make_decode_inputs(cfg, device="cuda", lengths=[5000, 777, 8203])
    scores, code = c_indexer(inp)
    assert code == 0
    keep = 256
    blocks, code = c_candidate_blocks(scores, inp["visible"], keep)
    assert code == 0
    s = scores.cpu().numpy()
    for r, n in enumerate(lengths):
        assert np.array_equal(blocks[r].cpu().numpy(), oracle.candidate_blocks(s[r, :n], n, keep)), f"row {r}"


def integer_inputs(lengths, seed):
    """Pools and queries of small integers: every score is an exact float."""
    cfg = small_config("cfg3", batch=len(lengths), seed=seed)
    inp, _ = make_decode_inputs(cfg, device="cuda", lengths=lengths)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    inp["index_pool"] = torch.randint(-3, 4, inp["index_pool"].shape, generator=gen, device="cuda").to(torch.bfloat16)
    inp["idx_q"] = torch.randint(-2, 3, inp["idx_q"].shape, generator=gen, device="cuda").float()
    inp["idx_w"] = torch.randint(-2, 3, inp["idx_w"].shape, generator=gen, device="cuda").float()
    return inp


def test_candidate_restricted_selection(cuda):
    lengths, ncand, k = [9000, 4097, 700], 512, 512
    inp = integer_inputs(lengths, 42)
    rng = np.random.default_rng(43)
    blocks = np.full((3, ncand), -1, np.int32)
    for r, n in enumerate(lengths):
        nblk = (n + 7) // 8
        chosen = np.sort(rng.choice(nblk, min(nblk, 300 + 50 * r), replace=False))
        chosen[-1] = nblk - 1  # the newest block, as a producer pins it
        blocks[r, :len(chosen)] = np.unique(chosen)
    out, code = c_candidate_select(inp, torch.from_numpy(blocks).cuda(), k)
    assert code == 0
    h = host(inp)
    for r, n in enumerate(lengths):
        positions = oracle.candidate_positions(blocks[r], n)
        keys = oracle.gather_rows(h["index_pool"], h["block_table"][r], positions)
        scores = oracle.index_scores(h["idx_q"][r:r + 1], keys, h["idx_w"][r:r + 1],
                                     np.arange(len(positions), dtype=np.int32)[None],
                                     np.array([len(positions)], np.int32))[0]
        expected = oracle.tiled_topk(scores, k, positions=positions)
        assert np.array_equal(out[r].cpu().numpy(), expected), f"row {r}"


@pytest.mark.parametrize("bad", [[3, 3], [5, 2], [-1, 4], [10_000], [-1]])
def test_candidate_lists_are_validated(cuda, bad):
    inp = integer_inputs([4096], 44)
    blocks = torch.full((1, 8), -1, dtype=torch.int32)
    blocks[0, :len(bad)] = torch.tensor(bad, dtype=torch.int32)
    out, code = c_candidate_select(inp, blocks.cuda(), 64)
    assert code == 1
    assert bool((out == -1).all())
