"""Merge of per-shard ranked lists on the B200 (dsr_topk_merge_lists): the exact
global top-k of the union, bit-exact against the reference's ranking rule
(index_selection.py:9-19) applied to every shard's entries at once."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from deepseekrpc_b200._native import call, ptr, stream_handle, library

pytestmark = pytest.mark.gpu


def shard_lists(rng, world, rows, k, span, *, short=(), ties=False):
    """Per-shard lists as the local top-k emits them: i32[world][2][rows][k], the
    scores' bit patterns then global ids (ascending, -1 padded); shard w owns the
    ids [w * span, (w + 1) * span)."""
    lists = np.full((world, 2, rows, k), -1, np.int32)
    for w in range(world):
        for r in range(rows):
            count = k // 3 if (w, r) in short else k
            ids = np.sort(rng.choice(span, count, replace=False)).astype(np.int32) + w * span
            s = rng.normal(size=count).astype(np.float32)
            if ties:
                s = np.round(s * 2) / 2
                s[rng.random(count) < 0.05] = -0.0
                s[rng.random(count) < 0.05] = 0.0
            s[rng.random(count) < 0.002] = np.nan
            s[rng.random(count) < 0.002] = np.inf
            lists[w, 0, r, :count] = s.view(np.int32)
            lists[w, 1, r, :count] = ids
    return lists


def expected(lists, k):
    world, _, rows, _ = lists.shape
    out = []
    for r in range(rows):
        ids = lists[:, 1, r].reshape(-1)
        scores = lists[:, 0, r].reshape(-1).view(np.float32)
        keep = ids >= 0
        out.append(oracle.tiled_topk(scores[keep], k, positions=ids[keep].astype(np.int64)))
    return np.stack(out)


def merge(lists, k):
    world, _, rows, _ = lists.shape
    lib = library()
    ws_bytes = lib.dsr_topk_merge_workspace_bytes(rows, world, k)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((rows, k), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.from_numpy(lists).cuda()
    call("dsr_topk_merge_lists", ptr(src), world, rows, k, ptr(out), ptr(ws), ws_bytes, ptr(err), stream_handle())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("world,k", [(1, 2048), (2, 2048), (3, 2048), (4, 2048), (8, 2048), (8, 512),
                                     (5, 100), (5, 1999), (7, 2048), (16, 2048), (3, 8192)])
def test_merge_matches_the_ranking_rule(cuda, world, k):
    # world * k up to 8192 takes the one-CTA-per-row merge, up to 16384 a cluster of
    # eight CTAs per row (5 x 1999: runs that straddle shards), above it the staged select
    rng = np.random.default_rng(100 + world * 7 + k)
    lists = shard_lists(rng, world, 4, k, 4 * k, short={(0, 1), (world - 1, 2)})
    assert np.array_equal(merge(lists, k), expected(lists, k))


@pytest.mark.parametrize("world", [2, 8])
def test_merge_with_heavy_ties_and_signed_zeros(cuda, world):
    rng = np.random.default_rng(300 + world)
    lists = shard_lists(rng, world, 3, 2048, 20000, ties=True)
    assert np.array_equal(merge(lists, 2048), expected(lists, 2048))


def test_merge_of_short_lists_takes_every_entry(cuda):
    rng = np.random.default_rng(7)
    k = 2048
    lists = shard_lists(rng, 4, 2, k, 3 * k, short={(w, r) for w in range(4) for r in range(2)})
    lists[1, :, 0] = -1  # an empty shard
    got = merge(lists, k)
    assert np.array_equal(got, expected(lists, k))
    assert (got[0] >= 0).sum() == 3 * (k // 3)
