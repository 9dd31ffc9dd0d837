"""Exact top-k on the B200: bit-exact against the reference's streaming merge (TiledIndexer)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import c_topk, dev

pytestmark = pytest.mark.gpu


def expected_rows(scores, lengths, k):
    return np.stack([oracle.tiled_topk(scores[r, :n], k) for r, n in enumerate(lengths)])


def test_topk_tie_fixture_at_decode_scale(cuda, golden):
    g = golden("topk_ties")
    scores = g["scores"][None]
    out, code = c_topk(dev(scores), dev(np.array([scores.shape[1]], np.int32)), int(g["keep"]))
    assert code == 0
    assert np.array_equal(out.cpu().numpy()[0], g["expected"])


def test_topk_ragged_rows_and_short_rows(cuda):
    rng = np.random.default_rng(21)
    lengths = [0, 1, 2047, 2048, 2049, 50000, 131072, 9000]
    stride = 131072
    scores = rng.normal(size=(len(lengths), stride)).astype(np.float32)
    scores[7, :9000] = np.round(scores[7, :9000])  # heavy ties
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), 2048)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, lengths, 2048))


def test_topk_long_rows_stream_through_the_copy_ring(cuda):
    # rows of several chunks per CTA: the bulk-copy ring wraps many times
    rng = np.random.default_rng(22)
    n = 700000
    scores = (np.round(rng.normal(size=(2, n)) * 8) / 8).astype(np.float32)
    out, code = c_topk(dev(scores), dev(np.array([n, 600001], np.int32)), 2048)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, [n, 600001], 2048))


def test_topk_threshold_bin_overflow_ranks_over_the_row(cuda):
    # more than 8192 entries share the threshold bin: all-equal scores, and a row
    # where 20000 entries tie exactly at the threshold value
    rng = np.random.default_rng(25)
    n = 60000
    scores = np.zeros((3, n), np.float32)
    scores[1] = rng.normal(size=n).astype(np.float32)
    scores[1, rng.choice(n, 20000, replace=False)] = 1.5
    scores[1, :100] = 9.0
    scores[2] = -0.0
    scores[2, 5::7] = 0.0
    lengths = [n, n, 50000]
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), 2048)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, lengths, 2048))
    assert out.cpu().numpy()[0].tolist() == list(range(2048))


@pytest.mark.parametrize("k", [1, 13, 512, 4096])
def test_topk_various_k(cuda, k):
    rng = np.random.default_rng(23 + k)
    scores = np.round(rng.normal(size=(3, 20000)) * 2).astype(np.float32)
    lengths = [20000, 7, 15000]
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), k)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, lengths, k))


def test_topk_negative_zero_equals_positive_zero(cuda):
    scores = np.array([[-0.0, 0.0, -0.0, 0.0, -1.0, 1.0]], np.float32)
    out, code = c_topk(dev(scores), dev(np.array([6], np.int32)), 3)
    assert code == 0
    assert out.cpu().numpy().tolist() == [[0, 1, 5]]  # the two lowest ids among the zeros


def test_topk_explicit_ids_skip_padding_and_return_scores(cuda):
    rng = np.random.default_rng(24)
    ranks, k = 4, 2048
    scores = np.full((2, ranks * k), -np.inf, np.float32)
    ids = np.full((2, ranks * k), -1, np.int32)
    for row in range(2):
        for r in range(ranks):
            count = k if r != 2 else 1500
            local = np.sort(rng.choice(65536, count, replace=False)) + r * 65536
            ids[row, r * k:r * k + count] = local
            scores[row, r * k:r * k + count] = np.round(rng.normal(size=count) * 3)
    lengths = np.array([ranks * k] * 2, np.int32)
    out, out_scores, code = c_topk(dev(scores), dev(lengths), k, ids=dev(ids), return_scores=True)
    assert code == 0
    for row in range(2):
        valid = ids[row] >= 0
        expected = oracle.tiled_topk(scores[row][valid], k, positions=ids[row][valid])
        assert np.array_equal(out.cpu().numpy()[row], expected)
        lookup = dict(zip(ids[row][valid].tolist(), scores[row][valid].tolist()))
        assert out_scores.cpu().numpy()[row].tolist() == [lookup[i] for i in expected.tolist()]


def test_topk_id_base_and_length_error(cuda):
    scores = torch.arange(100, dtype=torch.float32, device="cuda")[None]
    out, code = c_topk(scores, torch.tensor([100], dtype=torch.int32, device="cuda"), 4, id_base=1000)
    assert code == 0 and out.tolist() == [[1096, 1097, 1098, 1099]]
    out, code = c_topk(scores, torch.tensor([101], dtype=torch.int32, device="cuda"), 4)
    assert code == 1 and out.tolist() == [[-1, -1, -1, -1]]


def test_topk_each_resolution_path(cuda):
    # rows built so the threshold bin is resolved by each route: a few candidates
    # ranked pairwise, a candidate list ranked digit by digit, candidates beyond the
    # list ranked over the row, whole threshold bin selected, whole digit-1 bin
    # selected; and staged records beyond the last CTA's shared memory (walked from
    # L2) with a short and an overflowing candidate list
    rng = np.random.default_rng(26)
    n, k = 60000, 2048
    scores = (rng.normal(size=(8, n)) * 0.05).astype(np.float32)
    layouts = [
        [],                                              # pairwise ranking (plain normal scores)
        [(1000, 2.0), (3000, 1.0)],                      # 3000 tied in one digit-1 bin
        [(2048, 5.0)],                                   # the threshold bin is exactly k
        [(300, 3.0), (500, 1.125), (1248, 1.0625), (1000, 1.0)],  # cut at a digit-1 bin edge
        [(500, 4.0), (12000, 1.0)],                      # more candidates than the list holds
        [(1500, 2.0), (1000, 1.0)],                      # 1000 candidates: ranked digit by digit
        [(100, 2.0), (20000, 1.0)],                      # 20100 staged, 20000 candidates
        [],                                              # 18000 staged in one digit-0 bin
    ]
    for row, layout in enumerate(layouts):
        pos = rng.permutation(n)
        start = 0
        for count, value in layout:
            scores[row, pos[start:start + count]] = value
            start += count
    scores[0] = rng.normal(size=n).astype(np.float32)
    scores[7, rng.permutation(n)[:18000]] = rng.uniform(1.0, 1.25, 18000).astype(np.float32)
    lengths = [n] * 8
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), k)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, lengths, k))


def test_topk_ranks_nan_above_infinity(cuda):
    # torch's descending sort (the reference's merge_ranked) puts NaN first
    rng = np.random.default_rng(29)
    n = 40000
    scores = rng.normal(size=(2, n)).astype(np.float32)
    scores[0, rng.choice(n, 700, replace=False)] = np.nan
    scores[0, rng.choice(n, 900, replace=False)] = np.inf
    scores[1, rng.choice(n, 3000, replace=False)] = np.nan  # more NaN than k
    scores[1, :50] = -np.inf
    out, code = c_topk(dev(scores), dev(np.array([n, n - 7], np.int32)), 2048)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, [n, n - 7], 2048))


def test_topk_rows_not_16_byte_aligned(cuda):
    # an odd row stride leaves rows off 16-byte boundaries: plain loads, same result
    rng = np.random.default_rng(30)
    stride = 50001
    scores = np.round(rng.normal(size=(5, stride)) * 4).astype(np.float32)
    lengths = [stride, 50000, 3, 33333, 0]
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), 2048)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(scores, lengths, 2048))
    # valid ids increase along a row (the entry point's contract)
    ids = np.stack([np.sort(rng.choice(200000, stride, replace=False)).astype(np.int32) for _ in range(5)])
    ids[:, ::17] = -1
    out, code = c_topk(dev(scores), dev(np.array(lengths, np.int32)), 2048, ids=dev(ids))
    assert code == 0
    for row, m in enumerate(lengths):
        valid = ids[row, :m] >= 0
        expected = oracle.tiled_topk(scores[row, :m][valid], 2048, positions=ids[row, :m][valid])
        assert np.array_equal(out.cpu().numpy()[row], expected)


def test_topk_threshold_in_the_lowest_and_highest_bins(cuda):
    # thresholds at -inf (the lowest populated bin) and among NaN / +inf (the highest)
    n, k = 30000, 2048
    rows = np.zeros((4, n), np.float32)
    rows[0] = -np.inf
    rows[0, :1000] = np.arange(1000, dtype=np.float32)       # k-th largest is -inf
    rows[1] = np.inf
    rows[1, ::3] = np.nan                                     # 10,000 NaN above 20,000 +inf
    rows[2] = -np.inf
    rows[2, 5::7] = np.nan                                    # NaN, then -inf ties
    rows[3] = np.float32(-3.0e38)
    rows[3, 100:2100] = -np.inf                               # the most negative finite score
    lengths = [n] * 4
    out, code = c_topk(dev(rows), dev(np.array(lengths, np.int32)), k)
    assert code == 0
    assert np.array_equal(out.cpu().numpy(), expected_rows(rows, lengths, k))
