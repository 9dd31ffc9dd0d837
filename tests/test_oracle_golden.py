"""The CPU oracle reproduces the reference's own outputs (golden fixtures) bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle.ops import OracleError


def _bf(bits):
    return oracle.bf16_bits_to_f32(bits)


@pytest.mark.parametrize("name", ["sparse_kat", "sparse_dense"])
def test_sparse_attention_matches_reference_outputs(golden, name):
    g = golden(name)
    actual = oracle.sparse_attention(g["q"], _bf(g["window_bits"]), _bf(g["source_bits"]), g["ids"],
                                     g["sink"], scale=float(g["scale"]))
    assert np.array_equal(actual, g["expected"])


def test_sparse_attention_empty_row_is_zero(golden):
    g = golden("sparse_dense")
    assert np.array_equal(g["expected"][1], np.zeros_like(g["expected"][1]))


@pytest.mark.parametrize("name", ["index_kat", "index_visibility", "index_random"])
def test_index_scores_match_reference_outputs(golden, name):
    g = golden(name)
    actual = oracle.index_scores(g["q"], _bf(g["keys_bits"]), g["weights"], g["ids"], g["visible"])
    assert np.array_equal(actual, g["expected"])


def test_merge_ranked_tie_rule_matches_reference(golden):
    g = golden("merge_ranked")
    values = g["values"]
    for name in "abc":
        scores, ids = np.empty(0, np.float32), np.empty(0, np.int64)
        start = 0
        for count in g[f"pieces_{name}"]:
            scores, ids = oracle.merge_ranked(scores, ids, values[start:start + count],
                                              np.arange(start, start + count), keep=13)
            start += count
        assert np.array_equal(ids, g[f"ids_{name}"])
        assert np.array_equal(scores, g[f"scores_{name}"])
    _, ids = oracle.merge_ranked(np.empty(0, np.float32), np.empty(0, np.int64),
                                 np.array([9., 8., 7., np.inf], np.float32), np.arange(4), keep=2)
    assert ids.tolist() == g["pinned_ids"].tolist() == [3, 0]
    _, ids = oracle.merge_ranked(np.empty(0, np.float32), np.empty(0, np.int64), g["nan_values"],
                                 np.arange(len(g["nan_values"])), keep=8)
    assert ids.tolist() == g["nan_ids"].tolist() == [1, 4, 2, 8, 7, 0, 3, 6]


def test_tiled_topk_ties_match_reference_at_decode_scale(golden):
    g = golden("topk_ties")
    actual = oracle.tiled_topk(g["scores"], int(g["keep"]))
    assert np.array_equal(actual, g["expected"])


def test_tiled_selection_constructed_keys(golden):
    g = golden("tiled_select")
    keys = _bf(g["keys_bits"])
    for row, vis in enumerate(g["visible"]):
        scores = oracle.index_scores(g["q"][row:row + 1], keys[:vis], g["weights"][row:row + 1],
                                     np.arange(vis, dtype=np.int32)[None], np.array([vis], np.int32))[0]
        assert np.array_equal(oracle.tiled_topk(scores, 512, tile_rows=128), g["expected"][row])


def test_engram_decode_matches_reference(golden):
    g = golden("engram")
    bits, code = oracle.engram_decode(g["encoded"])
    assert code == 0
    assert np.array_equal(bits, g["expected_bits"])


def test_engram_nan_encoding_flags_code_2():
    encoded = np.zeros((1, 264), np.uint8)
    encoded[0, 3] = 0x7F  # E4M3 NaN
    bits, code = oracle.engram_decode(encoded)
    assert code == 2 and bits[0, 3] == 0


def test_oracle_refuses_invalid_slot_instead_of_substituting_a_row():
    with pytest.raises(OracleError, match="slot"):
        oracle.sparse_attention(np.ones((1, 1, 8), np.float32), np.ones((1, 8), np.float32),
                                np.ones((1, 8), np.float32), np.array([[2]], np.int32),
                                np.zeros(1, np.float32), scale=1.0)


def test_scatter_oracle_semantics():
    pool = np.zeros((13, 8), np.uint16)
    generations = np.arange(13, dtype=np.int64)
    values = np.arange(24, dtype=np.uint16).reshape(3, 8) + 0x3F80
    code = oracle.scatter_slots(pool, generations, np.array([9, 2, 12]), np.array([9, 2, 12]), values)
    assert code == 0 and np.array_equal(pool[[9, 2, 12]], values)
    stale = oracle.scatter_slots(pool, generations, np.array([9]), np.array([10]), values[:1])
    assert stale == 3
    dup = oracle.scatter_slots(pool, generations, np.array([4, 4]), np.array([4, 4]), values[:2])
    assert dup == 3 and np.array_equal(pool[4], values[0])
    nan_row = values[:1].copy()
    nan_row[0, 2] = 0x7FC0
    before = pool[5].copy()
    assert oracle.scatter_slots(pool, generations, np.array([5]), np.array([5]), nan_row) == 2
    assert pool[5, 2] == before[2] and pool[5, 3] == nan_row[0, 3]


def test_bf16_round_trip_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -2.5, 0.0, -0.0, np.inf], np.float32)
    b = oracle.f32_to_bf16_bits(x)
    back = oracle.bf16_bits_to_f32(b)
    assert back[0] == 1.0 and back[1] == 1.0 and back[2] == np.float32(1.0 + 2 ** -7)
    assert back[3] == -2.5 and np.isinf(back[6])


def test_candidate_restriction_matches_the_reference_known_answer():
    # the reference self-test's candidate lists and visibility (gpu_selftest.py:232-243):
    # a restricted selection scores every position of the listed blocks below visible
    blocks = [[2, 30, 64], [0, 127, 128], [3, 14, 80]]
    for row, visible in enumerate([513, 1025, 1025]):
        listed = np.array(blocks[row] + [-1] * 2045, np.int32)
        expected = [p for b in blocks[row] for p in range(b * 8, min(b * 8 + 8, visible))]
        assert oracle.candidate_positions(listed, visible).tolist() == expected


@pytest.mark.parametrize("listed,visible", [([3, 3], 64), ([5, 2], 64), ([-1, 4], 64), ([8], 64), ([-1], 10)])
def test_candidate_lists_are_validated_like_the_reference(listed, visible):
    with pytest.raises(OracleError):
        oracle.candidate_positions(np.array(listed, np.int32), visible)


def test_candidate_blocks_pin_the_newest_block_and_rank_by_block_max():
    scores = np.array([5, 1, 1, 1, 1, 1, 1, 1,   0, 0, 0, 9, 0, 0, 0, 0,   2, 2, 2, 2, 2, 2, 2, 2,
                       7, 7, -1], np.float32)
    # block maxima 5, 9, 2 and the partial newest block (pinned): keep 2 -> blocks 1 and 3
    assert oracle.candidate_blocks(scores, len(scores), keep=2).tolist() == [1, 3]
    # ties at equal block maxima go to the lower block id
    tied = np.zeros(32, np.float32)
    assert oracle.candidate_blocks(tied, 32, keep=2).tolist() == [0, 3]
