"""Reference drop-in ops on the B200 against the reference's golden outputs and the oracle.

Tolerances are the reference's own GPU self-test tolerances
(gpu_selftest.py:64,75): sparse attention rtol 5e-5 / atol 3e-6, index scores
rtol 8e-5 / atol 5e-6; scatter and Engram decode are bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import (bf16_from_bits, c_engram, c_index_scores, c_scatter, c_sparse_attention, dev)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["index_kat", "index_visibility", "index_random"])
def test_index_scores_golden(cuda, golden, name):
    g = golden(name)
    out, code = c_index_scores(dev(g["q"]), bf16_from_bits(g["keys_bits"]), dev(g["weights"]),
                               dev(g["ids"]), dev(g["visible"]))
    assert code == 0
    actual = out.cpu().numpy()
    expected = g["expected"]
    assert np.array_equal(np.isneginf(actual), np.isneginf(expected))
    finite = np.isfinite(expected)
    np.testing.assert_allclose(actual[finite], expected[finite], rtol=8e-5, atol=5e-6)


def test_index_scores_widened_bounds_64_heads(cuda):
    rng = np.random.default_rng(12)
    rows, heads, capacity, columns = 3, 64, 30000, 20000
    q = rng.normal(0, .3, (rows, heads, 128)).astype(np.float32)
    keys_bits = oracle.f32_to_bf16_bits(rng.normal(0, .3, (capacity, 128)))
    w = rng.normal(0, .2, (rows, heads)).astype(np.float32)
    ids = rng.integers(-1, capacity, (rows, columns)).astype(np.int32)
    visible = np.array([0, 15000, 30000], np.int32)
    out, code = c_index_scores(dev(q), bf16_from_bits(keys_bits), dev(w), dev(ids), dev(visible))
    assert code == 0
    expected = oracle.index_scores(q, oracle.bf16_bits_to_f32(keys_bits), w, ids, visible)
    actual = out.cpu().numpy()
    assert np.array_equal(np.isneginf(actual), np.isneginf(expected))
    finite = np.isfinite(expected)
    np.testing.assert_allclose(actual[finite], expected[finite], rtol=1e-4, atol=1e-5)


def test_index_scores_error_codes(cuda):
    q = torch.ones((2, 4, 128), device="cuda")
    keys = torch.ones((8, 128), dtype=torch.bfloat16, device="cuda")
    w = torch.ones((2, 4), device="cuda")
    ids = torch.tensor([[0, 8, -1], [1, 2, 3]], dtype=torch.int32, device="cuda")
    out, code = c_index_scores(q, keys, w, ids, torch.tensor([8, 8], dtype=torch.int32, device="cuda"))
    assert code == 1 and torch.isneginf(out[0, 1]) and torch.isneginf(out[0, 2]) and out[1, 0] == 512.0
    out, code = c_index_scores(q[1:], keys, w[1:], ids[1:], torch.tensor([9], dtype=torch.int32, device="cuda"))
    assert code == 1 and bool(torch.isneginf(out).all())
    w_nan = w.clone()
    w_nan[1, 2] = float("nan")
    _, code = c_index_scores(q, keys, w_nan, ids, torch.tensor([8, 8], dtype=torch.int32, device="cuda"))
    assert code in (1, 2)
    _, code = c_index_scores(q[1:], keys, w_nan[1:], ids[1:], torch.tensor([8], dtype=torch.int32, device="cuda"))
    assert code == 2


@pytest.mark.parametrize("name", ["sparse_kat", "sparse_dense"])
def test_sparse_attention_golden(cuda, golden, name):
    g = golden(name)
    out, code = c_sparse_attention(dev(g["q"]), bf16_from_bits(g["window_bits"]),
                                   bf16_from_bits(g["source_bits"]), dev(g["ids"]), dev(g["sink"]),
                                   float(g["scale"]))
    assert code == 0
    np.testing.assert_allclose(out.cpu().numpy(), g["expected"], rtol=5e-5, atol=3e-6)


def test_sparse_attention_widened_576_wide_64_heads(cuda):
    rng = np.random.default_rng(13)
    rows, heads, width, window_rows, source_rows, selected = 4, 64, 576, 128, 5000, 2176
    q = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(rng.normal(0, 1, (rows, heads, width))))
    window_bits = oracle.f32_to_bf16_bits(rng.normal(0, 1, (window_rows, width)))
    source_bits = oracle.f32_to_bf16_bits(rng.normal(0, 1, (source_rows, width)))
    ids = rng.integers(-1, window_rows + source_rows, (rows, selected)).astype(np.int32)
    ids[1, :50] = 7  # duplicates count
    ids[2] = -1      # empty row -> zeros
    sink = rng.normal(0, 1, heads).astype(np.float32)
    scale = 1 / np.sqrt(192)
    out, code = c_sparse_attention(dev(q), bf16_from_bits(window_bits), bf16_from_bits(source_bits), dev(ids),
                                   dev(sink), scale)
    assert code == 0
    expected = oracle.sparse_attention(q, oracle.bf16_bits_to_f32(window_bits),
                                       oracle.bf16_bits_to_f32(source_bits), ids, sink, scale=scale)
    np.testing.assert_allclose(out.cpu().numpy(), expected, rtol=1e-4, atol=1e-5)
    assert np.array_equal(out[2].cpu().numpy(), np.zeros((heads, width), np.float32))


def test_sparse_attention_invalid_id_flags_code_1(cuda):
    q = torch.ones((1, 2, 8), device="cuda")
    rows = torch.ones((3, 8), dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([[0, 6, -1]], dtype=torch.int32, device="cuda")
    _, code = c_sparse_attention(q, rows, rows, ids, torch.zeros(2, device="cuda"), 1.0)
    assert code == 1


def test_scatter_bit_preservation_and_refusals(cuda):
    rng = np.random.default_rng(14)
    pool_bits = np.zeros((13, 512), np.uint16)
    generations = np.arange(13, dtype=np.int64)
    values = oracle.f32_to_bf16_bits(rng.normal(0, .2, (3, 512)))
    pool = bf16_from_bits(pool_bits)
    gens = dev(generations)
    code = c_scatter(pool, gens, dev(np.array([9, 2, 12], np.int32)), dev(np.array([9, 2, 12])),
                     bf16_from_bits(values))
    assert code == 0
    assert np.array_equal(pool.view(torch.int16).cpu().numpy().view(np.uint16)[[9, 2, 12]], values)
    # stale generation, duplicate target, out of bounds, NaN element: compare with the oracle
    cases = [
        (np.array([9], np.int32), np.array([10]), values[:1]),
        (np.array([4, 4], np.int32), np.array([4, 4]), values[:2]),
        (np.array([13], np.int32), np.array([0]), values[:1]),
    ]
    nan_values = values[:1].copy()
    nan_values[0, 5] = 0x7FC0
    cases.append((np.array([6], np.int32), np.array([6]), nan_values))
    for slots, expected, vals in cases:
        ref_pool = pool.view(torch.int16).cpu().numpy().view(np.uint16).copy()
        ref_code = oracle.scatter_slots(ref_pool, generations, slots, expected, vals)
        code = c_scatter(pool, gens, dev(slots), dev(expected), bf16_from_bits(vals))
        assert code == ref_code != 0
        assert np.array_equal(pool.view(torch.int16).cpu().numpy().view(np.uint16), ref_pool)


def test_engram_golden(cuda, golden):
    g = golden("engram")
    out, code = c_engram(dev(g["encoded"]))
    assert code == 0
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), g["expected_bits"])


def test_engram_nan_encoding(cuda):
    encoded = np.zeros((2, 264), np.uint8)
    encoded[1, 9] = 0xFF
    out, code = c_engram(dev(encoded))
    bits, ref_code = oracle.engram_decode(encoded)
    assert code == ref_code == 2
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), bits)


def test_drop_in_module_signatures(cuda, golden):
    """The extension keeps the reference call convention: (value, status) pairs."""
    import deepseekrpc_b200
    ext = deepseekrpc_b200.extension()
    g = golden("sparse_kat")
    out, status = ext.sparse_attention(dev(g["q"]), bf16_from_bits(g["window_bits"]),
                                       bf16_from_bits(g["source_bits"]), dev(g["ids"]), dev(g["sink"]),
                                       float(g["scale"]))
    assert int(status.item()) == 0
    np.testing.assert_allclose(out.cpu().numpy(), g["expected"], rtol=5e-5, atol=3e-6)
    g = golden("index_kat")
    out, status = ext.index_scores(dev(g["q"]), bf16_from_bits(g["keys_bits"]), dev(g["weights"]),
                                   dev(g["ids"]), dev(g["visible"]))
    assert int(status.item()) == 0
    finite = np.isfinite(g["expected"])
    np.testing.assert_allclose(out.cpu().numpy()[finite], g["expected"][finite], rtol=8e-5, atol=5e-6)
    pool = torch.zeros((13, 512), dtype=torch.bfloat16, device="cuda")
    gens = torch.arange(13, dtype=torch.int64, device="cuda")
    slots = torch.tensor([9, 2, 12], dtype=torch.int32, device="cuda")
    values = torch.randn((3, 512), device="cuda").to(torch.bfloat16)
    assert int(ext.scatter_slots(pool, gens, slots, slots.long(), values).item()) == 0
    assert int(ext.scatter_slots(pool, gens, slots, slots.long() + 1, values).item()) == 3
    with pytest.raises(RuntimeError):
        ext.index_scores(dev(g["q"]).double(), bf16_from_bits(g["keys_bits"]), dev(g["weights"]),
                         dev(g["ids"]), dev(g["visible"]))
