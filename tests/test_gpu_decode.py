"""Paged decode path on the B200 (indexer -> top-k -> sparse MLA) against the oracle.

Tolerances: index scores within 1e-3 relative, checked two
ways: every key within 1e-3 of sum_h |w_h| |q_h.k| (the magnitude that bounds the
rounding of a signed-weight sum, which can cancel to near zero), and at least
99.9% of the keys within 1e-3 plain relative error; top-k bit-exact given
identical fp32 scores; attention max abs error <= 2e-2 and mean abs error <= 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import (assert_bf16_close, assert_scores, c_decode_step, c_indexer, c_mla, host,
                      oracle_attention, oracle_scores, score_bound)
from deepseekrpc_b200 import _native
from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs, small_config

pytestmark = pytest.mark.gpu
SCORE_RTOL = 1e-3


def check_scores(h, scores, b, min_share=0.999):
    """Within 1e-3 of the bound for every key, and within 1e-3 plain relative error
    for at least `min_share` of the keys (both reported by score_stats)."""
    n = int(h["visible"][b])
    ref = oracle_scores(h, b)
    assert_scores(scores[b, :n], ref, score_bound(h, b), SCORE_RTOL, min_share=min_share,
                  what=f"sequence {b} ({n} keys)")
    return ref


@pytest.mark.parametrize("idx_heads", [64, 32, 16])
def test_indexer_scores_ragged_batch(cuda, idx_heads):
    cfg = small_config("cfg3", batch=4, idx_heads=idx_heads, seed=31)
    inp, lengths = make_decode_inputs(cfg, lengths=[100, 4096, 9000, 70001])
    scores, code = c_indexer(inp)
    assert code == 0
    h = host(inp)
    s = scores.cpu().numpy()
    for b in range(4):
        check_scores(h, s, b)
        assert np.all(np.isnan(s[b, lengths[b]:]))  # nothing written past visible


def test_indexer_fp32_query_uses_hi_lo_split(cuda):
    cfg = small_config("cfg2", context=20000, seed=32)
    inp, _ = make_decode_inputs(cfg)
    inp["idx_q"] = inp["idx_q"] + torch.randn_like(inp["idx_q"]) * 1e-3  # not BF16-representable
    scores, code = c_indexer(inp)
    assert code == 0
    # q = bf16(q) + bf16(q - bf16(q)) carries ~16 of FP32's 24 mantissa bits, so the
    # score error is ~2^-17 of the bound: within 1e-3 of the bound everywhere, but
    # keys whose signed head terms cancel below ~1% of the bound exceed 1e-3 plain
    # relative error (about 2% of N(0,1) keys).  BF16-valued queries (the
    # reference's FP8 query, every BASELINE config) take the exact path above.
    check_scores(host(inp), scores.cpu().numpy(), 0, min_share=0.95)


def test_indexer_flags_bad_visibility_and_blocks(cuda):
    cfg = small_config("cfg2", context=1000, seed=33)
    inp, _ = make_decode_inputs(cfg)
    bad = dict(inp)
    bad["visible"] = inp["visible"] + 5000  # beyond the block table
    _, code = c_indexer(bad)
    assert code == 1
    bad = dict(inp)
    table = inp["block_table"].clone()
    table[0, 3] = 10 ** 6
    bad["block_table"] = table
    _, code = c_indexer(bad)
    assert code == 1


@pytest.mark.parametrize("heads", [64, 16])
def test_sparse_mla_against_oracle(cuda, heads):
    cfg = small_config("cfg2", context=9000, heads=heads, seed=34)
    inp, _ = make_decode_inputs(cfg)
    h = host(inp)
    rng = np.random.default_rng(34)
    topk = np.full((1, 2048), -1, np.int32)
    chosen = np.sort(rng.choice(9000, 1900, replace=False)).astype(np.int32)
    topk[0, :1900] = chosen
    out, code = c_mla(inp, torch.from_numpy(topk).cuda(), cfg.scale)
    assert code == 0
    assert_bf16_close(out.cpu().numpy()[0], oracle_attention(h, 0, topk[0], cfg.scale))


def test_sparse_mla_short_window_and_empty_selection(cuda):
    cfg = small_config("cfg2", context=37, seed=35)
    inp, _ = make_decode_inputs(cfg)
    h = host(inp)
    topk = np.full((1, 2048), -1, np.int32)
    out, code = c_mla(inp, torch.from_numpy(topk).cuda(), cfg.scale)
    assert code == 0
    assert_bf16_close(out.cpu().numpy()[0], oracle_attention(h, 0, topk[0], cfg.scale))
    topk[0, :3] = [0, 36, 40]  # 40 >= visible -> code 1
    _, code = c_mla(inp, torch.from_numpy(topk).cuda(), cfg.scale)
    assert code == 1


def run_step_and_check(cfg, lengths=None):
    inp, lengths = make_decode_inputs(cfg, lengths=lengths)
    out, topk, scores, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    h = host(inp)
    s = scores.cpu().numpy()
    t = topk.cpu().numpy()
    o = out.cpu().numpy()
    for b, n in enumerate(lengths):
        ref_scores = check_scores(h, s, b)
        # top-k: bit-exact against the reference ranking of the same fp32 scores
        assert np.array_equal(t[b], oracle.tiled_topk(s[b, :n], cfg.topk))
        # against the oracle's own scores the sets may differ only inside the rounding band
        ref_topk = oracle.tiled_topk(ref_scores, cfg.topk)
        diff = np.setxor1d(t[b][t[b] >= 0], ref_topk[ref_topk >= 0])
        if len(diff):
            threshold = np.sort(ref_scores)[::-1][min(cfg.topk, n) - 1]
            band = SCORE_RTOL * score_bound(h, b)[diff] + 1e-6
            assert np.all(np.abs(ref_scores[diff] - threshold) <= 2 * band)
        assert_bf16_close(o[b], oracle_attention(h, b, t[b], cfg.scale))
    return inp, lengths


def test_decode_step_config1(cuda):
    run_step_and_check(CONFIGS["cfg1"])


def test_decode_step_config2_full_size(cuda):
    run_step_and_check(CONFIGS["cfg2"])


def test_decode_step_ragged_batch(cuda):
    cfg = small_config("cfg3", batch=5, seed=36)
    run_step_and_check(cfg, lengths=[1, 130, 2048, 9000, 70000])


def test_decode_step_multiwave_batch(cuda):
    # 12 sequences x 17 tiles exceed one wave of CTAs: the persistent MLA kernel
    # walks several (tile, sequence) items per CTA with the next item's loads in flight
    cfg = small_config("cfg3", batch=12, seed=37)
    run_step_and_check(cfg, lengths=[300, 2047, 2048, 2049, 4000, 5100, 6000, 6500, 7000, 8191, 8192, 9000])


@pytest.mark.parametrize("heads", [64, 16])
def test_decode_step_ties_empty_rows_and_short_rows(cuda, heads):
    """The fused selection's paths in one batch: a row whose keys repeat 16 patterns
    (heavy ties, threshold bin within the parallel path), a row of 200,000 keys with
    one repeated pattern (every score equal: the threshold bin overflows and the
    row's first CTA resolves it alone; the lowest ids win), a row shorter than k
    (every key taken), an empty row (all padding) and an ordinary row.  With 64
    heads the attention runs as separate kernels (340 tile units); with 16 heads
    (85 units) inside the indexer launch, where each row's tiles wait for that
    row's ids (rows of at most k keys: the grid barrier; longer rows: the
    finisher's ready flag)."""
    cfg = small_config("cfg3", batch=5, seed=38, heads=heads)
    lengths = [9000, 200000, 1500, 0, 30000]
    inp, _ = make_decode_inputs(cfg, lengths=[max(n, 1) for n in lengths])
    inp["visible"] = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    inp["swa_len"] = torch.clamp(inp["visible"], max=128).to(torch.int32)
    table = inp["block_table"]
    pool = inp["index_pool"]
    for b, patterns in ((0, 16), (1, 1)):
        n = lengths[b]
        pos = torch.arange(n, device="cuda")
        rows = table[b].long()[pos // 64] * 64 + pos % 64
        pool[rows] = pool[rows[pos % patterns]]
    out, topk, scores, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    h = host(inp)
    s, t, o = scores.cpu().numpy(), topk.cpu().numpy(), out.cpu().numpy()
    for b, n in enumerate(lengths):
        assert np.array_equal(t[b], oracle.tiled_topk(s[b, :n], cfg.topk)), f"row {b}: top-k differs"
        assert_bf16_close(o[b], oracle_attention(h, b, t[b], cfg.scale))
    assert np.array_equal(t[1], np.arange(cfg.topk)), "equal scores select the lowest ids"
    assert np.array_equal(t[2][:1500], np.arange(1500)) and np.all(t[2][1500:] == -1)
    assert np.all(t[3] == -1)


@pytest.mark.parametrize("heads", [64, 16])
def test_decode_step_repeated_calls_reuse_the_workspace(cuda, heads):
    """The fused selection leaves its workspace zeroed (counters, histograms, row
    states and ready flags): the same workspace serves three calls in a row with
    the same results as fresh workspaces, with the attention in separate kernels
    (64 heads) and in the indexer launch (16 heads)."""
    cfg = small_config("cfg3", batch=3, seed=39, heads=heads)
    inp, lengths = make_decode_inputs(cfg, lengths=[40000, 2500, 70000])
    b, h, k = 3, cfg.heads, cfg.topk
    lib = _native.library()
    ws_bytes = lib.dsr_decode_workspace_bytes(b, max(lengths), h, k)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    from _helpers import status, finish
    from deepseekrpc_b200._native import call, ptr, stream_handle
    ref_out, ref_topk, _, code = c_decode_step(inp, k, cfg.scale)
    assert code == 0
    for _ in range(3):
        out = torch.empty((b, h, 512), device="cuda")
        topk = torch.empty((b, k), dtype=torch.int32, device="cuda")
        err = status()
        call("dsr_decode_step", ptr(inp["idx_q"]), ptr(inp["idx_w"]), inp["idx_q"].shape[1], ptr(inp["index_pool"]),
             ptr(inp["q"]), ptr(inp["kv_pool"]), h, inp["kv_pool"].shape[0] // 64, ptr(inp["block_table"]),
             inp["block_table"].shape[1], ptr(inp["visible"]), max(lengths), k, ptr(inp["swa"]), ptr(inp["swa_len"]),
             ptr(inp["sink"]), cfg.scale, ptr(out), ptr(topk), None, ptr(ws), ws_bytes, ptr(err), b, stream_handle())
        assert finish(err) == 0
        assert torch.equal(topk, ref_topk) and torch.equal(out, ref_out)
