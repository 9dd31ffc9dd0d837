"""Parity at the BASELINE geometries that the benchmark times.

- config 5: one 1,048,576-key sequence through dsr_decode_step (the bench times
  four of them, and the same sequence shape on every shard count);
- config 4: the prefill indexer over 266,240 keys with 64 queries sampled across
  the causal range 262,144..266,239, then the per-query top-k;
- config 3: the 32 seeded ragged lengths in [8192, 65536] with the fused append of
  the current token in the loop before the decode step.

Top-k bit-exact against the reference ranking of the GPU's own fp32 scores,
scores within the 1e-3 tolerance of test_gpu_decode (bound and plain relative
share), attention max abs <= 2e-2 and mean abs <= 2e-3 against the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import assert_bf16_close, assert_scores, c_decode_step, c_topk, finish, status
from deepseekrpc_b200._native import call, ptr, stream_handle
from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs, small_config

pytestmark = pytest.mark.gpu


def seq_rows(pool, table_row, positions):
    """Rows of logical positions of one sequence, gathered on the device, as host float32."""
    pos = torch.as_tensor(np.asarray(positions, np.int64), device=pool.device)
    rows = table_row.long()[pos // 64] * 64 + pos % 64
    return pool.index_select(0, rows).float().cpu().numpy()


def check_sequence(inp, b, n, out, topk, scores, scale, k=2048):
    """Scores, top-k and attention of sequence b (n visible keys) against the oracle."""
    table = inp["block_table"][b]
    keys = seq_rows(inp["index_pool"], table, np.arange(n))
    q = inp["idx_q"][b:b + 1].cpu().numpy()
    w = inp["idx_w"][b:b + 1].cpu().numpy()
    ref = oracle.index_scores(q, keys, w, np.arange(n, dtype=np.int32)[None], np.array([n], np.int32))[0]
    bound = (np.abs(w[0])[:, None] * np.abs(q[0].astype(np.float64) @ keys.T.astype(np.float64))).sum(0)
    got = scores[b, :n]
    assert_scores(got, ref, bound, what=f"sequence {b} ({n} keys)")
    assert np.array_equal(topk[b], oracle.tiled_topk(got, k)), f"sequence {b}: top-k differs"
    chosen = topk[b][topk[b] >= 0]
    source = seq_rows(inp["kv_pool"], table, chosen)
    window = inp["swa"][b, :int(inp["swa_len"][b])].float().cpu().numpy()
    sel = np.arange(len(window) + len(source), dtype=np.int32)[None]
    want = oracle.sparse_attention(inp["q"][b:b + 1].cpu().numpy(), window, source, sel,
                                   inp["sink"].cpu().numpy(), scale=scale)[0, :, :512]
    assert_bf16_close(out[b], want)


def test_config5_sequence_through_the_decode_step(cuda):
    cfg = CONFIGS["cfg5"]
    inp, lengths = make_decode_inputs(cfg, device="cuda", gen_device="cuda", lengths=[cfg.context])
    out, topk, scores, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    check_sequence(inp, 0, lengths[0], out.cpu().numpy(), topk.cpu().numpy(), scores.cpu().numpy(), cfg.scale)


def test_config5_batch_of_four_sequences(cuda):
    """The benchmarked config-5 step: four 1,048,576-key sequences in one call (every
    CTA's score range spans about 28,000 positions and some two rows)."""
    cfg = CONFIGS["cfg5"]
    inp, lengths = make_decode_inputs(cfg, device="cuda", gen_device="cuda", lengths=[cfg.context] * 4)
    out, topk, scores, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    t, s = topk.cpu().numpy(), scores.cpu().numpy()
    for b, n in enumerate(lengths):
        assert np.array_equal(t[b], oracle.tiled_topk(s[b, :n], cfg.topk)), f"sequence {b}: top-k differs"
    check_sequence(inp, 3, lengths[3], out.cpu().numpy(), t, s, cfg.scale)


def test_config4_prefill_geometry(cuda):
    cached, queries, k = 262144, 4096, 2048
    context = cached + queries
    cfg = small_config("cfg2", seed=0)
    inp, _ = make_decode_inputs(cfg, device="cuda", gen_device="cuda", lengths=[context])
    pool, table = inp["index_pool"], inp["block_table"][0].contiguous()
    gen = torch.Generator(device="cuda").manual_seed(4)
    q_all = torch.randn((queries, 64, 128), generator=gen, device="cuda").to(torch.bfloat16).float()
    w_all = torch.randn((queries, 64), generator=gen, device="cuda")
    # 64 queries across the causal range: the first, the last and 62 seeded others
    rng = np.random.default_rng(44)
    pick = np.unique(np.concatenate([[0, queries - 1], rng.choice(queries, 62, replace=False)]))[:64]
    pick_t = torch.as_tensor(pick, device="cuda")
    q, w = q_all[pick_t].contiguous(), w_all[pick_t].contiguous()
    visible = (cached + 1 + pick_t).to(torch.int32).contiguous()
    stride = context
    scores = torch.full((len(pick), stride), float("nan"), device="cuda")
    err = status()
    call("dsr_indexer_prefill", ptr(q), ptr(w), ptr(pool), pool.shape[0] // 64, ptr(table), table.shape[0],
         ptr(visible), ptr(scores), stride, ptr(err), len(pick), 64, stream_handle())
    assert finish(err) == 0
    out, code = c_topk(scores, visible, k)
    assert code == 0
    keys = seq_rows(pool, table, np.arange(context))
    hq, hw, s, o = q.cpu().numpy(), w.cpu().numpy(), scores.cpu().numpy(), out.cpu().numpy()
    for t in range(len(pick)):
        n = int(visible[t])
        ref = oracle.index_scores(hq[t:t + 1], keys[:n], hw[t:t + 1], np.arange(n, dtype=np.int32)[None],
                                  np.array([n], np.int32))[0]
        bound = (np.abs(hw[t])[:, None] * np.abs(hq[t].astype(np.float64) @ keys[:n].T.astype(np.float64))).sum(0)
        assert_scores(s[t, :n], ref, bound, what=f"query at position {n - 1}")
        assert np.all(np.isnan(s[t, n:])), "scores past a query's visible keys must stay untouched"
        assert np.array_equal(o[t], oracle.tiled_topk(s[t, :n], k)), f"query at position {n - 1}: top-k differs"


def test_config3_lengths_with_the_append_in_the_loop(cuda):
    cfg = CONFIGS["cfg3"]
    inp, lengths = make_decode_inputs(cfg, device="cuda", gen_device="cuda")
    B = len(lengths)
    rows = inp["kv_pool"].shape[0]
    generations = torch.zeros(rows, dtype=torch.int64, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(9)
    kv_new = torch.randn((B, 576), generator=gen, device="cuda").to(torch.bfloat16)
    ix_new = torch.randn((B, 128), generator=gen, device="cuda").to(torch.bfloat16)
    seq = torch.arange(B, dtype=torch.int32, device="cuda")
    positions = (inp["visible"] - 1).contiguous()  # the current token, published before selection
    expected = torch.zeros(B, dtype=torch.int64, device="cuda")
    err = status()
    call("dsr_append_kv_index", ptr(inp["kv_pool"]), ptr(inp["index_pool"]), ptr(generations), rows // 64,
         ptr(inp["block_table"]), B, inp["block_table"].shape[1], ptr(seq), ptr(positions), ptr(expected),
         ptr(kv_new), ptr(ix_new), ptr(inp["swa"]), ptr(err), B, stream_handle())
    assert finish(err) == 0
    # the appended rows landed: pools, ring row (L-1) % 128, generation 1
    for b, n in enumerate(lengths):
        r = int(inp["block_table"][b, (n - 1) // 64]) * 64 + (n - 1) % 64
        assert torch.equal(inp["kv_pool"][r], kv_new[b]) and torch.equal(inp["index_pool"][r], ix_new[b])
        assert torch.equal(inp["swa"][b, (n - 1) % 128], kv_new[b]) and int(generations[r]) == 1
    out, topk, scores, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    o, t, s = out.cpu().numpy(), topk.cpu().numpy(), scores.cpu().numpy()
    for b, n in enumerate(lengths):
        check_sequence(inp, b, n, o, t, s, cfg.scale)
