"""Prefill indexer GEMM on the B200: scores of many causal queries against one
paged sequence, checked against the oracle's index_scores row by row, and the
per-query top-k over them bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _helpers import c_topk, finish, status
from deepseekrpc_b200._native import call, ptr, stream_handle
from deepseekrpc_b200.workloads import make_decode_inputs, small_config

pytestmark = pytest.mark.gpu


def c_prefill(q, w, pool, table, visible, stride):
    scores = torch.full((q.shape[0], stride), float("nan"), device="cuda")
    err = status()
    call("dsr_indexer_prefill", ptr(q), ptr(w), ptr(pool), pool.shape[0] // 64, ptr(table), table.shape[0],
         ptr(visible), ptr(scores), stride, ptr(err), q.shape[0], q.shape[1], stream_handle())
    return scores, finish(err)


def sequence(context, seed):
    cfg = small_config("cfg2", seed=seed)
    inp, _ = make_decode_inputs(cfg, device="cuda", lengths=[context])
    return inp["index_pool"], inp["block_table"][0].contiguous()


@pytest.mark.parametrize("heads,exact", [(64, True), (32, False)])
def test_prefill_scores_match_the_oracle(cuda, heads, exact):
    context, queries = 5000, 37
    pool, table = sequence(context, 3)
    gen = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn((queries, heads, 128), generator=gen, device="cuda")
    if exact:
        q = q.to(torch.bfloat16).float()  # BF16-valued queries take the single-product path
    w = torch.randn((queries, heads), generator=gen, device="cuda")
    positions = torch.arange(context - queries, context, dtype=torch.int32, device="cuda")
    visible = positions + 1
    stride = (context + 63) // 64 * 64
    scores, code = c_prefill(q.contiguous(), w.contiguous(), pool, table, visible, stride)
    assert code == 0
    keys = oracle.gather_rows(pool.float().cpu().numpy(), table.cpu().numpy(), np.arange(context))
    hq, hw, s = q.cpu().numpy(), w.cpu().numpy(), scores.cpu().numpy()
    for t in range(queries):
        n = int(visible[t])
        ref = oracle.index_scores(hq[t:t + 1], keys[:n], hw[t:t + 1], np.arange(n, dtype=np.int32)[None],
                                  np.array([n], np.int32))[0]
        bound = (np.abs(hw[t])[:, None] * np.abs(hq[t].astype(np.float64) @ keys[:n].T.astype(np.float64))).sum(0)
        assert np.all(np.abs(s[t, :n] - ref) <= 1e-3 * bound + 1e-6), f"query {t}"
        assert np.all(np.isnan(s[t, n:])), "scores past a query's visible keys must stay untouched"


def test_prefill_topk_rows_are_exact(cuda):
    context, queries, k = 9000, 24, 2048
    pool, table = sequence(context, 4)
    gen = torch.Generator(device="cuda").manual_seed(12)
    q = torch.randn((queries, 64, 128), generator=gen, device="cuda").to(torch.bfloat16).float()
    w = torch.randn((queries, 64), generator=gen, device="cuda")
    visible = torch.arange(context - queries + 1, context + 1, dtype=torch.int32, device="cuda")
    stride = (context + 63) // 64 * 64
    scores, code = c_prefill(q, w, pool, table, visible, stride)
    assert code == 0
    out, code = c_topk(scores, visible, k)
    assert code == 0
    s = scores.cpu().numpy()
    for t in range(queries):
        n = int(visible[t])
        assert np.array_equal(out[t].cpu().numpy(), oracle.tiled_topk(s[t, :n], k)), f"query {t}"


def test_prefill_rejects_visibility_beyond_the_table(cuda):
    pool, table = sequence(1000, 5)
    q = torch.zeros((2, 64, 128), device="cuda")
    w = torch.zeros((2, 64), device="cuda")
    visible = torch.tensor([10, table.shape[0] * 64 + 1], dtype=torch.int32, device="cuda")
    _, code = c_prefill(q, w, pool, table, visible, table.shape[0] * 64 + 64)
    assert code == 1
