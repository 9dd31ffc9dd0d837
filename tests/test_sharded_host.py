"""Sequence-sharding host logic on CPU: shard plans, and the exchange layouts of
a sharded decode step over a real 2-rank gloo process group, checked against the
unsharded oracle (exact top-k, attention with the sink)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from deepseekrpc_b200.sharded import (ShardPlan, all_gather, gathered_lists, gathered_partials,
                                      local_block_table)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("lengths", [(4096,), (1048576,) * 4, (20000, 13000, 1, 64)])
def test_shard_plan_covers_every_position_once(world, lengths):
    plans = [ShardPlan(world, r, lengths) for r in range(world)]
    for b, n in enumerate(lengths):
        owned = []
        for p in plans:
            assert p.id_base % 64 == 0 and p.span % 64 == 0
            vis = p.local_visible()[b]
            owned.extend(range(p.id_base, p.id_base + vis))
        assert owned == list(range(n))
        assert sum(p.owns_tail(b) for p in plans) == 1
        assert sum(p.local_swa_len()[b] for p in plans) == min(128, n)


def test_local_block_table_takes_the_owned_columns():
    table = torch.arange(2 * 10, dtype=torch.int32).view(2, 10)
    plans = [ShardPlan(3, r, (640, 300)) for r in range(3)]  # 10 blocks -> spans of 4 blocks
    parts = [local_block_table(table, p) for p in plans]
    assert parts[0].tolist() == [[0, 1, 2, 3], [10, 11, 12, 13]]
    assert parts[2].tolist() == [[8, 9, -1, -1], [18, 19, -1, -1]]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _local_topk(scores_full, plan, k):
    """What each rank's dsr_indexer_topk_decode returns: the shard's top-k with global ids and scores."""
    batch = scores_full.shape[0]
    ids = np.full((batch, k), -1, np.int32)
    scores = np.full((batch, k), -np.inf, np.float32)
    for b, n in enumerate(plan.local_visible()):
        if n:
            pos = np.arange(plan.id_base, plan.id_base + n)
            sel = oracle.tiled_topk(scores_full[b, plan.id_base:plan.id_base + n], k, positions=pos)
            sel = sel[sel >= 0]
            ids[b, :len(sel)] = sel
            scores[b, :len(sel)] = scores_full[b, sel]
    return scores, ids


def _partial(q, rows, scale):
    """Unnormalised base-2 partial (m, l, o[:512]) of q over rows, no sink (float64)."""
    s = (q.astype(np.float64) @ rows.astype(np.float64).T) * scale * np.log2(np.e)  # [H, n]
    if rows.shape[0] == 0:
        return (np.full(q.shape[0], -np.inf), np.zeros(q.shape[0]), np.zeros((q.shape[0], 512)))
    m = s.max(axis=1)
    p = np.exp2(s - m[:, None])
    return m, p.sum(axis=1), p @ rows[:, :512].astype(np.float64)


def _exchange_worker(rank, world, port, failures):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)  # same draws on every rank
        lengths, k, heads, scale = (9000, 5000), 256, 4, 0.07
        batch, longest = len(lengths), max(lengths)
        scores_full = (np.round(rng.normal(size=(batch, longest)) * 4) / 4).astype(np.float32)  # ties
        kv = rng.normal(size=(batch, longest, 576)).astype(np.float32)
        swa = rng.normal(size=(batch, 128, 576)).astype(np.float32)
        q = rng.normal(size=(batch, heads, 576)).astype(np.float32)
        sink = rng.normal(size=heads).astype(np.float32)
        plan = ShardPlan(world, rank, lengths)

        # step 2: exchange of the local lists, merge to the exact global top-k
        sc, ids = _local_topk(scores_full, plan, k)
        # the send buffer dsr_indexer_topk_decode fills: [scores' bits ; ids]
        send = torch.stack((torch.from_numpy(sc).view(torch.int32), torch.from_numpy(ids)))
        s_all, i_all = gathered_lists(all_gather(send), world)
        assert s_all.shape == (batch, world * k) and i_all.shape == (batch, world * k)
        merged = []
        for b, n in enumerate(lengths):
            row_ids, row_s = i_all[b].numpy(), s_all[b].numpy()
            valid = row_ids >= 0
            assert np.all(np.diff(row_ids[valid]) > 0), "merged row ids must increase"
            got = oracle.tiled_topk(row_s[valid], k, positions=row_ids[valid])
            assert np.array_equal(got, oracle.tiled_topk(scores_full[b, :n], k)), f"row {b}"
            merged.append(got)

        # step 4: exchange of the per-shard partials, combine with the sink once
        o = np.zeros((batch, heads, 512), np.float32)
        m = np.zeros((batch, heads), np.float32)
        l = np.zeros((batch, heads), np.float32)
        swa_len = plan.local_swa_len()
        for b in range(batch):
            sel = merged[b][merged[b] >= 0]
            mine = sel[(sel >= plan.id_base) & (sel < plan.id_base + plan.local_visible()[b])]
            rows = np.concatenate([swa[b, :swa_len[b]], kv[b, mine]])
            mb, lb, ob = _partial(q[b], rows, scale)
            m[b], l[b], o[b] = mb, lb, ob
        # the send buffer dsr_sparse_mla_partial fills: [o | m | l]
        send = torch.cat((torch.from_numpy(o).reshape(-1), torch.from_numpy(m).reshape(-1),
                          torch.from_numpy(l).reshape(-1)))
        po, pm, pl = gathered_partials(all_gather(send), world, batch, heads)
        po, pm, pl = po.double().numpy(), pm.double().numpy(), pl.double().numpy()
        sk = np.tile(sink, batch).astype(np.float64) * np.log2(np.e)  # sink of pair (b, h) at b*H + h
        M = np.maximum(pm.max(axis=0), sk)
        w = np.exp2(pm - M)
        out = (po * w[:, :, None]).sum(axis=0) / ((pl * w).sum(axis=0) + np.exp2(sk - M))[:, None]
        out = out.reshape(batch, heads, 512)
        for b in range(batch):
            sel = merged[b][merged[b] >= 0]
            rows = np.concatenate([swa[b, :min(128, lengths[b])], kv[b, sel]])
            ids = np.arange(len(rows), dtype=np.int32)[None]
            ref = oracle.sparse_attention(q[b:b + 1], rows[:0], rows, ids, sink, scale=scale)[0, :, :512]
            np.testing.assert_allclose(out[b], ref, rtol=2e-5, atol=2e-5)
    except Exception as exc:  # reported to the parent, which fails the test
        failures.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_exchange_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    failures = ctx.SimpleQueue()
    mp.start_processes(_exchange_worker, args=(2, _free_port(), failures), nprocs=2, join=True,
                       start_method="spawn")
    assert failures.empty(), failures.get()
