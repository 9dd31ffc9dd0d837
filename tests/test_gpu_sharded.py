"""Sequence-sharded decode on one B200: every shard's kernels run in turn on the
same device (the all-gathers become concatenations in rank order), and the
result must match the unsharded decode step (top-k bit for bit) and the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _helpers import assert_bf16_close, c_decode_step, host, oracle_attention
from deepseekrpc_b200.sharded import ShardPlan, ShardedDecoder, local_block_table
from deepseekrpc_b200.workloads import make_decode_inputs, small_config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_sharded_step_matches_unsharded(cuda, world):
    cfg = small_config("cfg2")
    lengths = [20000, 13000, 700]
    inp, _ = make_decode_inputs(cfg, device="cuda", lengths=lengths)
    k = cfg.topk
    out_ref, topk_ref, _, code = c_decode_step(inp, k, cfg.scale)
    assert code == 0

    shards = []
    for rank in range(world):
        plan = ShardPlan(world, rank, tuple(lengths))
        table = local_block_table(inp["block_table"], plan)
        dec = ShardedDecoder(plan, cfg.heads, cfg.idx_heads, k, cfg.scale, inp["sink"], "cuda")
        shards.append((dec, table, dec.select_local(inp["idx_q"], inp["idx_w"], inp["index_pool"], table)))
    gathered = torch.cat([packed for _, _, packed in shards])  # rank-major, as all_gather_into_tensor
    for dec, _, _ in shards:
        assert torch.equal(dec.merge(gathered), topk_ref), "merged top-k differs from the unsharded step"
    partials = torch.cat([dec.attend_local(inp["q"], inp["kv_pool"], table, inp["swa"])
                          for dec, table, _ in shards])
    out = shards[0][0].combine(partials)
    torch.cuda.synchronize()
    for dec, _, _ in shards:
        assert int(dec.err.item()) == 0
    h = host(inp)
    ids = topk_ref.cpu().numpy()
    for b in range(len(lengths)):
        assert_bf16_close(out[b].cpu().numpy(), oracle_attention(h, b, ids[b], cfg.scale))
    assert (out - out_ref).abs().max().item() < 2e-2
