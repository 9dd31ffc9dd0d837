"""Few eager decode steps through the C ABI, for profiler captures.

    python -m deepseekrpc_b200.profile_step [--config cfg2] [--steps 4]

Runs `steps` decode steps (indexer -> top-k -> sparse MLA -> LSE combine, four
kernel launches each) of one BASELINE config on cuda:0 without CUDA graphs, so
that a profiler sees each kernel launch on its own, then checks the device
status.  Inputs are drawn on the GPU (seeded) and stay resident; one pool
replica, so a profiler's cache flush between replays makes each captured launch
read its pools from DRAM.
"""
from __future__ import annotations

import argparse
import sys

import torch

from deepseekrpc_b200 import _native
from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    parser.add_argument("--steps", type=int, default=4)
    parser.add_argument("--prefill", type=int, nargs=2, metavar=("QUERIES", "CONTEXT"),
                        help="instead: the prefill indexer GEMM, QUERIES causal queries ending at CONTEXT keys")
    parser.add_argument("--topk-rows", type=int, nargs=2, metavar=("ROWS", "CONTEXT"),
                        help="instead: the exact top-2048 (histogram pass + selection) of ROWS causal rows of "
                             "scores ending at CONTEXT keys, as in one of config 4's launches")
    args = parser.parse_args(argv)
    if args.prefill:
        return prefill(*args.prefill, args.steps)
    if args.topk_rows:
        return topk_rows(*args.topk_rows, args.steps)
    cfg = CONFIGS[args.config]
    torch.cuda.set_device(0)
    inp, lengths = make_decode_inputs(cfg, device="cuda:0", gen_device="cuda")
    lib = _native.library()
    batch, max_visible = len(lengths), max(lengths)
    ws_bytes = lib.dsr_decode_workspace_bytes(batch, max_visible, cfg.heads, cfg.topk)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda:0")
    out = torch.empty((batch, cfg.heads, 512), device="cuda:0")
    topk = torch.empty((batch, cfg.topk), dtype=torch.int32, device="cuda:0")
    err = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    for _ in range(args.steps):
        _native.call("dsr_decode_step", inp["idx_q"].data_ptr(), inp["idx_w"].data_ptr(), cfg.idx_heads,
                     inp["index_pool"].data_ptr(), inp["q"].data_ptr(), inp["kv_pool"].data_ptr(), cfg.heads,
                     inp["kv_pool"].shape[0] // 64, inp["block_table"].data_ptr(), inp["block_table"].shape[1],
                     inp["visible"].data_ptr(), max_visible, cfg.topk, inp["swa"].data_ptr(),
                     inp["swa_len"].data_ptr(), inp["sink"].data_ptr(), cfg.scale, out.data_ptr(),
                     topk.data_ptr(), None, ws.data_ptr(), ws_bytes, err.data_ptr(), batch,
                     _native.stream_handle())
    torch.cuda.synchronize()
    status = int(err.item())
    print(f"{args.steps} decode steps of {cfg.name}: device status {status}")
    return 0 if status == 0 else 1


def prefill(queries: int, context: int, steps: int) -> int:
    """`steps` launches of the prefill indexer (64 heads) on one seeded sequence."""
    from .workloads import small_config
    torch.cuda.set_device(0)
    inp, _ = make_decode_inputs(small_config("cfg2"), device="cuda:0", gen_device="cuda", lengths=[context])
    pool, table = inp["index_pool"], inp["block_table"][0].contiguous()
    gen = torch.Generator(device="cuda:0").manual_seed(4)
    q = torch.randn((queries, 64, 128), generator=gen, device="cuda:0").to(torch.bfloat16).float()
    w = torch.randn((queries, 64), generator=gen, device="cuda:0")
    visible = torch.arange(context - queries + 1, context + 1, dtype=torch.int32, device="cuda:0")
    scores = torch.empty((queries, context), device="cuda:0")
    err = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    for _ in range(steps):
        _native.call("dsr_indexer_prefill", q.data_ptr(), w.data_ptr(), pool.data_ptr(), pool.shape[0] // 64,
                     table.data_ptr(), table.shape[0], visible.data_ptr(), scores.data_ptr(), context,
                     err.data_ptr(), queries, 64, _native.stream_handle())
    torch.cuda.synchronize()
    status = int(err.item())
    print(f"{steps} prefill indexer launches, {queries} queries x {context} keys: device status {status}")
    return 0 if status == 0 else 1



def topk_rows(rows: int, context: int, steps: int) -> int:
    """`steps` launches of the standalone top-k over `rows` causal rows of seeded
    N(0, 64^2) scores (row r sees context - rows + 1 + r keys), histogram pass
    included, as the prefill path runs it over materialised scores."""
    torch.cuda.set_device(0)
    k = 2048
    gen = torch.Generator(device="cuda:0").manual_seed(3)
    scores = torch.randn((rows, context), generator=gen, device="cuda:0") * 64
    visible = torch.arange(context - rows + 1, context + 1, dtype=torch.int32, device="cuda:0")
    lib = _native.library()
    ws_bytes = lib.dsr_topk_workspace_bytes(rows, context)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda:0")
    out = torch.empty((rows, k), dtype=torch.int32, device="cuda:0")
    err = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    stream = _native.stream_handle(torch.cuda.current_stream())
    for _ in range(steps):
        _native.call("dsr_topk_select", scores.data_ptr(), None, visible.data_ptr(), out.data_ptr(), None,
                     err.data_ptr(), rows, context, k, 0, ws.data_ptr(), ws_bytes, stream)
    torch.cuda.synchronize()
    code = int(err.item())
    print(f"top-k {rows} x {context}: {steps} launches, device status {code}")
    return 0 if code == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
