"""Decode-step benchmark of the B200 attention hot path (indexer -> top-k -> sparse MLA).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    python bench.py --profile cfg2|cfg5 [B]|mla-cfg2|prefill Q C|topk-rows R C [--steps S]

Every N reports one workload: batch 4, context 1,048,576 per
sequence, 64 index heads, top-k 2048, 64 MLA heads over 576-wide rows, SWA 128.
N=1 (plain, or torch.distributed.run with one rank) runs it on one GPU through
dsr_decode_step; N>1 (one process per GPU under torch.distributed.run) shards
every sequence by contiguous position ranges across the ranks (sharded.py).
The pools are drawn chunk by chunk from generators seeded by (seed, sequence,
chunk), so every N -- and the CPU reference arm -- holds the same rows.
`value` is microseconds per decode step (lower is better), timed with CUDA
events around CUDA-graph replays of exactly K steps, max over ranks; the pools
(1.08 GB per step) exceed L2, and ranks whose share is smaller rotate pool
replicas.  `e2e` times the same steps through the C ABI with each step's query
inputs copied from pinned host memory and the attention output copied back
inside the timed region.  `parity_ok` checks the timed result (N=1: against the
CPU oracle; N>1: against a single-GPU decode of the same sequence).

The same line carries config 2 (batch 1, context 131,072: the 1-GPU latency
case, with its own roofline and rotated pool replicas for a cold L2), config 4
(chunked prefill indexer) and config 3 (batched decode with the append) as
named objects.  `--impl reference` times the reference's CPU equations (the
numpy oracle port) on this host's cores on config 5.  `--profile` runs a few
eager launches of one workload, without graphs, for ncu captures.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "µs per decode step (indexer+top-k+sparse attn) at 128K/1M ctx; HBM GB/s % peak"
DATA = ("synthetic: seeded N(0,1) rounded to BF16; long sequences drawn in 65,536-position chunks, "
        "each from a generator seeded by (seed, sequence, chunk), on the GPU")


def kernels_per_step(batch, heads, idx_heads, k):
    """This library's kernels one dsr_decode_step launches for the shape: 1 when
    the attention and combine run inside the cooperative indexer launch, else 3
    (indexer with the exact top-k, sparse MLA, LSE combine)."""
    from deepseekrpc_b200 import _native
    return int(_native.library().dsr_decode_step_launches(batch, heads, idx_heads, k))

# DRAM bytes per launch of the indexer, read from ncu captures of the same
# kernel (dram__bytes_read.sum + dram__bytes_write.sum; profiles/indexer_decode_cfg2.md):
# config 2 from a capture of the scores + top-k launch; config 5 from a
# one-sequence capture of the step's launch x 4 sequences
INDEXER_TRAFFIC = {"cfg2": 33875968, "cfg5": 1113096192}


# --------------------------------------------------------------------------- utils
def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), float(data["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def cfg5_config(world: int) -> dict:
    """The config object of the config-5 line: identical in both arms at every N."""
    from deepseekrpc_b200.workloads import CONFIGS
    cfg = CONFIGS["cfg5"]
    return {"workload": cfg.name, "batch": cfg.batch, "context": cfg.context, "topk": cfg.topk,
            "heads": cfg.heads, "idx_heads": cfg.idx_heads, "kv_dim": 576, "swa": 128, "block_tokens": 64,
            "l2": "inputs larger than L2: 1.08 GB of pools per step; a rank whose share is smaller rotates "
                  "pool replicas",
            "parallelism": f"sequence shards x{world}" if world > 1 else "single GPU"}


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the workload runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id, self.proc, self.lines = gpu_id, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50", "-i", self.gpu_id],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s, p in zip(sm, power) if p > 200] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(device_index: int) -> str:
    import torch
    props = torch.cuda.get_device_properties(device_index)
    try:
        return f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    except AttributeError:
        return str(device_index)


def set_cpu_threads():
    n = len(os.sched_getaffinity(0))
    os.environ.setdefault("OMP_NUM_THREADS", str(n))
    try:
        import torch
        torch.set_num_threads(n)
    except ImportError:
        pass
    return n


def capture(torch, fn, count, stream):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(count):
            fn(i)
    return graph


def time_replays(torch, graph, reps, stream):
    """Device time (ms) of `reps` replays, launched on `stream` and timed there."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def sequence_host(inp, b):
    """float32 numpy arrays of sequence b alone, as the oracle takes them: its
    visible pool rows gathered on the device in logical order (so the block
    table becomes the identity), its queries, SWA rows and the sink."""
    import numpy as np
    import torch
    n = int(inp["visible"][b])
    nb = (n + 63) // 64
    pos = torch.arange(n, device=inp["block_table"].device)
    rows = inp["block_table"][b].long()[pos // 64] * 64 + pos % 64
    out = {}
    for name, width in (("index_pool", 128), ("kv_pool", 576)):
        pool = torch.zeros((nb * 64, width), dtype=torch.float32, device=rows.device)
        pool[:n] = inp[name].index_select(0, rows).float()
        out[name] = pool.cpu().numpy()
    for key in ("idx_q", "idx_w", "q", "swa", "swa_len", "visible"):
        t = inp[key][b:b + 1]
        out[key] = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()
    out["sink"] = inp["sink"].float().cpu().numpy()
    out["block_table"] = np.arange(nb, dtype=np.int32)[None]
    return out


# ------------------------------------------------------------------ decode step
class DecodeRunner:
    """dsr_decode_step over `batch` consecutive sequences of an inputs dict,
    starting at sequence `row0` (a pool replica when every replica is one
    sequence of the dict), bound to the C ABI by pointer offsets."""

    def __init__(self, inp, lengths, cfg, batch, replicas):
        import torch
        from deepseekrpc_b200 import _native
        self.torch, self.native = torch, _native
        self.lib = _native.library()
        self.inp, self.cfg, self.batch, self.replicas = inp, cfg, batch, replicas
        self.L = max(lengths)
        self.stride = (self.L + 63) // 64 * 64
        self.heads, self.k = cfg.heads, cfg.topk
        self.ws_bytes = self.lib.dsr_decode_workspace_bytes(batch, self.L, self.heads, self.k)
        dev = inp["q"].device
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        # the fused indexer + exact top-k alone (the step's first launch, without attention)
        self.sel_ws_bytes = self.lib.dsr_indexer_topk_workspace_bytes(batch, self.L)
        self.sel_ws = torch.zeros(self.sel_ws_bytes, dtype=torch.uint8, device=dev)
        rows = batch * replicas
        self.out = torch.empty((rows, self.heads, 512), device=dev)
        self.topk = torch.empty((rows, self.k), dtype=torch.int32, device=dev)
        self.scores = torch.empty((rows, self.stride), device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pool_blocks = inp["kv_pool"].shape[0] // 64
        self.table_stride = inp["block_table"].shape[1]

    def _row(self, name, r):
        t = self.inp[name]
        return t.data_ptr() + r * self.batch * t.stride(0) * t.element_size()

    def _mine(self, t, r):
        return t.data_ptr() + r * self.batch * t.stride(0) * t.element_size()

    def step(self, r, stream=None, idx_q=None, idx_w=None, q=None, out=None, scores=False):
        """One decode step on replica r; pointer overrides select staged inputs/outputs."""
        s = self.native.stream_handle(stream)
        self.native.call("dsr_decode_step", idx_q or self._row("idx_q", r), idx_w or self._row("idx_w", r),
                         self.cfg.idx_heads, self.inp["index_pool"].data_ptr(), q or self._row("q", r),
                         self.inp["kv_pool"].data_ptr(), self.heads, self.pool_blocks,
                         self._row("block_table", r), self.table_stride, self._row("visible", r), self.L,
                         self.k, self._row("swa", r), self._row("swa_len", r), self.inp["sink"].data_ptr(),
                         self.cfg.scale, out or self._mine(self.out, r), self._mine(self.topk, r),
                         self._mine(self.scores, r) if scores else None, self.ws.data_ptr(), self.ws_bytes,
                         self.err.data_ptr(), self.batch, s)

    def indexer_select(self, r, stream=None):
        self.native.call("dsr_indexer_topk_decode", self._row("idx_q", r), self._row("idx_w", r),
                         self.cfg.idx_heads, self.inp["index_pool"].data_ptr(), self.pool_blocks,
                         self._row("block_table", r), self.table_stride, self._row("visible", r), self.L, self.k, 0,
                         self._mine(self.topk, r), None, self._mine(self.scores, r), self.sel_ws.data_ptr(),
                         self.sel_ws_bytes, self.err.data_ptr(), self.batch, self.native.stream_handle(stream))

    def mla_only(self, r, stream=None):
        mla_bytes = self.lib.dsr_mla_workspace_bytes(self.batch, self.heads, self.k)
        if not hasattr(self, "mla_ws"):
            self.mla_ws = self.torch.empty(mla_bytes, dtype=self.torch.uint8, device=self.out.device)
        self.native.call("dsr_sparse_mla_decode", self._row("q", r), self.inp["kv_pool"].data_ptr(),
                         self.pool_blocks, self._row("block_table", r), self.table_stride,
                         self._row("visible", r), self._mine(self.topk, r), self.k, self._row("swa", r),
                         self._row("swa_len", r), self.inp["sink"].data_ptr(), self.cfg.scale,
                         self._mine(self.out, r), self.mla_ws.data_ptr(), mla_bytes, self.err.data_ptr(),
                         self.batch, self.heads, self.native.stream_handle(stream))

    def indexer(self, r, stream=None):
        self.native.call("dsr_indexer_decode", self._row("idx_q", r), self._row("idx_w", r),
                         self.inp["index_pool"].data_ptr(), self.pool_blocks, self._row("block_table", r),
                         self.table_stride, self._row("visible", r), self._mine(self.scores, r), self.stride,
                         self.err.data_ptr(), self.batch, self.cfg.idx_heads, self.native.stream_handle(stream))


def timed_steps(torch, runner, K, W, stream, soak=0.0, sampler=None):
    """ms per step over exactly K graph-replayed steps (replica i % R for step i),
    after W warm-up steps and `soak` seconds of untimed load."""
    R = runner.replicas
    reps, rest = divmod(K, R)
    graph = capture(torch, lambda i: runner.step(i % R, stream=stream), R, stream) if reps else None
    tail = capture(torch, lambda i: runner.step(i % R, stream=stream), rest, stream) if rest else None
    warm = capture(torch, lambda i: runner.step(i % R, stream=stream), max(W, 1), stream)
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < soak:
            warm.replay()
            stream.synchronize()
        warm.replay()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        if tail is not None:
            tail.replay()
        end.record(stream)
        end.synchronize()
    return start.elapsed_time(end) / K


def indexer_alone_ms(torch, runner, K, stream):
    R = runner.replicas
    graph = capture(torch, lambda i: runner.indexer(i % R, stream=stream), R, stream)
    time_replays(torch, graph, 3, stream)
    reps = max(1, K // R)
    return time_replays(torch, graph, reps, stream) / (reps * R)


def e2e_ms(torch, runner, inp, K, stream, dev):
    """The same steps with their query inputs (index q, index weights, MLA q of the
    step's sequences) copied from one packed pinned host buffer and the attention
    output copied back to pinned host memory, both inside the timed region."""
    R, B = runner.replicas, runner.batch
    per = [inp[n][0].numel() for n in ("idx_q", "idx_w", "q")]
    n_in = B * sum(per)
    h_in = torch.empty((R, n_in), pin_memory=True)
    for r in range(R):
        rows = slice(r * B, (r + 1) * B)
        h_in[r] = torch.cat([inp[n][rows].reshape(-1).cpu() for n in ("idx_q", "idx_w", "q")])
    h_out = torch.empty((R, B, runner.heads, 512), pin_memory=True)
    d_in = torch.empty((R, n_in), device=dev)
    d_out = torch.empty((R, B, runner.heads, 512), device=dev)

    def step(i):
        r = i % R
        d_in[r].copy_(h_in[r], non_blocking=True)
        base = d_in[r].data_ptr()
        runner.step(r, stream=stream, idx_q=base, idx_w=base + 4 * B * per[0],
                    q=base + 4 * B * (per[0] + per[1]), out=d_out[r].data_ptr())
        h_out[r].copy_(d_out[r], non_blocking=True)

    graph = capture(torch, step, R, stream)
    time_replays(torch, graph, 3, stream)
    reps = max(1, K // R)
    ms = time_replays(torch, graph, reps, stream) / (reps * R)
    torch.cuda.synchronize()
    assert int(runner.err.item()) == 0
    assert torch.equal(h_out[0], runner.out[:B].cpu()), "e2e output differs from the device-resident run"
    return ms, n_in * 4, B * runner.heads * 512 * 4


def cpu_oracle_us(cfg, h, budget_s):
    """The oracle port of the reference's CPU path (oracle.decode_step: index_scores
    -> merge_ranked tiles -> sparse_attention) on sequence 0 of host arrays h;
    median µs over repeats until `budget_s` seconds have passed (at least one)."""
    import oracle
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        oracle.decode_step(h["idx_q"][:1], h["idx_w"][:1], h["index_pool"], h["q"][:1], h["kv_pool"],
                           h["block_table"][:1], h["visible"][:1], cfg.topk, h["swa"][:1], h["swa_len"][:1],
                           h["sink"], cfg.scale)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    return statistics.median(times) * 1e6, len(times)


def oracle_parity(cfg, h, n, gpu_scores, gpu_topk, gpu_out):
    """Sequence 0 of a GPU decode against the oracle: scores within 1e-3 of
    sum_h |w_h||q_h.k| (and the share within 1e-3 plain relative error),
    top-k bit-exact against the reference ranking of the GPU's own scores,
    attention max abs <= 2e-2 and mean abs <= 2e-3."""
    import numpy as np
    import oracle
    keys = oracle.gather_rows(h["index_pool"], h["block_table"][0], np.arange(n))
    q, w = h["idx_q"][:1], h["idx_w"][:1]
    ref = oracle.index_scores(q, keys, w, np.arange(n, dtype=np.int32)[None], np.array([n], np.int32))[0]
    bound = (np.abs(w[0])[:, None] * np.abs(q[0].astype(np.float64) @ keys.T.astype(np.float64))).sum(0)
    err = np.abs(gpu_scores.astype(np.float64) - ref)
    within = bool(np.all(err <= 1e-3 * bound + 1e-6))
    share = float(np.mean(err <= 1e-3 * np.abs(ref)))
    topk_ok = bool(np.array_equal(gpu_topk, oracle.tiled_topk(gpu_scores, cfg.topk)))
    chosen = gpu_topk[gpu_topk >= 0]
    source = oracle.gather_rows(h["kv_pool"], h["block_table"][0], chosen)
    window = h["swa"][0, :int(h["swa_len"][0])]
    sel = np.arange(len(window) + len(source), dtype=np.int32)[None]
    want = oracle.sparse_attention(h["q"][:1], window, source, sel, h["sink"], scale=cfg.scale)[0, :, :512]
    diff = np.abs(gpu_out.astype(np.float64) - want)
    ok = within and share >= 0.999 and topk_ok and diff.max() <= 2e-2 and diff.mean() <= 2e-3
    return {"parity_ok": bool(ok), "sequence": 0, "keys": n, "scores_within_bound": within,
            "scores_share_rel_1e-3": round(share, 6), "topk_bit_exact": topk_ok,
            "out_max_abs": float(diff.max()), "out_mean_abs": float(diff.mean()),
            "against": "CPU oracle (oracle/ops.py)"}


# ------------------------------------------------------------ config 2 (latency)
def cfg2_leg(args, dev, stream):
    """Config 2 (B=1, L=131,072): the 1-GPU latency case, R rotating pool
    replicas (every step from a cold L2), with its own roofline, per-kernel
    breakdown, step distribution, e2e and CPU baseline."""
    import torch
    from deepseekrpc_b200.workloads import CONFIGS, algorithmic_bytes, make_decode_inputs
    cfg = CONFIGS["cfg2"]
    R = args.replicas
    inp, lengths = make_decode_inputs(cfg, device=dev, gen_device="cuda", lengths=[cfg.context] * R)
    runner = DecodeRunner(inp, lengths, cfg, 1, R)
    hbm, _, peak_kind = peaks()
    with torch.cuda.stream(stream):
        for r in range(R):
            runner.step(r, stream=stream)
    torch.cuda.synchronize()
    assert int(runner.err.item()) == 0, f"config 2: device status {int(runner.err.item())}"
    K = args.cfg2_steps
    step_ms = timed_steps(torch, runner, K, args.warmup, stream)
    # per-step distribution: single-step graphs, an event pair around each replay
    singles = [capture(torch, lambda i, r=r: runner.step(r, stream=stream), 1, stream) for r in range(R)]
    samples = []
    with torch.cuda.stream(stream):
        for i in range(max(200, 25 * R)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            singles[i % R].replay()
            e1.record(stream)
            samples.append((e0, e1))
    torch.cuda.synchronize()
    per_step = sorted(a.elapsed_time(b) * 1e3 for a, b in samples[R:])
    del singles
    ix_ms = indexer_alone_ms(torch, runner, K, stream)
    breakdown = {"indexer_us": round(ix_ms * 1e3, 3)}
    # the exact top-k fused into the indexer launch: that launch minus the indexer alone
    g = capture(torch, lambda i: runner.indexer_select(i % R, stream=stream), R, stream)
    time_replays(torch, g, 3, stream)
    reps = max(1, K // R)
    fused_us = time_replays(torch, g, reps, stream) / (reps * R) * 1e3
    breakdown["indexer_select_us"] = round(fused_us, 3)
    breakdown["select_us"] = round(fused_us - ix_ms * 1e3, 3)
    g = capture(torch, lambda i: runner.mla_only(i % R, stream=stream), R, stream)
    time_replays(torch, g, 3, stream)
    breakdown["mla_combine_us"] = round(time_replays(torch, g, reps, stream) / (reps * R) * 1e3, 3)
    del g
    e2e, h2d, d2h = e2e_ms(torch, runner, inp, K, stream, dev)
    L = lengths[0]
    ix_bytes = L * (128 * 2 + 4) + cfg.idx_heads * (128 + 1) * 4
    step_bytes = algorithmic_bytes([L], cfg.heads, cfg.topk, cfg.idx_heads)
    achieved = ix_bytes / (ix_ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        threads = set_cpu_threads()
        us, n = cpu_oracle_us(cfg, sequence_host(inp, 0), args.cpu_budget / 2)
        cpu = {"value": round(us, 1), "unit": "us", "cores": threads, "kind": "port",
               "sample": f"{n} full config-2 decode steps (oracle/ops.py decode_step, numpy float32), median"}
    result = {
        "workload": cfg.name, "value": round(step_ms * 1e3, 3), "unit": "us", "steps": K,
        "config": {"batch": 1, "context": L, "topk": cfg.topk, "heads": cfg.heads, "idx_heads": cfg.idx_heads,
                   "l2": f"{R} rotating pool replicas, {R * step_bytes / 1e6:.0f} MB per rotation (> 2 x L2)"},
        "step_hbm": {"bytes": step_bytes, "achieved_gbs": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
                     "peak_gbs": hbm, "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm, 4),
                     "peak_kind": f"{peak_kind} HBM copy bandwidth"},
        "roofline": {"kernel": "indexer_decode", "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "traffic": INDEXER_TRAFFIC.get("cfg2"),
                     "algorithmic_bytes": ix_bytes, "launch_us": round(ix_ms * 1e3, 3),
                     "peak_kind": f"{peak_kind} HBM copy bandwidth"},
        "breakdown": breakdown,
        "step_distribution": {"median": round(statistics.median(per_step), 3),
                              "p10": round(per_step[len(per_step) // 10], 3),
                              "p90": round(per_step[(9 * len(per_step)) // 10], 3), "samples": len(per_step),
                              "unit": "us", "note": "single-step graph replays, an event pair each"},
        "e2e": {"value": round(e2e * 1e3, 3), "unit": "us", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "cpu_baseline": cpu,
        "gpu_launches_per_step": kernels_per_step(1, cfg.heads, cfg.idx_heads, cfg.topk),
    }
    del runner, inp
    torch.cuda.empty_cache()
    return result


# ------------------------------------------------------------ prefill (config 4)
def prefill_leg(dev, reps=5):
    """Config 4's indexer: 4096 causal queries at positions 262144..266239 against
    one 266,240-key paged sequence (tcgen05 GEMM, scores materialised), then the
    per-query top-2048 over them, 1024 rows per top-k launch (fewer, longer
    launches measured faster than 512-row ones: 4.45 against 4.64 ms)."""
    import torch
    from deepseekrpc_b200 import _native
    from deepseekrpc_b200.workloads import make_decode_inputs, small_config
    cached, queries, heads, k = 262144, 4096, 64, 2048
    context = cached + queries
    cfg = small_config("cfg2", seed=0)
    inp, _ = make_decode_inputs(cfg, device=dev, gen_device="cuda", lengths=[context])
    pool, table = inp["index_pool"], inp["block_table"][0].contiguous()
    gen = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn((queries, heads, 128), generator=gen, device=dev).to(torch.bfloat16).float()
    w = torch.randn((queries, heads), generator=gen, device=dev)
    visible = torch.arange(cached + 1, context + 1, dtype=torch.int32, device=dev)
    stride = context
    scores = torch.empty((queries, stride), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _native.library()
    chunk = 1024
    ws_bytes = lib.dsr_topk_workspace_bytes(chunk, stride)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty((queries, k), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    s = _native.stream_handle(stream)

    def indexer():
        _native.call("dsr_indexer_prefill", q.data_ptr(), w.data_ptr(), pool.data_ptr(), pool.shape[0] // 64,
                     table.data_ptr(), table.shape[0], visible.data_ptr(), scores.data_ptr(), stride,
                     err.data_ptr(), queries, heads, s)

    def topk():
        for r0 in range(0, queries, chunk):
            _native.call("dsr_topk_select", scores[r0].data_ptr(), None, visible[r0:].data_ptr(),
                         out[r0].data_ptr(), None, err.data_ptr(), min(chunk, queries - r0), stride, k, 0,
                         ws.data_ptr(), ws_bytes, s)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(reps):
                fn()
            end.record(stream)
        end.synchronize()
        return start.elapsed_time(end) / reps

    ix_ms = timed(indexer)
    tk_ms = timed(topk)
    assert int(err.item()) == 0, f"prefill device status {int(err.item())}"
    flops = 2.0 * heads * 128 * float(visible.double().sum().item())
    _, tf_peak, peak_kind = peaks()
    tflops = flops / (ix_ms * 1e-3) / 1e12
    del scores, ws
    torch.cuda.empty_cache()
    return {"workload": "cfg4: chunked prefill, 4096 causal queries vs 266,240 keys, 64 index heads, top-k 2048",
            "indexer_ms": round(ix_ms, 3), "indexer_tflops": round(tflops, 1),
            "indexer_frac": round(tflops / tf_peak, 4),
            "peak_tflops": tf_peak, "peak_kind": f"{peak_kind} bf16 (burst, kernel timed alone)",
            "flops": flops, "topk_ms": round(tk_ms, 3),
            "note": "scores materialised (4.36 GB, not counted as algorithmic); top-k over 1024-row launches"}


# --------------------------------------------------------- batched (config 3)
def batched_leg(dev, steps=50):
    """Config 3: 32 sequences of seeded ragged lengths in [8192, 65536] over one
    shared paged pool; each step appends one token per sequence (KV + index +
    SWA rows, generation-checked) and then decodes all 32."""
    import torch
    from deepseekrpc_b200 import _native
    from deepseekrpc_b200.workloads import CONFIGS, algorithmic_bytes, make_decode_inputs
    cfg = CONFIGS["cfg3"]
    inp, lengths = make_decode_inputs(cfg, device=dev, gen_device="cuda")
    B, L = len(lengths), max(lengths)
    lib = _native.library()
    rows = inp["kv_pool"].shape[0]
    generations = torch.zeros(rows, dtype=torch.int64, device=dev)
    seq = torch.arange(B, dtype=torch.int32, device=dev)
    positions = (inp["visible"] - 1).contiguous()
    expected = torch.zeros(B, dtype=torch.int64, device=dev)
    gen = torch.Generator(device=dev).manual_seed(9)
    kv_new = torch.randn((B, 576), generator=gen, device=dev).to(torch.bfloat16)
    ix_new = torch.randn((B, 128), generator=gen, device=dev).to(torch.bfloat16)
    ws_bytes = lib.dsr_decode_workspace_bytes(B, L, cfg.heads, cfg.topk)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty((B, cfg.heads, 512), device=dev)
    topk = torch.empty((B, cfg.topk), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step():
        s = _native.stream_handle(stream)
        _native.call("dsr_append_kv_index", inp["kv_pool"].data_ptr(), inp["index_pool"].data_ptr(),
                     generations.data_ptr(), rows // 64, inp["block_table"].data_ptr(), B,
                     inp["block_table"].shape[1], seq.data_ptr(), positions.data_ptr(), expected.data_ptr(),
                     kv_new.data_ptr(), ix_new.data_ptr(), inp["swa"].data_ptr(), err.data_ptr(), B, s)
        expected.add_(1)  # the rows' generation after this append
        _native.call("dsr_decode_step", inp["idx_q"].data_ptr(), inp["idx_w"].data_ptr(), cfg.idx_heads,
                     inp["index_pool"].data_ptr(), inp["q"].data_ptr(), inp["kv_pool"].data_ptr(), cfg.heads,
                     rows // 64, inp["block_table"].data_ptr(), inp["block_table"].shape[1],
                     inp["visible"].data_ptr(), L, cfg.topk, inp["swa"].data_ptr(), inp["swa_len"].data_ptr(),
                     inp["sink"].data_ptr(), cfg.scale, out.data_ptr(), topk.data_ptr(), None, ws.data_ptr(),
                     ws_bytes, err.data_ptr(), B, s)

    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"batched device status {int(err.item())}"
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / steps
    assert int(err.item()) == 0, f"batched device status {int(err.item())}"
    nbytes = algorithmic_bytes(lengths, cfg.heads, cfg.topk, cfg.idx_heads) + B * (576 + 128) * 2 * 2
    hbm, _, peak_kind = peaks()
    del inp, ws
    torch.cuda.empty_cache()
    return {"workload": cfg.name + ", append 1 token per sequence + decode", "value": round(ms * 1e3, 2),
            "unit": "us per batched step", "context_total": int(sum(lengths)), "bytes": nbytes,
            "achieved_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4), "peak_kind": f"{peak_kind} HBM",
            "steps": steps, "mode": "cuda graph per step (append, generation bump, decode)"}


# ---------------------------------------------------------------- single GPU
def run_single(args):
    """N=1: config 5 (4 x 1,048,576) on one GPU through dsr_decode_step."""
    import numpy as np
    import torch
    from deepseekrpc_b200.workloads import CONFIGS, algorithmic_bytes, long_context_inputs

    cfg = CONFIGS["cfg5"]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    lengths = [cfg.context] * cfg.batch
    inp = long_context_inputs(cfg, lengths, dev)
    runner = DecodeRunner(inp, lengths, cfg, cfg.batch, 1)
    stream = torch.cuda.Stream()
    hbm, _, peak_kind = peaks()
    with torch.cuda.stream(stream):  # eager warm-up (sets kernel attributes outside capture)
        runner.step(0, stream=stream)
    torch.cuda.synchronize()
    assert int(runner.err.item()) == 0, f"device status {int(runner.err.item())}"

    K, W = args.steps, args.warmup
    sampler = ClockSampler(gpu_id_for(0))
    with sampler:
        step_ms = timed_steps(torch, runner, K, W, stream, soak=args.soak)
    clocks = sampler.summary()
    assert int(runner.err.item()) == 0

    step_bytes = algorithmic_bytes(lengths, cfg.heads, cfg.topk, cfg.idx_heads)
    ix_ms = indexer_alone_ms(torch, runner, max(K, 10), stream)
    ix_bytes = sum(lengths) * (128 * 2 + 4) + cfg.batch * cfg.idx_heads * (128 + 1) * 4
    achieved = ix_bytes / (ix_ms * 1e-3) / 1e9
    e2e, h2d, d2h = e2e_ms(torch, runner, inp, K, stream, dev)

    # parity of the timed path: sequence 0 against the CPU oracle (one more step
    # that also returns its scores)
    with torch.cuda.stream(stream):
        runner.step(0, stream=stream, scores=True)
    torch.cuda.synchronize()
    assert int(runner.err.item()) == 0
    n = lengths[0]
    h = sequence_host(inp, 0)
    parity = oracle_parity(cfg, h, n, runner.scores[0, :n].cpu().numpy(), runner.topk[0].cpu().numpy(),
                           runner.out[0].cpu().numpy())

    cpu = None
    if not args.no_cpu_baseline:
        threads = set_cpu_threads()
        us, samples = cpu_oracle_us(cfg, h, args.cpu_budget)
        cpu = {"value": round(us * cfg.batch, 1), "unit": "us", "cores": threads, "kind": "port",
               "sample": f"{samples} decodes of sequence 0 (1,048,576 keys; oracle/ops.py decode_step, numpy "
                         f"float32), median x {cfg.batch} sequences"}
    del h, runner, inp
    torch.cuda.empty_cache()

    cfg2 = None if args.no_cfg2 else cfg2_leg(args, dev, stream)
    prefill = None if args.no_prefill else prefill_leg(dev)
    batched = None if args.no_batched else batched_leg(dev)

    result = {
        "metric": METRIC, "value": round(step_ms * 1e3, 3), "unit": "us", "n_gpus": 1, "steps": K,
        "warmup": W, "ms_per_step": round(step_ms, 6), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": DATA, "config": cfg5_config(1),
        "step_hbm": {"bytes": step_bytes, "achieved_gbs": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
                     "peak_gbs": hbm, "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm, 4),
                     "peak_kind": f"{peak_kind} HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"},
        "roofline": {"kernel": "indexer_decode", "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "traffic": INDEXER_TRAFFIC.get("cfg5"),
                     "algorithmic_bytes": ix_bytes, "launch_us": round(ix_ms * 1e3, 3),
                     "peak_kind": f"{peak_kind} HBM copy bandwidth"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e * 1e3, 3), "unit": "us", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": kernels_per_step(cfg.batch, cfg.heads, cfg.idx_heads, cfg.topk) * K,
        "parity_ok": parity["parity_ok"], "parity": parity,
        "clocks": clocks,
        "cfg2": cfg2,
        "prefill": prefill,
        "batched": batched,
    }
    print(json.dumps(result))


# ------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU path (the oracle port of its float32 equations) on
    config 5, rank 0 only: each step decodes sequence 0 (1,048,576 keys) and is
    scaled by the batch of four; same seeded rows as the GPU arm."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from deepseekrpc_b200.workloads import CONFIGS, long_context_inputs
    threads = set_cpu_threads()
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    cfg = CONFIGS["cfg5"]
    lengths = [cfg.context] * cfg.batch
    gen_device = "cuda" if torch.cuda.is_available() else "cpu"  # the GPU arm draws on the GPU
    inp = long_context_inputs(cfg, lengths, gen_device, sequences=[0])
    h = sequence_host(inp, 0)
    del inp
    if gen_device == "cuda":
        torch.cuda.empty_cache()
    for _ in range(min(args.warmup, 1)):
        cpu_oracle_us(cfg, h, 0.0)  # page-in, BLAS threads
    times = [cpu_oracle_us(cfg, h, 0.0)[0] * cfg.batch for _ in range(args.steps)]
    value = statistics.median(times)
    sample = (f"{args.steps} decodes of sequence 0 of config 5 (B=1, L=1,048,576) by the reference's CPU "
              f"equations (oracle/ops.py decode_step, numpy float32), median x {cfg.batch} sequences")
    data = DATA if gen_device == "cuda" else DATA + " (drawn on the CPU here: no GPU)"
    result = {
        "metric": METRIC, "impl": "reference", "value": round(value, 1), "unit": "us", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value / 1e3, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": data, "config": cfg5_config(world),
        "cpu_baseline": {"value": round(value, 1), "unit": "us", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result))


# ------------------------------------------------------------------ profiling
def run_profile(args):
    """A few eager launches of one workload on cuda:0, no CUDA graphs, so that a
    profiler sees each kernel launch on its own; exits nonzero on a device error."""
    import torch
    from deepseekrpc_b200 import _native
    from deepseekrpc_b200.workloads import CONFIGS, long_context_inputs, make_decode_inputs, small_config
    what, extra = args.profile[0], [int(x) for x in args.profile[1:]]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    if what in ("cfg1", "cfg2", "cfg3", "cfg5"):
        cfg = CONFIGS[what]
        if what == "cfg5":
            # optional: fewer sequences (a profiler capture small enough to replay)
            lengths = [cfg.context] * (extra[0] if extra else cfg.batch)
            inp = long_context_inputs(cfg, lengths, dev)
        else:
            inp, lengths = make_decode_inputs(cfg, device=dev, gen_device="cuda")
        runner = DecodeRunner(inp, lengths, cfg, len(lengths), 1)
        for _ in range(args.steps):
            runner.step(0)
        err = runner.err
        label = f"{args.steps} decode steps of {cfg.name}"
    elif what == "mla-cfg2":
        # the standalone sparse MLA + combine (the path of batches whose tiles
        # exceed one per SM, and of the sharded partials) at the config-2 shape,
        # over the top-k one decode step selected
        cfg = CONFIGS["cfg2"]
        inp, lengths = make_decode_inputs(cfg, device=dev, gen_device="cuda")
        runner = DecodeRunner(inp, lengths, cfg, 1, 1)
        runner.step(0)
        for _ in range(args.steps):
            runner.mla_only(0)
        err = runner.err
        label = f"{args.steps} standalone sparse MLA launches at the config-2 shape"
    elif what == "prefill":
        queries, context = extra
        inp, _ = make_decode_inputs(small_config("cfg2"), device=dev, gen_device="cuda", lengths=[context])
        pool, table = inp["index_pool"], inp["block_table"][0].contiguous()
        gen = torch.Generator(device=dev).manual_seed(4)
        q = torch.randn((queries, 64, 128), generator=gen, device=dev).to(torch.bfloat16).float()
        w = torch.randn((queries, 64), generator=gen, device=dev)
        visible = torch.arange(context - queries + 1, context + 1, dtype=torch.int32, device=dev)
        scores = torch.empty((queries, context), device=dev)
        for _ in range(args.steps):
            _native.call("dsr_indexer_prefill", q.data_ptr(), w.data_ptr(), pool.data_ptr(), pool.shape[0] // 64,
                         table.data_ptr(), table.shape[0], visible.data_ptr(), scores.data_ptr(), context,
                         err.data_ptr(), queries, 64, _native.stream_handle())
        label = f"{args.steps} prefill indexer launches, {queries} queries x {context} keys"
    elif what == "topk-rows":
        rows, context = extra
        k = 2048
        gen = torch.Generator(device=dev).manual_seed(3)
        scores = torch.randn((rows, context), generator=gen, device=dev) * 64
        visible = torch.arange(context - rows + 1, context + 1, dtype=torch.int32, device=dev)
        lib = _native.library()
        ws_bytes = lib.dsr_topk_workspace_bytes(rows, context)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        out = torch.empty((rows, k), dtype=torch.int32, device=dev)
        for _ in range(args.steps):
            _native.call("dsr_topk_select", scores.data_ptr(), None, visible.data_ptr(), out.data_ptr(), None,
                         err.data_ptr(), rows, context, k, 0, ws.data_ptr(), ws_bytes, _native.stream_handle())
        label = f"top-k {rows} x {context}: {args.steps} launches"
    else:
        raise SystemExit(f"unknown --profile workload {what!r}")
    torch.cuda.synchronize()
    code = int(err.item())
    print(f"{label}: device status {code}")
    return 0 if code == 0 else 1


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--replicas", type=int, default=8, help="config-2 pool replicas (cold L2 per step)")
    parser.add_argument("--cfg2-steps", type=int, default=2000, help="steps timed for the config-2 object")
    parser.add_argument("--soak", type=float, default=1.0, help="seconds of untimed warm-up load")
    parser.add_argument("--cpu-budget", type=float, default=15.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-cfg2", action="store_true", help="skip the config-2 latency object")
    parser.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill indexer leg")
    parser.add_argument("--no-batched", action="store_true", help="skip the config-3 batched decode leg")
    parser.add_argument("--profile", nargs="+", metavar="WORKLOAD",
                        help="cfg1|cfg2|cfg3|cfg5 [B], mla-cfg2, `prefill QUERIES CONTEXT` or `topk-rows ROWS CONTEXT`: "
                             "--steps eager launches for a profiler, then exit")
    args = parser.parse_args(argv)
    if args.profile:
        sys.exit(run_profile(args))
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus == 1 and world == 1:
        run_single(args)
    else:
        from deepseekrpc_b200 import sharded
        sharded.bench_main(args, METRIC, cfg5_config(world), DATA)


if __name__ == "__main__":
    main()
