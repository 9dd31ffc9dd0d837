"""Decode-step benchmark of the B200 attention hot path (indexer -> top-k -> sparse MLA).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N=1: BASELINE config 2 (batch 1, context 131072, 64 index heads, top-k 2048, 64
MLA heads over 576-wide rows, SWA 128).  N>1 (one process per GPU under
torch.distributed.run): config 5 (batch 4, context 1,048,576 per sequence)
sharded by contiguous position ranges across the ranks (sharded.py).
`value` is microseconds per decode step (lower is better), timed with CUDA
events around CUDA-graph replays of exactly K steps, max over ranks.  Each step
reads a different one of R pool replicas (R * working set > 2 x L2), so every
step starts from a cold L2.  `e2e` times the same steps through the C ABI with
the step's query inputs copied from pinned host memory and the attention output
copied back inside the timed region.  `--impl reference` times the reference's
CPU equations (the numpy oracle port) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import math
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
KERNELS_PER_STEP = 4  # indexer, top-k, sparse MLA, LSE combine


# --------------------------------------------------------------------------- utils
def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), float(data["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary, if any."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


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


# ------------------------------------------------------------------ decode step
class DecodeRunner:
    """Binds one decode step per pool replica to the C ABI (pointer offsets)."""

    def __init__(self, inp, lengths, cfg, replicas):
        import torch
        from deepseekrpc_b200 import _native
        self.torch, self.native = torch, _native
        self.lib = _native.library()
        self.inp, self.cfg, self.replicas = inp, cfg, replicas
        self.lengths = lengths
        self.L = lengths[0]
        self.stride = (self.L + 63) // 64 * 64
        self.heads, self.k = cfg.heads, cfg.topk
        self.ws_bytes = self.lib.dsr_decode_workspace_bytes(1, self.L, self.heads, self.k)
        dev = inp["q"].device
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.topk_ws_bytes = self.lib.dsr_topk_workspace_bytes(1, self.stride)
        self.topk_ws = torch.zeros(self.topk_ws_bytes, dtype=torch.uint8, device=dev)
        self.out = torch.empty((replicas, self.heads, 512), device=dev)
        self.topk = torch.empty((replicas, self.k), dtype=torch.int32, device=dev)
        self.scores = torch.empty((replicas, self.stride), device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pool_blocks = inp["kv_pool"].shape[0] // 64
        self.table_stride = inp["block_table"].shape[1]

    def _row(self, name, r):
        t = self.inp[name]
        return t.data_ptr() + r * t.stride(0) * t.element_size()

    def step(self, r, stream=None, idx_q=None, idx_w=None, q=None, out=None):
        """One decode step on replica r; pointer overrides select staged inputs/outputs."""
        s = self.native.stream_handle(stream)
        self.native.call("dsr_decode_step", idx_q or self._row("idx_q", r), idx_w or self._row("idx_w", r),
                         self.cfg.idx_heads, self.inp["index_pool"].data_ptr(), q or self._row("q", r),
                         self.inp["kv_pool"].data_ptr(), self.heads, self.pool_blocks,
                         self._row("block_table", r), self.table_stride, self._row("visible", r), self.L,
                         self.k, self._row("swa", r), self._row("swa_len", r), self.inp["sink"].data_ptr(),
                         self.cfg.scale, out or self.out[r].data_ptr(), self.topk[r].data_ptr(), None,
                         self.ws.data_ptr(), self.ws_bytes, self.err.data_ptr(), 1, s)

    def topk_only(self, r, stream=None):
        self.native.call("dsr_topk_select", self.scores[r].data_ptr(), None, self._row("visible", r),
                         self.topk[r].data_ptr(), None, self.err.data_ptr(), 1, self.stride, self.k, 0,
                         self.topk_ws.data_ptr(), self.topk_ws_bytes, self.native.stream_handle(stream))

    def mla_only(self, r, stream=None):
        mla_bytes = self.lib.dsr_mla_workspace_bytes(1, self.heads, self.k)
        if not hasattr(self, "mla_ws"):
            self.mla_ws = self.torch.empty(mla_bytes, dtype=self.torch.uint8, device=self.out.device)
        self.native.call("dsr_sparse_mla_decode", self._row("q", r), self.inp["kv_pool"].data_ptr(),
                         self.pool_blocks, self._row("block_table", r), self.table_stride,
                         self._row("visible", r), self.topk[r].data_ptr(), self.k, self._row("swa", r),
                         self._row("swa_len", r), self.inp["sink"].data_ptr(), self.cfg.scale,
                         self.out[r].data_ptr(), self.mla_ws.data_ptr(), mla_bytes, self.err.data_ptr(), 1,
                         self.heads, self.native.stream_handle(stream))

    def indexer(self, r, stream=None):
        self.native.call("dsr_indexer_decode", self._row("idx_q", r), self._row("idx_w", r),
                         self.inp["index_pool"].data_ptr(), self.pool_blocks, self._row("block_table", r),
                         self.table_stride, self._row("visible", r), self.scores[r].data_ptr(), self.stride,
                         self.err.data_ptr(), 1, self.cfg.idx_heads, self.native.stream_handle(stream))


def capture(torch, fn, count, stream):
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(count):
            fn(i)
    return graph


def time_replays(torch, graph, reps, stream):
    """Device time of `reps` replays, launched on `stream` and timed there."""
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


def cpu_reference_step_us(cfg, host, lengths, budget_s, threads):
    """Times the oracle port of the reference CPU path on one decode step."""
    import oracle
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        oracle.decode_step(host["idx_q"][:1], host["idx_w"][:1], host["index_pool"], host["q"][:1],
                           host["kv_pool"], host["block_table"][:1], host["visible"][:1], cfg.topk,
                           host["swa"][:1], host["swa_len"][:1], host["sink"], cfg.scale)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 1:
            break
    return statistics.median(times) * 1e6, len(times)


def cpu_config_baselines(budget_s, threads):
    """The oracle port of the reference CPU path on configs 1, 3 and 5 (bounded
    samples; per-step estimates scale the sampled sequences by their keys)."""
    import torch
    import oracle
    from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs

    def one_row_us(cfg, host, row, budget):
        times = []
        t_end = time.perf_counter() + budget
        while True:
            t0 = time.perf_counter()
            oracle.decode_step(host["idx_q"][row:row + 1], host["idx_w"][row:row + 1], host["index_pool"],
                               host["q"][row:row + 1], host["kv_pool"], host["block_table"][row:row + 1],
                               host["visible"][row:row + 1], cfg.topk, host["swa"][row:row + 1],
                               host["swa_len"][row:row + 1], host["sink"], cfg.scale)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() > t_end:
                break
        return statistics.median(times) * 1e6, len(times)

    def to_host(inp, rows):
        out = {}
        for key, v in inp.items():
            t = v if key in ("index_pool", "kv_pool", "sink") else v[:rows]
            out[key] = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()
        return out

    result = {}
    cfg = CONFIGS["cfg1"]
    inp, lengths = make_decode_inputs(cfg, device="cuda:0", gen_device="cuda")
    us, n = one_row_us(cfg, to_host(inp, 1), 0, budget_s / 4)
    result["cfg1"] = {"value": round(us, 1), "unit": "us per step", "cores": threads, "kind": "port",
                      "sample": f"{n} full steps, median"}
    del inp
    cfg = CONFIGS["cfg3"]
    inp, lengths = make_decode_inputs(cfg, device="cuda:0", gen_device="cuda")
    host = to_host(inp, 2)
    del inp
    torch.cuda.empty_cache()
    per_key = []
    for row in range(2):
        us, n = one_row_us(cfg, host, row, budget_s / 8)
        per_key.append(us / lengths[row])
    est = sum(per_key) / 2 * sum(lengths)
    result["cfg3"] = {"value": round(est, 1), "unit": "us per step (estimate)", "cores": threads, "kind": "port",
                      "sample": f"sequences 0-1 (L = {lengths[0]}, {lengths[1]}) timed, scaled by the batch's "
                                f"{sum(lengths)} keys"}
    del host
    cfg = CONFIGS["cfg5"]
    inp, lengths = make_decode_inputs(cfg, device="cuda:0", gen_device="cuda", lengths=[cfg.context])
    host = to_host(inp, 1)
    del inp
    torch.cuda.empty_cache()
    us, n = one_row_us(cfg, host, 0, budget_s / 4)
    result["cfg5"] = {"value": round(us * cfg.batch, 1), "unit": "us per step (estimate)", "cores": threads,
                      "kind": "port", "sample": f"{n} decodes of one 1,048,576-key sequence, median x 4 sequences"}
    return result


def host_copy(inp, replica=0):
    import torch
    result = {}
    for key, v in inp.items():
        if key in ("index_pool", "kv_pool", "sink"):
            t = v
        else:
            t = v[replica:replica + 1]
        result[key] = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()
    return result


def set_cpu_threads():
    n = len(os.sched_getaffinity(0))
    os.environ.setdefault("OMP_NUM_THREADS", str(n))
    try:
        import torch
        torch.set_num_threads(n)
    except ImportError:
        pass
    return n


# ------------------------------------------------------------ prefill (config 4)
def prefill_leg(dev, reps=5):
    """Config 4's indexer: 4096 causal queries at positions 262144..266239 against
    one 266,240-key paged sequence (tcgen05 GEMM, scores materialised), then the
    per-query top-2048 over them, 512 rows per top-k launch."""
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
    chunk = 512
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
            "note": "scores materialised (4.36 GB, not counted as algorithmic); top-k over 512-row launches"}


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
    return {"workload": cfg.name + ", append 1 token per sequence + decode", "value": round(ms * 1e3, 2),
            "unit": "us per batched step", "context_total": int(sum(lengths)), "bytes": nbytes,
            "achieved_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4), "peak_kind": f"{peak_kind} HBM",
            "steps": steps, "mode": "cuda graph per step (append, generation bump, decode)"}


# ---------------------------------------------------------------- single GPU
def run_single(args):
    import torch
    from deepseekrpc_b200.workloads import CONFIGS, algorithmic_bytes, make_decode_inputs
    from deepseekrpc_b200 import _native

    cfg = CONFIGS["cfg2"]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    R = args.replicas
    inp, lengths = make_decode_inputs(cfg, device=dev, gen_device="cuda", lengths=[cfg.context] * R)
    runner = DecodeRunner(inp, lengths, cfg, R)
    stream = torch.cuda.Stream()
    hbm_peak, tf_peak, peak_kind = peaks()

    # eager warm-up (sets kernel attributes outside capture) + error check
    with torch.cuda.stream(stream):
        for r in range(R):
            runner.step(r, stream=stream)
    torch.cuda.synchronize()
    assert int(runner.err.item()) == 0, f"device status {int(runner.err.item())}"

    K, W = args.steps, args.warmup
    reps = max(1, K // R)
    graph = capture(torch, lambda i: runner.step(i % R, stream=stream), R, stream)
    rest = K - reps * R
    tail = capture(torch, lambda i: runner.step(i % R, stream=stream), rest, stream) if rest else None
    warm = capture(torch, lambda i: runner.step(i % R, stream=stream), max(W, 1), stream)

    sampler = ClockSampler(gpu_id_for(0))
    with sampler, torch.cuda.stream(stream):
        # soak: clocks settle under this exact workload before and while timing
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < args.soak:
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
        step_ms = start.elapsed_time(end) / K
    clocks = sampler.summary()
    assert int(runner.err.item()) == 0

    # per-step distribution: one single-step graph per replica, an event pair
    # around each replay (rotation kept, so every step starts from a cold L2)
    singles = [capture(torch, lambda i, r=r: runner.step(r, stream=stream), 1, stream) for r in range(R)]
    samples = []
    with torch.cuda.stream(stream):
        for i in range(max(200, 25 * R)):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            singles[i % R].replay()
            e1.record(stream)
            samples.append((e0, e1))
    torch.cuda.synchronize()
    per_step = sorted(a.elapsed_time(b) * 1e3 for a, b in samples[R:])
    step_dist = {"median": round(statistics.median(per_step), 3),
                 "p10": round(per_step[len(per_step) // 10], 3),
                 "p90": round(per_step[(9 * len(per_step)) // 10], 3),
                 "samples": len(per_step), "unit": "us",
                 "note": "single-step graph replays, an event pair each (includes one graph launch per step)"}
    del singles

    # dominant kernel (indexer) timed alone, same replica rotation
    ix_graph = capture(torch, lambda i: runner.indexer(i % R, stream=stream), R, stream)
    time_replays(torch, ix_graph, 3, stream)
    ix_reps = max(1, K // R)
    ix_ms = time_replays(torch, ix_graph, ix_reps, stream) / (ix_reps * R)
    # per-kernel breakdown: each stage alone, same replica rotation
    breakdown = {}
    topk_g = capture(torch, lambda i: runner.topk_only(i % R, stream=stream), R, stream)
    time_replays(torch, topk_g, 3, stream)
    breakdown["topk_us"] = round(time_replays(torch, topk_g, reps, stream) / (reps * R) * 1e3, 3)
    mla_g = capture(torch, lambda i: runner.mla_only(i % R, stream=stream), R, stream)
    time_replays(torch, mla_g, 3, stream)
    breakdown["mla_combine_us"] = round(time_replays(torch, mla_g, reps, stream) / (reps * R) * 1e3, 3)

    L = lengths[0]
    ix_bytes = L * (128 * 2 + 4) + cfg.idx_heads * (128 + 1) * 4
    step_bytes = algorithmic_bytes([L], cfg.heads, cfg.topk, cfg.idx_heads)
    achieved = ix_bytes / (ix_ms * 1e-3) / 1e9
    traffic = profile_traffic("indexer_decode_cfg2")

    # e2e through the C ABI: each step's query inputs (index q, index weights, MLA q)
    # travel host->device from one packed pinned buffer, the attention output
    # device->host; both copies sit inside the timed region.
    n_iq, n_iw, n_q = (inp["idx_q"][0].numel(), inp["idx_w"][0].numel(), inp["q"][0].numel())
    n_in = n_iq + n_iw + n_q
    h_in = torch.empty((R, n_in), pin_memory=True)
    for r in range(R):
        h_in[r, :n_iq] = inp["idx_q"][r].flatten().cpu()
        h_in[r, n_iq:n_iq + n_iw] = inp["idx_w"][r].flatten().cpu()
        h_in[r, n_iq + n_iw:] = inp["q"][r].flatten().cpu()
    h_out = torch.empty((R, cfg.heads, 512), pin_memory=True)
    d_in = torch.empty((R, n_in), device=dev)
    d_out = torch.empty((R, cfg.heads, 512), device=dev)

    def e2e_step(i):
        r = i % R
        d_in[r].copy_(h_in[r], non_blocking=True)
        base = d_in[r].data_ptr()
        runner.step(r, stream=stream, idx_q=base, idx_w=base + 4 * n_iq, q=base + 4 * (n_iq + n_iw),
                    out=d_out[r].data_ptr())
        h_out[r].copy_(d_out[r], non_blocking=True)

    e2e_mode = "cuda graph"
    try:
        e2e_graph = capture(torch, e2e_step, R, stream)
        time_replays(torch, e2e_graph, 3, stream)
        e2e_ms = time_replays(torch, e2e_graph, reps, stream) / (reps * R)
    except RuntimeError:
        e2e_mode = "eager copies + per-step launches"
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(3 * R):
                e2e_step(i)
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for i in range(reps * R):
                e2e_step(i)
            end.record(stream)
        end.synchronize()
        e2e_ms = start.elapsed_time(end) / (reps * R)
    h2d = n_in * 4
    d2h = h_out[0].numel() * 4
    assert int(runner.err.item()) == 0
    torch.cuda.synchronize()
    assert torch.equal(h_out[0], runner.out[0].cpu()), "e2e output differs from the device-resident run"

    # CPU baseline: the reference's CPU equations (oracle port) on this host
    cpu = None
    if not args.no_cpu_baseline:
        threads = set_cpu_threads()
        host = host_copy(inp, 0)
        us, samples = cpu_reference_step_us(cfg, host, lengths, args.cpu_budget, threads)
        cpu = {"value": round(us, 1), "unit": "us", "cores": threads, "kind": "port",
               "sample": f"{samples} full config-2 decode steps (oracle/ops.py decode_step, numpy float32), "
                         "median"}
        cpu["other_configs"] = cpu_config_baselines(args.cpu_budget, threads)

    # config 5 through the sharded code on this one GPU: the N=1 point of the
    # 1/2/4/8 scaling series that `--gpus N` reports for config 5
    scaling_base = None
    if not args.no_scaling_base:
        from deepseekrpc_b200 import sharded
        scaling_base = sharded.single_gpu_base(max(3, min(K, 200)), 3, dev)

    prefill = None if args.no_prefill else prefill_leg(dev)
    batched = None if args.no_batched else batched_leg(dev)

    result = {
        "metric": METRIC, "value": round(step_ms * 1e3, 3), "unit": "us", "n_gpus": 1, "steps": K,
        "warmup": W, "ms_per_step": round(step_ms, 6), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1), BF16 pools)",
        "config": {"workload": cfg.name, "batch": 1, "context": L, "topk": cfg.topk, "heads": cfg.heads,
                   "idx_heads": cfg.idx_heads, "kv_dim": 576, "swa": 128, "block_tokens": 64,
                   "l2": f"inputs larger than L2: {R} rotating pool replicas, "
                         f"{R * step_bytes / 1e6:.0f} MB per rotation",
                   "parallelism": "single GPU"},
        "step_hbm": {"bytes": step_bytes, "achieved_gbs": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
                     "peak_gbs": hbm_peak, "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm_peak, 4),
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
        "roofline": {"kernel": "indexer_decode", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "traffic": traffic, "algorithmic_bytes": ix_bytes, "launch_us": round(ix_ms * 1e3, 3),
                     "peak_kind": f"{peak_kind} HBM copy bandwidth"},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": "us", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "mode": e2e_mode},
        "gpu_launches": KERNELS_PER_STEP * K,
        "breakdown": dict(breakdown, indexer_us=round(ix_ms * 1e3, 3)),
        "step_distribution": step_dist,
        "clocks": clocks,
        "scaling_base": scaling_base,
        "prefill": prefill,
        "batched": batched,
    }
    print(json.dumps(result))


# ------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs
    threads = set_cpu_threads()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    # N=1: config 2, as the GPU arm; N>1: config 5, timed on one of its four
    # identical 1,048,576-position sequences and scaled by four (a bounded sample)
    sharded_cfg = world > 1
    cfg = CONFIGS["cfg5"] if sharded_cfg else CONFIGS["cfg2"]
    seqs = cfg.batch if sharded_cfg else 1
    inp, lengths = make_decode_inputs(cfg, device="cpu", gen_device="cpu",
                                      lengths=[cfg.context] if sharded_cfg else None)
    host = host_copy(inp, 0)
    steps = min(args.steps, 3) if sharded_cfg else args.steps
    cpu_reference_step_us(cfg, host, lengths, 0.0, threads)  # warm-up (page-in, BLAS threads)
    times = []
    for _ in range(steps):
        us, _ = cpu_reference_step_us(cfg, host, lengths, 0.0, threads)
        times.append(us * seqs)
    value = statistics.median(times)
    sample = (f"{steps} decode steps of one config-5 sequence (B=1, L=1,048,576) of the reference CPU "
              f"equations (oracle/ops.py) x {seqs} sequences, median" if sharded_cfg else
              f"{steps} full config-2 decode steps of the reference CPU equations (oracle/ops.py), median")
    result = {
        "metric": METRIC, "impl": "reference", "value": round(value, 1), "unit": "us", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(value / 1e3, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), BF16-valued pools)",
        "config": {"workload": cfg.name, "batch": seqs, "context": lengths[0], "topk": cfg.topk,
                   "heads": cfg.heads, "idx_heads": cfg.idx_heads, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 1), "unit": "us", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result))


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20000)
    parser.add_argument("--warmup", type=int, default=50)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--replicas", type=int, default=8)
    parser.add_argument("--soak", type=float, default=1.0, help="seconds of untimed warm-up load")
    parser.add_argument("--cpu-budget", type=float, default=15.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-scaling-base", action="store_true",
                        help="skip the 1-GPU config-5 point of the scaling series")
    parser.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill indexer leg")
    parser.add_argument("--no-batched", action="store_true", help="skip the config-3 batched decode leg")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    if args.impl == "reference":
        if args.steps > 20:
            args.steps = 20  # each CPU step takes a fraction of a second; keep the run bounded
        run_reference(args)
        return
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_single(args)
    else:
        from deepseekrpc_b200 import sharded
        sharded.bench_main(args, METRIC)


if __name__ == "__main__":
    main()
