"""Sequence-sharded sparse-attention decode across the GPUs of one node.

One process per GPU (torch.distributed, NCCL).  Rank r of G owns the logical
positions [r*S, (r+1)*S) of every sequence, S = the shard span (a multiple of
the 64-token block), in its own index-key and KV pools; the SWA rows live on
the rank that owns each sequence's tail.  A decode step is

  1. local indexer scores over the owned positions, local exact top-k with
     global ids (id_base = r*S), scores returned with the ids;
  2. one all-gather of the (score, id) lists; every rank merges the G lists
     into the exact global top-k with the same tie rule (the union of the local
     top-k sets holds the global top-k under that total order), so every rank
     holds the same selection without a second exchange;
  3. local sparse-MLA partial (m, l, o) over the selected rows it owns (plus the
     SWA rows on the tail owner), without the sink;
  4. one all-gather of the partials and a log-sum-exp combine that adds the
     sink exactly once.

There is no reference counterpart (the reference decodes on one GPU); the
single-GPU semantics it must reproduce are TiledIndexer.select
(index_selection.py:79-124) followed by sparse_attention with the sink
(native/operations.cu:30-82).

The exchange/layout helpers are plain torch and run on any backend (the CPU
tests use gloo); the per-rank compute goes through the C ABI and needs the
built library and a B200.
"""
from __future__ import annotations

import json
import os
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native
from .workloads import BLOCK, INDEX_DIM, KV_DIM, SWA_ROWS, V_DIM, CONFIGS

# ----------------------------------------------------------------- planning


@dataclass(frozen=True)
class ShardPlan:
    """Position ownership of rank `rank` out of `world` for a batch of sequences."""

    world: int
    rank: int
    lengths: tuple  # visible positions of each sequence (the query sits at L-1)

    @property
    def span(self) -> int:
        """Positions per shard: the longest sequence's blocks split evenly."""
        blocks = (max(self.lengths) + BLOCK - 1) // BLOCK
        return ((blocks + self.world - 1) // self.world) * BLOCK

    @property
    def id_base(self) -> int:
        return self.rank * self.span

    def local_visible(self) -> list[int]:
        """Owned visible positions of each sequence: [id_base, id_base + n)."""
        base, span = self.id_base, self.span
        return [max(0, min(n - base, span)) for n in self.lengths]

    def owns_tail(self, b: int) -> bool:
        """The rank holding position L_b - 1 also holds that sequence's SWA rows."""
        n = self.lengths[b]
        return n > 0 and self.id_base <= n - 1 < self.id_base + self.span

    def local_swa_len(self) -> list[int]:
        return [min(SWA_ROWS, n) if self.owns_tail(b) else 0 for b, n in enumerate(self.lengths)]

    def local_blocks(self) -> int:
        return self.span // BLOCK


def local_block_table(full_table: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    """Columns of a global block table owned by `plan` (block j of the shard = global
    block id_base/64 + j), padded with -1 past the table's end."""
    first = plan.id_base // BLOCK
    cols = plan.local_blocks()
    out = torch.full((full_table.shape[0], cols), -1, dtype=torch.int32, device=full_table.device)
    take = max(0, min(cols, full_table.shape[1] - first))
    if take:
        out[:, :take] = full_table[:, first:first + take]
    return out.contiguous()


# ------------------------------------------------------------ exchange layouts
#
# Send buffers are written in place by the kernels and all-gathered rank-major:
#   top-k lists: i32 [2][B][k] per rank (the scores' bit patterns, then the
#                global ids, -1 padded) -> gathered [G*2][B][k], read by
#                dsr_topk_merge_lists;
#   partials:    f32 [o (B*H*512) | m (B*H) | l (B*H)] per rank -> gathered
#                [G][...], read by dsr_lse_combine_packed.
# The two decoders below restate those layouts on the host (tests, inspection).


def gathered_lists(gathered: torch.Tensor, world: int):
    """Gathered top-k lists -> scores f32[B, G*k], ids i32[B, G*k], ids increasing along a row."""
    g = gathered.view(world, 2, gathered.shape[-2], gathered.shape[-1])
    b, k = g.shape[2], g.shape[3]
    scores = g[:, 0].permute(1, 0, 2).reshape(b, world * k).contiguous().view(torch.float32)
    ids = g[:, 1].permute(1, 0, 2).reshape(b, world * k).contiguous()
    return scores, ids


def gathered_partials(gathered: torch.Tensor, world: int, batch: int, heads: int):
    """Gathered partials -> o f32[G, B*H, 512], m f32[G, B*H], l f32[G, B*H] (base-2 m)."""
    bh = batch * heads
    g = gathered.view(world, bh * (V_DIM + 2))
    return (g[:, :bh * V_DIM].reshape(world, bh, V_DIM), g[:, bh * V_DIM:bh * (V_DIM + 1)],
            g[:, bh * (V_DIM + 1):])


def all_gather(tensor: torch.Tensor, group=None) -> torch.Tensor:
    """Rank-major concatenation along dim 0."""
    world = dist.get_world_size(group)
    out = torch.empty((world * tensor.shape[0],) + tuple(tensor.shape[1:]), dtype=tensor.dtype,
                      device=tensor.device)
    dist.all_gather_into_tensor(out, tensor.contiguous(), group=group)
    return out


class _DeviceView:
    """A raw device allocation as a torch tensor (CUDA array interface)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """All-gather of one fixed-size payload per rank over NVLink peer mappings.

    Every rank allocates an exchange buffer (dsr_p2p_alloc), the 64-byte CUDA IPC
    handles travel through the process group once (all_gather_object), and each
    rank maps its peers' buffers (dsr_p2p_open).  `all_gather(payload)` launches
    dsr_p2p_allgather on the stream: the payload of rank r lands in slot r of every
    rank's buffer, and the returned tensor (`gathered`, rank-major, the same
    memory every call) is complete when that kernel is.  No collective library
    runs per step; the kernels are capturable in a CUDA graph.  All ranks must
    issue the same exchanges in the same order, as the collective would require.
    """

    def __init__(self, payload_shape, dtype: torch.dtype, device, group=None, chunks: int | None = None):
        import ctypes
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise ValueError("the peer exchange spans 1 to 8 ranks of one node")
        self.lib = _native.library()
        self.dtype, self.payload_shape = dtype, tuple(payload_shape)
        numel = 1
        for d in self.payload_shape:
            numel *= d
        self.payload_bytes = numel * torch.empty((), dtype=dtype).element_size()
        if self.payload_bytes % 16:
            raise ValueError("exchange payloads are whole 16-byte units")
        self.chunks = chunks or max(1, min(16, self.payload_bytes // 65536))
        size = self.lib.dsr_p2p_buffer_bytes(self.world, self.payload_bytes)
        buf = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _native.call("dsr_p2p_alloc", size, ctypes.addressof(buf), ctypes.addressof(handle))
        self._local = buf.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for w, h in enumerate(handles):
            if w == self.rank:
                ptrs.append(self._local)
                continue
            peer = ctypes.c_void_p()
            raw = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            _native.call("dsr_p2p_open", ctypes.addressof(raw), ctypes.addressof(peer))
            self._opened.append(peer.value)
            ptrs.append(peer.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        typestr = {torch.int32: "<i4", torch.float32: "<f4"}[dtype]
        self.gathered = torch.as_tensor(
            _DeviceView(self._local + 256, (self.world,) + self.payload_shape, typestr), device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        dist.barrier(group)  # every peer mapping exists before the first exchange

    def all_gather(self, payload: torch.Tensor, stream=None) -> torch.Tensor:
        if payload.dtype != self.dtype or tuple(payload.shape) != self.payload_shape or not payload.is_contiguous():
            raise ValueError("payload does not match the exchange's shape and dtype")
        import ctypes
        _native.call("dsr_p2p_allgather", payload.data_ptr(), self.payload_bytes,
                     ctypes.cast(self._ptrs, ctypes.c_void_p), self.rank, self.world, self.payload_bytes,
                     self.chunks, self.err.data_ptr(), _native.stream_handle(stream))
        return self.gathered

    def close(self) -> None:
        """After every rank's last exchange has completed (a barrier), unmap and free."""
        if self._local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        for peer in self._opened:
            _native.call("dsr_p2p_close", peer)
        self._opened = []
        self.gathered = None
        _native.call("dsr_p2p_free", self._local)
        self._local = None


# ------------------------------------------------------------- per-rank step


class ShardedDecoder:
    """Buffers and C-ABI calls of one rank's sharded decode step."""

    def __init__(self, plan: ShardPlan, heads: int, idx_heads: int, topk: int, scale: float,
                 sink: torch.Tensor, device):
        self.plan, self.heads, self.idx_heads, self.k, self.scale = plan, heads, idx_heads, topk, scale
        self.lib = _native.library()
        B = len(plan.lengths)
        self.batch = B
        self.span = plan.span
        dev = torch.device(device)
        self.visible = torch.tensor(plan.local_visible(), dtype=torch.int32, device=dev)
        self.swa_len = torch.tensor(plan.local_swa_len(), dtype=torch.int32, device=dev)
        self.send_lists = torch.empty((2, B, topk), dtype=torch.int32, device=dev)
        self.ix_bytes = self.lib.dsr_indexer_topk_workspace_bytes(B, self.span)
        self.ix_ws = torch.zeros(self.ix_bytes, dtype=torch.uint8, device=dev)
        self.merge_bytes = self.lib.dsr_topk_merge_workspace_bytes(B, plan.world, topk)
        self.merge_ws = torch.zeros(self.merge_bytes, dtype=torch.uint8, device=dev)
        self.ids = torch.empty((B, topk), dtype=torch.int32, device=dev)
        self.mla_bytes = self.lib.dsr_mla_workspace_bytes(B, heads, topk)
        self.mla_ws = torch.zeros(self.mla_bytes, dtype=torch.uint8, device=dev)
        bh = B * heads
        self.send_partial = torch.empty(bh * (V_DIM + 2), device=dev)
        self.o = self.send_partial[:bh * V_DIM]
        self.m = self.send_partial[bh * V_DIM:bh * (V_DIM + 1)]
        self.l = self.send_partial[bh * (V_DIM + 1):]
        self.out = torch.empty((B, heads, V_DIM), device=dev)
        self.sink = sink.float().contiguous().to(dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    # the phases, so a single-GPU emulation can run them shard by shard
    def select_local(self, idx_q, idx_w, index_pool, block_table, stream=None):
        """Local indexer + exact top-k (global ids and scores) into the send buffer."""
        p = _native.ptr
        _native.call("dsr_indexer_topk_decode", p(idx_q), p(idx_w), self.idx_heads, p(index_pool),
                     index_pool.shape[0] // BLOCK, p(block_table), block_table.shape[1], p(self.visible),
                     self.span, self.k, self.plan.id_base, p(self.send_lists[1]), p(self.send_lists[0]), None,
                     p(self.ix_ws), self.ix_bytes, p(self.err), self.batch, _native.stream_handle(stream))
        return self.send_lists

    def merge(self, gathered, stream=None):
        """Exact global top-k from the gathered lists (identical on every rank)."""
        p = _native.ptr
        _native.call("dsr_topk_merge_lists", p(gathered), self.plan.world, self.batch, self.k, p(self.ids),
                     p(self.merge_ws), self.merge_bytes, p(self.err), _native.stream_handle(stream))
        return self.ids

    def attend_local(self, q, kv_pool, block_table, swa, stream=None):
        """This rank's unnormalised partial (o, m, l) into the send buffer."""
        p = _native.ptr
        _native.call("dsr_sparse_mla_partial", p(q), p(kv_pool), kv_pool.shape[0] // BLOCK, p(block_table),
                     block_table.shape[1], p(self.visible), p(self.ids), self.k, self.plan.id_base, p(swa),
                     p(self.swa_len), float(self.scale), p(self.o), p(self.m), p(self.l), p(self.mla_ws),
                     self.mla_bytes, p(self.err), self.batch, self.heads, _native.stream_handle(stream))
        return self.send_partial

    def combine(self, gathered, stream=None):
        p = _native.ptr
        _native.call("dsr_lse_combine_packed", p(gathered), self.plan.world, p(self.sink), p(self.out),
                     p(self.err), self.batch, self.heads, _native.stream_handle(stream))
        return self.out

    def use_peer_exchange(self, group=None) -> None:
        """Exchange lists and partials over NVLink peer mappings instead of the
        collective library (every rank of `group` on this node)."""
        dev = self.err.device
        self.exchanges = (PeerExchange(tuple(self.send_lists.shape), torch.int32, dev, group),
                          PeerExchange(tuple(self.send_partial.shape), torch.float32, dev, group))

    def close(self) -> None:
        for x in getattr(self, "exchanges", ()) or ():
            x.close()
        self.exchanges = None

    def _gather(self, which: int, payload, group, stream):
        exchanges = getattr(self, "exchanges", None)
        if exchanges:
            return exchanges[which].all_gather(payload, stream)
        return all_gather(payload, group)

    def exchange_status(self) -> int:
        """Worst device status of the peer exchanges (0 without them)."""
        return max((int(x.err.item()) for x in getattr(self, "exchanges", ()) or ()), default=0)

    def step(self, inputs, group=None, stream=None):
        """One full decode step with the two exchanges; returns out f32[B, H, 512]."""
        lists = self.select_local(inputs["idx_q"], inputs["idx_w"], inputs["index_pool"],
                                  inputs["block_table"], stream)
        self.merge(self._gather(0, lists, group, stream), stream)
        partial = self.attend_local(inputs["q"], inputs["kv_pool"], inputs["block_table"], inputs["swa"], stream)
        return self.combine(self._gather(1, partial, group, stream), stream)


# ------------------------------------------------------------------ inputs


def make_shard_inputs(cfg, plan: ShardPlan, device, layout_seed: int | None = None):
    """Seeded synthetic inputs of one rank: its own paged pools for the owned
    positions [id_base, id_base + span) of every sequence, drawn chunk by chunk
    from generators seeded by (config seed, sequence, chunk) -- so every world
    size holds the same logical rows -- and laid out by a per-rank permutation;
    the queries, weights, SWA rows and sink (identical on every rank; swa_len is
    nonzero on the tail owner only)."""
    from .workloads import long_context_inputs
    seed = 7919 * (plan.rank + 1) if layout_seed is None else layout_seed
    return long_context_inputs(cfg, plan.lengths, device, start=plan.id_base, span=plan.span, layout_seed=seed)


# ------------------------------------------------------------------- bench


def _capture(fn, stream):
    """fn() captured as a CUDA graph on `stream` (all ranks together), or None."""
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph, stream=stream):
            fn()
    except RuntimeError:
        graph = None
    ok = torch.tensor([1 if graph is not None else 0], device=torch.cuda.current_device())
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)  # the same choice on every rank
    torch.cuda.synchronize()
    return graph if int(ok.item()) == 1 else None


def _timed_steps(fn, steps, stream, dev, group=None) -> float:
    """ms per step: CUDA events on `stream` around `steps` calls, barrier and
    synchronize on both sides, max over ranks."""
    dist.barrier(group)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for i in range(steps):
            fn(i)
        end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    dist.barrier(group)
    ms = torch.tensor([start.elapsed_time(end) / steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=group)
    return float(ms.item())


# kernels of this library launched per sharded step: indexer with its local
# top-k (one cooperative launch), list exchange, merge, MLA partial (tiles +
# in-shard combine), partial exchange, cross-shard combine
LAUNCHES_PER_STEP = 7


def replicas_for_cold_l2(per_rank_bytes: int, device) -> int:
    """Pool replicas a rank rotates through so that every step reads its pools
    from DRAM: enough that R x the step's bytes exceed twice the L2 cache."""
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    return max(1, -(-int(2.2 * l2) // max(1, per_rank_bytes)))


def single_gpu_reference(cfg, lengths, seq: int, device):
    """Sequence `seq` decoded alone on this GPU through dsr_decode_step (whole
    pools, same seeded rows): the (ids i32[k], out f32[heads, 512]) the sharded
    step must reproduce."""
    from .workloads import long_context_inputs
    inp = long_context_inputs(cfg, lengths, device, sequences=[seq], layout_seed=12345)
    lib = _native.library()
    n = int(lengths[seq])
    ws_bytes = lib.dsr_decode_workspace_bytes(1, n, cfg.heads, cfg.topk)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)
    out = torch.empty((1, cfg.heads, V_DIM), device=device)
    ids = torch.empty((1, cfg.topk), dtype=torch.int32, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    p = _native.ptr
    _native.call("dsr_decode_step", p(inp["idx_q"]), p(inp["idx_w"]), cfg.idx_heads, p(inp["index_pool"]),
                 p(inp["q"]), p(inp["kv_pool"]), cfg.heads, inp["kv_pool"].shape[0] // BLOCK,
                 p(inp["block_table"]), inp["block_table"].shape[1], p(inp["visible"]), n, cfg.topk,
                 p(inp["swa"]), p(inp["swa_len"]), p(inp["sink"]), float(cfg.scale), p(out), p(ids), None, p(ws),
                 ws_bytes, p(err), 1, _native.stream_handle(torch.cuda.current_stream(device)))
    torch.cuda.synchronize(device)
    if int(err.item()) != 0:
        raise RuntimeError(f"single-GPU reference step: device status {int(err.item())}")
    return ids[0], out[0]


def parity_against_single_gpu(cfg, lengths, ids, out, device, seq: int = 0, group=None) -> dict:
    """Every rank compares its merged top-k (bit for bit) and its combined output
    (BF16 tolerance: max abs <= 2e-2, mean abs <= 2e-3) for sequence `seq` with
    rank 0's single-GPU decode of that sequence; all ranks agree on the verdict."""
    rank = dist.get_rank(group)
    ref_ids = torch.empty((cfg.topk,), dtype=torch.int32, device=device)
    ref_out = torch.empty((cfg.heads, V_DIM), device=device)
    if rank == 0:
        r_ids, r_out = single_gpu_reference(cfg, lengths, seq, device)
        ref_ids.copy_(r_ids)
        ref_out.copy_(r_out)
        torch.cuda.empty_cache()
    dist.broadcast(ref_ids, 0, group=group)
    dist.broadcast(ref_out, 0, group=group)
    diff = (out[seq] - ref_out).abs()
    ids_ok = bool(torch.equal(ids[seq], ref_ids))
    max_abs, mean_abs = float(diff.max().item()), float(diff.mean().item())
    ok = torch.tensor([1 if ids_ok and max_abs <= 2e-2 and mean_abs <= 2e-3 else 0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    return {"parity_ok": bool(ok.item()), "sequence": seq, "topk_identical": ids_ok,
            "out_max_abs": max_abs, "out_mean_abs": mean_abs,
            "against": "dsr_decode_step of the same sequence on one GPU (same seeded rows)"}


PHASES = ("indexer_topk", "exchange_lists", "merge", "mla_partial", "exchange_partials", "combine")


def phase_breakdown(dec: "ShardedDecoder", replicas, stream, dev, steps: int = 20) -> dict:
    """What each launch of a step adds (PHASES order), the way the benchmark runs
    it: for n = 1..6 the first n launches of every step captured as CUDA graphs
    (one step per pool replica, all ranks together), timed over `steps` replays
    like the step itself (max over ranks); a phase's cost is the growth of that
    time when it joins.  An exchange's cost includes waiting for the slowest
    peer."""
    R = len(replicas)

    def prefix(n):
        def one(inp):
            lists = dec.select_local(inp["idx_q"], inp["idx_w"], inp["index_pool"], inp["block_table"], stream)
            if n >= 2:
                gathered = dec._gather(0, lists, None, stream)
            if n >= 3:
                dec.merge(gathered, stream)
            if n >= 4:
                partial = dec.attend_local(inp["q"], inp["kv_pool"], inp["block_table"], inp["swa"], stream)
            if n >= 5:
                gathered = dec._gather(1, partial, None, stream)
            if n >= 6:
                dec.combine(gathered, stream)
        return lambda: [one(replicas[i]) for i in range(R)]

    cumulative = []
    for n in range(1, len(PHASES) + 1):
        fn = prefix(n)
        with torch.cuda.stream(stream):
            fn()
        graph = _capture(fn, stream)
        run = (lambda i: graph.replay()) if graph is not None else (lambda i: fn())
        cumulative.append(_timed_steps(run, steps, stream, dev) / R * 1e3)
        graph = None
    added = [cumulative[0]] + [cumulative[i] - cumulative[i - 1] for i in range(1, len(PHASES))]
    return {"note": "us per step of CUDA graphs holding the first n launches of every step, n = 1..6; "
                    "each phase = the growth when it joins; max over ranks",
            "cumulative": [round(x, 2) for x in cumulative],
            **{name: round(x, 2) for name, x in zip(PHASES, added)}}


def bench_main(args, metric: str, config: dict, data: str) -> None:
    """bench.py --gpus N under torch.distributed.run: config 5 sharded over N ranks.

    `value` = µs per decode step of the whole job (4 sequences x 1,048,576
    positions, fixed as N grows: strong scaling), max over ranks of CUDA-event
    time around K steps, barrier + synchronize on both sides.  Each rank rotates
    through R copies of its pools when its share of a step is too small to
    evict L2 by itself.  `e2e` repeats the steps with each rank's query inputs
    copied from pinned host memory and the attention output copied back inside
    the timed region.  After timing, every rank checks its result against a
    single-GPU decode of sequence 0 (`parity_ok`)."""
    from datetime import timedelta
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    graph = e2e_graph = None
    dec = None
    try:
        from .workloads import algorithmic_bytes
        cfg = CONFIGS["cfg5"]
        lengths = tuple([cfg.context] * cfg.batch)
        plan = ShardPlan(world, rank, lengths)
        inputs = make_shard_inputs(cfg, plan, dev)
        total_bytes = algorithmic_bytes(list(lengths), cfg.heads, cfg.topk, cfg.idx_heads)
        R = replicas_for_cold_l2(total_bytes // world, dev)
        replicas = [inputs] + [dict(inputs, index_pool=inputs["index_pool"].clone(),
                                    kv_pool=inputs["kv_pool"].clone()) for _ in range(R - 1)]
        dec = ShardedDecoder(plan, cfg.heads, cfg.idx_heads, cfg.topk, cfg.scale, inputs["sink"], dev)
        # the two exchanges: NVLink peer stores (default) or the collective library
        exchange = os.environ.get("DSR_EXCHANGE", "peer")
        if exchange == "peer" and world > 1:
            dec.use_peer_exchange()
        else:
            exchange = "nccl"
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                dec.step(replicas[i % R], stream=stream)
        torch.cuda.synchronize()
        assert int(dec.err.item()) == 0 and dec.exchange_status() == 0, \
            f"rank {rank}: device status {int(dec.err.item())}/{dec.exchange_status()}"
        # R steps (one per replica: kernels and both exchanges) as one CUDA graph,
        # plus a graph of the K mod R remaining steps; every rank captures, so the
        # exchanges line up; eager steps if capture is refused
        K = args.steps
        reps, rest = divmod(K, R)

        def steps_fn(n):
            return lambda: [dec.step(replicas[i % R], stream=stream) for i in range(n)]

        graph = _capture(steps_fn(R), stream) if reps else None
        tail = _capture(steps_fn(rest), stream) if rest else None
        graphed = (graph is not None or not reps) and (tail is not None or not rest)
        if graphed:
            def run(i):
                if i < reps:
                    graph.replay()
                else:
                    tail.replay()
            calls = reps + (1 if rest else 0)
        else:
            def run(i):
                dec.step(replicas[i % R], stream=stream)
            calls = K
        step_ms = _timed_steps(run, calls, stream, dev) * calls / K

        # end to end: query inputs host -> device, output device -> host, every step
        names = ("idx_q", "idx_w", "q")
        sizes = [inputs[n].numel() for n in names]
        h_in = torch.empty(sum(sizes), pin_memory=True)
        h_in.copy_(torch.cat([inputs[n].reshape(-1).cpu() for n in names]))
        d_in = torch.empty(sum(sizes), device=dev)
        staged = []
        for rep in replicas:
            st = dict(rep)
            off = 0
            for n, size in zip(names, sizes):
                st[n] = d_in[off:off + size].view(inputs[n].shape)
                off += size
            staged.append(st)
        h_out = torch.empty(tuple(dec.out.shape), pin_memory=True)

        def e2e_step(i):
            d_in.copy_(h_in, non_blocking=True)
            out = dec.step(staged[i % R], stream=stream)
            h_out.copy_(out, non_blocking=True)

        with torch.cuda.stream(stream):
            for i in range(3):
                e2e_step(i)
        e2e_graph = _capture(lambda: [e2e_step(i) for i in range(R)], stream)
        if e2e_graph is not None:
            e2e_calls = max(1, K // R)
            e2e_ms = _timed_steps(lambda i: e2e_graph.replay(), e2e_calls, stream, dev) / R
        else:
            e2e_ms = _timed_steps(e2e_step, K, stream, dev)
        torch.cuda.synchronize()
        assert int(dec.err.item()) == 0 and dec.exchange_status() == 0
        assert torch.equal(h_out, dec.out.cpu()), "e2e output differs from the device-resident run"

        phases = phase_breakdown(dec, replicas, stream, dev)
        parity = parity_against_single_gpu(cfg, lengths, dec.ids, dec.out, dev)
        graph = tail = e2e_graph = None  # graphs holding exchange work go before the process group
        if rank == 0:
            print(json.dumps({
                "metric": metric, "value": round(step_ms * 1e3, 3), "unit": "us", "n_gpus": world,
                "steps": K, "warmup": args.warmup, "ms_per_step": round(step_ms, 6),
                "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": data, "config": config,
                "step_hbm": {"bytes": total_bytes, "achieved_gbs": round(total_bytes / (step_ms * 1e-3) / 1e9, 1),
                             "per_rank_bytes": total_bytes // world},
                "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": "us",
                        "h2d_bytes_per_step": world * h_in.numel() * 4,
                        "d2h_bytes_per_step": world * h_out.numel() * 4},
                "gpu_launches": LAUNCHES_PER_STEP * K,
                "parity_ok": parity["parity_ok"], "parity": parity, "phases_us": phases,
                "exchange": ("NVLink peer stores (dsr_p2p_allgather)" if exchange == "peer" else "NCCL all_gather"),
                "replicas": R,
                "l2": f"{R} pool replica(s) per rank rotated, {R * total_bytes // world / 1e6:.0f} MB per rotation "
                      f"(> 2 x L2)" if R > 1 else "inputs larger than L2 on every rank",
                "mode": "cuda graph per step" if graphed else "eager launches",
            }))
    finally:
        graph = tail = e2e_graph = None
        if dec is not None:
            dec.close()
        dist.destroy_process_group()
