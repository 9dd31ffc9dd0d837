"""Synthetic decode workloads with the shapes of the BASELINE configurations.

The reference publishes no dataset for this path; every input is seeded
synthetic data with the configured shapes and value distributions
(N(0,1) rounded to BF16; index weights N(0,1)/8 in config 1).  Draw order on a
torch.Generator seeded with the config seed: [context lengths (config 3)],
index q, index-key pool, index weights, MLA q, KV pool, SWA rows, sink, block
permutation.  The query of sequence b sits at position L_b - 1 and is already
appended, so visible = L_b and the SWA window holds min(128, L_b) rows.

Pools are paged in 64-token blocks; the logical blocks of all sequences are
laid out over the physical blocks by a seeded random permutation.

Long contexts (config 5, and any sequence sharded across GPUs) are drawn in
chunks of CHUNK positions, each from its own generator seeded by (config seed,
sequence, chunk): a rank that owns positions [start, start + span) draws only
the chunks it owns, and every shard count -- one GPU, two, four, eight, or the
CPU reference arm -- holds the same index keys and KV rows at every logical
position.  The queries, weights, SWA rows and sink come from one generator
seeded by the config seed, drawn on every rank alike.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK = 64
INDEX_DIM = 128
KV_DIM = 576
V_DIM = 512
SWA_ROWS = 128


@dataclass(frozen=True)
class DecodeConfig:
    name: str
    batch: int
    context: int                 # fixed context length (0 = drawn per sequence)
    heads: int                   # MLA query heads
    idx_heads: int = 64
    topk: int = 2048
    scale: float = 1 / math.sqrt(192)
    weight_scale: float = 1.0
    seed: int = 0
    context_range: tuple = field(default=(0, 0))  # inclusive range for drawn lengths

    def lengths(self, gen: torch.Generator | None = None) -> list[int]:
        if self.context:
            return [self.context] * self.batch
        lo, hi = self.context_range
        return torch.randint(lo, hi + 1, (self.batch,), generator=gen).tolist()


CONFIGS = {
    # BASELINE.json configs[0..4]
    "cfg1": DecodeConfig("cfg1: decode B=1 L=4096, MLA 16 heads", 1, 4096, 16, weight_scale=1 / 8),
    "cfg2": DecodeConfig("cfg2: decode B=1 L=131072, MLA 64 heads", 1, 131072, 64),
    "cfg3": DecodeConfig("cfg3: batched decode B=32 L~U[8192,65536]", 32, 0, 64,
                         context_range=(8192, 65536)),
    "cfg5": DecodeConfig("cfg5: decode B=4 L=1048576", 4, 1048576, 64, seed=1),
}


def small_config(base: str, **overrides) -> DecodeConfig:
    """A config with the base's geometry and overridden sizes (tests)."""
    from dataclasses import replace
    return replace(CONFIGS[base], **overrides)


def _normal_bf16(shape, gen, device):
    return torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)


def make_decode_inputs(cfg: DecodeConfig, device="cuda", gen_device="cpu", lengths=None):
    """Seeded inputs of one decode step; tensors live on `device`.

    gen_device="cpu" reproduces the documented CPU draw order exactly (tests);
    gen_device="cuda" draws on the GPU (same distributions, different stream of
    numbers) for the large benchmark pools.
    """
    gen = torch.Generator(device=gen_device)
    gen.manual_seed(cfg.seed)
    if lengths is None:
        lengths = cfg.lengths(torch.Generator().manual_seed(cfg.seed) if not cfg.context else None)
    batch = len(lengths)
    blocks_per_seq = [(n + BLOCK - 1) // BLOCK for n in lengths]
    total_blocks = sum(blocks_per_seq)
    max_blocks = max(blocks_per_seq)
    rows = total_blocks * BLOCK
    idx_q = _normal_bf16((batch, cfg.idx_heads, INDEX_DIM), gen, gen_device)
    index_pool = _normal_bf16((rows, INDEX_DIM), gen, gen_device)
    idx_w = torch.randn((batch, cfg.idx_heads), generator=gen, device=gen_device) * cfg.weight_scale
    q = _normal_bf16((batch, cfg.heads, KV_DIM), gen, gen_device)
    kv_pool = _normal_bf16((rows, KV_DIM), gen, gen_device)
    swa = _normal_bf16((batch, SWA_ROWS, KV_DIM), gen, gen_device)
    sink = torch.randn((cfg.heads,), generator=gen, device=gen_device)
    perm = torch.randperm(total_blocks, generator=gen, device=gen_device).to(torch.int32)
    table = torch.full((batch, max_blocks), -1, dtype=torch.int32)
    start = 0
    perm_cpu = perm.cpu()
    for b, nb in enumerate(blocks_per_seq):
        table[b, :nb] = perm_cpu[start:start + nb]
        start += nb
    visible = torch.tensor(lengths, dtype=torch.int32)
    swa_len = torch.clamp(visible, max=SWA_ROWS).to(torch.int32)
    out = dict(idx_q=idx_q.float(), idx_w=idx_w.float(), index_pool=index_pool, q=q.float(),
               kv_pool=kv_pool, swa=swa, sink=sink.float(), block_table=table, visible=visible,
               swa_len=swa_len)
    return {k: v.to(device).contiguous() for k, v in out.items()}, lengths


def algorithmic_bytes(lengths, heads, topk=2048, idx_heads=64):
    """Bytes one decode step must move at minimum (the roofline numerator).

    Index keys of every visible position (256 B each), the selected KV rows and
    the SWA rows (1152 B each), plus the FP32 query/weight inputs and the FP32
    output at the kernel boundary.
    """
    total = 0
    for n in lengths:
        sel = min(topk, n) + min(SWA_ROWS, n)
        total += n * INDEX_DIM * 2 + sel * KV_DIM * 2
        total += idx_heads * INDEX_DIM * 4 + idx_heads * 4 + heads * KV_DIM * 4 + heads * V_DIM * 4
    return total


# ------------------------------------------------------------- long contexts
CHUNK = 65536  # positions per seeded chunk of a long sequence (1024 pool blocks)


def _chunk_generator(cfg: DecodeConfig, seq: int, chunk: int, device) -> torch.Generator:
    gen = torch.Generator(device=device)
    gen.manual_seed((cfg.seed + 1) * 1_000_003 + seq * 65_537 + chunk)
    return gen


def chunk_rows(cfg: DecodeConfig, seq: int, chunk: int, device):
    """Index keys bf16[CHUNK, 128] and KV rows bf16[CHUNK, 576] of positions
    [chunk * CHUNK, (chunk + 1) * CHUNK) of sequence `seq`, N(0,1) rounded to BF16."""
    gen = _chunk_generator(cfg, seq, chunk, device)
    index = _normal_bf16((CHUNK, INDEX_DIM), gen, device)
    kv = _normal_bf16((CHUNK, KV_DIM), gen, device)
    return index, kv


def query_inputs(cfg: DecodeConfig, batch: int, device):
    """The step's queries and per-sequence state, identical on every rank: index q
    [B,H,128], index weights [B,H], MLA q [B,heads,576] (BF16-valued, FP32 storage),
    SWA rows bf16[B,128,576], sink f32[heads]."""
    gen = torch.Generator(device=device)
    gen.manual_seed(cfg.seed)
    idx_q = _normal_bf16((batch, cfg.idx_heads, INDEX_DIM), gen, device)
    idx_w = torch.randn((batch, cfg.idx_heads), generator=gen, device=device) * cfg.weight_scale
    q = _normal_bf16((batch, cfg.heads, KV_DIM), gen, device)
    swa = _normal_bf16((batch, SWA_ROWS, KV_DIM), gen, device)
    sink = torch.randn((cfg.heads,), generator=gen, device=device)
    return dict(idx_q=idx_q.float().contiguous(), idx_w=idx_w.float().contiguous(), q=q.float().contiguous(),
                swa=swa.contiguous(), sink=sink.float().contiguous())


def long_context_inputs(cfg: DecodeConfig, lengths, device, start: int = 0, span: int | None = None,
                        layout_seed: int = 0, sequences=None):
    """Pools holding positions [start, start + span) of every sequence (clipped to
    its length), drawn chunk by chunk (chunk_rows) and laid out in 64-row pool
    blocks by a seeded permutation.  Returns the query_inputs() tensors plus
    index_pool, kv_pool, block_table i32[B, span / 64] (local block j = positions
    start + 64j ...), visible i32[B] (owned positions) and swa_len i32[B]
    (min(128, L) for the sequences whose last position lies in the range, else 0).
    `sequences` (default all) restricts the pools to those sequences, keeping the
    batch order of the given list."""
    lengths = list(lengths)
    seqs = list(range(len(lengths))) if sequences is None else list(sequences)
    if span is None:
        span = (max(lengths) + BLOCK - 1) // BLOCK * BLOCK
    if start % BLOCK or span % BLOCK:
        raise ValueError("shard ranges are whole 64-position blocks")
    dev = torch.device(device)
    local = [max(0, min(lengths[b] - start, span)) for b in seqs]
    blocks = [(n + BLOCK - 1) // BLOCK for n in local]
    total = max(1, sum(blocks))
    index_pool = torch.zeros((total * BLOCK, INDEX_DIM), dtype=torch.bfloat16, device=dev)
    kv_pool = torch.zeros((total * BLOCK, KV_DIM), dtype=torch.bfloat16, device=dev)
    layout = torch.Generator(device=dev)
    layout.manual_seed(layout_seed)
    perm = torch.randperm(total, generator=layout, device=dev).to(torch.int32)
    table = torch.full((len(seqs), span // BLOCK), -1, dtype=torch.int32, device=dev)
    first = 0
    for i, (b, n) in enumerate(zip(seqs, local)):
        nb = blocks[i]
        table[i, :nb] = perm[first:first + nb]
        first += nb
        for c in range(start // CHUNK, (start + n - 1) // CHUNK + 1 if n else start // CHUNK):
            lo, hi = max(start, c * CHUNK), min(start + n, (c + 1) * CHUNK)
            index, kv = chunk_rows(cfg, b, c, dev)
            pos = torch.arange(lo - start, hi - start, device=dev)
            rows = table[i].long()[pos // BLOCK] * BLOCK + pos % BLOCK
            index_pool.index_copy_(0, rows, index[lo - c * CHUNK:hi - c * CHUNK])
            kv_pool.index_copy_(0, rows, kv[lo - c * CHUNK:hi - c * CHUNK])
            del index, kv
    out = query_inputs(cfg, len(lengths), dev)
    if sequences is not None:
        sel = torch.as_tensor(seqs, device=dev)
        out = {k: (v if k == "sink" else v.index_select(0, sel).contiguous()) for k, v in out.items()}
    out.update(index_pool=index_pool, kv_pool=kv_pool, block_table=table.contiguous(),
               visible=torch.tensor(local, dtype=torch.int32, device=dev),
               swa_len=torch.tensor([min(SWA_ROWS, lengths[b]) if start <= lengths[b] - 1 < start + span else 0
                                     for b in seqs], dtype=torch.int32, device=dev))
    return out
