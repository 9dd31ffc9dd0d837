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
