"""Index selection with the interface of the reference's TiledIndexer, on the
fused sm_100a kernels.

The reference (src/deepseekrpc/index_selection.py:9-124) scores a query's
visible logical positions tile by tile through `index_scores`, ranks them with
`merge_ranked` (higher score first, lower logical id on ties) keeping 512, and
can also produce 2048 candidate blocks of 8 positions (block maximum, newest
block pinned) or restrict a later indexer to such blocks.  Here every step runs
on the device: one kernel scores all visible positions of every row through the
paged pool's block table and a second selects the exact top-k from the
indexer's own score histogram; the candidate modes are two more device passes.
Tiling does not change an exact selection, so `tile_rows` is kept for interface
parity and validated only.  Rows of a selection share one pool; there is no CPU
fallback.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from .cuda_ops import ValidationError


def merge_ranked(scores, ids, new_scores, new_ids, *, keep: int):
    """Exact ranking of two (score, id) lists: higher score first, then lower id;
    -0.0 equals +0.0 (index_selection.py:9-19).  Runs on the tensors' device."""
    scores, ids = torch.cat((scores, new_scores)), torch.cat((ids, new_ids))
    by_id = torch.argsort(ids, stable=True)
    order = by_id[torch.argsort(scores[by_id], descending=True, stable=True)[:keep]]
    return scores[order], ids[order]


@dataclass(frozen=True)
class IndexSelection:
    topk: torch.Tensor                      # i32 [rows, keep], ascending, -1 padded
    candidate_blocks: torch.Tensor | None   # i32 [rows, 2048] when produced


@dataclass(frozen=True)
class PagedIndexKeys:
    """The index-key pool of a batch of sequences: bf16 [pool_blocks*64, 128] rows
    and an i32 [rows, table_stride] block table (logical block j -> physical block)."""
    pool: torch.Tensor
    block_table: torch.Tensor

    @property
    def device(self):
        return self.pool.device


def _integer(value, what, low, high):
    if isinstance(value, bool) or not isinstance(value, int) or not low <= value <= high:
        raise ValidationError(f"{what} must be an integer in [{low}, {high}]")
    return value


class TiledIndexer:
    """Dense or candidate-restricted top-k selection of logical key positions."""

    def __init__(self, *, tile_rows: int = 8192, keep: int = 512, candidate_keep: int = 2048):
        self.tile_rows = _integer(tile_rows, "index key tile rows", 8, 8192)
        if tile_rows % 8:
            raise ValidationError("index key tiles must align with candidate blocks of eight")
        self.keep = _integer(keep, "selected keys", 1, 8192)
        self.candidate_keep = _integer(candidate_keep, "candidate blocks", 1, 8192)

    def select(self, pool: PagedIndexKeys, query, weights, visible_counts, *, produce_candidates: bool = False,
               candidate_blocks=None) -> IndexSelection:
        rows = len(visible_counts)
        table = pool.block_table
        if (not query.is_cuda or query.dtype != torch.float32 or query.dim() != 3 or query.shape[0] != rows or
                query.shape[1] not in (16, 32, 64) or query.shape[2] != 128 or not query.is_contiguous() or
                weights.device != query.device or weights.dtype != torch.float32 or
                weights.shape != query.shape[:2] or not weights.is_contiguous() or
                pool.pool.device != query.device or pool.pool.dtype != torch.bfloat16 or
                pool.pool.dim() != 2 or pool.pool.shape[1] != 128 or pool.pool.shape[0] % 64 or
                table.device != query.device or table.dtype != torch.int32 or table.dim() != 2 or
                table.shape[0] != rows or not table.is_contiguous() or
                (produce_candidates and candidate_blocks is not None)):
            raise ValidationError("index selection state, precision, query geometry or candidate mode mismatch")
        for visible in visible_counts:
            _integer(int(visible), "visible logical index keys", 0, table.shape[1] * 64)
        visible = torch.tensor([int(v) for v in visible_counts], dtype=torch.int32, device=query.device)
        err = torch.zeros(1, dtype=torch.int32, device=query.device)
        lib, p = _native.library(), _native.ptr
        stream = _native.stream_handle()
        heads, pool_blocks = query.shape[1], pool.pool.shape[0] // 64
        topk = torch.empty((rows, self.keep), dtype=torch.int32, device=query.device)
        blocks_out = None
        if candidate_blocks is not None:
            if (candidate_blocks.dtype != torch.int32 or candidate_blocks.device != query.device or
                    candidate_blocks.dim() != 2 or candidate_blocks.shape[0] != rows or
                    not candidate_blocks.is_contiguous()):
                raise ValidationError("candidate block tensor does not match the pinned topology")
            ncand = candidate_blocks.shape[1]
            ws_bytes = lib.dsr_candidate_select_workspace_bytes(rows, ncand)
            ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=query.device)
            _native.call("dsr_candidate_select", p(query), p(weights), heads, p(pool.pool), pool_blocks, p(table),
                         table.shape[1], p(visible), p(candidate_blocks), ncand, self.keep, p(topk), p(ws), ws_bytes,
                         p(err), rows, stream)
        else:
            max_visible = max(1, int(visible.max().item()) if rows else 1)
            stride = (max_visible + 63) // 64 * 64
            scores = torch.empty((rows, stride), device=query.device) if produce_candidates else None
            ws_bytes = lib.dsr_indexer_topk_workspace_bytes(rows, max_visible)
            ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=query.device)
            _native.call("dsr_indexer_topk_decode", p(query), p(weights), heads, p(pool.pool), pool_blocks, p(table),
                         table.shape[1], p(visible), max_visible, self.keep, 0, p(topk), None, p(scores), p(ws),
                         ws_bytes, p(err), rows, stream)
            if produce_candidates:
                blocks_out = torch.empty((rows, self.candidate_keep), dtype=torch.int32, device=query.device)
                cb_bytes = lib.dsr_candidate_blocks_workspace_bytes(rows, stride, self.candidate_keep)
                cb_ws = torch.zeros(cb_bytes, dtype=torch.uint8, device=query.device)
                _native.call("dsr_candidate_blocks", p(scores), p(visible), rows, stride, self.candidate_keep,
                             p(blocks_out), p(cb_ws), cb_bytes, p(err), stream)
        code = int(err.item())
        if code:
            raise ValidationError(f"index selection rejected its input or pool state (code {code})")
        return IndexSelection(topk, blocks_out)
