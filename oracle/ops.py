"""numpy restatement of the reference hot-path equations (test infrastructure only).

Each function cites the reference lines it follows (paths inside the
Protonburn35/DeepSeekRPC project).  Differences from the reference functions are
limited to removing their fixture-size bounds (rows <= 64, heads <= 32,
keys <= 8192, width <= 512) and to returning an error code where the CUDA op
reports one through its status tensor.
"""
from __future__ import annotations

import math

import numpy as np

ERR_ID, ERR_NONFINITE, ERR_SCATTER = 1, 2, 3


class OracleError(ValueError):
    """Raised where the reference raises ValidationError."""


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = 0x7FC0
    return rounded


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------- sparse attention (a4)
def sparse_attention(query, window_kv, source_kv, indices, sink, *, scale):
    """reference_attention.py:13-31 (sparse_attention_reference), unbounded.

    out[r,h] = sum_i e^{s_i - M} kv_i / (sum_i e^{s_i - M} + e^{sink_h - M}),
    s_i = scale * kv_i . q[r,h] over the non-padding ids of row r (duplicates
    count), M = max(sink_h, max_i s_i).  kv = concat(window, source).
    """
    query = np.asarray(query)
    if (query.ndim != 3 or window_kv.ndim != 2 or source_kv.ndim != 2 or
            query.shape[2] != window_kv.shape[1] or query.shape[2] != source_kv.shape[1] or
            indices.shape[0] != query.shape[0] or sink.shape != (query.shape[1],) or
            not math.isfinite(scale) or scale <= 0):
        raise OracleError("invalid attention fixture")
    kv = np.concatenate([window_kv, source_kv]).astype(np.float32)
    if indices.dtype != np.int32 or np.any(indices < -1) or np.any(indices >= len(kv)):
        raise OracleError("invalid sparse reference slot")
    output = np.zeros_like(query, dtype=np.float32)
    for row in range(len(query)):
        selected = kv[indices[row][indices[row] >= 0]]
        for head in range(query.shape[1]):
            logits = selected @ query[row, head].astype(np.float32) * np.float32(scale)
            maximum = max(float(sink[head]), float(np.max(logits, initial=-np.inf)))
            exp = np.exp(logits - maximum)
            output[row, head] = (exp @ selected) / (exp.sum() + np.exp(np.float32(sink[head] - maximum)))
    return output


# ----------------------------------------------------------- index scores (a1)
def index_scores(query, keys, weights, indices, visible):
    """reference_attention.py:34-47 (index_scores_reference), unbounded.

    out[r,c] = sum_h w[r,h] * max(q[r,h] . keys[id], 0) for 0 <= id < visible[r],
    -inf otherwise (padding -1 or id >= visible).
    """
    if (query.ndim != 3 or query.shape[2] != 128 or keys.ndim != 2 or keys.shape[1] != 128 or
            weights.shape != query.shape[:2] or indices.ndim != 2 or indices.shape[0] != len(query) or
            visible.shape != (len(query),) or np.any(visible < 0) or np.any(visible > len(keys))):
        raise OracleError("invalid index fixture")
    if indices.dtype != np.int32 or np.any(indices < -1) or np.any(indices >= len(keys)):
        raise OracleError("invalid index reference slot")
    out = np.full(indices.shape, -np.inf, dtype=np.float32)
    for row in range(len(query)):
        valid = (indices[row] >= 0) & (indices[row] < visible[row])
        dot = query[row].astype(np.float32) @ keys[indices[row, valid]].astype(np.float32).T
        out[row, valid] = (np.maximum(dot, 0) * weights[row, :, None]).sum(axis=0)
    return out


# ------------------------------------------------------------- top-k (a2, a3)
def merge_ranked(scores, ids, new_scores, new_ids, *, keep):
    """index_selection.py:9-19: exact streaming ranking, lower ids break ties.

    Stable argsort by id, then stable descending argsort by score (-0.0 == +0.0).
    torch's descending sort ranks NaN above +inf; numpy's would rank it last, so
    NaN is ordered by a leading key of its own.
    """
    scores = np.concatenate([np.asarray(scores, np.float32), np.asarray(new_scores, np.float32)])
    ids = np.concatenate([np.asarray(ids, np.int64), np.asarray(new_ids, np.int64)])
    order = np.argsort(ids, kind="stable")
    s = scores[order]
    nan = np.isnan(s)
    order = order[np.lexsort((np.where(nan, np.float32(0), -s), ~nan))[:keep]]
    return scores[order], ids[order]


def tiled_topk(scores_row, keep, *, tile_rows=8192, positions=None):
    """TiledIndexer._select's dense selection (index_selection.py:79-120) for one row.

    scores_row[i] is the score of logical position positions[i] (default i).
    Tiles of tile_rows positions are merged with merge_ranked(keep); the chosen
    ids are returned sorted ascending and padded with -1 to `keep`.
    """
    scores_row = np.asarray(scores_row, np.float32)
    n = len(scores_row)
    positions = np.arange(n, dtype=np.int64) if positions is None else np.asarray(positions, np.int64)
    best_s = np.empty(0, np.float32)
    best_i = np.empty(0, np.int64)
    for start in range(0, n, tile_rows):
        best_s, best_i = merge_ranked(best_s, best_i, scores_row[start:start + tile_rows],
                                      positions[start:start + tile_rows], keep=keep)
    out = np.full(keep, -1, np.int32)
    chosen = np.sort(best_i).astype(np.int32)
    out[:len(chosen)] = chosen
    return out


# ------------------------------------------------------ candidate blocks (a2)
def candidate_blocks(scores_row, visible, keep=2048, *, tile_rows=8192):
    """TiledIndexer._select's candidate production (index_selection.py:108-119) for one row.

    Per tile of tile_rows positions, the scores (padded with -inf to a multiple
    of 8) are max-reduced over blocks of 8 positions, the block holding position
    visible-1 is pinned to +inf, and the blocks are ranked with merge_ranked
    (keep); the chosen block ids come back sorted ascending, -1 padded to `keep`.
    """
    scores_row = np.asarray(scores_row, np.float32)[:visible]
    best_s = np.empty(0, np.float32)
    best_i = np.empty(0, np.int64)
    for start in range(0, visible, tile_rows):
        tile = scores_row[start:start + tile_rows]
        if len(tile) % 8:
            tile = np.concatenate([tile, np.full(8 - len(tile) % 8, -np.inf, np.float32)])
        blocks = tile.reshape(-1, 8)
        reduced = np.where(np.isnan(blocks).any(axis=1), np.float32(np.nan), blocks.max(axis=1)).astype(np.float32)
        ids = np.arange(start // 8, start // 8 + len(reduced), dtype=np.int64)
        reduced[ids == (visible - 1) // 8] = np.inf
        best_s, best_i = merge_ranked(best_s, best_i, reduced, ids, keep=keep)
    out = np.full(keep, -1, np.int32)
    chosen = np.sort(best_i).astype(np.int32)
    out[:len(chosen)] = chosen
    return out


def candidate_positions(blocks_row, visible):
    """Logical positions a candidate-restricted indexer scores (index_selection.py:62-90):
    every position of each listed block (ascending, -1 padded) below `visible`.
    Raises OracleError where the reference raises ValidationError: blocks not
    strictly increasing, a block after padding, a block past the visible keys,
    or no position at all for a nonempty query."""
    last, padded, positions = -1, False, []
    for block in blocks_row:
        block = int(block)
        if block == -1:
            padded = True
            continue
        if padded or block <= last or not 0 <= block < (visible + 7) // 8:
            raise OracleError("candidate blocks are stale, duplicated or out of order")
        last = block
        positions.extend(range(block * 8, min(block * 8 + 8, visible)))
    if visible and not positions:
        raise OracleError("a nonempty index query has no published candidate blocks")
    return np.asarray(positions, np.int64)


# --------------------------------------------------------------- scatter (a6)
def scatter_slots(pool_bits, generations, slots, expected, value_bits):
    """native/operations.cu:144-161 (scatter_kernel) semantics on bf16 bit arrays.

    In place on pool_bits; returns the status code (0 = ok).  A row is refused
    (code 3) when its slot is out of bounds, repeats an earlier row's slot, or
    its generation differs from expected; elements whose bf16 exponent is all
    ones are skipped with code 2.  Generations are not modified.
    """
    code = 0
    capacity = len(pool_bits)
    for row, slot in enumerate(slots.tolist()):
        valid = 0 <= slot < capacity and slot not in slots[:row].tolist()
        if not valid or generations[slot] != expected[row]:
            code = code or ERR_SCATTER
            continue
        values = value_bits[row]
        bad = (values & 0x7F80) == 0x7F80
        if bad.any():
            code = code or ERR_NONFINITE
        pool_bits[slot, ~bad] = values[~bad]
    return code


# ---------------------------------------------------------------- engram decode
def engram_decode(encoded):
    """native/operations.cu:125-142 / engram_storage.py:103-119: FP8 E4M3 x UE8M0 -> bf16 bits.

    Returns (bits uint16[rows,256], code).  NaN encodings and a 255 scale give
    code 2 and value 0, as the CUDA kernel does.
    """
    encoded = np.asarray(encoded, np.uint8)
    values = encoded[:, :256]
    exponent = ((values >> 3) & 15).astype(np.int32)
    mantissa = (values & 7).astype(np.float32)
    magnitude = np.where(exponent == 0, np.ldexp(mantissa, -9),
                         np.ldexp(1 + mantissa / 8, exponent - 7)).astype(np.float32)
    magnitude = np.where((values & 128) != 0, -magnitude, magnitude)
    scales = encoded[:, 256:]
    scale_values = np.ldexp(np.ones(scales.shape, dtype=np.float32), scales.astype(np.int32) - 127)
    with np.errstate(over="ignore", invalid="ignore"):
        output = (magnitude.reshape(-1, 8, 32) * scale_values[..., None]).reshape(-1, 256)
    nan_code = ((exponent == 15) & (mantissa == 7)) | (np.repeat(scales, 32, axis=1) == 255)
    code = 0
    if nan_code.any():
        code = ERR_NONFINITE
    output = np.where(nan_code, np.float32(0), output).astype(np.float32)
    bits = f32_to_bf16_bits(output)
    if not np.all(np.isfinite(output[~nan_code])) or not np.all(np.isfinite(bf16_bits_to_f32(bits))):
        code = code or ERR_NONFINITE
    return bits, code


# ------------------------------------------------------ paged decode step (new)
def gather_rows(pool, block_table_row, positions):
    """Rows of a paged pool [blocks*64, width] for logical positions."""
    positions = np.asarray(positions, np.int64)
    return pool[block_table_row[positions // 64].astype(np.int64) * 64 + positions % 64]


def decode_step(idx_q, idx_w, index_pool, q, kv_pool, block_table, visible, k, swa, swa_len, sink,
                scale, *, dv=512, tile_rows=8192, return_scores=False):
    """Reference decode step on paged pools, composed from the reference equations.

    Per sequence b: the lightning-indexer scores of positions [0, visible[b])
    (index_scores over the keys gathered through the block table), the exact
    top-k of TiledIndexer (tiles of tile_rows, merge_ranked), then
    sparse_attention of q[b] over [SWA rows ; selected KV rows] with the sink,
    keeping the first dv output columns (the MLA value width).
    Pools are float32 arrays holding bf16 values.
    """
    batch = len(q)
    out = np.zeros((batch, q.shape[1], dv), np.float32)
    topk = np.full((batch, k), -1, np.int32)
    scores_all = []
    for b in range(batch):
        n = int(visible[b])
        keys = gather_rows(index_pool, block_table[b], np.arange(n))
        ids = np.arange(n, dtype=np.int32)[None]
        scores = index_scores(idx_q[b:b + 1], keys, idx_w[b:b + 1], ids, np.array([n], np.int32))[0]
        scores_all.append(scores)
        topk[b] = tiled_topk(scores, k, tile_rows=tile_rows)
        chosen = topk[b][topk[b] >= 0]
        source = gather_rows(kv_pool, block_table[b], chosen)
        window = swa[b, :int(swa_len[b])]
        sel = np.arange(len(window) + len(source), dtype=np.int32)[None]
        out[b] = sparse_attention(q[b:b + 1], window, source, sel, sink, scale=scale)[0, :, :dv]
    if return_scores:
        return out, topk, scores_all
    return out, topk
