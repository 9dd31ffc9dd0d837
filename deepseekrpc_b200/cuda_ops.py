"""Checked device operations with the interface of the reference's cuda_ops module.

The reference wraps its `deepseekrpc_cuda` extension in checked calls
(src/deepseekrpc/cuda_ops.py:11-50): `extension()` insists on a CUDA device and
ABI generation 2, every op returns `[value, status]`, and a nonzero device
status becomes `ValidationError` after the op completes ("tentative writes
require rollback").  This module keeps those names, arguments and error
behaviour over this package's sm_100a extension, and adds the same checked
form for the fused decode-path ops.  There is no CPU fallback: without a CUDA
device or the built extension every call raises.
"""
from __future__ import annotations

import math
from functools import lru_cache


class ValidationError(ValueError):
    """An input or device state the operation refused (the reference's ValidationError)."""


@lru_cache(maxsize=1)
def extension():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("a real CUDA device is required; CPU inference fallback is not supported")
    from . import extension as load
    module = load()
    if module.abi_version() != 2:
        raise RuntimeError("native extension ABI does not match this source")
    return module


def _status(status):
    # the op is complete once its status is read: a nonzero code is a refusal
    code = int(status.item())
    if code:
        raise ValidationError(f"native CUDA operation rejected input/state (code {code}); "
                              "tentative writes require rollback")


def _result(result):
    value, status = result
    _status(status)
    return value


# ------------------------------------------------------------ reference ops
def sparse_attention(query, window_kv, source_kv, indices, sink, *, scale: float):
    if not math.isfinite(scale) or scale <= 0:
        raise ValidationError("invalid attention scale")
    return _result(extension().sparse_attention(query, window_kv, source_kv, indices, sink, scale))


def index_scores(query, keys, weights, indices, visible):
    return _result(extension().index_scores(query, keys, weights, indices, visible))


def decode_engram(encoded):
    return _result(extension().engram_decode(encoded))


def scatter_slots(pool, generations, slots, expected_generations, values):
    _status(extension().scatter_slots(pool, generations, slots, expected_generations, values))


# ----------------------------------------------------------- decode-path ops
def topk_select(scores, lengths, k: int, *, ids=None, id_base: int = 0, return_scores: bool = False):
    """Exact top-k per row (ids ascending, -1 padded); ties go to the lower id."""
    result = extension().topk_select(scores, lengths, k, ids, id_base, return_scores)
    _status(result[1])
    return (result[0], result[2]) if return_scores else result[0]


def indexer_decode(query, weights, index_pool, block_table, visible, score_stride: int):
    return _result(extension().indexer_decode(query, weights, index_pool, block_table, visible, score_stride))


def sparse_mla_decode(query, kv_pool, block_table, visible, topk, swa, swa_len, sink, *, scale: float):
    if not math.isfinite(scale) or scale <= 0:
        raise ValidationError("invalid attention scale")
    return _result(extension().sparse_mla_decode(query, kv_pool, block_table, visible, topk, swa, swa_len,
                                                 sink, scale))


def decode_step(idx_q, idx_w, index_pool, query, kv_pool, block_table, visible, max_visible: int, k: int,
                swa, swa_len, sink, *, scale: float, return_scores: bool = False):
    """Indexer -> exact top-k -> sparse MLA in one device chain; returns (out, topk[, scores])."""
    if not math.isfinite(scale) or scale <= 0:
        raise ValidationError("invalid attention scale")
    result = extension().decode_step(idx_q, idx_w, index_pool, query, kv_pool, block_table, visible,
                                     max_visible, k, swa, swa_len, sink, scale, return_scores)
    _status(result[2])
    return (result[0], result[1], result[3]) if return_scores else (result[0], result[1])


def append_kv_index(kv_pool, index_pool, generations, block_table, seq, positions, expected, kv_values,
                    index_values, swa=None):
    """Generation-checked append; a refused row raises ValidationError and was not written."""
    _status(extension().append_kv_index(kv_pool, index_pool, generations, block_table, seq, positions,
                                        expected, kv_values, index_values, swa))
