"""C-ABI call wrappers and reference computations shared by the GPU tests."""
from __future__ import annotations

import numpy as np
import torch

import oracle
from deepseekrpc_b200 import _native
from deepseekrpc_b200._native import call, ptr, stream_handle


def dev(array, dtype=None):
    t = torch.as_tensor(np.asarray(array))
    if dtype is not None:
        t = t.to(dtype)
    return t.contiguous().cuda()


def bf16_from_bits(bits):
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16).contiguous().cuda()


def status():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def finish(err):
    torch.cuda.synchronize()
    return int(err.item())


# ---------------------------------------------------------------- legacy ops
def c_index_scores(q, keys, w, ids, visible):
    out = torch.empty(ids.shape, dtype=torch.float32, device="cuda")
    err = status()
    call("dsr_index_scores", ptr(q), ptr(keys), ptr(w), ptr(ids), ptr(visible), ptr(out), ptr(err),
         q.shape[0], q.shape[1], ids.shape[1], keys.shape[0], stream_handle())
    return out, finish(err)


def c_sparse_attention(q, window, source, ids, sink, scale):
    out = torch.empty_like(q)
    err = status()
    call("dsr_sparse_attention", ptr(q), ptr(window), ptr(source), ptr(ids), ptr(sink), ptr(out),
         ptr(err), q.shape[0], q.shape[1], q.shape[2], window.shape[0], source.shape[0], ids.shape[1],
         float(scale), stream_handle())
    return out, finish(err)


def c_scatter(pool, generations, slots, expected, values):
    err = status()
    call("dsr_scatter_slots", ptr(pool), ptr(generations), ptr(slots), ptr(expected), ptr(values),
         ptr(err), slots.shape[0], pool.shape[1], pool.shape[0], stream_handle())
    return finish(err)


def c_engram(encoded):
    out = torch.empty((encoded.shape[0], 256), dtype=torch.bfloat16, device="cuda")
    err = status()
    call("dsr_engram_decode", ptr(encoded), ptr(out), ptr(err), encoded.shape[0], stream_handle())
    return out, finish(err)


# ------------------------------------------------------------------- top-k
def c_topk(scores, lengths, k, ids=None, id_base=0, return_scores=False):
    rows, stride = scores.shape
    out = torch.empty((rows, k), dtype=torch.int32, device="cuda")
    out_s = torch.empty((rows, k), dtype=torch.float32, device="cuda") if return_scores else None
    err = status()
    ws_bytes = _native.library().dsr_topk_workspace_bytes(rows, stride)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    call("dsr_topk_select", ptr(scores), ptr(ids), ptr(lengths), ptr(out), ptr(out_s), ptr(err), rows,
         stride, k, id_base, ptr(ws), ws_bytes, stream_handle())
    c_topk.last_ws = ws
    code = finish(err)
    return (out, out_s, code) if return_scores else (out, code)


# ------------------------------------------------------------ decode path
def c_indexer(inp, score_stride=None):
    b = inp["idx_q"].shape[0]
    stride = score_stride or inp["block_table"].shape[1] * 64
    scores = torch.full((b, stride), float("nan"), dtype=torch.float32, device="cuda")
    err = status()
    call("dsr_indexer_decode", ptr(inp["idx_q"]), ptr(inp["idx_w"]), ptr(inp["index_pool"]),
         inp["index_pool"].shape[0] // 64, ptr(inp["block_table"]), inp["block_table"].shape[1],
         ptr(inp["visible"]), ptr(scores), stride, ptr(err), b, inp["idx_q"].shape[1], stream_handle())
    return scores, finish(err)


def c_mla(inp, topk, scale):
    b, h = inp["q"].shape[:2]
    k = topk.shape[1]
    ws_bytes = _native.library().dsr_mla_workspace_bytes(b, h, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((b, h, 512), dtype=torch.float32, device="cuda")
    err = status()
    call("dsr_sparse_mla_decode", ptr(inp["q"]), ptr(inp["kv_pool"]), inp["kv_pool"].shape[0] // 64,
         ptr(inp["block_table"]), inp["block_table"].shape[1], ptr(inp["visible"]), ptr(topk), k,
         ptr(inp["swa"]), ptr(inp["swa_len"]), ptr(inp["sink"]), float(scale), ptr(out), ptr(ws), ws_bytes,
         ptr(err), b, h, stream_handle())
    return out, finish(err)


def c_decode_step(inp, k, scale, return_scores=True):
    b, h = inp["q"].shape[:2]
    max_visible = int(inp["visible"].max().item())
    stride = (max_visible + 63) // 64 * 64
    lib = _native.library()
    ws_bytes = lib.dsr_decode_workspace_bytes(b, max_visible, h, k)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((b, h, 512), dtype=torch.float32, device="cuda")
    topk = torch.empty((b, k), dtype=torch.int32, device="cuda")
    scores = torch.full((b, stride), float("nan"), dtype=torch.float32, device="cuda") if return_scores else None
    err = status()
    call("dsr_decode_step", ptr(inp["idx_q"]), ptr(inp["idx_w"]), inp["idx_q"].shape[1],
         ptr(inp["index_pool"]), ptr(inp["q"]), ptr(inp["kv_pool"]), h, inp["kv_pool"].shape[0] // 64,
         ptr(inp["block_table"]), inp["block_table"].shape[1], ptr(inp["visible"]), max_visible, k,
         ptr(inp["swa"]), ptr(inp["swa_len"]), ptr(inp["sink"]), float(scale), ptr(out), ptr(topk),
         ptr(scores), ptr(ws), ws_bytes, ptr(err), b, stream_handle())
    return out, topk, scores, finish(err)


# ------------------------------------------------------- oracle references
def host(inp):
    """float32 numpy copies of a decode input dict."""
    result = {}
    for key, value in inp.items():
        v = value.float() if value.dtype == torch.bfloat16 else value
        result[key] = v.cpu().numpy()
    return result


def oracle_scores(h, b):
    n = int(h["visible"][b])
    keys = oracle.gather_rows(h["index_pool"], h["block_table"][b], np.arange(n))
    return oracle.index_scores(h["idx_q"][b:b + 1], keys, h["idx_w"][b:b + 1],
                               np.arange(n, dtype=np.int32)[None], np.array([n], np.int32))[0]


def score_bound(h, b):
    """sum_h |w_h| * |q_h . k| per key: the scale of the score's rounding error."""
    n = int(h["visible"][b])
    keys = oracle.gather_rows(h["index_pool"], h["block_table"][b], np.arange(n)).astype(np.float64)
    dot = h["idx_q"][b].astype(np.float64) @ keys.T
    return (np.abs(h["idx_w"][b])[:, None] * np.abs(dot)).sum(0)


def oracle_attention(h, b, ids, scale):
    chosen = ids[ids >= 0]
    source = oracle.gather_rows(h["kv_pool"], h["block_table"][b], chosen)
    window = h["swa"][b, :int(h["swa_len"][b])]
    sel = np.arange(len(window) + len(source), dtype=np.int32)[None]
    return oracle.sparse_attention(h["q"][b:b + 1], window, source, sel, h["sink"], scale=scale)[0, :, :512]


def assert_bf16_close(actual, expected, max_abs=2e-2, mean_abs=2e-3):
    diff = np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))
    assert np.all(np.isfinite(actual))
    assert diff.max() <= max_abs, f"max abs error {diff.max():.3e} > {max_abs}"
    assert diff.mean() <= mean_abs, f"mean abs error {diff.mean():.3e} > {mean_abs}"


def score_stats(got, ref, bound, rtol=1e-3):
    """Agreement of GPU index scores with the oracle's.

    The pass criterion is |got - ref| <= rtol * bound + 1e-6 with bound =
    sum_h |w_h| |q_h . k| (the magnitude that bounds the rounding of a sum of
    signed-weight terms, which can cancel to near zero).  Reported beside it:
    the plain relative error |got - ref| / |ref| (max over keys with |ref| above
    1e-3 of its bound, where cancellation is mild) and the share of all keys
    within rtol plain relative error (|ref| = 0 counts only when got is 0 too).
    """
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bound = np.asarray(bound, np.float64)
    err = np.abs(got - ref)
    mild = np.abs(ref) > 1e-3 * bound
    rel = err / np.maximum(np.abs(ref), 1e-300)
    return {
        "keys": int(len(ref)),
        "within_bound": bool(np.all(err <= rtol * bound + 1e-6)),
        "max_err_over_bound": float(np.max(err / (bound + 1e-30))) if len(ref) else 0.0,
        "max_rel_mild": float(np.max(rel[mild])) if mild.any() else 0.0,
        "share_rel_within": float(np.mean(err <= rtol * np.abs(ref))) if len(ref) else 1.0,
    }


def assert_scores(got, ref, bound, rtol=1e-3, min_share=0.999, what="scores"):
    """Every key within rtol of the bound; at most max(2, (1 - min_share) * keys)
    keys beyond rtol plain relative error (a short sequence may hold one or two
    keys whose head terms cancel to ~1e-4 of the bound)."""
    stats = score_stats(got, ref, bound, rtol)
    assert np.all(np.isfinite(got)), f"{what}: non-finite score"
    assert stats["within_bound"], f"{what}: {stats}"
    n = stats["keys"]
    bad = round((1.0 - stats["share_rel_within"]) * n)
    assert bad <= max(2, int((1.0 - min_share) * n)), f"{what}: {stats}"
    print(f"{what}: {stats}")
    return stats
