"""Ring-offset pools -- the reference's own pool layout -- on the B200.

The reference keeps one flat pool per (kind, layer) in which logical row p lives
at slot (p + offset) % slots, the offset a SHA-256 hash of (run, role, kind,
layer) (bootstrap.py:185-192, cache_pool.py:24-113).  Here the same logical rows
are laid out both ways -- paged (a seeded block permutation) and ring-offset
(hash-like offsets, not multiples of 64, wrapping around the end of the slots,
several sequences' regions in one tensor) -- and the ring entry points must give
the paged ones' scores bit for bit, the same top-k, attention within the
oracle's tolerance, and the oracle's append (two pools, two generation arrays).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import oracle
from oracle.append import ERR_NONFINITE, ERR_SCATTER, append_kv_index_ring, ring_rows
from _helpers import assert_bf16_close, c_decode_step, c_indexer, finish, host, oracle_attention, status
from deepseekrpc_b200 import _native
from deepseekrpc_b200._native import call, ptr, stream_handle
from deepseekrpc_b200.workloads import CONFIGS, make_decode_inputs, small_config

pytestmark = pytest.mark.gpu


def hashed_offset(kind: str, layer: int, slots: int) -> int:
    """An offset drawn the way the reference's boot draws its pools' offsets."""
    digest = hashlib.sha256(f"ring-test/2/{kind}/{layer}".encode()).digest()
    return int.from_bytes(digest[:8], "little") % slots


def ring_layout(lengths, kind, extra=(37, 0, 515, 3)):
    """Ring descriptors i64[B,3] for regions packed one after another: slots =
    length + extra (at least 1), hash-like offsets; returns (ring, rows)."""
    ring, first = [], 0
    for b, n in enumerate(lengths):
        slots = max(1, n + extra[b % len(extra)])
        ring.append((first, slots, hashed_offset(kind, b, slots)))
        first += slots
    return np.asarray(ring, np.int64), first


def to_ring(pool, table, lengths, ring, rows, width):
    """The logical rows of paged pool `pool` placed at their ring rows (other rows: NaN
    bit patterns, so that any read of a wrong row shows)."""
    out = torch.full((rows, width), float("nan"), dtype=torch.bfloat16, device="cuda")
    for b, n in enumerate(lengths):
        pos = torch.arange(n, device="cuda")
        src = table[b].long()[pos // 64] * 64 + pos % 64
        first, slots, offset = (int(x) for x in ring[b])
        dst = first + (pos + offset) % slots
        out[dst] = pool[src]
    return out.contiguous()


def ring_inputs(inp, lengths):
    """Ring-offset copies of a paged decode input: index and KV pools with their own
    offsets, and the SWA ring as a 128-slot windows pool per sequence."""
    ix_ring, ix_rows = ring_layout(lengths, "index_keys")
    kv_ring, kv_rows = ring_layout(lengths, "sources", extra=(5, 64, 1, 300))
    out = dict(inp)
    out["index_pool"] = to_ring(inp["index_pool"], inp["block_table"], lengths, ix_ring, ix_rows, 128)
    out["kv_pool"] = to_ring(inp["kv_pool"], inp["block_table"], lengths, kv_ring, kv_rows, 576)
    # windows pools: slot (p + offset) % 128 holds position p (paged layout: slot p % 128)
    B = len(lengths)
    swa_ring = np.asarray([(128 * b, 128, hashed_offset("windows", b, 128)) for b in range(B)], np.int64)
    swa = torch.empty((B * 128, 576), dtype=torch.bfloat16, device="cuda")
    for b, n in enumerate(lengths):
        for p in range(max(0, n - 128), n):
            swa[128 * b + (p + int(swa_ring[b, 2])) % 128] = inp["swa"][b, p % 128]
    out["swa_pool"] = swa
    out["rings"] = {k: torch.from_numpy(v).cuda() for k, v in
                    (("index", ix_ring), ("kv", kv_ring), ("swa", swa_ring))}
    out["rows"] = {"index": ix_rows, "kv": kv_rows, "swa": B * 128}
    return out


LENGTHS = [9000, 130, 4096, 20001]


def test_ring_layouts_wrap_at_unaligned_offsets():
    wraps = []
    for kind, extra in (("index_keys", (37, 0, 515, 3)), ("sources", (5, 64, 1, 300))):
        ring, _ = ring_layout(LENGTHS, kind, extra)
        for (first, slots, offset), n in zip(ring, LENGTHS):
            assert offset % 64, "offsets off the 64-row grid"
            wraps.append(n > int(slots) - int(offset))
            if wraps[-1]:
                assert (int(slots) - int(offset)) % 128, "the wrap falls inside a 128-key tile"
    assert any(wraps) and not all(wraps), "the layouts hold wrapping and non-wrapping sequences"


def c_indexer_ring(r, stride):
    b = r["idx_q"].shape[0]
    scores = torch.full((b, stride), float("nan"), device="cuda")
    err = status()
    call("dsr_indexer_decode_ring", ptr(r["idx_q"]), ptr(r["idx_w"]), ptr(r["index_pool"]), r["rows"]["index"],
         ptr(r["rings"]["index"]), ptr(r["visible"]), ptr(scores), stride, ptr(err), b, r["idx_q"].shape[1],
         stream_handle())
    return scores, finish(err)


def c_decode_step_ring(r, k, scale):
    b, h = r["q"].shape[:2]
    max_visible = int(r["visible"].max().item())
    stride = (max_visible + 63) // 64 * 64
    ws_bytes = _native.library().dsr_decode_workspace_bytes(b, max_visible, h, k)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty((b, h, 512), device="cuda")
    topk = torch.empty((b, k), dtype=torch.int32, device="cuda")
    scores = torch.full((b, stride), float("nan"), device="cuda")
    err = status()
    call("dsr_decode_step_ring", ptr(r["idx_q"]), ptr(r["idx_w"]), r["idx_q"].shape[1], ptr(r["index_pool"]),
         r["rows"]["index"], ptr(r["rings"]["index"]), ptr(r["q"]), ptr(r["kv_pool"]), r["rows"]["kv"],
         ptr(r["rings"]["kv"]), h, ptr(r["visible"]), max_visible, k, ptr(r["swa_pool"]), r["rows"]["swa"],
         ptr(r["rings"]["swa"]), ptr(r["swa_len"]), ptr(r["sink"]), float(scale), ptr(out), ptr(topk), ptr(scores),
         ptr(ws), ws_bytes, ptr(err), b, stream_handle())
    return out, topk, scores, finish(err)


def test_ring_indexer_equals_the_paged_indexer(cuda):
    cfg = small_config("cfg3", batch=len(LENGTHS), seed=61)
    inp, lengths = make_decode_inputs(cfg, lengths=LENGTHS)
    r = ring_inputs(inp, lengths)
    stride = inp["block_table"].shape[1] * 64
    paged, code = c_indexer(inp, stride)
    assert code == 0
    ring, code = c_indexer_ring(r, stride)
    assert code == 0
    for b, n in enumerate(lengths):
        assert torch.equal(ring[b, :n], paged[b, :n]), f"sequence {b}: ring scores differ from the paged ones"
        assert torch.isnan(ring[b, n:]).all(), "nothing is written past the visible keys"


def test_ring_decode_step_matches_the_paged_step_and_the_oracle(cuda):
    cfg = small_config("cfg3", batch=len(LENGTHS), seed=62)
    inp, lengths = make_decode_inputs(cfg, lengths=LENGTHS)
    r = ring_inputs(inp, lengths)
    out_p, topk_p, scores_p, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    out_r, topk_r, scores_r, code = c_decode_step_ring(r, cfg.topk, cfg.scale)
    assert code == 0
    assert torch.equal(topk_r, topk_p), "the ring step selected other rows"
    h = host(inp)
    t = topk_r.cpu().numpy()
    for b in range(len(lengths)):
        assert torch.equal(scores_r[b, :lengths[b]], scores_p[b, :lengths[b]])
        assert_bf16_close(out_r[b].cpu().numpy(), oracle_attention(h, b, t[b], cfg.scale))
    assert (out_r - out_p).abs().max().item() < 1e-3


def test_ring_decode_step_at_the_million_key_geometry(cuda):
    """Four ragged sequences near 1,048,576 keys: every CTA's score range spans
    more than one staging chunk, so the selection stages only the 32-key groups
    whose maxima reach the threshold bin, and in the wrapped second run those
    groups start at positions off the 128-key tile grid."""
    cfg = CONFIGS["cfg5"]
    lengths = [1048576, 1000003, 917505, 1040001]
    inp, lengths = make_decode_inputs(cfg, device="cuda", gen_device="cuda", lengths=lengths)
    r = ring_inputs(inp, lengths)
    out_p, topk_p, scores_p, code = c_decode_step(inp, cfg.topk, cfg.scale)
    assert code == 0
    out_r, topk_r, scores_r, code = c_decode_step_ring(r, cfg.topk, cfg.scale)
    assert code == 0
    assert torch.equal(topk_r, topk_p), "the ring step selected other rows"
    for b, n in enumerate(lengths):
        assert torch.equal(scores_r[b, :n], scores_p[b, :n]), f"sequence {b}: ring scores differ"
    t, s = topk_r.cpu().numpy(), scores_r.cpu().numpy()
    for b, n in enumerate(lengths):
        assert np.array_equal(t[b], oracle.tiled_topk(s[b, :n], cfg.topk)), f"sequence {b}: top-k differs"
    assert (out_r - out_p).abs().max().item() < 1e-3


def test_ring_visibility_beyond_the_slots_is_refused(cuda):
    cfg = small_config("cfg3", batch=2, seed=63)
    inp, lengths = make_decode_inputs(cfg, lengths=[3000, 500])
    r = ring_inputs(inp, lengths)
    ring = r["rings"]["index"].clone()
    ring[1, 1] = 499  # slots below the visible count
    r["rings"] = dict(r["rings"], index=ring)
    _, code = c_indexer_ring(r, 3008)
    assert code == 1
    ring = r["rings"]["index"].clone()
    ring[1, 1], ring[1, 2] = 600, 600  # offset outside [0, slots)
    r["rings"] = dict(r["rings"], index=ring)
    _, code = c_indexer_ring(r, 3008)
    assert code == 1


def test_ring_append_two_pools_against_the_oracle(cuda):
    rng = np.random.default_rng(64)
    lengths = [300, 5000, 64, 1200]
    kv_ring, kv_rows = ring_layout(lengths, "sources")
    ix_ring, ix_rows = ring_layout(lengths, "index_keys", extra=(1, 9, 200, 77))
    kv = oracle.f32_to_bf16_bits(rng.normal(size=(kv_rows, 576)).astype(np.float32))
    ix = oracle.f32_to_bf16_bits(rng.normal(size=(ix_rows, 128)).astype(np.float32))
    kv_gen = rng.integers(0, 4, size=kv_rows).astype(np.int64)
    ix_gen = rng.integers(0, 4, size=ix_rows).astype(np.int64)
    dev = {name: torch.from_numpy(a.copy() if a.dtype != np.uint16 else a.view(np.int16).copy()).cuda()
           for name, a in (("kv", kv), ("ix", ix), ("kv_gen", kv_gen), ("ix_gen", ix_gen))}
    d_kv_ring, d_ix_ring = torch.from_numpy(kv_ring).cuda(), torch.from_numpy(ix_ring).cuda()

    def append(seq, positions, kv_exp, ix_exp, kv_vals, ix_vals):
        err = status()
        # every argument tensor stays referenced until the launch has completed
        args = dict(kv_exp=torch.tensor(kv_exp, dtype=torch.int64, device="cuda"),
                    ix_exp=torch.tensor(ix_exp, dtype=torch.int64, device="cuda"),
                    seq=torch.tensor(seq, dtype=torch.int32, device="cuda"),
                    pos=torch.tensor(positions, dtype=torch.int32, device="cuda"),
                    kv_vals=torch.from_numpy(kv_vals.view(np.int16)).cuda(),
                    ix_vals=torch.from_numpy(ix_vals.view(np.int16)).cuda())
        call("dsr_append_kv_index_ring", ptr(dev["kv"]), kv_rows, ptr(d_kv_ring), ptr(dev["kv_gen"]),
             ptr(args["kv_exp"]), ptr(dev["ix"]), ix_rows, ptr(d_ix_ring), ptr(dev["ix_gen"]), ptr(args["ix_exp"]),
             len(lengths), ptr(args["seq"]), ptr(args["pos"]), ptr(args["kv_vals"]), ptr(args["ix_vals"]),
             ptr(err), len(seq), stream_handle())
        code = finish(err)
        del args
        codes = append_kv_index_ring(kv, kv_gen, ring_rows(kv_ring, kv_rows, seq, positions), kv_exp, ix, ix_gen,
                                     ring_rows(ix_ring, ix_rows, seq, positions), ix_exp, kv_vals, ix_vals)
        assert np.array_equal(dev["kv"].cpu().numpy().view(np.uint16), kv)
        assert np.array_equal(dev["ix"].cpu().numpy().view(np.uint16), ix)
        assert np.array_equal(dev["kv_gen"].cpu().numpy(), kv_gen)
        assert np.array_equal(dev["ix_gen"].cpu().numpy(), ix_gen)
        return code, codes

    def expected(seq, positions):
        kr = ring_rows(kv_ring, kv_rows, seq, positions)
        ir = ring_rows(ix_ring, ix_rows, seq, positions)
        return ([int(kv_gen[r]) if r >= 0 else 0 for r in kr], [int(ix_gen[r]) if r >= 0 else 0 for r in ir])

    def values(n):
        return (oracle.f32_to_bf16_bits(rng.normal(size=(n, 576)).astype(np.float32)),
                oracle.f32_to_bf16_bits(rng.normal(size=(n, 128)).astype(np.float32)))

    # 1. one token per sequence for three steps, including rows past the wrap point
    positions = [n - 1 for n in lengths]
    for _ in range(3):
        seq = list(range(len(lengths)))
        ke, ie = expected(seq, positions)
        code, codes = append(seq, positions, ke, ie, *values(len(seq)))
        assert code == 0 and not codes
        positions = [p + 1 for p in positions]
    # 2. each refusal in its own batch next to valid rows
    cases = {"stale_kv": ERR_SCATTER, "stale_index": ERR_SCATTER, "repeat": ERR_SCATTER,
             "sequence": ERR_SCATTER, "nan": ERR_NONFINITE}
    for case, want in cases.items():
        seq, pos = [0, 1, 3], [10, 4000, 900]
        ke, ie = expected(seq, pos)
        kv_vals, ix_vals = values(3)
        if case == "stale_kv":
            ke[1] += 1
        elif case == "stale_index":
            ie[2] += 1
        elif case == "repeat":
            seq, pos = seq + [1], pos + [4000]
            ke, ie = ke + [ke[1]], ie + [ie[1]]
            kv_vals, ix_vals = values(4)
        elif case == "sequence":
            seq, pos = seq + [7], pos + [3]
            ke, ie = ke + [0], ie + [0]
            kv_vals, ix_vals = values(4)
        elif case == "nan":
            ix_vals[0, 5] = 0x7FC0
        code, codes = append(seq, pos, ke, ie, kv_vals, ix_vals)
        assert codes == {want} and code == want, (case, code, codes)


def test_ring_ops_through_the_torch_extension(cuda):
    """The same ring step through deepseekrpc_cuda (the module the reference's runtime imports)."""
    import deepseekrpc_b200
    ext = deepseekrpc_b200.extension()
    cfg = small_config("cfg3", batch=2, seed=65)
    inp, lengths = make_decode_inputs(cfg, lengths=[7000, 300])
    r = ring_inputs(inp, lengths)
    out_c, topk_c, _, code = c_decode_step_ring(r, cfg.topk, cfg.scale)
    assert code == 0
    out, topk, err = ext.decode_step_ring(r["idx_q"], r["idx_w"], r["index_pool"], r["rings"]["index"], r["q"],
                                          r["kv_pool"], r["rings"]["kv"], r["visible"], max(lengths), cfg.topk,
                                          r["swa_pool"], r["rings"]["swa"], r["swa_len"], r["sink"], cfg.scale)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(topk, topk_c) and torch.equal(out, out_c)
    scores, err = ext.indexer_decode_ring(r["idx_q"], r["idx_w"], r["index_pool"], r["rings"]["index"],
                                          r["visible"], 7040)
    sel = ext.topk_select(scores, r["visible"], cfg.topk)
    out2, err2 = ext.sparse_mla_decode_ring(r["q"], r["kv_pool"], r["rings"]["kv"], r["visible"], sel[0],
                                            r["swa_pool"], r["rings"]["swa"], r["swa_len"], r["sink"], cfg.scale)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(sel[1].item()) == 0 and int(err2.item()) == 0
    assert torch.equal(sel[0], topk_c), "select (indexer + top-k) then attend gives the same rows"
    assert (out2 - out_c).abs().max().item() < 1e-5
