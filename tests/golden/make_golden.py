"""Generate the golden fixtures of the hot path from the reference's own code.

Run once in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference <path-to-DeepSeekRPC>/src

It imports the reference's CPU functions (reference_attention.sparse_attention_reference,
reference_attention.index_scores_reference, index_selection.merge_ranked,
engram_storage.decode_fp8_rows, cache_pool.SlotMap) and records their outputs on
seeded inputs shaped like the reference's own known-answer tests
(src/deepseekrpc/gpu_selftest.py:55-101,209-246, tests/test_reference_attention.py,
tests/test_index_selection.py, tests/test_cache_pool.py).  The outputs are written
next to this script as .npz / .json files and committed; nothing at test time
imports the reference.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bf16_round(a):
    import torch
    t = torch.as_tensor(np.asarray(a, np.float32)).to(torch.bfloat16)
    return t.float().numpy(), t.view(torch.int16).numpy().view(np.uint16)


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the reference's src/ directory")
    args = parser.parse_args(argv)
    sys.path.insert(0, args.reference)
    import torch
    from deepseekrpc.cache_pool import SlotMap
    from deepseekrpc.engram_storage import decode_fp8_rows
    from deepseekrpc.index_selection import merge_ranked
    from deepseekrpc.jsonutil import ValidationError
    from deepseekrpc.reference_attention import index_scores_reference, sparse_attention_reference
    from deepseekrpc.state import Operation

    out = {}

    # 1. sparse attention KAT: sink, duplicates, padding, empty row (gpu_selftest.py:55-64)
    rng = np.random.default_rng(5501)
    q = rng.normal(0, .2, (3, 64, 512)).astype(np.float32)
    window, window_bits = bf16_round(rng.normal(0, .3, (7, 512)))
    source, source_bits = bf16_round(rng.normal(0, .3, (11, 512)))
    ids = np.array([[0, 6, 7, 17, -1, -1], [5, 5, 9, 10, -1, 11], [-1] * 6], np.int32)
    sink = rng.normal(0, .3, 64).astype(np.float32)
    expected = sparse_attention_reference(q, window, source, ids, sink, scale=512 ** -.5)
    out["sparse_kat"] = dict(q=q, window_bits=window_bits, source_bits=source_bits, ids=ids, sink=sink,
                             scale=np.float32(512 ** -.5), expected=expected)

    # 2. sparse attention vs dense softmax geometry (tests/test_reference_attention.py:10-27)
    rng = np.random.default_rng(41)
    q = (rng.normal(size=(3, 2, 512)) / 4).astype(np.float32)
    window, window_bits = bf16_round(rng.normal(size=(5, 512)))
    source, source_bits = bf16_round(rng.normal(size=(7, 512)))
    ids = np.array([[0, 7, 7, -1], [-1, -1, -1, -1], [1, 4, 11, -1]], np.int32)
    sink = np.array([1.7, -0.9], np.float32)
    expected = sparse_attention_reference(q, window, source, ids, sink, scale=512 ** -0.5)
    out["sparse_dense"] = dict(q=q, window_bits=window_bits, source_bits=source_bits, ids=ids, sink=sink,
                               scale=np.float32(512 ** -0.5), expected=expected)

    # 3. index scores KAT: signed weights, causal visibility (gpu_selftest.py:66-75)
    rng = np.random.default_rng(6601)
    q = rng.normal(0, .3, (5, 32, 128)).astype(np.float32)
    keys, keys_bits = bf16_round(rng.normal(0, .3, (19, 128)))
    w = rng.normal(0, .2, (5, 32)).astype(np.float32)
    ids = np.tile(np.array([0, 1, 18, 8, 8, -1, 3, 9], np.int32), (5, 1))
    visible = np.array([0, 1, 9, 18, 19], np.int32)
    expected = index_scores_reference(q, keys, w, ids, visible)
    out["index_kat"] = dict(q=q, keys_bits=keys_bits, weights=w, ids=ids, visible=visible, expected=expected)

    # 4. index ReLU-before-weights and visibility (tests/test_reference_attention.py:30-44)
    rng = np.random.default_rng(1017)
    q = (rng.normal(size=(3, 32, 128)) / 8).astype(np.float32)
    keys, keys_bits = bf16_round(rng.normal(size=(97, 128)))
    w = (rng.normal(size=(3, 32)) / 16).astype(np.float32)
    ids = np.tile(np.arange(-1, 97, dtype=np.int32), (3, 1))
    visible = np.array([0, 42, 97], np.int32)
    expected = index_scores_reference(q, keys, w, ids, visible)
    out["index_visibility"] = dict(q=q, keys_bits=keys_bits, weights=w, ids=ids, visible=visible,
                                   expected=expected)

    # 5. index scores, a larger in-bound random case (rows 16, heads 32, 2048 keys)
    rng = np.random.default_rng(7701)
    q, _ = bf16_round(rng.normal(size=(16, 32, 128)))
    keys, keys_bits = bf16_round(rng.normal(size=(2048, 128)))
    w = (rng.normal(size=(16, 32)) / 8).astype(np.float32)
    ids = np.stack([rng.permutation(2048)[:1024] for _ in range(16)]).astype(np.int32)
    ids[:, ::37] = -1
    visible = rng.integers(0, 2049, 16).astype(np.int32)
    visible[0], visible[1] = 0, 2048
    expected = index_scores_reference(q, keys, w, ids, visible)
    out["index_random"] = dict(q=q, keys_bits=keys_bits, weights=w, ids=ids, visible=visible,
                               expected=expected)

    # 6. merge_ranked: explicit ties across odd tile splits (tests/test_index_selection.py:58-84)
    rng = np.random.default_rng(1017)
    values = rng.normal(size=57).astype(np.float32)
    values[[0, 11, 56]] = 1.75
    merge = {"values": values}
    for name, pieces in (("a", (17, 14, 26)), ("b", (1, 8, 7, 29, 12)), ("c", (57,))):
        s, i, start = torch.empty(0), torch.empty(0, dtype=torch.int64), 0
        for count in pieces:
            s, i = merge_ranked(s, i, torch.from_numpy(values[start:start + count]),
                                torch.arange(start, start + count), keep=13)
            start += count
        merge[f"pieces_{name}"] = np.array(pieces, np.int64)
        merge[f"ids_{name}"] = i.numpy()
        merge[f"scores_{name}"] = s.numpy()
    s, i = merge_ranked(torch.empty(0), torch.empty(0, dtype=torch.int64),
                        torch.tensor([9., 8., 7., float("inf")]), torch.arange(4), keep=2)
    merge["pinned_ids"] = i.numpy()
    # NaN scores: torch's descending sort ranks them above +inf
    nan_values = np.array([1., np.nan, np.inf, -0.0, np.nan, -np.inf, 0.0, 2., np.inf, 0.0], np.float32)
    s, i = merge_ranked(torch.empty(0), torch.empty(0, dtype=torch.int64), torch.from_numpy(nan_values),
                        torch.arange(len(nan_values)), keep=8)
    merge["nan_values"], merge["nan_ids"] = nan_values, i.numpy()
    out["merge_ranked"] = merge

    # 7. tie-heavy top-2048 over 131072 scores through 8192-wide tiles (TiledIndexer merge)
    rng = np.random.default_rng(8801)
    n, keep = 131072, 2048
    scores = (np.round(rng.normal(size=n) * 4) / 4).astype(np.float32)
    scores[rng.integers(0, n, 3000)] = 0.0
    scores[rng.integers(0, n, 3000)] = -0.0
    scores[rng.integers(0, n, 500)] = 2.25  # a tie group straddling the threshold
    s, i = torch.empty(0), torch.empty(0, dtype=torch.int64)
    for start in range(0, n, 8192):
        s, i = merge_ranked(s, i, torch.from_numpy(scores[start:start + 8192]),
                            torch.arange(start, min(n, start + 8192)), keep=keep)
    out["topk_ties"] = dict(scores=scores, keep=np.int64(keep), expected=np.sort(i.numpy()).astype(np.int32))

    # 8. tiled selection with constructed keys (gpu_selftest.py:209-246), tiles of 128
    keys = np.zeros((1025, 128), np.float32)
    positions = np.arange(1025)
    keys[:, 0], keys[:, 1] = positions // 256, (positions % 256) / 256
    keys, keys_bits = bf16_round(keys)
    q = np.zeros((3, 32, 128), np.float32)
    q[:, 0, 0], q[:, 0, 1] = 256., 1.
    w = np.zeros((3, 32), np.float32)
    w[:, 0] = [1., -1., 1.]
    visible = np.array([513, 1025, 1025], np.int32)
    topk = np.full((3, 512), -1, np.int32)
    for row, vis in enumerate(visible):
        s, i = torch.empty(0), torch.empty(0, dtype=torch.int64)
        for start in range(0, vis, 128):
            logical = np.arange(start, min(vis, start + 128))
            tile_scores = index_scores_reference(q[row:row + 1], keys[logical], w[row:row + 1],
                                                 np.arange(len(logical), dtype=np.int32)[None],
                                                 np.array([len(logical)], np.int32))[0]
            s, i = merge_ranked(s, i, torch.from_numpy(tile_scores), torch.from_numpy(logical), keep=512)
        chosen = np.sort(i.numpy()).astype(np.int32)
        topk[row, :len(chosen)] = chosen
    analytic = np.stack([np.arange(1, 513), np.arange(512), np.arange(513, 1025)]).astype(np.int32)
    assert np.array_equal(topk, analytic)
    out["tiled_select"] = dict(q=q, keys_bits=keys_bits, weights=w, visible=visible, expected=topk)

    # 9. Engram FP8 decode (gpu_selftest.py:77-85)
    encoded = np.empty((5, 264), np.uint8)
    values = np.arange(256, dtype=np.uint8)
    values[[127, 255]] = 0
    encoded[:, :256] = values
    encoded[:, 256:] = np.array([0, 64, 126, 127, 130], np.uint8)[:, None]
    decoded = torch.from_numpy(decode_fp8_rows(encoded)).to(torch.bfloat16)
    out["engram"] = dict(encoded=encoded, expected_bits=decoded.view(torch.int16).numpy().view(np.uint16))

    for name, arrays in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **arrays)

    # 10. SlotMap trace: offsets, partial acceptance, duplicate refusal (tests/test_cache_pool.py)
    trace = []
    rng = np.random.default_rng(9901)
    for slots, offset in ((3, 0), (3, 2), (8, 5), (16, 11)):
        mapping = SlotMap(slots, context=64, offset=offset, max_mutations=16)
        mapping.reset("a" * 32, 0)
        start, number = 0, 1
        steps = []
        for _ in range(12):
            rows = int(rng.integers(1, 5))
            op = Operation("a" * 32, "b" * 32, 0, number, "c" * 32, "d" * 64, start, rows)
            number += 1
            mapping.begin(op)
            logical = list(range(start, start + rows))
            if rng.random() < 0.2 and rows > 1:
                logical[-1] = logical[0] + slots  # same physical slot twice -> refused
            try:
                result = mapping.reserve(logical, list(range(start, start + rows)))
                reserved = [list(map(int, result[0])), list(map(int, result[1]))]
                error = None
            except ValidationError as e:
                reserved, error = None, str(e)
            accepted = int(rng.integers(0, rows + 1))
            mapping.finish(op, accepted)
            probe = list(range(max(0, start - slots - 2), start + rows))
            physical = []
            for p in probe:
                try:
                    physical.append(mapping.physical([p])[0])
                except ValidationError:
                    physical.append(None)
            steps.append(dict(start=start, rows=rows, logical=logical, reserved=reserved, error=error,
                              accepted=accepted, probe=probe, physical=physical,
                              generations=mapping.generations.tolist(), logical_map=mapping.logical.tolist()))
            start += accepted if error is None else 0
        trace.append(dict(slots=slots, offset=offset, steps=steps))
    (HERE / "slotmap_trace.json").write_text(json.dumps(trace))

    # 11. SlotMap windows: several write batches per window (the journal spans
    # them), ring wrap-around (context > slots, hash-like offsets), out-of-order
    # producing tokens, oversized windows and undo-journal exhaustion
    windows = []
    rng = np.random.default_rng(9902)
    for slots, offset, journal in ((8, 3, 6), (64, 37, 16), (100, 91, 64), (1000, 517, 64)):
        mapping = SlotMap(slots, context=4 * slots, offset=offset, max_mutations=journal)
        mapping.reset("e" * 32, 3)
        start, number, steps = 0, 1, []
        for _ in range(16):
            rows = int(rng.integers(1, min(64, 4 * slots - start) + 1)) if rng.random() > 0.1 else 65
            op = Operation("e" * 32, "b" * 32, 3, number, "c" * 32, "d" * 64, start, rows)
            number += 1
            record = dict(start=start, rows=rows, begin_error=None, batches=[])
            try:
                mapping.begin(op)
            except ValidationError as e:
                record["begin_error"] = str(e)
                steps.append(record)
                continue
            token = start
            for _ in range(int(rng.integers(1, 4))):
                if token >= start + rows:
                    break
                n = int(rng.integers(1, start + rows - token + 1))
                logical = list(range(token, token + n))
                tokens = list(range(token, token + n))
                if rng.random() < 0.15 and n > 1:
                    tokens[-1], tokens[0] = tokens[0], tokens[-1]  # producing tokens go backwards
                if rng.random() < 0.15:
                    logical[-1] = logical[0] + slots  # one slot twice
                try:
                    result = mapping.reserve(logical, tokens)
                    batch = dict(logical=logical, tokens=tokens,
                                 reserved=[list(map(int, result[0])), list(map(int, result[1]))], error=None)
                    token += n
                except ValidationError as e:
                    batch = dict(logical=logical, tokens=tokens, reserved=None, error=str(e))
                record["batches"].append(batch)
            accepted = int(rng.integers(0, token - start + 1))
            rejected = [(int(i), int(m.slot), int(m.previous_generation)) for i, m in mapping.rejected(op, accepted)]
            mapping.finish(op, accepted)
            probe = list(range(max(0, start - slots - 2), start + rows))
            physical = []
            for q in probe:
                try:
                    physical.append(mapping.physical([q])[0])
                except ValidationError:
                    physical.append(None)
            record.update(accepted=accepted, rejected=rejected, probe=probe, physical=physical,
                          generations=mapping.generations.tolist(), logical_map=mapping.logical.tolist())
            steps.append(record)
            start += accepted
        windows.append(dict(slots=slots, offset=offset, journal=journal, context=4 * slots, steps=steps))
    (HERE / "slotmap_windows.json").write_text(json.dumps(windows))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
