"""CPU checks of the append and pool restatements (no GPU).

The fused append's oracle must equal the reference's two checked scatters plus
its bump (scatter_slots on the KV pool and on the index pool, then
generations = expected + 1, native/operations.cu:144-161 and cache_pool.py:309)
whenever the whole batch passes, and must depart from them only as documented:
a row with a non-finite element is refused whole.  The two pool restatements
(this library's whole-batch refusal and the reference's partial writes) must
reach the same state after write -> finish(accepted = 0).
"""
from __future__ import annotations

import numpy as np

import oracle
from oracle.append import ERR_NONFINITE, ERR_SCATTER, append_kv_index, paged_rows, ring_rows


def _bits(rng, shape):
    return oracle.f32_to_bf16_bits(rng.normal(size=shape).astype(np.float32))


def _setup(rng, rows=256):
    return _bits(rng, (rows, 576)), _bits(rng, (rows, 128)), rng.integers(0, 4, size=rows).astype(np.int64)


def test_valid_batch_equals_two_reference_scatters_and_the_bump():
    rng = np.random.default_rng(11)
    kv, ix, gen = _setup(rng)
    rows = rng.choice(256, size=20, replace=False).astype(np.int64)
    expected = gen[rows].copy()
    kv_new, ix_new = _bits(rng, (20, 576)), _bits(rng, (20, 128))
    seq = np.arange(20)
    positions = np.arange(20) * 7
    swa = _bits(rng, (20, 128, 576))
    a_kv, a_ix, a_gen, a_swa = kv.copy(), ix.copy(), gen.copy(), swa.copy()
    assert append_kv_index(a_kv, a_ix, a_gen, rows, seq, positions, expected, kv_new, ix_new, a_swa) == set()
    r_kv, r_ix, r_gen = kv.copy(), ix.copy(), gen.copy()
    slots = rows.astype(np.int32)
    assert oracle.scatter_slots(r_kv, r_gen, slots, expected, kv_new) == 0
    assert oracle.scatter_slots(r_ix, r_gen, slots, expected, ix_new) == 0
    r_gen[rows] = expected + 1
    assert np.array_equal(a_kv, r_kv) and np.array_equal(a_ix, r_ix) and np.array_equal(a_gen, r_gen)
    for i in range(20):
        assert np.array_equal(a_swa[seq[i], positions[i] % 128], kv_new[i])


def test_row_level_refusal_is_the_only_departure():
    rng = np.random.default_rng(12)
    kv, ix, gen = _setup(rng)
    rows = np.array([3, 9, 40], np.int64)
    expected = gen[rows].copy()
    kv_new, ix_new = _bits(rng, (3, 576)), _bits(rng, (3, 128))
    kv_new[1, 5] = 0x7F80  # +inf in the KV half of row 1
    a_kv, a_ix, a_gen = kv.copy(), ix.copy(), gen.copy()
    codes = append_kv_index(a_kv, a_ix, a_gen, rows, [0, 1, 2], [0, 1, 2], expected, kv_new, ix_new)
    assert codes == {ERR_NONFINITE}
    # row 1 refused whole: KV, index and generation untouched
    assert np.array_equal(a_kv[9], kv[9]) and np.array_equal(a_ix[9], ix[9]) and a_gen[9] == gen[9]
    # the reference scatter writes row 1's finite elements instead (the documented difference)
    r_kv, r_gen = kv.copy(), gen.copy()
    assert oracle.scatter_slots(r_kv, r_gen, rows.astype(np.int32), expected, kv_new) == ERR_NONFINITE
    assert not np.array_equal(r_kv[9], kv[9]) and r_kv[9, 5] == kv[9, 5]
    # rows 0 and 2 are written identically by both
    assert np.array_equal(a_kv[[3, 40]], r_kv[[3, 40]])


def test_scatter_checks_follow_the_reference_rule():
    rng = np.random.default_rng(13)
    kv, ix, gen = _setup(rng)
    rows = np.array([5, -1, 5, 7], np.int64)  # in bounds, out of bounds, repeated, stale
    expected = gen[[5, 0, 5, 7]].copy()
    expected[3] += 1
    kv_new, ix_new = _bits(rng, (4, 576)), _bits(rng, (4, 128))
    a_kv, a_ix, a_gen = kv.copy(), ix.copy(), gen.copy()
    codes = append_kv_index(a_kv, a_ix, a_gen, rows, [0, 1, 2, 3], [0, 1, 2, 3], expected, kv_new, ix_new)
    assert codes == {ERR_SCATTER}
    assert np.array_equal(a_kv[5], kv_new[0]) and a_gen[5] == expected[0] + 1
    assert np.array_equal(a_kv[7], kv[7]) and a_gen[7] == gen[7]


def test_paged_and_ring_addressing():
    table = np.array([[3, 0, -1], [1, 2, 4]], np.int32)
    rows = paged_rows(table, 5, [0, 0, 0, 1, 2, 0], [5, 64, 130, 191, 0, -1])
    assert rows.tolist() == [3 * 64 + 5, 0 * 64 + 0, -1, 4 * 64 + 63, -1, -1]
    ring = np.array([[0, 100, 37], [100, 50, 0]], np.int64)
    rows = ring_rows(ring, 150, [0, 0, 1, 1, 2], [0, 70, 49, 50, 0])
    assert rows.tolist() == [37, (70 + 37) % 100, 149, 100, -1]


def test_both_pool_restatements_agree_after_rollback():
    rng = np.random.default_rng(14)
    ours, ref = oracle.PoolOracle(32, 128, 16), oracle.ReferenceRowPool(32, 128, 16)
    for pool in (ours, ref):
        pool.data[:] = 0
    # an accepted batch, then a refused batch (a NaN element, a stale generation), both rolled back
    batches = [([1, 2, 3], [0, 0, 0], False), ([4, 5], [0, 0], True), ([6, 2], [0, 0], False)]
    journal = []
    for slots, expected, poison in batches:
        values = _bits(rng, (len(slots), 128))
        if poison:
            values[1, 17] = 0x7FC0
        start = len(journal)
        codes = [pool.write(slots, expected, values, start) for pool in (ours, ref)]
        assert (codes[0] == 0) == (codes[1] == 0)
        journal += [(start + i, s, e) for i, (s, e) in enumerate(zip(slots, expected))]
    for pool in (ours, ref):
        pool.finish(journal)
    assert np.array_equal(ours.data, ref.data) and np.array_equal(ours.generations, ref.generations)
    assert not ours.data.any() and not ours.generations.any()
