"""CPU restatement of the fused KV + index-key + SWA append (test infrastructure only).

The reference appends one decode step's rows with two checked scatters and a
ring write: AttentionState.publish_source writes the KV source pool and the
index-key pool through DeviceRowPool.write (attention_state.py:183-192), each a
scatter_kernel launch (native/operations.cu:144-161) followed, when the whole
batch passed, by the generation bump `generations[slot] = expected + 1`
(cache_pool.py:309); forward_mqa then writes the 128-slot SWA windows pool
(vllm_attention.py:261), whose SlotMap refuses a batch that repeats a ring slot
(cache_pool.py:86-88).

Per row, in batch order, the checks of scatter_kernel are kept as they are:
  - the physical row is out of bounds                      -> code 3, row skipped
  - an earlier row of the batch targets the same row        -> code 3, row skipped
  - generations[row] != expected[i]                         -> code 3, row skipped
and the SWA rule of the windows pool: with a ring, an earlier row of the same
sequence at the same ring row p % 128                        -> code 3, row skipped.

Deliberate departure of the B200 library, restated here so that the tests pin it
row by row: scatter_kernel writes the finite elements of a row and skips the
non-finite ones (code 2); the fused append refuses the whole row instead (code 2,
nothing of the row written: not the KV row, not the index row, not the ring row,
no bump).  And the bump is per written row, where the reference bumps the batch
only when its scatter status is 0 (with status 0 both agree).

Status: the device reports the first failing row's code in an unspecified order;
`append_kv_index` returns the set of codes raised, and a batch whose rows fail
with one code only has a definite status.
"""
from __future__ import annotations

import numpy as np

ERR_NONFINITE, ERR_SCATTER = 2, 3
SWA_ROWS = 128


def _nonfinite(bits) -> bool:
    return bool(np.any((np.asarray(bits, np.uint16) & 0x7F80) == 0x7F80))


def paged_rows(block_table, pool_blocks, seq, positions):
    """Physical pool row of each appended row through a block table, -1 when the
    sequence, the position or the table entry lies outside the pool."""
    rows = np.full(len(seq), -1, np.int64)
    table_rows, stride = block_table.shape
    for i, (s, p) in enumerate(zip(np.asarray(seq).tolist(), np.asarray(positions).tolist())):
        if not (0 <= s < table_rows and p >= 0 and p // 64 < stride):
            continue
        blk = int(block_table[s, p // 64])
        if 0 <= blk < pool_blocks:
            rows[i] = blk * 64 + p % 64
    return rows


def ring_rows(ring, pool_rows, seq, positions):
    """Physical pool row of each appended row in a ring-offset pool:
    ring[s] = (first, slots, offset) -> first + (p + offset) % slots
    (the reference SlotMap's slot = (logical + offset) % slots, cache_pool.py:24-113,
    placed at row `first` of a shared pool); -1 outside the pool."""
    rows = np.full(len(seq), -1, np.int64)
    for i, (s, p) in enumerate(zip(np.asarray(seq).tolist(), np.asarray(positions).tolist())):
        if not (0 <= s < len(ring) and p >= 0):
            continue
        first, slots, offset = (int(x) for x in ring[s])
        if slots <= 0 or not 0 <= offset < slots or first < 0 or first + slots > pool_rows:
            continue
        rows[i] = first + (p + offset) % slots
    return rows


def append_kv_index(kv_pool, index_pool, generations, rows, seq, positions, expected, kv_values,
                    index_values, swa=None, swa_rows=None):
    """Applies one append batch in place; returns the set of status codes raised.

    kv_pool u16[R, 576], index_pool u16[R, 128] (BF16 bit patterns),
    generations i64[R]; rows i64[n] the physical row of each new row (-1 = out of
    bounds, see paged_rows / ring_rows); swa u16[B, 128, 576] or None;
    swa_rows (optional) i64[n] ring row of each new row (default p % 128).
    """
    codes = set()
    seq = np.asarray(seq).tolist()
    positions = np.asarray(positions).tolist()
    rows = np.asarray(rows).tolist()
    ring_of = (list(np.asarray(swa_rows).tolist()) if swa_rows is not None
               else [p % SWA_ROWS for p in positions])
    for i, row in enumerate(rows):
        # scatter_kernel's checks (operations.cu:149-153)
        valid = row >= 0 and row not in rows[:i]
        if valid and swa is not None:
            valid = all(not (seq[j] == seq[i] and ring_of[j] == ring_of[i]) for j in range(i))
        if not valid or generations[row] != expected[i]:
            codes.add(ERR_SCATTER)
            continue
        # departure: a row with any non-finite element is refused whole
        if _nonfinite(kv_values[i]) or _nonfinite(index_values[i]):
            codes.add(ERR_NONFINITE)
            continue
        kv_pool[row] = kv_values[i]
        index_pool[row] = index_values[i]
        if swa is not None:
            swa[seq[i], ring_of[i]] = kv_values[i]
        generations[row] = expected[i] + 1  # cache_pool.py:309
    return codes


def append_kv_index_ring(kv_pool, kv_generations, kv_rows, kv_expected, index_pool, index_generations,
                         index_rows, index_expected, kv_values, index_values):
    """The append over two ring-offset pools with their own generations (the
    reference's source and index-key DeviceRowPools, each written by
    DeviceRowPool.write with its own expected generations, cache_pool.py:289-313).

    kv_rows / index_rows: the target row of each new row in each pool (ring_rows;
    -1 = out of bounds).  A row is refused (code 3) when either target is out of
    bounds, repeats an earlier row's target in its pool, or either generation
    differs from its expected value; a row with a non-finite element is refused
    whole (code 2, the departure documented above).  Written rows bump both
    generations to expected + 1.  Returns the set of codes raised."""
    codes = set()
    kv_rows = np.asarray(kv_rows).tolist()
    index_rows = np.asarray(index_rows).tolist()
    for i, (kr, ir) in enumerate(zip(kv_rows, index_rows)):
        valid = kr >= 0 and ir >= 0 and kr not in kv_rows[:i] and ir not in index_rows[:i]
        if (not valid or kv_generations[kr] != kv_expected[i] or
                index_generations[ir] != index_expected[i]):
            codes.add(ERR_SCATTER)
            continue
        if _nonfinite(kv_values[i]) or _nonfinite(index_values[i]):
            codes.add(ERR_NONFINITE)
            continue
        kv_pool[kr] = kv_values[i]
        index_pool[ir] = index_values[i]
        kv_generations[kr] = kv_expected[i] + 1
        index_generations[ir] = index_expected[i] + 1
    return codes
