"""CPU restatement of the reference's DeviceRowPool data semantics (test infrastructure only).

Follows src/deepseekrpc/cache_pool.py:289-352 (write: undo backup of the target
rows, checked scatter with expected generations, generation bump; finish: the
rejected mutations restored newest first from their backups and previous
generations), cache_pool.py:255-274 (restore_rows: fresh rows only, generation
1) and snapshot_state.py:205-216 (row tiles by logical id, slot =
(logical + offset) % slots, non-finite rows refused).  Host metadata follows the
reference SlotMap, which the tests pin separately against a recorded trace of
the reference itself.  Data are BF16 bit patterns (uint16).
"""
from __future__ import annotations

import numpy as np

from .ops import scatter_slots


class PoolOracle:
    def __init__(self, slots: int, width: int, undo_rows: int):
        self.data = np.zeros((slots, width), np.uint16)
        self.generations = np.zeros(slots, np.int64)
        self.undo = np.zeros((undo_rows, width), np.uint16)

    @staticmethod
    def _nonfinite(bits):
        return bool(np.any((np.asarray(bits, np.uint16) & 0x7F80) == 0x7F80))

    def write(self, slots, expected, values, undo_start):
        """cache_pool.py:293-310: backup, checked scatter, bump.  Returns the device
        status (0, 3 = bounds/repeat/generation, 2 = non-finite); a refused batch
        leaves only its backup written (this library writes a batch whole or not at all)."""
        slots = list(slots)
        for i, s in enumerate(slots):
            if 0 <= s < len(self.data):
                self.undo[undo_start + i] = self.data[s]
        bad = any(s < 0 or s >= len(self.data) for s in slots) or len(set(slots)) != len(slots)
        bad = bad or any(self.generations[s] != e for s, e in zip(slots, expected))
        if bad:
            return 3
        if self._nonfinite(values):
            return 2
        for i, s in enumerate(slots):
            self.data[s] = values[i]
            self.generations[s] = expected[i] + 1
        return 0

    def finish(self, rejected_journal_order):
        """cache_pool.py:336-352: (journal index, slot, previous generation) entries,
        restored newest first."""
        for index, slot, previous in reversed(list(rejected_journal_order)):
            self.data[slot] = self.undo[index]
            self.generations[slot] = previous

    def restore(self, slots, values):
        """cache_pool.py:255-274 (after the host checks): rows written, generation 1."""
        for i, s in enumerate(slots):
            self.data[s] = values[i]
            self.generations[s] = 1

    def gather(self, logical, offset):
        """snapshot_state.py:205-216: rows of logical ids, in order; None if non-finite."""
        rows = self.data[(np.asarray(logical, np.int64) + offset) % len(self.data)]
        return None if self._nonfinite(rows) else rows.copy()


class ReferenceRowPool:
    """The reference's own DeviceRowPool.write / finish data path, partial writes
    included (cache_pool.py:289-313,336-352): the target rows are backed up, the
    batch is scattered by scatter_kernel's rule (native/operations.cu:144-161,
    restated by oracle.scatter_slots: refused rows skipped, non-finite elements
    skipped, the rest written), and the generations are bumped only when the
    scatter status is 0; a failed write needs finish(accepted=0), which restores
    the rejected mutations newest first.  PoolOracle above restates this
    library's whole-batch refusal; the two must agree on every end state after
    finish."""

    def __init__(self, slots: int, width: int, undo_rows: int):
        self.data = np.zeros((slots, width), np.uint16)
        self.generations = np.zeros(slots, np.int64)
        self.undo = np.zeros((undo_rows, width), np.uint16)

    def write(self, slots, expected, values, undo_start):
        slots = np.asarray(slots, np.int32)
        for i, s in enumerate(slots.tolist()):
            self.undo[undo_start + i] = self.data[s]  # index_select into the undo rows (cache_pool.py:300)
        code = scatter_slots(self.data, self.generations, slots, np.asarray(expected, np.int64),
                             np.asarray(values, np.uint16))
        if code == 0:
            self.generations[slots] = np.asarray(expected, np.int64) + 1  # cache_pool.py:309
        return code

    def finish(self, rejected_journal_order):
        for index, slot, previous in reversed(list(rejected_journal_order)):
            self.data[slot] = self.undo[index]
            self.generations[slot] = previous
