"""Row pools with the interface of the reference's cache_pool module, on the
device transactions of this package (dsr_pool_*).

`SlotMap` is the host metadata (cache_pool.py:24-153): slot = (logical + offset)
% slots, one generation per slot bumped by every write, a journal of mutations
that `finish(operation, accepted)` rolls back past the accepted prefix.
`DeviceRowPool` (cache_pool.py:156-360) keeps a BF16 [slots, width] pool, its
int64 generations and an undo log on one CUDA device.  Where the reference
gathers the backup, synchronises, scatters, bumps the generations and
synchronises again, `write` here is one launch (dsr_pool_write: the whole batch
checked, backed up and written, or refused with nothing but the backup written)
and `finish` one more (dsr_pool_rollback).  Snapshot tiles stream through
dsr_pool_gather / dsr_pool_restore in the reference's wire format (rows of a
tile in logical order, BF16 bits little-endian).  There is no CPU fallback.
"""
from __future__ import annotations

import re
import threading
from contextlib import contextmanager
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np

from . import _native
from .cuda_ops import ValidationError

I64_MAX = (1 << 63) - 1
U64_MAX = (1 << 64) - 1


def _integer(value, name: str, low: int, high: int) -> int:
    if type(value) is not int or not low <= value <= high:
        raise ValidationError(f"{name} must be an integer in [{low}, {high}]")
    return value


def _hex_id(value, size: int, name: str) -> str:
    if not isinstance(value, str) or not re.fullmatch(r"[0-9a-f]{%d}" % size, value):
        raise ValidationError(f"invalid {name} identity")
    return value


@dataclass(frozen=True)
class Operation:
    """The fields of the reference's state.Operation a pool reads (state.py:23-40)."""
    session: str
    epoch: int
    start: int
    rows: int

    def __post_init__(self):
        _hex_id(self.session, 32, "session")
        _integer(self.epoch, "epoch", 0, U64_MAX)
        _integer(self.start, "start position", 0, 1048576)
        _integer(self.rows, "operation rows", 1, min(4096, 1048576 - self.start))


class SlotMutation(NamedTuple):
    """One journal entry, as the pool's rollback reads it back."""
    token_position: int
    slot: int
    previous_logical: int
    previous_generation: int


def _refuse(reason: str, message: str):
    """A ValidationError (the reference's exception type) tagged with a short reason."""
    error = ValidationError(message)
    error.reason = reason
    raise error


def _int_array(values, name: str, low: int, high: int) -> np.ndarray:
    """Python ints in [low, high] as an int64 array (bools and floats refused)."""
    values = list(values)
    if any(type(v) is not int for v in values):
        _refuse("type", f"{name}: integers required")
    arr = np.asarray(values, dtype=np.int64) if values else np.zeros(0, np.int64)
    if arr.size and (arr.min() < low or arr.max() > high):
        _refuse("range", f"{name}: outside [{low}, {high}]")
    return arr


class SlotMap:
    """Host metadata of one ring-offset row pool: which logical row each physical
    slot holds and its generation, plus the undo journal of the open window.

    Semantics are the reference SlotMap's (src/deepseekrpc/cache_pool.py:24-153),
    pinned by a recorded trace of it: slot = (logical + offset) % slots; a write
    batch of 1..64 rows inside the active window, in non-decreasing producing-token
    order, with no repeated slot, bumps each slot's generation; `physical` accepts
    only rows still held under their own logical id with a nonzero generation;
    `finish(operation, accepted)` puts back every mutation produced by a token at
    or past start + accepted, newest first.  The representation is this module's
    own: the per-slot state lives in two int64 arrays, the journal in four
    preallocated arrays (structure of arrays, `max_mutations` entries), and every
    batch is validated and applied with vectorised numpy operations.
    """

    def __init__(self, slots: int, *, context: int, offset: int, max_mutations: int = 64):
        self.slots = _integer(slots, "slot count", 1, 1048576)
        self.context = _integer(context, "logical capacity", slots, 1048576)
        self.offset = _integer(offset, "slot offset", 0, slots - 1)
        self.max_mutations = _integer(max_mutations, "journal capacity", 1, 4096)
        self.logical = np.full(slots, -1, dtype=np.int64)      # logical row held by each slot
        self.generations = np.zeros(slots, dtype=np.int64)     # 0 = never written in this epoch
        self._j_token = np.zeros(max_mutations, np.int64)      # journal: producing token,
        self._j_slot = np.zeros(max_mutations, np.int64)       #   target slot,
        self._j_logical = np.zeros(max_mutations, np.int64)    #   the slot's previous logical row
        self._j_generation = np.zeros(max_mutations, np.int64)  #   and its previous generation
        self._j_len = 0
        self.epoch, self.session, self.active = -1, None, None

    # ----------------------------------------------------------------- views
    @property
    def metadata_bytes(self) -> int:
        return self.logical.nbytes + self.generations.nbytes

    @property
    def journal(self) -> list:
        """The open window's mutations in write order."""
        n = self._j_len
        return [SlotMutation(int(t), int(s), int(lg), int(g)) for t, s, lg, g in
                zip(self._j_token[:n], self._j_slot[:n], self._j_logical[:n], self._j_generation[:n])]

    def slot_of(self, logical):
        """Physical slot(s) of logical row(s)."""
        return (np.asarray(logical, dtype=np.int64) + self.offset) % self.slots if np.ndim(logical) \
            else (int(logical) + self.offset) % self.slots

    # -------------------------------------------------------------- epochs
    def _new_epoch(self, session: str, epoch: int) -> None:
        self.session, self.epoch = session, epoch
        self.logical.fill(-1)
        self.generations.fill(0)

    def reset(self, session: str, epoch: int) -> None:
        _hex_id(session, 32, "pool session")
        _integer(epoch, "pool epoch", 0, I64_MAX)
        if self.active is not None:
            _refuse("busy", "pool reset while a window is open")
        if epoch <= self.epoch:
            _refuse("epoch", f"pool reset to epoch {epoch}, not after the current epoch {self.epoch}")
        self._new_epoch(session, epoch)

    def discard_for_reset(self, session: str, epoch: int) -> None:
        """Drops the open window and every row under a strictly newer epoch."""
        _hex_id(session, 32, "pool session")
        _integer(epoch, "pool epoch", 0, I64_MAX)
        if epoch <= self.epoch:
            _refuse("epoch", f"pool discard to epoch {epoch}, not after the current epoch {self.epoch}")
        self.active, self._j_len = None, 0
        self._new_epoch(session, epoch)

    # ------------------------------------------------------------- windows
    def begin(self, operation) -> None:
        if self.active is not None:
            _refuse("busy", "a window is already open on this pool")
        if operation.session != self.session or operation.epoch != self.epoch:
            _refuse("stale", "window belongs to another session or epoch")
        if operation.rows > 64 or operation.start + operation.rows > self.context:
            _refuse("bounds", "window is longer than 64 rows or ends past the logical capacity")
        self.active = operation

    def _check_batch(self, logical_positions, token_positions):
        """Validates a write batch as a whole; returns (logical, tokens, slots) arrays."""
        if self.active is None:
            _refuse("idle", "pool write without an open window")
        n = len(logical_positions)
        if n != len(token_positions) or not 1 <= n <= 64:
            _refuse("shape", "write batch must hold 1..64 rows with one producing token each")
        if self._j_len + n > self.max_mutations:
            _refuse("journal", "undo journal is full")
        logical = _int_array(logical_positions, "logical rows", 0, self.context - 1)
        window = self.active
        first = int(self._j_token[self._j_len - 1]) if self._j_len else window.start
        tokens = _int_array(token_positions, "producing tokens", first, window.start + window.rows - 1)
        if np.any(np.diff(tokens) < 0):
            _refuse("order", "producing tokens go backwards")
        slots = (logical + self.offset) % self.slots
        if len(np.unique(slots)) != n:
            _refuse("repeat", "write batch targets one slot twice")
        if np.any(self.generations[slots] == I64_MAX):
            _refuse("exhausted", "slot generation exhausted; start a new epoch")
        return logical, tokens, slots

    def prepare(self, logical_positions, token_positions):
        """Validates a batch; returns (mutations, slots, current generations) without applying it."""
        logical, tokens, slots = self._check_batch(logical_positions, token_positions)
        gens = self.generations[slots]
        mutations = [SlotMutation(int(t), int(s), int(lg), int(g))
                     for t, s, lg, g in zip(tokens, slots, self.logical[slots], gens)]
        return mutations, slots.tolist(), gens.tolist()

    def reserve(self, logical_positions, token_positions):
        """Validates and applies a batch: journals each slot's previous state, then
        claims the slots for the new rows at generation + 1.  Returns (slots,
        previous generations) -- the expected generations of the device write."""
        logical, tokens, slots = self._check_batch(logical_positions, token_positions)
        n, j = len(slots), self._j_len
        previous = self.generations[slots].copy()
        self._j_token[j:j + n] = tokens
        self._j_slot[j:j + n] = slots
        self._j_logical[j:j + n] = self.logical[slots]
        self._j_generation[j:j + n] = previous
        self._j_len = j + n
        self.logical[slots] = logical
        self.generations[slots] = previous + 1
        return slots.tolist(), previous.tolist()

    # ---------------------------------------------------------------- reads
    def physical(self, logical_positions):
        """Slots of live logical rows; -1 passes through as padding."""
        values = list(logical_positions)
        if not values:
            return []
        padded = np.asarray([v == -1 and type(v) is int for v in values])
        live = _int_array([v for v, pad in zip(values, padded) if not pad], "visible logical rows", 0,
                          self.context - 1)
        out = np.full(len(values), -1, np.int64)
        slots = (live + self.offset) % self.slots
        if np.any(self.logical[slots] != live) or np.any(self.generations[slots] == 0):
            _refuse("absent", "a visible row is missing or its slot now holds another row")
        out[~padded] = slots
        return out.tolist()

    # ------------------------------------------------------------- prefixes
    def validate_prefix(self, count: int) -> None:
        _integer(count, "retained rows", 0, self.slots)
        if self.active is not None:
            _refuse("busy", "prefix retention while a window is open")
        logical = np.arange(count, dtype=np.int64)
        slots = (logical + self.offset) % self.slots
        if np.any(self.logical[slots] != logical) or np.any(self.generations[slots] <= 0):
            _refuse("absent", "retained prefix has missing or overwritten rows")

    def retain_prefix(self, session: str, epoch: int, count: int) -> None:
        """Keeps rows 0..count-1 (each at generation 1) under a newer epoch."""
        _hex_id(session, 32, "retained prefix session")
        _integer(epoch, "retained prefix epoch", self.epoch + 1, I64_MAX)
        self.validate_prefix(count)
        keep = (self.logical >= 0) & (self.logical < count)
        self.logical[~keep] = -1
        self.generations[:] = keep
        self.session, self.epoch = session, epoch
        self._j_len = 0

    # --------------------------------------------------------------- commit
    def rejected(self, operation, accepted: int):
        """(journal index, mutation) of the mutations produced at or past
        start + accepted, newest first."""
        _integer(accepted, "accepted rows", 0, operation.rows)
        if self.active != operation:
            _refuse("stale", "commit targets another window")
        n = self._j_len
        idx = np.nonzero(self._j_token[:n] >= operation.start + accepted)[0][::-1]
        return [(int(i), SlotMutation(int(self._j_token[i]), int(self._j_slot[i]), int(self._j_logical[i]),
                                      int(self._j_generation[i]))) for i in idx]

    def finish(self, operation, accepted: int) -> None:
        """Closes the window; the rejected mutations are undone newest first, so a
        slot written twice ends with the state before its first rejected write."""
        rejected = self.rejected(operation, accepted)
        if rejected:
            order = np.asarray([i for i, _ in rejected], np.int64)  # newest first; the last write wins
            for i in order:
                s = self._j_slot[i]
                self.logical[s] = self._j_logical[i]
                self.generations[s] = self._j_generation[i]
        self._j_len = 0
        self.active = None


MAX_PAYLOAD = 1024 * 1024  # bytes per snapshot record chunk (protocol.py:15)


class DeviceRowPool:
    """One BF16 [slots, width] pool with int64 generations and an undo log on a CUDA
    device (cache_pool.py:156-360).  Width up to 576 (the MLA KV rows; the
    reference's pools stop at 512).  Every public method holds the pool's lock."""

    def __init__(self, slots: int, width: int, *, context: int, offset: int, admitted_bytes: int,
                 device="cuda:0", max_mutations: int = 64):
        import torch
        _integer(width, "BF16 cache width", 1, 576)
        _integer(admitted_bytes, "BF16 cache pool admission", 1, 1 << 40)
        self.map = SlotMap(slots, context=context, offset=offset, max_mutations=max_mutations)
        self.width = width
        dev = torch.device(device)
        if dev.type != "cuda" or not torch.cuda.is_available():
            raise RuntimeError("BF16 cache pools require a real CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.payload_bytes = slots * width * 2
        self.allocation_bytes = (self.payload_bytes + slots * 8 + max_mutations * (width * 2 + 256) +
                                 64 * (width * 2 + 32))
        self.admission_bytes = self.allocation_bytes + self.map.metadata_bytes
        if self.admission_bytes > admitted_bytes:
            raise ValidationError("eager BF16 payload, map, generations and undo exceed admission")
        self._mutex, self._needs_rollback, self.closed = threading.RLock(), False, False
        _native.library()  # the device transactions must be available
        with torch.cuda.device(dev):
            self.data = torch.zeros((slots, width), dtype=torch.bfloat16, device=dev)
            self.generations = torch.zeros(slots, dtype=torch.int64, device=dev)
            self._undo = torch.zeros((max_mutations, width), dtype=torch.bfloat16, device=dev)
            self._err = torch.zeros(1, dtype=torch.int32, device=dev)
            self._tile = torch.empty((1024, width), dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize(dev)

    # ------------------------------------------------------------ helpers
    def _open(self):
        if self.closed:
            raise ValidationError("BF16 cache pool is closed")

    def _status(self, what: str) -> int:
        code = int(self._err.item())  # synchronises the stream, as the reference does
        self._err.zero_()
        return code

    def _device_ints(self, values, dtype):
        import torch
        return torch.tensor(values, dtype=dtype).to(self.device, non_blocking=True)

    # ------------------------------------------------------ window control
    def reset(self, session: str, epoch: int) -> None:
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            self.map.reset(session, epoch)
            self.generations.zero_()
            torch.cuda.synchronize(self.device)
            self._needs_rollback = False

    def begin(self, operation) -> None:
        with self._mutex:
            self._open()
            if self._needs_rollback:
                raise ValidationError("cache requires rollback before another window")
            self.map.begin(operation)

    def discard_for_reset(self, session: str, epoch: int) -> None:
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            torch.cuda.synchronize(self.device)
            self.map.discard_for_reset(session, epoch)
            self.generations.zero_()
            torch.cuda.synchronize(self.device)
            self._needs_rollback = False

    def retain_prefix(self, session: str, epoch: int, count: int) -> None:
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            if self._needs_rollback:
                raise ValidationError("failed tentative writes cannot be retained as an encoder prefix")
            self.map.retain_prefix(session, epoch, count)
            self.generations.copy_(torch.from_numpy(self.map.generations))
            torch.cuda.synchronize(self.device)

    # -------------------------------------------------------- transactions
    def write(self, logical_positions, token_positions, values) -> None:
        """Checked batch write with its undo backup: one device launch
        (dsr_pool_write); a refused batch leaves the pool needing rollback."""
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            if (self._needs_rollback or values.device != self.device or values.dtype != torch.bfloat16 or
                    tuple(values.shape) != (len(logical_positions), self.width) or not values.is_contiguous()):
                raise ValidationError("cache scatter state, shape or BF16 storage mismatch")
            start = len(self.map.journal)
            slots, previous = self.map.reserve(logical_positions, token_positions)
            p = _native.ptr
            d_slots = self._device_ints(slots, torch.int32)
            d_prev = self._device_ints(previous, torch.int64)
            stream = _native.stream_handle()
            try:
                _native.call("dsr_pool_write", p(self.data), p(self.generations), self.map.slots, self.width,
                             p(d_slots), p(d_prev), p(values), len(slots), p(self._undo), self._undo.shape[0],
                             start, p(self._err), stream)
                code = self._status("write")
            except BaseException:
                self._needs_rollback = True
                raise
            if code:
                self._needs_rollback = True
                raise ValidationError(f"native CUDA operation rejected input/state (code {code}); "
                                      "tentative writes require rollback")

    def physical(self, logical_positions):
        with self._mutex:
            self._open()
            if self._needs_rollback:
                raise ValidationError("failed tentative cache writes cannot be consumed")
            return self.map.physical(logical_positions)

    @contextmanager
    def read_window(self, operation):
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            if self._needs_rollback or self.map.active != operation:
                raise ValidationError("cache consumer targets a failed or stale window")
            try:
                yield self.data
            finally:
                torch.cuda.synchronize(self.device)

    def finish(self, operation, accepted: int) -> None:
        """Commits the accepted prefix; the rejected rows get their backup and previous
        generation back in one launch (dsr_pool_rollback)."""
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            if self._needs_rollback and accepted != 0:
                raise ValidationError("failed cache operation requires complete abort")
            rejected = self.map.rejected(operation, accepted)[::-1]  # journal order
            if rejected:
                p = _native.ptr
                d_slots = self._device_ints([m.slot for _, m in rejected], torch.int32)
                d_prev = self._device_ints([m.previous_generation for _, m in rejected], torch.int64)
                d_undo = self._device_ints([i for i, _ in rejected], torch.int32)
                try:
                    _native.call("dsr_pool_rollback", p(self.data), p(self.generations), self.map.slots,
                                 self.width, p(self._undo), self._undo.shape[0], p(d_slots), p(d_prev), p(d_undo),
                                 len(rejected), p(self._err), _native.stream_handle())
                    code = self._status("rollback")
                except BaseException:
                    self._needs_rollback = True
                    raise
                if code:
                    self._needs_rollback = True
                    raise ValidationError(f"native CUDA operation rejected input/state (code {code}); "
                                          "tentative writes require rollback")
            else:
                torch.cuda.synchronize(self.device)
            self.map.finish(operation, accepted)
            self._needs_rollback = False

    # ------------------------------------------------------------ snapshots
    def restore_rows(self, logical_positions, values) -> None:
        """Applies a validated snapshot tile into a fresh, quiescent epoch (dsr_pool_restore)."""
        import torch
        with self._mutex, torch.cuda.device(self.device):
            self._open()
            if (self.map.active is not None or self._needs_rollback or not 1 <= len(logical_positions) <= 1024 or
                    values.device != self.device or values.dtype != torch.bfloat16 or
                    tuple(values.shape) != (len(logical_positions), self.width) or not values.is_contiguous()):
                raise ValidationError("snapshot restore tile differs from its quiescent BF16 pool")
            slots, used = [], set()
            for logical in logical_positions:
                _integer(logical, "restored logical cache row", 0, self.map.context - 1)
                slot = self.map.slot_of(logical)
                if self.map.generations[slot] or slot in used:
                    raise ValidationError("snapshot repeats or overwrites a restored physical row")
                slots.append(slot)
                used.add(slot)
            p = _native.ptr
            d_logical = self._device_ints(list(logical_positions), torch.int64)
            _native.call("dsr_pool_restore", p(self.data), p(self.generations), self.map.slots, self.width,
                         self.map.offset, p(d_logical), p(values), len(slots), p(self._err), _native.stream_handle())
            code = self._status("restore")
            if code:
                raise ValidationError(f"native CUDA operation rejected input/state (code {code})")
            self.map.logical[slots] = list(logical_positions)
            self.map.generations[slots] = 1

    def snapshot_tiles(self, logical_positions):
        """Snapshot record of these logical rows: tiles of up to min(1024, 1 MiB / row
        bytes) rows in logical order, BF16 bits little-endian (snapshot_state.py:205-216)."""
        import torch
        logical_positions = list(logical_positions)
        step = min(1024, MAX_PAYLOAD // (self.width * 2))
        for start in range(0, len(logical_positions), step):
            rows = logical_positions[start:start + step]
            with self._mutex, torch.cuda.device(self.device):
                self._open()
                self.physical(rows)  # live and not overwritten
                p = _native.ptr
                d_logical = self._device_ints(rows, torch.int64)
                tile = self._tile[:len(rows)]
                _native.call("dsr_pool_gather", p(self.data), p(self.generations), self.map.slots, self.width,
                             self.map.offset, p(d_logical), len(rows), p(tile), p(self._err), _native.stream_handle())
                code = self._status("gather")
                if code == 2:
                    raise ValidationError("snapshot encountered nonfinite live state")
                if code:
                    raise ValidationError(f"snapshot rows are not live (code {code})")
                yield tile.view(torch.int16).cpu().numpy().view(np.uint16).tobytes()

    def close(self) -> None:
        import torch
        with self._mutex:
            if not self.closed:
                torch.cuda.synchronize(self.device)
                self.data = self.generations = self._undo = self._tile = None
                self.closed = True
