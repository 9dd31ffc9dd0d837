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


@dataclass(frozen=True)
class SlotMutation:
    token_position: int
    slot: int
    previous_logical: int
    previous_generation: int


class SlotMap:
    """Host slot metadata of one pool (cache_pool.py:24-153)."""

    def __init__(self, slots: int, *, context: int, offset: int, max_mutations: int = 64):
        self.slots = _integer(slots, "cache slots", 1, 1048576)
        self.context = _integer(context, "cache logical capacity", slots, 1048576)
        self.offset = _integer(offset, "local physical slot offset", 0, slots - 1)
        self.max_mutations = _integer(max_mutations, "undo row capacity", 1, 4096)
        self.logical = np.full(slots, -1, dtype=np.int64)
        self.generations = np.zeros(slots, dtype=np.int64)
        self.epoch, self.session, self.active = -1, None, None
        self.journal: list[SlotMutation] = []

    @property
    def metadata_bytes(self) -> int:
        return self.logical.nbytes + self.generations.nbytes

    def slot_of(self, logical: int) -> int:
        return (logical + self.offset) % self.slots

    def reset(self, session: str, epoch: int) -> None:
        _hex_id(session, 32, "cache session")
        _integer(epoch, "cache epoch", 0, I64_MAX)
        if self.active is not None or epoch <= self.epoch:
            raise ValidationError("cache reset requires quiescence and a newer epoch")
        self.session, self.epoch = session, epoch
        self.logical[:] = -1
        self.generations[:] = 0

    def discard_for_reset(self, session: str, epoch: int) -> None:
        _hex_id(session, 32, "cache session")
        _integer(epoch, "cache epoch", 0, I64_MAX)
        if epoch <= self.epoch:
            raise ValidationError("discarded cache recovery requires a newer epoch")
        self.active = None
        self.journal = []
        self.reset(session, epoch)

    def begin(self, operation) -> None:
        if (self.active is not None or operation.epoch != self.epoch or operation.session != self.session or
                operation.rows > 64 or operation.start + operation.rows > self.context):
            raise ValidationError("cache window is active, stale or exceeds its admitted bounds")
        self.active = operation

    def prepare(self, logical_positions, token_positions):
        """Validates a batch against the active window; returns (mutations, slots, generations)."""
        if self.active is None:
            raise ValidationError("cache mutation requires an active window")
        count = len(logical_positions)
        if count != len(token_positions) or not 1 <= count <= 64:
            raise ValidationError("cache row batch is empty or outside the admitted bound")
        if len(self.journal) + count > self.max_mutations:
            raise ValidationError("cache undo row capacity exhausted")
        last_token = self.journal[-1].token_position if self.journal else self.active.start
        window_end = self.active.start + self.active.rows - 1
        mutations, slots, generations, used = [], [], [], set()
        for logical, token in zip(logical_positions, token_positions):
            _integer(logical, "cache logical position", 0, self.context - 1)
            _integer(token, "cache producing token", last_token, window_end)
            last_token = token
            slot = self.slot_of(logical)
            if slot in used:
                raise ValidationError("one scatter batch repeats a physical cache slot")
            used.add(slot)
            generation = int(self.generations[slot])
            if generation == I64_MAX:
                raise ValidationError("cache generation exhausted; coordinated new epoch required")
            mutations.append(SlotMutation(token, slot, int(self.logical[slot]), generation))
            slots.append(slot)
            generations.append(generation)
        return mutations, slots, generations

    def reserve(self, logical_positions, token_positions):
        mutations, slots, generations = self.prepare(logical_positions, token_positions)
        for logical, m in zip(logical_positions, mutations):  # the whole batch was validated
            self.logical[m.slot] = logical
            self.generations[m.slot] = m.previous_generation + 1
        self.journal.extend(mutations)
        return slots, generations

    def physical(self, logical_positions):
        out = []
        for logical in logical_positions:
            if logical == -1:
                out.append(-1)
                continue
            _integer(logical, "visible cache logical position", 0, self.context - 1)
            slot = self.slot_of(logical)
            if self.logical[slot] != logical or self.generations[slot] == 0:
                raise ValidationError("cache row is absent or its physical slot was overwritten")
            out.append(slot)
        return out

    def validate_prefix(self, count: int) -> None:
        _integer(count, "retained compressed rows", 0, self.slots)
        if self.active is not None:
            raise ValidationError("prefix retention requires quiescent cache metadata")
        logical = np.arange(count, dtype=np.int64)
        slots = (logical + self.offset) % self.slots
        if np.any(self.logical[slots] != logical) or np.any(self.generations[slots] <= 0):
            raise ValidationError("retained encoder prefix has missing or overwritten source rows")

    def retain_prefix(self, session: str, epoch: int, count: int) -> None:
        _hex_id(session, 32, "retained prefix session")
        _integer(epoch, "retained prefix epoch", self.epoch + 1, I64_MAX)
        self.validate_prefix(count)
        keep = (self.logical >= 0) & (self.logical < count)
        self.logical[~keep] = -1
        self.generations[:] = keep
        self.session, self.epoch = session, epoch
        self.journal = []

    def rejected(self, operation, accepted: int):
        """(journal index, mutation) of the rows past the accepted prefix, newest first."""
        _integer(accepted, "cache accepted prefix", 0, operation.rows)
        if self.active != operation:
            raise ValidationError("cache commit targets another operation")
        boundary = operation.start + accepted
        return [(i, m) for i, m in reversed(list(enumerate(self.journal))) if m.token_position >= boundary]

    def finish(self, operation, accepted: int) -> None:
        for _, m in self.rejected(operation, accepted):
            self.logical[m.slot] = m.previous_logical
            self.generations[m.slot] = m.previous_generation
        self.journal = []
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
