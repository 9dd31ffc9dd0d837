"""Row-pool transactions on the B200 (dsr_pool_*), through the DeviceRowPool mirror, against
the oracle's restatement of the reference's DeviceRowPool (cache_pool.py:289-352) and its
snapshot row streaming (snapshot_state.py:205-216, cache_pool.py:255-274)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from deepseekrpc_b200.cache_pool import DeviceRowPool, Operation
from deepseekrpc_b200.cuda_ops import ValidationError

pytestmark = pytest.mark.gpu
S = "c" * 32


def bf16_rows(rng, n, width):
    bits = oracle.f32_to_bf16_bits(rng.normal(size=(n, width)).astype(np.float32))
    return bits, torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda().contiguous()


def device_state(pool):
    return (pool.data.view(torch.int16).cpu().numpy().view(np.uint16), pool.generations.cpu().numpy())


class Mirror:
    """A DeviceRowPool and the oracle driven by the same host journal."""

    def __init__(self, slots=64, width=576, offset=5, context=256, undo=64):
        self.pool = DeviceRowPool(slots, width, context=context, offset=offset, admitted_bytes=1 << 30,
                                  max_mutations=undo)
        self.ref = oracle.PoolOracle(slots, width, undo)
        # the reference's own write path (partial writes, bump only on success):
        # after every finish its state must equal the device's too
        self.ref_partial = oracle.ReferenceRowPool(slots, width, undo)
        self.width = width

    def write(self, rng, logical, tokens, poison=False):
        bits, values = bf16_rows(rng, len(logical), self.width)
        if poison:
            bits[0, 3] = 0x7FC0
            values = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda().contiguous()
        start = len(self.pool.map.journal)
        try:
            self.pool.write(logical, tokens, values)
        finally:
            if len(self.pool.map.journal) > start:  # the host reserved the batch: mirror it
                new = self.pool.map.journal[start:]
                for ref in (self.ref, self.ref_partial):
                    ref.write([m.slot for m in new], [m.previous_generation for m in new], bits, start)

    def finish(self, op, accepted):
        rejected = self.pool.map.rejected(op, accepted)[::-1]
        self.pool.finish(op, accepted)
        for ref in (self.ref, self.ref_partial):
            ref.finish([(i, m.slot, m.previous_generation) for i, m in rejected])

    def check(self):
        """After a finish: the device equals both restatements (whole-batch refusal and
        the reference's partial writes) bit for bit."""
        data, gens = device_state(self.pool)
        assert np.array_equal(data, self.ref.data) and np.array_equal(gens, self.ref.generations)
        assert np.array_equal(data, self.ref_partial.data), "end state differs from the reference's write -> finish"
        assert np.array_equal(gens, self.ref_partial.generations)


def test_random_transactions_match_the_reference_semantics(cuda):
    rng = np.random.default_rng(71)
    m = Mirror()
    m.pool.reset(S, 1)
    start, epoch = 0, 1
    for _ in range(24):
        rows = int(rng.integers(1, 6))
        op = Operation(S, epoch, start, rows)
        m.pool.begin(op)
        token = start
        for _ in range(int(rng.integers(1, 3))):  # one or two write batches per window
            n = int(rng.integers(1, rows - (token - start) + 1)) if token < start + rows else 0
            if n == 0:
                break
            logical = list(range(token, token + n))
            m.write(rng, logical, list(range(token, token + n)))
            token += n
        accepted = int(rng.integers(0, token - start + 1))
        m.finish(op, accepted)
        m.check()
        start += accepted


def test_refused_batch_rolls_back_to_the_previous_state(cuda):
    rng = np.random.default_rng(72)
    m = Mirror(slots=16, width=128, offset=3)
    m.pool.reset(S, 1)
    op = Operation(S, 1, 0, 4)
    m.pool.begin(op)
    m.write(rng, [0, 1], [0, 1])
    m.finish(op, 2)
    before = device_state(m.pool)
    op = Operation(S, 1, 2, 4)
    m.pool.begin(op)
    m.write(rng, [2], [2])
    with pytest.raises(ValidationError):  # a NaN element refuses the whole batch on the device
        m.write(rng, [3, 4], [3, 4], poison=True)
    with pytest.raises(ValidationError):
        m.pool.physical([0])  # failed tentative writes cannot be consumed
    with pytest.raises(ValidationError):
        m.pool.finish(op, 1)  # a failed operation needs a complete abort
    m.finish(op, 0)
    m.check()
    data, gens = device_state(m.pool)
    assert np.array_equal(data, before[0]) and np.array_equal(gens, before[1])
    # a device generation that disagrees with the host map is refused (status 3)
    m.pool.generations[m.pool.map.slot_of(5)] = 7
    op = Operation(S, 1, 2, 4)
    m.pool.begin(op)
    with pytest.raises(ValidationError):
        m.pool.write([5], [2], bf16_rows(rng, 1, 128)[1])
    m.pool.finish(op, 0)  # the rollback puts back the host map's previous generation
    assert int(m.pool.generations[m.pool.map.slot_of(5)]) == 0


def test_rejected_rewrite_of_one_slot_restores_the_earliest_backup(cuda):
    rng = np.random.default_rng(73)
    m = Mirror(slots=8, width=64, offset=0, context=64)
    m.pool.reset(S, 1)
    op = Operation(S, 1, 0, 3)
    m.pool.begin(op)
    m.write(rng, [0], [0])
    m.finish(op, 1)
    op = Operation(S, 1, 1, 6)
    m.pool.begin(op)
    m.write(rng, [1, 2], [1, 2])
    m.write(rng, [9], [3])   # logical 9 lands on slot 1 again (8 slots)
    m.write(rng, [10], [4])  # and logical 10 on slot 2
    m.finish(op, 1)          # keeps logical 1 only: slot 1 must hold logical 1's row
    m.check()
    assert m.pool.physical([0, 1]) == [0, 1]


def test_snapshot_tiles_and_restore_round_trip(cuda):
    rng = np.random.default_rng(74)
    width, count = 576, 1500  # two snapshot tiles of up to 910 rows (1 MiB each)
    src = DeviceRowPool(2048, width, context=4096, offset=77, admitted_bytes=1 << 31)
    src.reset(S, 1)
    ref = oracle.PoolOracle(2048, width, 64)
    for start in range(0, count, 64):
        n = min(64, count - start)
        op = Operation(S, 1, start, n)
        src.begin(op)
        bits, values = bf16_rows(rng, n, width)
        src.write(list(range(start, start + n)), list(range(start, start + n)), values)
        src.finish(op, n)
        ref.restore([(p + 77) % 2048 for p in range(start, start + n)], bits)
    tiles = list(src.snapshot_tiles(range(count)))
    assert [len(t) for t in tiles] == [910 * width * 2, (count - 910) * width * 2]
    assert b"".join(tiles) == ref.gather(list(range(count)), 77).tobytes()
    # restore the record into a fresh pool with another offset, as snapshot_restore does
    dst = DeviceRowPool(2048, width, context=4096, offset=5, admitted_bytes=1 << 31)
    dst.reset(S, 3)
    blob = np.frombuffer(b"".join(tiles), np.uint16).reshape(count, width)
    for start in range(0, count, 1024):
        rows = blob[start:start + 1024]
        values = torch.from_numpy(rows.view(np.int16).copy()).view(torch.bfloat16).cuda()
        dst.restore_rows(list(range(start, start + len(rows))), values)
    assert b"".join(dst.snapshot_tiles(range(count))) == b"".join(tiles)
    with pytest.raises(ValidationError):  # a live row is never overwritten by a restore
        dst.restore_rows([3], torch.zeros((1, width), dtype=torch.bfloat16, device="cuda"))
    # non-finite live state is refused by the snapshot
    src.data[(12 + 77) % 2048, 5] = float("inf")
    with pytest.raises(ValidationError):
        list(src.snapshot_tiles(range(20)))
