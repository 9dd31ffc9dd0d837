"""Fused KV + index-key + SWA append (dsr_append_kv_index) against the oracle's
restatement of the reference's checked scatter and generation bump
(native/operations.cu:144-161, cache_pool.py:309, vllm_attention.py:261).

Pools, the SWA ring and the generations are compared bit for bit after every
batch; every refusal case (out of bounds, a repeated row, a stale generation, a
repeated SWA ring row, NaN in the KV half, Inf in the index half) runs in a batch
of its own next to valid rows, so its status code is definite, and the refused
rows must stay untouched.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle.append import ERR_NONFINITE, ERR_SCATTER, append_kv_index, paged_rows
from _helpers import finish, status
from deepseekrpc_b200._native import call, ptr, stream_handle

pytestmark = pytest.mark.gpu


def bits_tensor(bits):
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).cuda()


def host_bits(t):
    return t.cpu().numpy().view(np.uint16)


class Pools:
    """Device pools and their host copies, paged in 64-row blocks by a seeded permutation."""

    def __init__(self, rng, lengths, spare_blocks=8):
        self.lengths = list(lengths)
        blocks = [(n + 1 + 63) // 64 + 1 for n in lengths]  # room for the appended positions
        total = sum(blocks) + spare_blocks
        perm = rng.permutation(total).astype(np.int32)
        self.table = np.full((len(lengths), max(blocks)), -1, np.int32)
        start = 0
        for b, nb in enumerate(blocks):
            self.table[b, :nb] = perm[start:start + nb]
            start += nb
        self.pool_blocks = total
        rows = total * 64
        self.kv = oracle.f32_to_bf16_bits(rng.normal(size=(rows, 576)).astype(np.float32))
        self.ix = oracle.f32_to_bf16_bits(rng.normal(size=(rows, 128)).astype(np.float32))
        self.swa = oracle.f32_to_bf16_bits(rng.normal(size=(len(lengths), 128, 576)).astype(np.float32))
        self.gen = rng.integers(0, 5, size=rows).astype(np.int64)
        self.d_kv, self.d_ix, self.d_swa = bits_tensor(self.kv), bits_tensor(self.ix), bits_tensor(self.swa)
        self.d_gen = torch.from_numpy(self.gen.copy()).cuda()
        self.d_table = torch.from_numpy(self.table).cuda()

    def append(self, seq, positions, expected, kv_bits, ix_bits, use_swa=True):
        n = len(seq)
        err = status()
        d_seq = torch.tensor(seq, dtype=torch.int32, device="cuda")
        d_pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
        d_exp = torch.tensor(expected, dtype=torch.int64, device="cuda")
        d_kvv, d_ixv = bits_tensor(kv_bits), bits_tensor(ix_bits)
        call("dsr_append_kv_index", ptr(self.d_kv), ptr(self.d_ix), ptr(self.d_gen), self.pool_blocks,
             ptr(self.d_table), self.table.shape[0], self.table.shape[1], ptr(d_seq), ptr(d_pos), ptr(d_exp),
             ptr(d_kvv), ptr(d_ixv), ptr(self.d_swa) if use_swa else None, ptr(err), n, stream_handle())
        code = finish(err)
        rows = paged_rows(self.table, self.pool_blocks, seq, positions)
        codes = append_kv_index(self.kv, self.ix, self.gen, rows, seq, positions, expected, kv_bits, ix_bits,
                                self.swa if use_swa else None)
        return code, codes

    def check(self):
        assert np.array_equal(host_bits(self.d_kv), self.kv), "KV pool differs from the oracle"
        assert np.array_equal(host_bits(self.d_ix), self.ix), "index-key pool differs from the oracle"
        assert np.array_equal(host_bits(self.d_swa), self.swa), "SWA ring differs from the oracle"
        assert np.array_equal(self.d_gen.cpu().numpy(), self.gen), "generations differ from the oracle"

    def expected_for(self, seq, positions):
        rows = paged_rows(self.table, self.pool_blocks, seq, positions)
        return [int(self.gen[r]) if r >= 0 else 0 for r in rows]


def new_rows(rng, n):
    kv = oracle.f32_to_bf16_bits(rng.normal(size=(n, 576)).astype(np.float32))
    ix = oracle.f32_to_bf16_bits(rng.normal(size=(n, 128)).astype(np.float32))
    return kv, ix


def test_ragged_batch_of_32_sequences_appends_bit_exact(cuda):
    rng = np.random.default_rng(301)
    lengths = rng.integers(100, 3000, size=32)
    p = Pools(rng, lengths)
    seq = list(range(32))
    positions = [int(n) for n in lengths]
    for step in range(3):  # consecutive steps: each expects the previous step's bump
        expected = p.expected_for(seq, positions)
        kv, ix = new_rows(rng, 32)
        code, codes = p.append(seq, positions, expected, kv, ix)
        assert code == 0 and not codes
        p.check()
        positions = [q + 1 for q in positions]


def test_append_without_swa_ring_and_speculative_rows(cuda):
    rng = np.random.default_rng(302)
    p = Pools(rng, [500, 70, 1000])
    # six consecutive rows of one sequence and one each of the others, no ring
    seq = [0] * 6 + [1, 2]
    positions = [500 + i for i in range(6)] + [70, 1000]
    kv, ix = new_rows(rng, len(seq))
    code, codes = p.append(seq, positions, p.expected_for(seq, positions), kv, ix, use_swa=False)
    assert code == 0 and not codes
    p.check()


CASES = ["bounds", "duplicate", "stale", "ring", "nan_kv", "inf_index"]


@pytest.mark.parametrize("case", CASES)
def test_refused_rows_leave_nothing_behind(cuda, case):
    rng = np.random.default_rng(303 + CASES.index(case))
    lengths = [200, 900, 64, 4000]
    p = Pools(rng, lengths)
    seq = [0, 1, 2, 3]
    positions = [200, 900, 64, 4000]
    expected = p.expected_for(seq, positions)
    kv, ix = new_rows(rng, 4)
    want = ERR_SCATTER
    if case == "bounds":
        # a position past the block table, an unmapped block, a sequence past the table
        seq += [1, 2, 9]
        positions += [p.table.shape[1] * 64 + 5, 64 * (p.table.shape[1] - 1), 3]
        expected += [0, 0, 0]
        p.table[2, -1] = -1
        p.d_table.copy_(torch.from_numpy(p.table))
        extra_kv, extra_ix = new_rows(rng, 3)
        kv, ix = np.concatenate([kv, extra_kv]), np.concatenate([ix, extra_ix])
    elif case == "duplicate":
        seq.append(1)
        positions.append(900)
        expected.append(expected[1])
        extra_kv, extra_ix = new_rows(rng, 1)
        kv, ix = np.concatenate([kv, extra_kv]), np.concatenate([ix, extra_ix])
    elif case == "stale":
        expected[2] += 1
    elif case == "ring":
        # positions 900 and 772 of sequence 1 share ring row 900 % 128
        seq.append(1)
        positions.append(772)
        expected += p.expected_for([1], [772])
        extra_kv, extra_ix = new_rows(rng, 1)
        kv, ix = np.concatenate([kv, extra_kv]), np.concatenate([ix, extra_ix])
    elif case == "nan_kv":
        kv[1, 37] = 0x7FC1
        want = ERR_NONFINITE
    elif case == "inf_index":
        ix[3, 127] = 0xFF80
        want = ERR_NONFINITE
    kv_before, ix_before, gen_before = p.kv.copy(), p.ix.copy(), p.gen.copy()
    code, codes = p.append(seq, positions, expected, kv, ix)
    assert codes == {want}, f"oracle raised {codes}"
    assert code == want, f"device status {code}, expected {want}"
    p.check()
    # the refused row's targets are untouched and the valid rows were appended
    rows = paged_rows(p.table, p.pool_blocks, seq, positions)
    written = [i for i, r in enumerate(rows) if r >= 0 and p.gen[r] == expected[i] + 1]
    assert len(written) >= 3
    if case in ("nan_kv", "inf_index", "stale"):
        bad = {"nan_kv": 1, "inf_index": 3, "stale": 2}[case]
        r = rows[bad]
        assert np.array_equal(p.kv[r], kv_before[r]) and np.array_equal(p.ix[r], ix_before[r])
        assert p.gen[r] == gen_before[r]
