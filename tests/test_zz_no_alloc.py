"""Allocation-free top-k entry point (dsr_topk_select_noalloc).

It must give exactly what dsr_topk_select gives with a caller workspace, call
after call on the library's fixed scratch, and refuse sizes beyond that scratch
before touching a device.  The file sorts last so the GPU case also runs after
every other test has used the device.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _helpers import c_topk, dev, finish, status
from deepseekrpc_b200 import _native
from deepseekrpc_b200._native import ptr, stream_handle

SCRATCH_BYTES = 16 << 20  # DSR_TOPK_NOALLOC_BYTES


def c_topk_noalloc(scores, lengths, k, ids=None, id_base=0):
    rows, stride = scores.shape
    out = torch.empty((rows, k), dtype=torch.int32, device="cuda")
    out_s = torch.empty((rows, k), dtype=torch.float32, device="cuda")
    err = status()
    rc = _native.library().dsr_topk_select_noalloc(ptr(scores), ptr(ids), ptr(lengths), ptr(out), ptr(out_s),
                                                   ptr(err), rows, stride, k, id_base, stream_handle())
    assert rc == 0, _native.last_error()
    return out, out_s, finish(err)


def test_noalloc_refuses_sizes_beyond_its_scratch_without_a_device():
    lib = _native.library()
    assert lib.dsr_topk_workspace_bytes(8, 131072) <= SCRATCH_BYTES < lib.dsr_topk_workspace_bytes(16, 131072)
    # 16 rows x 131072 entries need more than the fixed scratch: refused on the host
    assert lib.dsr_topk_select_noalloc(1, None, 1, 1, None, 1, 16, 131072, 2048, 0, None) == _native.DSR_EINVAL
    assert "scratch" in _native.last_error()
    assert lib.dsr_topk_select_noalloc(1, None, 1, 1, None, 1, 1, 1 << 30, 2048, 0, None) == _native.DSR_EINVAL
    # ids past int32 (id_base + entries) are refused before any CUDA call too
    assert lib.dsr_topk_select_noalloc(1, None, 1, 1, None, 1, 1, 4096, 2048, (1 << 31) - 4096, None) == \
        _native.DSR_EINVAL
    assert "id_base" in _native.last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_on_consecutive_calls(cuda):
    rng = np.random.default_rng(97)
    # call 1: ragged rows at the largest accepted size, normal scores
    lengths1 = [131072, 0, 2047, 50000, 131072, 9000, 1, 70000]
    s1 = rng.normal(size=(8, 131072)).astype(np.float32)
    s1[5, :9000] = np.round(s1[5, :9000])  # heavy ties
    # call 2: another shape, explicit ids with -1 holes, a k that exceeds some rows
    n2 = 40000
    s2 = (np.round(rng.normal(size=(3, n2)) * 4) / 4).astype(np.float32)
    ids2 = np.tile(np.arange(n2, dtype=np.int32) * 3, (3, 1))
    ids2[:, 7::11] = -1
    lengths2 = [n2, 3000, 25000]
    cases = [(dev(s1), dev(np.array(lengths1, np.int32)), 2048, None),
             (dev(s2), dev(np.array(lengths2, np.int32)), 4096, dev(ids2))]
    for repeat in range(2):  # the scratch is reused call after call
        for scores, lengths, k, ids in cases:
            want, want_s, want_code = c_topk(scores, lengths, k, ids=ids, return_scores=True)
            got, got_s, code = c_topk_noalloc(scores, lengths, k, ids=ids)
            assert code == want_code == 0
            assert torch.equal(got, want), f"ids differ (repeat {repeat}, k {k})"
            assert torch.equal(got_s, want_s), f"scores differ (repeat {repeat}, k {k})"
