"""NVLink peer exchange (dsr_p2p_*) on two GPUs of one node: the all-gather agrees with
NCCL's, and the sharded decode step gives the same bits with either exchange."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs of one node")
def test_peer_exchange_matches_nccl_on_two_gpus():
    worker = Path(__file__).resolve().parent / "_peer_worker.py"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), str(worker)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "PEER_EXCHANGE_OK" in proc.stdout


def test_exchange_wait_runs_out_without_a_peer(cuda):
    """A world-2 exchange whose second buffer is a local one that no peer ever
    signals: the bounded arrival wait gives up with DSR_ERR_TIMEOUT after about
    2 s (no hang), and the local epoch still advances past the abandoned step."""
    import ctypes
    import time

    from deepseekrpc_b200 import _native
    from deepseekrpc_b200._native import call, ptr, stream_handle
    from deepseekrpc_b200.sharded import _DeviceView

    lib = _native.library()
    payload = torch.arange(64, dtype=torch.int32, device=cuda)
    size = lib.dsr_p2p_buffer_bytes(2, payload.numel() * 4)
    buffers, handle = [], (ctypes.c_uint8 * 64)()
    for _ in range(2):
        buf = ctypes.c_void_p()
        call("dsr_p2p_alloc", size, ctypes.addressof(buf), ctypes.addressof(handle))
        buffers.append(buf.value)
    table = (ctypes.c_void_p * 2)(*buffers)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for attempt in (1, 2):
            err.zero_()
            t0 = time.perf_counter()
            call("dsr_p2p_allgather", ptr(payload), payload.numel() * 4, ctypes.cast(table, ctypes.c_void_p), 0, 2,
                 payload.numel() * 4, 1, ptr(err), stream_handle())
            torch.cuda.synchronize()
            elapsed = time.perf_counter() - t0
            assert int(err.item()) == _native.DSR_ERR_TIMEOUT, f"attempt {attempt}: status {int(err.item())}"
            assert elapsed < 10.0, f"the wait took {elapsed:.1f} s"
            control = torch.as_tensor(_DeviceView(buffers[0], (16,), "<i4"), device=cuda).clone()
            assert int(control[8].item()) == attempt, "the epoch did not advance past the timed-out exchange"
            # this rank's own slot arrived in the local buffer; the silent peer's did not
            assert int(control[0].item()) == attempt and int(control[1].item()) == 0
    finally:
        torch.cuda.synchronize()
        for b in buffers:
            call("dsr_p2p_free", b)
