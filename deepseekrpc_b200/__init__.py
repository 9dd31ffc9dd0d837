"""B200-native (sm_100a) implementation of DeepSeekRPC's attention hot path.

Layers:
  include/dsr_b200.h / libdsr_b200.so   C ABI over the hand-written kernels (_native: ctypes)
  deepseekrpc_cuda (torch extension)    the reference module's op names on that ABI
  cuda_ops, index_selection             host-side mirrors of the reference modules
  sharded                               sequence sharding across GPUs (NCCL)
  workloads                             seeded BASELINE-config inputs
"""
from __future__ import annotations

import importlib
import sys

__all__ = ["extension"]


def extension():
    """The `deepseekrpc_cuda` torch extension built in this package.

    Also registers it under the top-level name `deepseekrpc_cuda`, so code
    written against the reference (`import deepseekrpc_cuda`) binds to it.
    Raises ImportError when the extension has not been built.
    """
    module = sys.modules.get("deepseekrpc_cuda")
    if module is None or not getattr(module, "__file__", "").startswith(__path__[0]):
        import torch  # noqa: F401  (loads libc10/libtorch before the extension)
        module = importlib.import_module(".deepseekrpc_cuda", __name__)
        sys.modules["deepseekrpc_cuda"] = module
    if module.abi_version() != 2:
        raise RuntimeError("deepseekrpc_cuda ABI does not match this source")
    return module
