"""ctypes binding of the C ABI (include/dsr_b200.h) in libdsr_b200.so.

This is the plain-pointer boundary a non-PyTorch host (cgo, JNI, N-API, ctypes)
binds; the parity tests call the kernels through it.  Loading fails loudly
when the library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from functools import lru_cache
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdsr_b200.so"

DSR_OK, DSR_EINVAL, DSR_ECUDA, DSR_ENODEV = 0, -1, -2, -3
DSR_ERR_ID, DSR_ERR_NONFINITE, DSR_ERR_SCATTER, DSR_ERR_TIMEOUT = 1, 2, 3, 4

_P = c_void_p  # every device pointer travels as an opaque address

# name -> (restype, argtypes); mirrors include/dsr_b200.h exactly
SIGNATURES = {
    "dsr_abi_version": (c_int, []),
    "dsr_last_error": (c_char_p, []),
    "dsr_device_check": (c_int, []),
    "dsr_index_scores": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P]),
    "dsr_sparse_attention": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64,
                                     c_int64, c_int64, c_float, _P]),
    "dsr_scatter_slots": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, _P]),
    "dsr_engram_decode": (c_int, [_P, _P, _P, c_int64, _P]),
    "dsr_topk_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "dsr_topk_select": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P, c_size_t,
                                _P]),
    "dsr_topk_select_noalloc": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64,
                                        _P]),
    "dsr_indexer_decode": (c_int, [_P, _P, _P, c_int64, _P, c_int64, _P, _P, c_int64, _P, c_int64,
                                   c_int64, _P]),
    "dsr_indexer_prefill": (c_int, [_P, _P, _P, c_int64, _P, c_int64, _P, _P, c_int64, _P, c_int64,
                                    c_int64, _P]),
    "dsr_candidate_blocks_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "dsr_candidate_blocks": (c_int, [_P, _P, c_int64, c_int64, c_int64, _P, _P, c_size_t, _P, _P]),
    "dsr_candidate_select_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "dsr_candidate_select": (c_int, [_P, _P, c_int64, _P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64,
                                     _P, _P, c_size_t, _P, c_int64, _P]),
    "dsr_mla_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "dsr_sparse_mla_decode": (c_int, [_P, _P, c_int64, _P, c_int64, _P, _P, c_int64, _P, _P, _P,
                                      c_float, _P, _P, c_size_t, _P, c_int64, c_int64, _P]),
    "dsr_sparse_mla_partial": (c_int, [_P, _P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64, _P, _P,
                                       c_float, _P, _P, _P, _P, c_size_t, _P, c_int64, c_int64, _P]),
    "dsr_indexer_topk_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "dsr_indexer_topk_decode": (c_int, [_P, _P, c_int64, _P, c_int64, _P, c_int64, _P, c_int64, c_int64,
                                        c_int64, _P, _P, _P, _P, c_size_t, _P, c_int64, _P]),
    "dsr_topk_merge_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "dsr_topk_merge_lists": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, c_size_t, _P, _P]),
    "dsr_lse_combine_packed": (c_int, [_P, c_int64, _P, _P, _P, c_int64, c_int64, _P]),
    "dsr_append_kv_index": (c_int, [_P, _P, _P, c_int64, _P, c_int64, c_int64, _P, _P, _P, _P, _P,
                                    _P, _P, c_int64, _P]),
    "dsr_lse_combine": (c_int, [_P, _P, _P, c_int64, _P, _P, _P, _P, _P, c_int64, c_int64, c_int64,
                                _P]),
    "dsr_pool_write": (c_int, [_P, _P, c_int64, c_int64, _P, _P, _P, c_int64, _P, c_int64, c_int64, _P, _P]),
    "dsr_pool_rollback": (c_int, [_P, _P, c_int64, c_int64, _P, c_int64, _P, _P, _P, c_int64, _P, _P]),
    "dsr_pool_gather": (c_int, [_P, _P, c_int64, c_int64, c_int64, _P, c_int64, _P, _P, _P]),
    "dsr_pool_restore": (c_int, [_P, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, _P, _P]),
    "dsr_p2p_buffer_bytes": (c_size_t, [c_int64, c_int64]),
    "dsr_p2p_alloc": (c_int, [c_size_t, _P, _P]),
    "dsr_p2p_open": (c_int, [_P, _P]),
    "dsr_p2p_close": (c_int, [_P]),
    "dsr_p2p_free": (c_int, [_P]),
    "dsr_p2p_allgather": (c_int, [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int64, _P, _P]),
    "dsr_decode_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "dsr_decode_step_launches": (c_int, [c_int64, c_int64, c_int64, c_int64]),
    "dsr_indexer_decode_ring": (c_int, [_P, _P, _P, c_int64, _P, _P, _P, c_int64, _P, c_int64, c_int64, _P]),
    "dsr_sparse_mla_decode_ring": (c_int, [_P, _P, c_int64, _P, _P, _P, c_int64, _P, c_int64, _P, _P, _P,
                                           c_float, _P, _P, c_size_t, _P, c_int64, c_int64, _P]),
    "dsr_decode_step_ring": (c_int, [_P, _P, c_int64, _P, c_int64, _P, _P, _P, c_int64, _P, c_int64, _P,
                                     c_int64, c_int64, _P, c_int64, _P, _P, _P, c_float, _P, _P, _P, _P,
                                     c_size_t, _P, c_int64, _P]),
    "dsr_append_kv_index_ring": (c_int, [_P, c_int64, _P, _P, _P, _P, c_int64, _P, _P, _P, c_int64, _P, _P,
                                         _P, _P, _P, c_int64, _P]),
    "dsr_decode_step": (c_int, [_P, _P, c_int64, _P, _P, _P, c_int64, c_int64, _P, c_int64, _P,
                                c_int64, c_int64, _P, _P, _P, c_float, _P, _P, _P, _P, c_size_t, _P,
                                c_int64, _P]),
}


class NativeError(RuntimeError):
    """A host-side refusal (argument/bound violation or launch failure)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (code {code})")
        self.code = code


@lru_cache(maxsize=1)
def library() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing; run `python -m deepseekrpc_b200.build` "
                          "(there is no CPU fallback for these kernels)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def last_error() -> str:
    return (library().dsr_last_error() or b"").decode()


def call(name: str, *args) -> int:
    """Calls a C-ABI entry point and raises NativeError on a nonzero host return."""
    rc = getattr(library(), name)(*args)
    if rc != DSR_OK:
        raise NativeError(rc, last_error())
    return rc


def ptr(tensor) -> int | None:
    """Device address of a torch tensor (None for None)."""
    return None if tensor is None else tensor.data_ptr()


def stream_handle(stream=None) -> int:
    """cudaStream_t of a torch stream (default: the current stream)."""
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream
