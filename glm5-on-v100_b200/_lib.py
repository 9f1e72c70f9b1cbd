"""ctypes binding of libdsa_b200.so — the C ABI declared in include/dsa_b200.h.

The library is REQUIRED: there is no CPU or PyTorch fallback. ``lib()`` raises
``DsaLibraryError`` when the shared object is missing (build it with
``python glm5-on-v100_b200/build.py``).
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsa_b200.so")

# status codes (include/dsa_b200.h)
DSA_OK = 0
DSA_ERR_INVALID = 1
DSA_ERR_UNSUPPORTED = 2
DSA_ERR_TIMEOUT = 3
DSA_ERR_CUDA = 4
DSA_ERR_WORKSPACE = 5
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "TIMEOUT", 4: "CUDA", 5: "WORKSPACE"}

# element / cache formats
DSA_F16 = 0
DSA_BF16 = 1
DSA_F32 = 2
DSA_FP8_DS_MLA = 3
DSA_FP8_IDXK = 4

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_d = ctypes.c_double

# name -> (restype, argtypes); one entry per function of include/dsa_b200.h
SIGNATURES = {
    "dsa_last_error": (ctypes.c_char_p, []),
    "dsa_version": (_i, []),
    "dsa_device_error": (_i, [_i]),
    "dsa_selftest_wait_timeout": (_i, [_i64, _p]),
    "dsa_sparse_mla_decode_workspace_bytes": (_sz, [_i, _i, _i]),
    "dsa_sparse_mla_decode_plan": (_i, [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i),
                                        ctypes.POINTER(_sz), ctypes.POINTER(_i)]),
    "dsa_sparse_mla_decode": (_i, [_p, _i, _p, _p, _i, _p, _i, _i64, _i, _p, _i64, _p, _i64, _i, _p,
                                   _i, _i, _i, _d, _p, _sz, _p]),
    "dsa_sparse_mla_decode_noalloc": (_i, [_p, _i, _p, _p, _i, _p, _i, _i64, _i, _p, _i64, _p, _i64, _i,
                                           _p, _i, _i, _i, _d, _p]),
    "dsa_indexer_logits": (_i, [_p, _i64, _i, _p, _i, _p, _i, _i64, _i, _p, _i, _p, _i64, _i, _p, _i,
                                _i, _p, _p]),
    "dsa_indexer_logits_packed": (_i, [_p, _i64, _i, _p, _i, _p, _i, _i64, _i, _p, _i, _p, _i64, _i,
                                       _p, _i, _p]),
    "dsa_decode_topk": (_i, [_p, _i64, _p, _i64, _i, _p, _p, _i, _i, _p]),
    "dsa_topk_rows": (_i, [_p, _i64, _p, _i64, _i, _p, _i, _i, _p]),
    "dsa_indexer_k_store": (_i, [_p, _i, _i64, _p, _i, _i, _p, _i, _p]),
    "dsa_indexer_shard_merge": (_i, [_p, _i64, _p, _p, _i, _i, _i, _i, _p]),
    "dsa_indexer_shard_merge_p2p": (_i, [_p, _i64, _p, _p, _p, _i, _i, _i, _i, _i, _i64, _i64, _p, _p]),
    "dsa_ipc_alloc": (_i, [_i64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "dsa_ipc_free": (_i, [_p]),
    "dsa_ipc_open": (_i, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "dsa_ipc_close": (_i, [_p]),
    "dsa_ipc_flag_set": (_i, [ctypes.c_uint64, _i, _i, _p, _p]),
    "dsa_ipc_slot_wait": (_i, [_p, _i, _i, _i64, _p, _p]),
    "dsa_indexer_shard_stage": (_i, [_p, _p, _i64, _p, _i64, _i, _i, _p, _p]),
    "dsa_topk_rows_payload": (_i, [_p, _i64, _p, _i64, _i, _p, _p, _i, _i, _i, _p]),
    "dsa_shard_exchange_topk": (_i, [_p, _i64, _i, _p, _p, _i, _i, _i, _p, _i64, _p, _i, _i, _p, _i64, _p, _p]),
    "dsa_shard_exchange_merge": (_i, [_p, _i64, _p, _p, _i, _i, _i, _i, _i64, _p, _i64, _p, _p]),
    "dsa_concat_and_cache_ds_mla": (_i, [_p, _i64, _p, _i64, _p, _i64, _i, _p, _i, _p, _p, _i64, _i, _p]),
    "dsa_indexer_qk_store": (_i, [_p, _i, _p, _i, _p, _i, _i64, _p, _i64, _p, _i64, _i, _p, _p, ctypes.c_float, _p,
                                  _p, _i64, _i, ctypes.c_float, _p, _i, _i, _p]),
}


class DsaLibraryError(ImportError):
    """libdsa_b200.so is missing or does not export the expected ABI."""


class DsaError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        super().__init__(f"{fn} failed [{STATUS_NAMES.get(status, status)}]: {message}")


_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise DsaLibraryError(
                    f"{LIB_PATH} not found: the DSA CUDA library is required (no fallback). "
                    "Build it with `python glm5-on-v100_b200/build.py`.")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                try:
                    fn = getattr(handle, name)
                except AttributeError as e:
                    raise DsaLibraryError(f"{LIB_PATH} does not export {name}") from e
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


# Debug mode (DSA_B200_CHECK_DEVICE=1): after every successful call the hook
# that ops.py installs synchronises the device and raises if a bounded wait
# inside a kernel expired (the sticky status word of dsa_device_error).
CHECK_DEVICE = os.environ.get("DSA_B200_CHECK_DEVICE", "0") not in ("", "0")
post_call_hook = None


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise DsaError on failure."""
    fn = getattr(lib(), name)
    st = fn(*args)
    if st != DSA_OK:
        msg = lib().dsa_last_error().decode(errors="replace")
        raise DsaError(name, st, msg)
    if CHECK_DEVICE and post_call_hook is not None:
        post_call_hook(name)
