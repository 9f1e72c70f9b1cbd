"""B200 (sm_100a) DSA sparse-attention hot path: a drop-in for the SM70 DSA ops
of bayley/glm5-on-v100.

Layout:
  csrc/                 CUDA kernels + C ABI (libdsa_b200.so, include/dsa_b200.h)
  _lib.py               ctypes binding of the C ABI (no fallback when missing)
  ops.py                torch ops + wrappers with the reference's _sm70_ops API
  sparse_attn_indexer.py  indexer orchestration (K store, logits, top-k, sharding)
  mla_sparse.py         sparse MLA decode / prefill glue (spec-as-decode rows)
  build.py              nvcc build of the library

The package directory name contains '-', so import it with
``importlib.import_module("glm5-on-v100_b200")``; it also registers itself as
``glm5_on_v100_b200``.
"""
import sys as _sys

from . import _lib  # noqa: F401
from . import ops  # noqa: F401
from .ops import (  # noqa: F401
    persistent_topk,
    sm70_decode_topk,
    sm70_indexer_k_store,
    sm70_indexer_logits,
    sm70_indexer_logits_packed,
    sm70_indexer_shard_merge,
    sm70_indexer_shard_merge_p2p,
    sm70_ipc_alloc,
    sm70_ipc_flag_set,
    sm70_ipc_open,
    sm70_ipc_slot_wait,
    sm70_sparse_mla_decode,
)
from . import sparse_attn_indexer  # noqa: F401  (registers the sm70_sparse_indexer op)
from .sparse_attn_indexer import sm70_sparse_indexer  # noqa: F401

_sys.modules.setdefault("glm5_on_v100_b200", _sys.modules[__name__])
