"""CPU: the C-ABI library loads, exports every entry point include/dsa_b200.h
declares, and rejects bad arguments with a status code before touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def declared_functions():
    names = []
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(dsa_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "dsa_sparse_mla_decode" in names and "dsa_indexer_logits" in names
    assert len(names) >= 17


def test_library_exports_every_declared_symbol(dsa):
    lib_path = dsa._lib.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(dsa_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    # the Python binding covers the same set
    assert set(dsa._lib.SIGNATURES) == set(declared_functions())


def test_version_and_error_text(dsa):
    lib = dsa._lib.lib()
    assert lib.dsa_version() >> 16 == 1
    assert isinstance(lib.dsa_last_error(), bytes)


def test_argument_validation_without_gpu(dsa):
    L = dsa._lib
    lib = L.lib()
    null = None
    # negative batch
    st = lib.dsa_sparse_mla_decode(null, 0, null, null, 0, null, 0, 0, 64, null, 0, null, 0, 0, null, -1, 64, 2048,
                                   1.0, null, 0, null)
    assert st == L.DSA_ERR_INVALID
    assert b"negative" in lib.dsa_last_error()
    # zero-size work is a no-op success
    assert lib.dsa_sparse_mla_decode(null, 0, null, null, 0, null, 0, 0, 64, null, 0, null, 0, 0, null, 0, 64, 2048,
                                     1.0, null, 0, null) == L.DSA_OK
    # unsupported indexer head count
    st = lib.dsa_indexer_logits(ctypes.c_void_p(16), 128, 128, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, 10,
                                64, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 4, 4, ctypes.c_void_p(16), 2, 65,
                                null, null)
    assert st == L.DSA_ERR_UNSUPPORTED
    # non power-of-two page
    st = lib.dsa_indexer_logits(ctypes.c_void_p(16), 128, 128, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 0, 10,
                                48, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 4, 4, ctypes.c_void_p(16), 2, 32,
                                null, null)
    assert st == L.DSA_ERR_INVALID
    # top-k size limit
    assert lib.dsa_topk_rows(ctypes.c_void_p(16), 8192, ctypes.c_void_p(16), 8192, 8192, ctypes.c_void_p(16), 1,
                             8192, null) == L.DSA_ERR_UNSUPPORTED
    # shard merge limits
    assert lib.dsa_indexer_shard_merge(ctypes.c_void_p(16), 2048, ctypes.c_void_p(16), null, 0, 9, 4, 2048,
                                       null) == L.DSA_ERR_UNSUPPORTED
    assert lib.dsa_indexer_shard_merge(ctypes.c_void_p(16), 2048, ctypes.c_void_p(16), null, -1, 2, 4, 2048,
                                       null) == L.DSA_ERR_INVALID
    # fp8 indexer store requires head_dim 128
    assert lib.dsa_indexer_k_store(ctypes.c_void_p(16), L.DSA_FP8_IDXK, 10, ctypes.c_void_p(16), 0, 64,
                                   ctypes.c_void_p(16), 3, null) == L.DSA_ERR_UNSUPPORTED


def test_python_wrapper_raises_on_bad_dtype(dsa):
    import torch

    o = torch.empty(1, 1, 512)
    with pytest.raises(RuntimeError):
        dsa.ops._sparse_mla_decode_impl(o, torch.empty(1, 1), torch.empty(1, 1, 576), torch.empty(1, 64, 576),
                                        torch.empty(1, 8, dtype=torch.int32), torch.empty(1, 1, dtype=torch.int32),
                                        torch.empty(1, dtype=torch.int32), 1.0)


def test_torch_ops_registered_with_reference_schemas(dsa):
    import torch

    ns = torch.ops.dsa_b200

    def args(op):
        sch = op.default._schema
        return [(a.name, bool(a.alias_info and a.alias_info.is_write)) for a in sch.arguments]

    assert args(ns.sm70_sparse_mla_decode) == [("o", True), ("lse", True), ("q", False), ("kv_cache", False),
                                               ("idx", False), ("block_table", False), ("seq_lens", False),
                                               ("scale", False)]
    assert args(ns.sm70_indexer_logits)[0] == ("score", True)
    assert args(ns.sm70_indexer_logits)[-1] == ("hist", True)
    for name in ["sm70_indexer_logits_packed", "sm70_decode_topk", "sm70_indexer_k_store", "sm70_indexer_shard_merge",
                 "sm70_indexer_shard_merge_p2p", "sm70_ipc_alloc", "sm70_ipc_open", "sm70_ipc_flag_set",
                 "sm70_ipc_slot_wait", "persistent_topk"]:
        assert hasattr(ns, name), name
    # the layer op: reference signature with topk_indices_buffer mutated (sai.py:1089-1119)
    assert args(ns.sm70_sparse_indexer) == [("k_cache_prefix", False), ("kv_cache", False), ("q", False),
                                            ("k", False), ("weights", False), ("topk_tokens", False),
                                            ("head_dim", False), ("max_model_len", False),
                                            ("topk_indices_buffer", True)]


def test_sparse_indexer_op_without_metadata_returns_buffer(dsa):
    """A profiling / dummy run (no forward-context metadata) leaves the buffer
    untouched and returns it, as the reference does (sai.py:543-544)."""
    import torch

    sai = dsa.sparse_attn_indexer
    buf = torch.full((3, 4), 5, dtype=torch.int32)
    out = sai._sm70_sparse_indexer_impl("layers.0.k_cache", torch.empty(0), torch.empty(0), torch.empty(3, 128),
                                        torch.empty(0), 4, 128, 1024, buf)
    assert out is buf and int(buf.sum()) == 60
