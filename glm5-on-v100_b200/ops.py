"""Torch-facing operators of the DSA hot path — a drop-in for the reference's
``vllm._sm70_ops`` wrappers (reference/_sm70_ops.py:1848-1991) and the
``torch.ops._C.sm70_*`` schemas they call (csrc/torch_bindings.cpp hunk of
patches/glm5-v100-sm70-full.patch), plus the upstream ``persistent_topk`` op
the SM70 indexer uses (reference/sparse_attn_indexer.py:632-639).

Every operator is registered under the ``dsa_b200`` torch library namespace with
the reference's schema (same argument names, order, mutability and return
type) and a fake implementation, and every wrapper below has the reference's
Python signature. The CUDA implementation is the C ABI of libdsa_b200.so,
called on the current stream with raw device pointers; argument checks mirror
the reference's TORCH_CHECKs and raise RuntimeError.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib as L

NAMESPACE = "dsa_b200"

# Device-side waits of the P2P shard exchange give up after this long and
# report DSA_ERR_TIMEOUT instead of hanging (the reference's spins are
# unbounded, csrc/attention/sm70_mla_decode.cu:2196).
P2P_TIMEOUT_NS = int(float(os.environ.get("DSA_B200_P2P_TIMEOUT_S", "5")) * 1e9)

_DTYPE = {torch.float16: L.DSA_F16, torch.bfloat16: L.DSA_BF16, torch.float32: L.DSA_F32}
DSMLA_ROW_BYTES = 656
IDXK_FP8_ROW_BYTES = 132


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _rowmajor(t, name):
    _check(t.dim() == 2 and t.stride(1) == 1, f"{name} must be 2-D with unit inner stride")


def _int32(t, name):
    _check(t.dtype == torch.int32, f"{name} must be int32")


# ----------------------------------------------------------------- impls
def decode_plan(B: int, n_head: int, topk: int, kv_format: int) -> dict:
    """How the decode op runs a problem on the current device: slices of the
    top-k axis per row, how many merge inside one thread-block cluster, the
    workspace bytes and the kernel launches per call."""
    s, c, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    ws = ctypes.c_size_t()
    L.call("dsa_sparse_mla_decode_plan", B, n_head, topk, kv_format, ctypes.byref(s), ctypes.byref(c),
           ctypes.byref(ws), ctypes.byref(n))
    return {"n_splits": s.value, "cluster_size": c.value, "workspace_bytes": ws.value, "launches": n.value}


def _sparse_mla_decode_impl(o, lse, q, kv_cache, idx, block_table, seq_lens, scale):
    _check(q.is_cuda and kv_cache.is_cuda, "q and kv_cache must be CUDA tensors")
    _check(q.dtype in (torch.float16, torch.bfloat16), "q must be fp16 or bf16")
    _check(o.dtype in (torch.float16, torch.bfloat16), "o must be fp16 or bf16")
    _check(lse.dtype == torch.float32, "lse must be fp32")
    _int32(idx, "idx")
    _int32(block_table, "block_table")
    _int32(seq_lens, "seq_lens")
    if kv_cache.dtype == torch.uint8:
        _check(kv_cache.size(-1) == DSMLA_ROW_BYTES, "fp8 kv_cache last dim must be 656 (fp8_ds_mla layout)")
        fmt, row = L.DSA_FP8_DS_MLA, DSMLA_ROW_BYTES
    else:
        _check(kv_cache.dtype in (torch.float16, torch.bfloat16) and kv_cache.size(-1) == 576,
               "kv_cache must be fp16/bf16 [.., page, 576] or uint8 fp8_ds_mla [.., page, 656]")
        fmt, row = _DTYPE[kv_cache.dtype], 576
    _check(q.dim() == 3 and q.size(2) == 576, "q last dim must be 576")
    _check(o.dim() == 3 and o.size(2) == 512, "o last dim must be 512")
    _check(q.is_contiguous() and o.is_contiguous() and lse.is_contiguous() and kv_cache.is_contiguous(),
           "q, o, lse and kv_cache must be contiguous")
    B, H = q.size(0), q.size(1)
    _check(tuple(o.shape[:2]) == (B, H) and tuple(lse.shape) == (B, H), "o/lse shape mismatch with q")
    _rowmajor(idx, "idx")
    _rowmajor(block_table, "block_table")
    _check(idx.size(0) >= B and block_table.size(0) >= B and seq_lens.numel() >= B,
           "idx/block_table/seq_lens have fewer rows than q")
    topk = idx.size(1)
    page = kv_cache.size(-2)
    n_rows = kv_cache.numel() // row
    with torch.cuda.device(q.device):
        ws_bytes = decode_plan(B, H, topk, fmt)["workspace_bytes"]
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        L.call("dsa_sparse_mla_decode", _vp(o), _DTYPE[o.dtype], _vp(lse), _vp(q), _DTYPE[q.dtype],
               _vp(kv_cache), fmt, n_rows, page, _vp(idx), idx.stride(0), _vp(block_table),
               block_table.stride(0), block_table.size(1), _vp(seq_lens.contiguous()), B, H, topk,
               float(scale), _vp(ws), ws_bytes, _stream(q.device))


def _k_cache_format(k_cache):
    if k_cache.dtype == torch.uint8:
        _check(k_cache.size(-1) == IDXK_FP8_ROW_BYTES, "fp8 indexer k_cache last dim must be 132")
        return L.DSA_FP8_IDXK, IDXK_FP8_ROW_BYTES
    _check(k_cache.dtype in (torch.float16, torch.bfloat16), "k_cache must be fp16, bf16 or uint8 (fp8)")
    _check(k_cache.size(-1) == 128, "indexer head_dim must be 128")
    return _DTYPE[k_cache.dtype], 128


def _logits_common(score, k_cache, weights, block_table, seq_lens):
    _check(score.dtype == torch.float32, "score must be fp32")
    _check(weights.dtype in _DTYPE, "weights must be fp16, bf16 or fp32")
    _int32(block_table, "block_table")
    _int32(seq_lens, "seq_lens")
    _rowmajor(score, "score")
    _rowmajor(block_table, "block_table")
    _check(k_cache.is_contiguous() and weights.is_contiguous(), "k_cache and weights must be contiguous")
    fmt, row = _k_cache_format(k_cache)
    page = k_cache.size(-2)
    _check(page > 0 and (page & (page - 1)) == 0, "indexer cache page size must be a power of two")
    return fmt, k_cache.numel() // row, page


def _indexer_logits_impl(score, q, k_cache, weights, block_table, seq_lens, hist):
    _check(q.dtype in (torch.float16, torch.bfloat16), "q must be fp16 or bf16")
    _check(q.dim() == 3 and q.size(2) == 128, "indexer head_dim must be 128")
    _check(q.is_contiguous(), "q must be contiguous")
    fmt, n_rows, page = _logits_common(score, k_cache, weights, block_table, seq_lens)
    B, Hi = q.size(0), q.size(1)
    _check(tuple(weights.shape) == (B, Hi), "weights must be [B, n_ihead]")
    hp = None
    if hist is not None:
        _check(hist.dtype == torch.int32 and hist.is_contiguous() and tuple(hist.shape) == (B, 4096),
               "hist must be contiguous int32 [B, 4096]")
        hp = _vp(hist)
    with torch.cuda.device(q.device):
        L.call("dsa_indexer_logits", _vp(score), score.stride(0), score.size(1), _vp(q), _DTYPE[q.dtype],
               _vp(k_cache), fmt, n_rows, page, _vp(weights), _DTYPE[weights.dtype], _vp(block_table),
               block_table.stride(0), block_table.size(1), _vp(seq_lens.contiguous()), B, Hi, hp,
               _stream(q.device))


def _indexer_logits_packed_impl(score, q_packed, k_cache, weights, block_table, seq_lens):
    _check(q_packed.dtype in (torch.float16, torch.bfloat16) and q_packed.is_contiguous(),
           "q_packed must be contiguous fp16/bf16")
    fmt, n_rows, page = _logits_common(score, k_cache, weights, block_table, seq_lens)
    B = score.size(0)
    nqt = (B + 15) // 16
    _check(tuple(q_packed.shape) == (32, nqt, 8, 16, 16), "q_packed must be [32, ceil(B/16), 8, 16, 16]")
    _check(tuple(weights.shape) == (B, 32), "weights must be [B, 32]")
    with torch.cuda.device(score.device):
        L.call("dsa_indexer_logits_packed", _vp(score), score.stride(0), score.size(1), _vp(q_packed),
               _DTYPE[q_packed.dtype], _vp(k_cache), fmt, n_rows, page, _vp(weights), _DTYPE[weights.dtype],
               _vp(block_table), block_table.stride(0), block_table.size(1), _vp(seq_lens.contiguous()), B,
               _stream(score.device))


def _decode_topk_impl(idx, score, seq_lens, hist, k):
    _check(score.dtype == torch.float32, "score must be fp32")
    _int32(idx, "idx")
    _int32(seq_lens, "seq_lens")
    _rowmajor(idx, "idx")
    _rowmajor(score, "score")
    B = score.size(0)
    _check(idx.size(0) == B and idx.size(1) == k, "idx must be [B, K]")
    _check(hist.dtype == torch.int32 and hist.is_contiguous() and tuple(hist.shape) == (B, 4096),
           "hist must be contiguous int32 [B, 4096]")
    with torch.cuda.device(score.device):
        L.call("dsa_decode_topk", _vp(idx), idx.stride(0), _vp(score), score.stride(0), score.size(1),
               _vp(seq_lens.contiguous()), _vp(hist), B, int(k), _stream(score.device))


def _persistent_topk_impl(score, lens, topk_idx, workspace, k, max_seq_len):
    _check(score.dtype == torch.float32, "score must be fp32")
    _int32(topk_idx, "topk_idx")
    _int32(lens, "lengths")
    _rowmajor(score, "score")
    _rowmajor(topk_idx, "topk_idx")
    n = score.size(0)
    _check(lens.numel() == n and topk_idx.size(0) == n and topk_idx.size(1) >= k, "topk shape mismatch")
    with torch.cuda.device(score.device):
        L.call("dsa_topk_rows", _vp(topk_idx), topk_idx.stride(0), _vp(score), score.stride(0), score.size(1),
               _vp(lens.reshape(-1).contiguous()), n, int(k), _stream(score.device))


def _indexer_k_store_impl(kv_cache, k, slot_mapping):
    _check(kv_cache.is_cuda and k.is_cuda, "kv_cache and k must be CUDA tensors")
    _check(k.dtype in (torch.float16, torch.bfloat16), "k must be fp16 or bf16")
    _int32(slot_mapping, "slot_mapping")
    _check(kv_cache.is_contiguous() and k.is_contiguous(), "kv_cache and k must be contiguous")
    head_dim = k.size(-1)
    n_tok = k.size(0)
    if kv_cache.dtype == torch.uint8:
        _check(head_dim == 128, "fp8 indexer store requires head_dim == 128")
        _check(kv_cache.size(-1) == IDXK_FP8_ROW_BYTES, "fp8 indexer kv_cache last dim must be 132")
        fmt, row = L.DSA_FP8_IDXK, IDXK_FP8_ROW_BYTES
    else:
        _check(kv_cache.dtype in (torch.float16, torch.bfloat16), "kv_cache must be fp16, bf16 or uint8 (fp8)")
        fmt, row = _DTYPE[kv_cache.dtype], head_dim
    if n_tok == 0:
        return
    with torch.cuda.device(k.device):
        L.call("dsa_indexer_k_store", _vp(kv_cache), fmt, kv_cache.numel() // row, _vp(k), _DTYPE[k.dtype],
               head_dim, _vp(slot_mapping.contiguous()), n_tok, _stream(k.device))


def _shard_merge_impl(out, allf, dst_rows, dst_base, topk):
    _check(allf.is_cuda and allf.is_contiguous() and allf.dim() == 3, "allf must be contiguous [tp, R, 2K] cuda")
    _check(allf.dtype == torch.float32, "allf must be fp32")
    _check(out.dtype == torch.int32 and out.dim() == 2 and out.stride(1) == 1, "out must be int32 [rows, >=K]")
    tp, R = allf.size(0), allf.size(1)
    _check(allf.size(2) == 2 * topk, "allf last dim must be 2*topk")
    _check(dst_base >= 0 or dst_rows.numel() == R, "need dst_rows when dst_base < 0")
    dp = _vp(dst_rows.contiguous()) if dst_base < 0 else None
    with torch.cuda.device(allf.device):
        L.call("dsa_indexer_shard_merge", _vp(out), out.stride(0), _vp(allf), dp, int(dst_base), tp, R,
               int(topk), _stream(allf.device))


_ERR_FLAGS: dict = {}


def p2p_error_flag(device) -> torch.Tensor:
    """Per-device int32 word the bounded P2P waits set to DSA_ERR_TIMEOUT."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = _ERR_FLAGS.get(device)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR_FLAGS[device] = t
    return t


class DsaDeviceError(RuntimeError):
    """A bounded wait inside a kernel of this library expired: the launch
    returned without finishing its output (the status word of
    dsa_device_error)."""


def device_error(device=None, reset: bool = False) -> int:
    """The library's sticky device status on `device` (0, or DSA_ERR_TIMEOUT
    after an expired wait); synchronises with the device. reset clears it."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        v = int(L.lib().dsa_device_error(1 if reset else 0))
    if v < 0:
        raise L.DsaError("dsa_device_error", -v, L.lib().dsa_last_error().decode(errors="replace"))
    return v


def check_device_status(device=None) -> None:
    """Synchronise `device` and raise DsaDeviceError (clearing the status) if
    a bounded wait in one of this library's kernels expired since the last
    check."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    torch.cuda.synchronize(dev)
    v = device_error(dev, reset=True)
    if v != 0:
        raise DsaDeviceError(f"a bounded device wait expired on {dev}: status {L.STATUS_NAMES.get(v, v)}; "
                             "the outputs of the launches since the last check are incomplete")


def selftest_wait_timeout(timeout_s: float = 0.01, device=None) -> None:
    """Launch one block whose mbarrier wait cannot complete: after timeout_s of
    device time it records DSA_ERR_TIMEOUT and returns (tests the bounded-wait
    path without a fault)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        L.call("dsa_selftest_wait_timeout", int(timeout_s * 1e9), _stream(dev))


def _check_after_call(name: str) -> None:
    # debug mode only; never inside a CUDA-graph capture (no synchronisation there)
    if name in ("dsa_device_error", "dsa_selftest_wait_timeout") or name.startswith("dsa_ipc"):
        return
    if torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing():
        check_device_status()


L.post_call_hook = _check_after_call


def check_p2p_status(device) -> None:
    """Raise if a bounded P2P wait on `device` timed out (synchronises)."""
    f = p2p_error_flag(device)
    v = int(f.item())
    if v != 0:
        f.zero_()
        raise RuntimeError(f"P2P shard exchange wait failed on {device}: status {L.STATUS_NAMES.get(v, v)}")


def p2p_failed(device) -> bool:
    """True (and the error word cleared) if a bounded P2P wait on `device`
    expired since the last check; synchronises with the device."""
    f = p2p_error_flag(device)
    v = int(f.item())
    if v != 0:
        f.zero_()
    return v != 0


def shard_stage(slot_rows, vals, idx) -> None:
    """slot_rows f32 [R, 2K] <- [vals | idx bits]; skipped on the device when
    an earlier P2P wait failed (the slot may still be read by a peer)."""
    R, K = vals.shape
    _check(slot_rows.dtype == torch.float32 and slot_rows.is_contiguous() and tuple(slot_rows.shape) == (R, 2 * K),
           "slot_rows must be contiguous f32 [R, 2K]")
    _check(vals.dtype == torch.float32 and idx.dtype == torch.int32 and vals.stride(1) == 1 and idx.stride(1) == 1,
           "vals f32 / idx int32 with unit inner stride")
    with torch.cuda.device(slot_rows.device):
        L.call("dsa_indexer_shard_stage", _vp(slot_rows), _vp(vals), vals.stride(0), _vp(idx), idx.stride(0), R, K,
               _vp(p2p_error_flag(slot_rows.device)), _stream(slot_rows.device))


def topk_rows_payload(pay, score, lens, hist, k: int, pos_off: int) -> None:
    """Local top-k of a key shard written as payload rows pay[:, :k] = values,
    pay[:, k:2k] = positions + pos_off (f32 bits); hist (or None) is consumed
    and zeroed."""
    _check(score.dtype == torch.float32 and pay.dtype == torch.float32, "score and pay must be fp32")
    _rowmajor(score, "score")
    _rowmajor(pay, "pay")
    _int32(lens, "lengths")
    B = score.size(0)
    _check(pay.size(0) >= B and pay.size(1) >= 2 * k, "pay must be [B, >= 2k]")
    hp = None
    if hist is not None:
        _check(hist.dtype == torch.int32 and hist.is_contiguous() and tuple(hist.shape) == (B, 4096),
               "hist must be contiguous int32 [B, 4096]")
        hp = _vp(hist)
    with torch.cuda.device(score.device):
        L.call("dsa_topk_rows_payload", _vp(pay), pay.stride(0), _vp(score), score.stride(0), score.size(1),
               _vp(lens.reshape(-1).contiguous()), hp, B, int(k), int(pos_off), _stream(score.device))


def shard_exchange_topk(ex, score, lens, hist, k: int, pos_off: int) -> None:
    """Decode exchange, stage half: this rank's local top-k rows into slot
    (seq & 1) of ex.buf, then staged = seq (no host sequencing; see
    dsa_shard_exchange_topk)."""
    _check(score.dtype == torch.float32, "score must be fp32")
    _rowmajor(score, "score")
    B = score.size(0)
    hp = None
    if hist is not None:
        _check(hist.dtype == torch.int32 and hist.is_contiguous() and tuple(hist.shape) == (B, 4096),
               "hist must be contiguous int32 [B, 4096]")
        hp = _vp(hist)
    with torch.cuda.device(score.device):
        L.call("dsa_shard_exchange_topk", _vp(score), score.stride(0), score.size(1), _vp(lens), hp, B, int(k),
               int(pos_off), ctypes.c_void_p(ex.buf.data_ptr()), ex.slot_bytes, ex.flag_arr, ex.tp, ex.rank,
               _vp(ex.ctl), P2P_TIMEOUT_NS, _vp(p2p_error_flag(score.device)), _stream(score.device))


def shard_exchange_merge(ex, out, R: int) -> None:
    """Decode exchange, merge half: the global top-k of rows 0..R-1 from every
    rank's slot into out[0:R] (ascending, -1 first), then merged = seq."""
    _check(out.dtype == torch.int32 and out.dim() == 2 and out.stride(1) == 1, "out must be int32 2-D")
    with torch.cuda.device(out.device):
        L.call("dsa_shard_exchange_merge", _vp(out), out.stride(0), ex.data_arr, ex.flag_arr, ex.tp, ex.rank, int(R),
               ex.K, ex.slot_bytes, _vp(ex.ctl), P2P_TIMEOUT_NS, _vp(p2p_error_flag(out.device)),
               _stream(out.device))


def _u64_array(t, tp):
    _check(t.device.type == "cpu" and t.dtype == torch.int64 and t.numel() >= tp, "pointer tensors must be CPU int64")
    arr = (ctypes.c_uint64 * tp)(*[int(x) for x in t.reshape(-1)[:tp].tolist()])
    return arr


def _shard_merge_p2p_impl(out, data_ptrs, flag_ptrs, dst_rows, dst_base, topk, tp, R, seq, slot_off):
    _check(out.dtype == torch.int32 and out.dim() == 2 and out.stride(1) == 1, "out must be int32 2-D")
    _check(dst_base >= 0 or dst_rows.numel() == R, "need dst_rows when dst_base < 0")
    dptr = _u64_array(data_ptrs, tp)
    fptr = _u64_array(flag_ptrs, tp)
    dp = _vp(dst_rows.contiguous()) if dst_base < 0 else None
    with torch.cuda.device(out.device):
        L.call("dsa_indexer_shard_merge_p2p", _vp(out), out.stride(0), dptr, fptr, dp, int(dst_base), int(topk),
               int(tp), int(R), int(seq), int(slot_off), P2P_TIMEOUT_NS, _vp(p2p_error_flag(out.device)),
               _stream(out.device))


class _IpcBuffer:
    """Owns a cudaMalloc'd IPC-exportable allocation; exposed to torch via
    __cuda_array_interface__ and freed when the last tensor view dies."""

    def __init__(self, ptr: int, nbytes: int):
        self.ptr = ptr
        self.nbytes = nbytes
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}

    def __del__(self):
        try:
            L.lib().dsa_ipc_free(ctypes.c_void_p(self.ptr))
        except Exception:
            pass


def _ipc_alloc_impl(nbytes):
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    L.call("dsa_ipc_alloc", int(nbytes), ctypes.byref(ptr), handle)
    buf = torch.as_tensor(_IpcBuffer(ptr.value, int(nbytes)), device=torch.device("cuda", torch.cuda.current_device()))
    h = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).clone()
    return [buf, h]


def _ipc_open_impl(handle):
    _check(handle.device.type == "cpu" and handle.numel() == 64, "handle must be a 64-byte CPU tensor")
    ptr = ctypes.c_void_p()
    L.call("dsa_ipc_open", bytes(handle.to(torch.uint8).numpy().tobytes()), ctypes.byref(ptr))
    return int(ptr.value)


def _ipc_flag_set_impl(flag_ptr, which, seq):
    dev = torch.device("cuda", torch.cuda.current_device())
    L.call("dsa_ipc_flag_set", int(flag_ptr), int(which), int(seq), _vp(p2p_error_flag(dev)), _stream(dev))


def _ipc_slot_wait_impl(flag_ptrs, tp, min_seq):
    dev = torch.device("cuda", torch.cuda.current_device())
    L.call("dsa_ipc_slot_wait", _u64_array(flag_ptrs, tp), int(tp), int(min_seq), P2P_TIMEOUT_NS,
           _vp(p2p_error_flag(dev)), _stream(dev))


def _rope_args(positions, cos_sin_cache):
    if positions is None:
        return None, None, 0
    _check(positions.dtype == torch.int64 and positions.is_contiguous(), "positions must be contiguous int64")
    _check(cos_sin_cache is not None and cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous() and
           cos_sin_cache.dim() == 2 and cos_sin_cache.size(1) == 64,
           "cos_sin_cache must be contiguous f32 [max_pos, 64] (32 cos | 32 sin)")
    return _vp(positions), _vp(cos_sin_cache), cos_sin_cache.size(0)


def _concat_and_cache_ds_mla_impl(kv_c, k_pe, kv_cache, slot_mapping, positions, cos_sin_cache, is_neox):
    _check(kv_c.dtype in (torch.float16, torch.bfloat16) and k_pe.dtype == kv_c.dtype,
           "kv_c and k_pe must be fp16 or bf16, the same dtype")
    _check(kv_c.dim() == 2 and kv_c.size(1) == 512 and kv_c.stride(1) == 1, "kv_c must be [T, 512], unit inner stride")
    k_pe = k_pe.reshape(k_pe.size(0), -1)
    _check(k_pe.size(1) == 64 and k_pe.stride(1) == 1, "k_pe must be [T, 64] (or [T, 1, 64])")
    _check(kv_cache.dtype == torch.uint8 and kv_cache.size(-1) == DSMLA_ROW_BYTES and kv_cache.is_contiguous(),
           "kv_cache must be contiguous uint8 fp8_ds_mla [n_blocks, page, 656]")
    _int32(slot_mapping, "slot_mapping")
    n = kv_c.size(0)
    if n == 0:
        return
    pp, cp, max_pos = _rope_args(positions, cos_sin_cache)
    with torch.cuda.device(kv_c.device):
        L.call("dsa_concat_and_cache_ds_mla", _vp(kv_cache), kv_cache.numel() // DSMLA_ROW_BYTES, _vp(kv_c),
               kv_c.stride(0), _vp(k_pe), k_pe.stride(0), _DTYPE[kv_c.dtype], _vp(slot_mapping.contiguous()), n, pp, cp,
               max_pos, int(bool(is_neox)), _stream(kv_c.device))


def _indexer_qk_store_impl(q_out, weights_out, kv_cache, q, kw, slot_mapping, ln_weight, ln_bias, ln_eps, positions,
                           cos_sin_cache, is_neox, weight_scale):
    _check(q.dtype in (torch.float16, torch.bfloat16) and kw.dtype == q.dtype, "q and kw must be fp16 or bf16, same dtype")
    _check(q.dim() == 3 and q.size(2) == 128 and q.stride(2) == 1 and q.stride(1) == 128,
           "q must be [T, n_head, 128] with contiguous heads")
    T, H = q.size(0), q.size(1)
    _check(kw.dim() == 2 and kw.size(0) == T and kw.size(1) == 128 + H and kw.stride(1) == 1,
           "kw must be [T, 128 + n_head] (k then weight logits)")
    _check(q_out.dtype in (torch.float16, torch.bfloat16) and q_out.is_contiguous() and tuple(q_out.shape) == (T, H, 128),
           "q_out must be contiguous fp16/bf16 [T, n_head, 128]")
    _check(weights_out.dtype in _DTYPE and weights_out.is_contiguous() and tuple(weights_out.shape) == (T, H),
           "weights_out must be contiguous [T, n_head]")
    fmt, row = _k_cache_format(kv_cache)
    _check(kv_cache.is_contiguous(), "kv_cache must be contiguous")
    _int32(slot_mapping, "slot_mapping")
    for t, name in ((ln_weight, "ln_weight"), (ln_bias, "ln_bias")):
        _check(t is None or (t.dtype == torch.float32 and t.is_contiguous() and t.numel() == 128),
               f"{name} must be f32 [128]")
    if T == 0:
        return
    pp, cp, max_pos = _rope_args(positions, cos_sin_cache)
    with torch.cuda.device(q.device):
        L.call("dsa_indexer_qk_store", _vp(q_out), _DTYPE[q_out.dtype], _vp(weights_out), _DTYPE[weights_out.dtype],
               _vp(kv_cache), fmt, kv_cache.numel() // row, _vp(q), q.stride(0), _vp(kw), kw.stride(0),
               _DTYPE[q.dtype], _vp(ln_weight), _vp(ln_bias), float(ln_eps), pp, cp, max_pos, int(bool(is_neox)),
               float(weight_scale), _vp(slot_mapping.contiguous()), T, H, _stream(q.device))


# ------------------------------------------------------ torch registration
_lib_def = torch.library.Library(NAMESPACE, "DEF")
_SCHEMAS = {
    "sm70_sparse_mla_decode": ("(Tensor! o, Tensor! lse, Tensor q, Tensor kv_cache, Tensor idx, "
                               "Tensor block_table, Tensor seq_lens, float scale) -> ()",
                               _sparse_mla_decode_impl, "CUDA"),
    "sm70_indexer_logits": ("(Tensor! score, Tensor q, Tensor k_cache, Tensor weights, Tensor block_table, "
                            "Tensor seq_lens, Tensor!? hist) -> ()", _indexer_logits_impl, "CUDA"),
    "sm70_indexer_logits_packed": ("(Tensor! score, Tensor q_packed, Tensor k_cache, Tensor weights, "
                                   "Tensor block_table, Tensor seq_lens) -> ()",
                                   _indexer_logits_packed_impl, "CUDA"),
    "sm70_decode_topk": ("(Tensor! idx, Tensor score, Tensor seq_lens, Tensor hist, int k) -> ()",
                         _decode_topk_impl, "CUDA"),
    "persistent_topk": ("(Tensor score, Tensor lengths, Tensor! output, Tensor workspace, int k, "
                        "int max_seq_len) -> ()", _persistent_topk_impl, "CUDA"),
    "sm70_indexer_k_store": ("(Tensor! kv_cache, Tensor k, Tensor slot_mapping) -> ()",
                             _indexer_k_store_impl, "CUDA"),
    "sm70_indexer_shard_merge": ("(Tensor! out, Tensor allf, Tensor dst_rows, int dst_base, int topk) -> ()",
                                 _shard_merge_impl, "CUDA"),
    "sm70_indexer_shard_merge_p2p": ("(Tensor! out, Tensor data_ptrs, Tensor flag_ptrs, Tensor dst_rows, "
                                     "int dst_base, int topk, int tp, int R, int seq, int slot_off) -> ()",
                                     _shard_merge_p2p_impl, "CUDA"),
    "sm70_ipc_alloc": ("(int bytes) -> Tensor[]", _ipc_alloc_impl, "CompositeExplicitAutograd"),
    "sm70_ipc_open": ("(Tensor handle) -> int", _ipc_open_impl, "CPU"),
    "sm70_ipc_flag_set": ("(int flag_ptr, int which, int seq) -> ()", _ipc_flag_set_impl,
                          "CompositeExplicitAutograd"),
    "sm70_ipc_slot_wait": ("(Tensor flag_ptrs, int tp, int min_seq) -> ()", _ipc_slot_wait_impl, "CPU"),
    # cache writers (no SM70 op in the reference: the upstream writer and the
    # indexer's torch producer, with the rotary embedding fused in)
    "concat_and_cache_ds_mla": ("(Tensor kv_c, Tensor k_pe, Tensor! kv_cache, Tensor slot_mapping, "
                                "Tensor? positions, Tensor? cos_sin_cache, bool is_neox) -> ()",
                                _concat_and_cache_ds_mla_impl, "CUDA"),
    "indexer_qk_store": ("(Tensor! q_out, Tensor! weights_out, Tensor! kv_cache, Tensor q, Tensor kw, "
                         "Tensor slot_mapping, Tensor? ln_weight, Tensor? ln_bias, float ln_eps, Tensor? positions, "
                         "Tensor? cos_sin_cache, bool is_neox, float weight_scale) -> ()",
                         _indexer_qk_store_impl, "CUDA"),
}
for _name, (_schema, _fn, _key) in _SCHEMAS.items():
    _lib_def.define(_name + _schema)
    _lib_def.impl(_name, _fn, _key)


def _noop_fake(*args, **kwargs):
    return None


for _name in ("sm70_sparse_mla_decode", "sm70_indexer_logits", "sm70_indexer_logits_packed", "sm70_decode_topk",
              "persistent_topk", "sm70_indexer_k_store", "sm70_indexer_shard_merge",
              "sm70_indexer_shard_merge_p2p", "concat_and_cache_ds_mla", "indexer_qk_store"):
    torch.library.register_fake(f"{NAMESPACE}::{_name}")(_noop_fake)


def _op(name):
    return getattr(getattr(torch.ops, NAMESPACE), name)


# ---------------------------------------- reference-compatible wrappers
def sm70_sparse_mla_decode(o, lse, q, kv_cache, idx, block_table, seq_lens, scale: float) -> None:
    """Sparse (top-k) MLA decode/prefill: writes o [B,H,512] (fp16/bf16) and lse [B,H] fp32."""
    _op("sm70_sparse_mla_decode")(o, lse, q, kv_cache, idx, block_table, seq_lens, scale)


def sm70_indexer_logits(score, q, k_cache, weights, block_table, seq_lens, hist=None) -> None:
    """DSA indexer logits -> score [B, max_kv] fp32 (pad = -inf); optional fused
    level-1 top-k histogram into a pre-zeroed int32 [B, 4096] `hist`."""
    _op("sm70_indexer_logits")(score, q, k_cache, weights, block_table, seq_lens, hist)


def sm70_indexer_logits_packed(score, q_packed, k_cache, weights, block_table, seq_lens) -> None:
    """Indexer logits from the packed q layout [32, ceil(B/16), 8, 16, 16]."""
    _op("sm70_indexer_logits_packed")(score, q_packed, k_cache, weights, block_table, seq_lens)


def sm70_decode_topk(idx, score, seq_lens, hist, k: int) -> None:
    """Exact top-k positions of score rows (p < seq_lens), ascending, -1 padded."""
    _op("sm70_decode_topk")(idx, score, seq_lens, hist, k)


def persistent_topk(score, lengths, output, workspace, k: int, max_seq_len: int) -> None:
    """Per-row top-k with the upstream persistent_topk signature (workspace unused)."""
    _op("persistent_topk")(score, lengths, output, workspace, k, max_seq_len)


def sm70_indexer_k_store(kv_cache, k, slot_mapping) -> None:
    """Indexer-K scatter into the paged cache (skips slot < 0)."""
    _op("sm70_indexer_k_store")(kv_cache, k, slot_mapping)


def sm70_indexer_shard_merge(out, allf, dst_rows, dst_base: int, topk: int) -> None:
    _op("sm70_indexer_shard_merge")(out, allf, dst_rows, dst_base, topk)


def sm70_indexer_shard_merge_p2p(out, data_ptrs, flag_ptrs, dst_rows, dst_base: int, topk: int, tp: int, R: int,
                                 seq: int, slot_off: int) -> None:
    _op("sm70_indexer_shard_merge_p2p")(out, data_ptrs, flag_ptrs, dst_rows, dst_base, topk, tp, R, seq, slot_off)


def sm70_ipc_alloc(nbytes: int):
    return _op("sm70_ipc_alloc")(nbytes)


def sm70_ipc_open(handle) -> int:
    return _op("sm70_ipc_open")(handle)


def sm70_ipc_flag_set(flag_ptr: int, which: int, seq: int) -> None:
    _op("sm70_ipc_flag_set")(flag_ptr, which, seq)


def sm70_ipc_slot_wait(flag_ptrs, tp: int, min_seq: int) -> None:
    _op("sm70_ipc_slot_wait")(flag_ptrs, tp, min_seq)


def concat_and_cache_mla(kv_c, k_pe, kv_cache, slot_mapping, kv_cache_dtype: str = "fp8_ds_mla", scale=None,
                         positions=None, cos_sin_cache=None, is_neox: bool = False) -> None:
    """Latent-cache writer with the upstream signature (concat_and_cache_mla,
    kv_cache_dtype "fp8_ds_mla"; scale is unused by that format). Given
    positions and a cos/sin table, the rotary embedding of k_pe is applied
    on the way in (k_pe is then the un-rotated key)."""
    _check(kv_cache_dtype == "fp8_ds_mla", f"only the fp8_ds_mla cache is written here (got {kv_cache_dtype})")
    _op("concat_and_cache_ds_mla")(kv_c, k_pe, kv_cache, slot_mapping, positions, cos_sin_cache, is_neox)


def indexer_qk_store(q_out, weights_out, kv_cache, q, kw, slot_mapping, ln_weight=None, ln_bias=None,
                     ln_eps: float = 1e-6, positions=None, cos_sin_cache=None, is_neox: bool = False,
                     weight_scale: float = 1.0) -> None:
    """The indexer's q / k / weights producer fused into the K store: k =
    LayerNorm(kw[:, :128]) + rotary into the cache rows, q_out = rotary(q),
    weights_out = kw[:, 128:] * weight_scale."""
    _op("indexer_qk_store")(q_out, weights_out, kv_cache, q, kw, slot_mapping, ln_weight, ln_bias, float(ln_eps),
                            positions, cos_sin_cache, is_neox, float(weight_scale))
