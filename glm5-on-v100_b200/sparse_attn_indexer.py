"""Lightning-indexer orchestration: K store, decode and prefill top-k, key
sharding across tensor-parallel ranks and the exact shard merge.

Mirrors ``_sm70_sparse_indexer`` (reference/sparse_attn_indexer.py:528-1071)
and the P2P exchange state ``_sm70_p2p_state`` (:44-106) without vLLM's
forward context: the indexer metadata is passed explicitly (``IndexerMeta``).
Every device computation goes through the ops of ``ops.py`` (libdsa_b200.so).

Differences from the reference, by design:
  * decode rows are not chunked into groups of < 8: the logits kernel builds
    the fused histogram for any batch (the reference's B >= 8 kernel could not,
    sai.py:595-601);
  * prefill sub-blocks are sized by a score-buffer budget instead of a fixed
    128 rows (results are per row, so identical);
  * shard merges take any tp in [1, 8] and any K <= 2048 (the reference's
    fused kernels: tp in [2, 4], K == 2048);
  * device waits of the P2P exchange are bounded; after one expires on any
    rank, every rank (agreeing over the host) redoes the step through the
    all-gather path and stays on it (the reference falls back only when its
    init fails, sai.py:100-105);
  * decode rows can be key-sharded too (ShardConfig.decode), with an
    exchange whose sequence number lives on the device.
"""
from __future__ import annotations

import contextlib
import ctypes
import logging
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch

from . import ops

logger = logging.getLogger(__name__)

KEY_TILE = 64              # key-span granularity of a launch (sai.py:681)
SCORE_BUDGET_BYTES = 1 << 29  # fp32 score buffer per prefill sub-block


@dataclass
class DecodeMeta:
    block_table: torch.Tensor  # [nd, max_blocks] int32
    seq_lens: torch.Tensor     # [nd] or [nd, next_n] int


@dataclass
class PrefillChunk:
    token_start: int
    cu_seqlen_ks: torch.Tensor    # [n_q] cumulative KV starts (flattened-KV offsets)
    cu_seqlen_ke: torch.Tensor    # [n_q] cumulative KV ends
    block_table: torch.Tensor     # [num_reqs, max_blocks]
    num_reqs: int
    query_start_loc_cpu: Optional[List[int]] = None  # request bounds within the chunk
    _causal_max_cache: dict = field(default_factory=dict)


@dataclass
class IndexerMeta:
    slot_mapping: torch.Tensor
    num_decode_tokens: int = 0
    decode: Optional[DecodeMeta] = None
    prefill_chunks: List[PrefillChunk] = field(default_factory=list)


@dataclass
class ShardConfig:
    """Key sharding of indexer scoring across tp ranks (prefill: sai.py:726-880;
    decode rows too when `decode` is set) and the state of its merge."""
    tp: int = 1
    rank: int = 0
    min_ctx: int = 16384               # VLLM_SM70_IDXER_TP_SHARD_MIN_CTX default
    group: object = None               # torch.distributed group for the all-gather
    cpu_group: object = None           # gloo group: IPC handle exchange and the ranks' agreement
    merge: str = "fused"               # "p2p" | "fused" | "torch"
    rows_cap: int = 1024               # P2P slot capacity (max_num_batched_tokens)
    decode: bool = False               # also split every decode row's keys across the ranks
    backend: object = None             # ops module (or a stand-in with its IPC/merge functions)
    agree: Optional[Callable] = None   # AND over the ranks (default: all_reduce MIN on cpu_group)
    gather: Optional[Callable] = None  # [R, 2K] -> [tp*R, 2K] (default: NCCL all_gather_into_tensor)
    p2p: object = None                 # P2PExchange, built on the first merge
    decode_exchange: object = None     # DecodeExchange, built on the first sharded decode step
    p2p_init_failed: bool = False
    p2p_failed: bool = False           # set on every rank together: P2P is off from then on


# Per-chunk (tok_lo, n_q, ke) entries handed to the sparse prefill attention
# (the reference's _SM70_PREFILL_META bridge, sai.py:85-92, :1070).
PREFILL_META: dict = {}


# ----------------------------------------------------------- pure helpers
def shard_span(max_kv: int, tp: int, rank: int, page: int, kt: int = KEY_TILE):
    """(off, span) of this rank's contiguous key span (sai.py:797-806)."""
    unit = max(kt, page)
    per = ((max_kv + tp - 1) // tp + unit - 1) // unit * unit
    off = rank * per
    span = min(per, max(max_kv - off, 0))
    span = max(span, page)
    return off, span


def request_bounds(chunk: PrefillChunk, n_q: int) -> List[int]:
    """Authoritative per-request query bounds of a chunk (sai.py:692-725)."""
    if chunk.query_start_loc_cpu is not None:
        return [int(x) for x in chunk.query_start_loc_cpu]
    if chunk.num_reqs == 1:
        return [0, n_q]
    raise RuntimeError("prefill chunk with several requests needs query_start_loc_cpu")


def sub_blocks(lo: int, hi: int, max_kv_hint: int):
    """Row sub-blocks of a request segment, sized so the fp32 score buffer
    stays within SCORE_BUDGET_BYTES (the reference uses 128 rows, sai.py:763)."""
    rows = max(128, (SCORE_BUDGET_BYTES // max(4 * max_kv_hint, 1)) // 64 * 64)
    for a in range(lo, hi, rows):
        yield a, min(a + rows, hi)


def pack_payload(pending, K: int, device) -> torch.Tensor:
    """Pending (row_lo, n_rows, vals [n,K] f32, gidx [n,K] i32) -> [R, 2K] f32 (sai.py:953-961)."""
    R = sum(p[1] for p in pending)
    fused = torch.empty((R, 2 * K), dtype=torch.float32, device=device)
    ro = 0
    for _, n_r, lv, gi in pending:
        fused[ro:ro + n_r, :K] = lv
        fused[ro:ro + n_r, K:] = gi.view(torch.float32)
        ro += n_r
    return fused


def destination(pending, device):
    """(dst_rows tensor, dst_base): contiguous pending rows use dst_base (sai.py:915-941)."""
    contig = True
    exp_row = pending[0][0]
    for row_lo, n_r, _, _ in pending:
        if row_lo != exp_row:
            contig = False
            break
        exp_row = row_lo + n_r
    if contig:
        return torch.empty(0, dtype=torch.int32, device=device), pending[0][0]
    dst = torch.cat([torch.arange(r0, r0 + n, dtype=torch.int32, device=device) for r0, n, _, _ in pending])
    return dst, -1


def torch_merge_epilogue(allf: torch.Tensor, K: int):
    """The reference's torch.topk merge (sai.py:1007-1030): [tp, R, 2K] -> [R, K] ids."""
    tp, R, _ = allf.shape
    av = allf[:, :, :K].permute(1, 0, 2).reshape(R, tp * K)
    ai = allf[:, :, K:].permute(1, 0, 2).reshape(R, tp * K).contiguous().view(torch.int32)
    mv, mp = torch.topk(av, K, dim=1)
    mi = ai.gather(1, mp)
    return torch.where(torch.isinf(mv), torch.full_like(mi, -1), mi).to(torch.int32)


# ------------------------------------------------------------- P2P state
class _IpcSlots:
    """Two payload slots and a {staged, merged} flag pair in CUDA IPC memory,
    opened on every rank of the shard group (sai.py:44-106)."""

    def __init__(self, device, tp: int, rank: int, K: int, rows_cap: int, cpu_group=None,
                 all_gather_object: Optional[Callable] = None, backend=ops):
        import torch.distributed as dist

        self.backend = backend
        self.device = device
        self.tp, self.rank, self.K, self.rows_cap = tp, rank, K, rows_cap
        self.slot_bytes = (rows_cap * 2 * K * 4 + 15) // 16 * 16
        self.buf, handle = backend.sm70_ipc_alloc(2 * self.slot_bytes)
        self.fbuf, fhandle = backend.sm70_ipc_alloc(64)
        payload = (handle.numpy().tobytes(), fhandle.numpy().tobytes())
        objs: list = [None] * tp
        (all_gather_object or (lambda o, p: dist.all_gather_object(o, p, group=cpu_group)))(objs, payload)
        data_ptrs, flag_ptrs = [], []
        for i, (h, fh) in enumerate(objs):
            if i == rank:
                data_ptrs.append(self.buf.data_ptr())
                flag_ptrs.append(self.fbuf.data_ptr())
            else:
                data_ptrs.append(backend.sm70_ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
                flag_ptrs.append(backend.sm70_ipc_open(torch.frombuffer(bytearray(fh), dtype=torch.uint8)))
        self.data_ptrs_t = torch.tensor(data_ptrs, dtype=torch.int64)
        self.flag_ptrs_t = torch.tensor(flag_ptrs, dtype=torch.int64)
        self.data_arr = (ctypes.c_uint64 * tp)(*data_ptrs)
        self.flag_arr = (ctypes.c_uint64 * tp)(*flag_ptrs)
        self.my_flag_ptr = self.fbuf.data_ptr()


class P2PExchange(_IpcSlots):
    """Host-sequenced exchange of the prefill merge (sai.py:885-952). Per merge
    with sequence seq: slot = seq & 1; wait until every peer merged seq-2
    (slot reuse), stage my payload, publish staged = seq, merge reading all
    peers' slots, publish merged = seq. Every device wait is bounded
    (ops.P2P_TIMEOUT_NS); after one expires the rank's error word is set, the
    stage and both flag stores of that merge do nothing, and the merge kernel
    returns at once, so no peer reads a half-written slot. The caller learns
    of it from backend.p2p_failed()."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.seq = 0

    def merge(self, pending, out: torch.Tensor) -> None:
        K, be = self.K, self.backend
        R = sum(p[1] for p in pending)
        self.seq += 1
        seq = self.seq
        soff = (seq & 1) * self.slot_bytes
        if seq > 2:
            be.sm70_ipc_slot_wait(self.flag_ptrs_t, self.tp, seq - 2)
        slot_view = self.buf[soff:soff + R * 2 * K * 4].view(torch.float32).view(R, 2 * K)
        ro = 0
        for _, n_r, lv, gi in pending:
            be.shard_stage(slot_view[ro:ro + n_r], lv, gi)
            ro += n_r
        be.sm70_ipc_flag_set(self.my_flag_ptr, 0, seq)
        dst, base = destination(pending, out.device)
        be.sm70_indexer_shard_merge_p2p(out, self.data_ptrs_t, self.flag_ptrs_t, dst, base, K, self.tp, R, seq, soff)
        be.sm70_ipc_flag_set(self.my_flag_ptr, 1, seq)


class DecodeExchange(_IpcSlots):
    """Device-sequenced exchange of the key-sharded decode indexer: the
    sequence number lives in a device control block (ctl[0]) that the merge
    kernel advances, so a decode step (logits -> local top-k into my slot ->
    merge over peer slots) is stream-ordered device work a CUDA graph can
    replay (dsa_shard_exchange_topk / dsa_shard_exchange_merge). No
    reference counterpart: the reference shards prefill only."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.ctl = torch.zeros(4, dtype=torch.int32, device=self.buf.device)

    def topk_stage(self, score, lens, hist, pos_off: int) -> None:
        self.backend.shard_exchange_topk(self, score, lens, hist, self.K, pos_off)

    def merge(self, out: torch.Tensor, R: int) -> None:
        self.backend.shard_exchange_merge(self, out, R)


def all_ranks_ok(ok: bool, shard: "ShardConfig") -> bool:
    """AND of `ok` over the shard group, on the host (gloo cpu_group), so that
    every rank takes the same merge path in the same step."""
    if shard.tp <= 1:
        return ok
    if shard.agree is not None:
        return bool(shard.agree(ok))
    import torch.distributed as dist

    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=shard.cpu_group)
    return bool(t.item())


def _p2p_state(device, shard: ShardConfig, K: int) -> Optional[P2PExchange]:
    if shard.p2p is None and not shard.p2p_init_failed:
        try:
            shard.p2p = P2PExchange(device, shard.tp, shard.rank, K, shard.rows_cap, shard.cpu_group,
                                    backend=shard.backend or ops)
            logger.info("P2P shard merge initialised (tp=%d, rows_cap=%d)", shard.tp, shard.rows_cap)
        except Exception:
            logger.exception("P2P shard merge init failed on this rank")
            shard.p2p_init_failed = True
    return shard.p2p


def merge_shards(pending, topk_indices_buffer: torch.Tensor, K: int, shard: ShardConfig) -> None:
    """Exact global top-K of the rows in `pending` from every rank's local
    candidates, written to topk_indices_buffer (sai.py:881-1030).

    merge="p2p": every rank first agrees (host AND over the group) that its
    exchange exists; after the merge every rank reports whether one of its
    bounded waits expired, and if any did, ALL ranks redo this step through
    the all-gather path and stay on it (the reference falls back only when
    init fails, sai.py:100-105). Ranks therefore never run different
    collectives."""
    if not pending:
        return
    device = topk_indices_buffer.device
    R = sum(p[1] for p in pending)
    if shard.merge == "p2p" and not shard.p2p_failed:
        st = _p2p_state(device, shard, K)
        if not all_ranks_ok(st is not None, shard):
            shard.p2p_failed = True
            logger.warning("P2P shard merge unavailable on some rank; every rank uses the all-gather path")
        elif R <= st.rows_cap:  # R is the same on every rank: all take this branch together
            st.merge(pending, topk_indices_buffer)
            if all_ranks_ok(not st.backend.p2p_failed(device), shard):
                return
            shard.p2p_failed = True
            logger.warning("P2P shard merge wait expired on some rank; every rank redoes the step through the "
                           "all-gather path and stays on it")
    fused = pack_payload(pending, K, device)
    if shard.gather is not None:
        allf = shard.gather(fused)
    else:
        import torch.distributed as dist

        allf = torch.empty((shard.tp * R, 2 * K), dtype=torch.float32, device=device)
        dist.all_gather_into_tensor(allf, fused, group=shard.group)
    allf = allf.view(shard.tp, R, 2 * K)
    if shard.merge == "torch":
        mi = torch_merge_epilogue(allf, K)
        ro = 0
        for row_lo, n_r, _, _ in pending:
            topk_indices_buffer[row_lo:row_lo + n_r, :K].copy_(mi[ro:ro + n_r])
            ro += n_r
        return
    dst, base = destination(pending, device)
    (shard.backend or ops).sm70_indexer_shard_merge(topk_indices_buffer, allf.contiguous(), dst, base, K)


def decode_span(max_kv: int, shard: ShardConfig, page: int):
    """(off, span, pg_lo, pg_hi) of this rank's contiguous key span of every
    decode row (the prefill split of sai.py:797-806 over the block-table
    width, so the span is fixed per rank and a captured step needs no host
    sync)."""
    off, span = shard_span(max_kv, shard.tp, shard.rank, page)
    pg_lo = min(off // page, max(max_kv // page - 1, 0))
    pg_hi = max(min(max_kv // page, (off + span + page - 1) // page), pg_lo + 1)
    return off, (pg_hi - pg_lo) * page, pg_lo, pg_hi


def decode_indexer_sharded(q, kv_cache, weights, block_table, seq_lens, topk_tokens, out_idx, shard: ShardConfig,
                           bufs: Optional[dict] = None) -> None:
    """Key-sharded decode indexer: this rank scores keys [off, off+span) of
    every row (with the fused histogram), selects its local top-K straight
    into payload rows, and the exact merge over all ranks writes the global
    top-K of every row to out_idx on every rank.

    merge="p2p" runs the device-sequenced DecodeExchange (no host sync; the
    caller checks ops.p2p_failed at a point of its choosing); otherwise the
    payload goes through the NCCL all-gather and the fused merge kernel."""
    nd = q.shape[0]
    page = kv_cache.shape[1]
    max_kv = block_table.shape[1] * page
    off, span, pg_lo, pg_hi = decode_span(max_kv, shard, page)
    bufs = {} if bufs is None else bufs
    if bufs.get("shape") != (nd, span, topk_tokens):
        dev = q.device
        bufs.update(shape=(nd, span, topk_tokens), score=torch.empty((nd, span), dtype=torch.float32, device=dev),
                    hist=torch.zeros((nd, 4096), dtype=torch.int32, device=dev),
                    pay=torch.empty((nd, 2 * topk_tokens), dtype=torch.float32, device=dev))
    seg_bt = block_table[:, pg_lo:pg_hi]
    sl = (seq_lens.to(torch.int32) - off).clamp_(0, span)
    ops.sm70_indexer_logits(bufs["score"], q, kv_cache, weights, seg_bt, sl, bufs["hist"])
    if shard.merge == "p2p":
        ex = shard.decode_exchange
        if ex is None:
            ex = DecodeExchange(q.device, shard.tp, shard.rank, topk_tokens, shard.rows_cap, shard.cpu_group,
                                backend=shard.backend or ops)
            shard.decode_exchange = ex
        ex.topk_stage(bufs["score"], sl, bufs["hist"], off)
        ex.merge(out_idx, nd)
        return
    pay = bufs["pay"]
    ops.topk_rows_payload(pay, bufs["score"], sl, bufs["hist"], topk_tokens, off)
    pend = [(0, nd, pay[:, :topk_tokens], pay[:, topk_tokens:].contiguous().view(torch.int32))]
    merge_shards(pend, out_idx, topk_tokens, shard)


# ------------------------------------------------------------ main entry
def sparse_indexer(meta: IndexerMeta, kv_cache: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                   weights: torch.Tensor, topk_tokens: int, topk_indices_buffer: torch.Tensor,
                   shard: Optional[ShardConfig] = None, fused_decode_topk: bool = True) -> torch.Tensor:
    """One DSA indexer layer: store this step's keys, then write every
    token's top-k logical key positions (ascending, -1 padded) to
    topk_indices_buffer[:num_tokens, :topk_tokens].

    kv_cache: paged indexer-K cache [nb, page, 128] fp16/bf16 or [nb, page,
    132] uint8 (fp8); q [T, Hi, 128]; k [T, 128]; weights [T, Hi] (already
    scaled by softmax_scale * Hi^-0.5, as Indexer.forward does).
    """
    shard = shard or ShardConfig()
    n = k.shape[0]
    slot = meta.slot_mapping[:n].to(torch.int32)
    kin = k[:n] if k.dtype in (torch.float16, torch.bfloat16) else k[:n].to(torch.float16)
    ops.sm70_indexer_k_store(kv_cache, kin.contiguous(), slot)
    topk_indices_buffer[:n] = -1
    page = kv_cache.shape[1]

    nd = meta.num_decode_tokens
    if nd > 0 and meta.decode is not None:
        bt = meta.decode.block_table.to(torch.int32)
        seq = meta.decode.seq_lens
        if seq.dim() == 2:
            seq = seq[:, -1].contiguous()
        seq = seq.to(torch.int32)
        max_kv = bt.shape[1] * page
        score = torch.empty((nd, max_kv), dtype=torch.float32, device=q.device)
        topk_idx = topk_indices_buffer[:nd, :topk_tokens]
        if shard.tp > 1 and shard.decode:
            decode_indexer_sharded(q[:nd].contiguous(), kv_cache, weights[:nd].contiguous(), bt, seq, topk_tokens,
                                   topk_idx, shard)
        elif fused_decode_topk:
            hist = torch.zeros((nd, 4096), dtype=torch.int32, device=q.device)
            ops.sm70_indexer_logits(score, q[:nd].contiguous(), kv_cache, weights[:nd].contiguous(), bt, seq, hist)
            ops.sm70_decode_topk(topk_idx, score, seq, hist, topk_tokens)
        else:
            ops.sm70_indexer_logits(score, q[:nd].contiguous(), kv_cache, weights[:nd].contiguous(), bt, seq)
            ops.persistent_topk(score, seq.view(nd, 1), topk_idx, score, topk_tokens, max_kv)

    entries = []
    for chunk in meta.prefill_chunks:
        entries.append(_prefill_chunk(chunk, kv_cache, q, weights, topk_tokens, topk_indices_buffer, shard, page))
    if meta.prefill_chunks:
        PREFILL_META["chunks"] = entries
    return topk_indices_buffer


def _prefill_chunk(chunk: PrefillChunk, kv_cache, q, weights, topk_tokens, topk_indices_buffer, shard, page):
    ke = (chunk.cu_seqlen_ke - chunk.cu_seqlen_ks).to(torch.int32)  # true causal lengths (sai.py:661-673)
    n_q = ke.shape[0]
    tok_lo = chunk.token_start
    bt_chunk = chunk.block_table.to(torch.int32)
    full_kv = bt_chunk.shape[1] * page
    bounds = request_bounds(chunk, n_q)
    pending = []
    for r in range(chunk.num_reqs):
        lo, hi = bounds[r], bounds[r + 1]
        if hi <= lo:
            continue
        for lo2, hi2 in sub_blocks(lo, hi, full_kv):
            n_seg = hi2 - lo2
            ke_seg = ke[lo2:hi2].contiguous()
            causal_max = chunk._causal_max_cache.get((lo2, hi2))
            if causal_max is None:  # one host sync per sub-block, shared by all layers
                causal_max = int(ke_seg.max().item())
                chunk._causal_max_cache[(lo2, hi2)] = causal_max
            max_kv = min(full_kv, (causal_max + KEY_TILE - 1) // KEY_TILE * KEY_TILE)
            max_kv = max(max_kv, page)
            q_slice = q[tok_lo + lo2:tok_lo + hi2].contiguous()
            w_slice = weights[tok_lo + lo2:tok_lo + hi2].contiguous()
            topk_idx = topk_indices_buffer[tok_lo + lo2:tok_lo + hi2, :topk_tokens]
            if shard.tp > 1 and causal_max >= shard.min_ctx:
                off, span = shard_span(max_kv, shard.tp, shard.rank, page)
                pg_lo = off // page
                pg_hi = max(min(bt_chunk.shape[1], (off + span + page - 1) // page), pg_lo + 1)
                seg_bt = bt_chunk[r:r + 1, pg_lo:pg_hi].expand(n_seg, pg_hi - pg_lo).contiguous()
                sl_raw = ke_seg - off
                sl_local = sl_raw.clamp(1, span).contiguous()
                score = torch.empty((n_seg, span), dtype=torch.float32, device=q.device)
                ops.sm70_indexer_logits(score, q_slice, kv_cache, w_slice, seg_bt, sl_local)
                if shard.rank > 0:  # rows whose reach ends before this span (sai.py:818-835)
                    score[:, 0].masked_fill_(sl_raw <= 0, float("-inf"))
                loc_idx = torch.empty((n_seg, topk_tokens), dtype=torch.int32, device=q.device)
                ops.persistent_topk(score, sl_local.view(n_seg, 1), loc_idx, score, topk_tokens, span)
                neg = loc_idx < 0
                loc_val = score.gather(1, loc_idx.clamp(min=0).to(torch.long))
                loc_val.masked_fill_(neg, float("-inf"))
                gidx = torch.where(neg, loc_idx, loc_idx + off)
                pending.append((tok_lo + lo2, n_seg, loc_val, gidx))
            else:
                bt_cols = min(bt_chunk.shape[1], (max_kv + page - 1) // page)
                seg_bt = bt_chunk[r:r + 1, :bt_cols].expand(n_seg, bt_cols).contiguous()
                score = torch.empty((n_seg, max_kv), dtype=torch.float32, device=q.device)
                ops.sm70_indexer_logits(score, q_slice, kv_cache, w_slice, seg_bt, ke_seg)
                ops.persistent_topk(score, ke_seg.view(n_seg, 1), topk_idx, score, topk_tokens, max_kv)
    if pending:
        merge_shards(pending, topk_indices_buffer, topk_tokens, shard)
    return (tok_lo, n_q, ke)


# -------------------------------------------------- the layer's custom op
# vLLM's forward context stand-in: the per-step indexer metadata of every
# layer, keyed by the layer's k-cache prefix, plus the layer group's key
# sharding (the reference reads get_forward_context().attn_metadata,
# sai.py:541-546).
_FORWARD: dict = {"attn_metadata": None, "shard": None}


@contextlib.contextmanager
def forward_context(attn_metadata: Optional[dict], shard: Optional[ShardConfig] = None):
    """Makes `attn_metadata` ({k_cache_prefix: IndexerMeta}) and `shard` the
    state that ``sm70_sparse_indexer`` reads for the duration of a step."""
    old = dict(_FORWARD)
    _FORWARD.update(attn_metadata=attn_metadata, shard=shard)
    try:
        yield
    finally:
        _FORWARD.update(old)


def _sm70_sparse_indexer_impl(k_cache_prefix: str, kv_cache: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                              weights: torch.Tensor, topk_tokens: int, head_dim: int, max_model_len: int,
                              topk_indices_buffer: torch.Tensor) -> torch.Tensor:
    """Body of the vllm::sm70_sparse_indexer custom op (sai.py:528-1071): a
    profiling / dummy run without metadata returns the buffer untouched
    (sai.py:543-544); otherwise the layer's metadata drives sparse_indexer."""
    md = _FORWARD["attn_metadata"]
    if not isinstance(md, dict):
        return topk_indices_buffer
    if k.shape[-1] != head_dim:
        raise RuntimeError(f"sm70_sparse_indexer: k head dim {k.shape[-1]} != head_dim {head_dim}")
    sparse_indexer(md[k_cache_prefix], kv_cache, q, k, weights, topk_tokens, topk_indices_buffer,
                   shard=_FORWARD["shard"])
    return topk_indices_buffer


def _sm70_sparse_indexer_fake(k_cache_prefix, kv_cache, q, k, weights, topk_tokens, head_dim, max_model_len,
                              topk_indices_buffer):
    return topk_indices_buffer


# schema of the reference's registration (direct_register_custom_op with
# mutates_args=["topk_indices_buffer"], sai.py:1089-1095)
ops._lib_def.define("sm70_sparse_indexer(str k_cache_prefix, Tensor kv_cache, Tensor q, Tensor k, Tensor weights, "
                    "int topk_tokens, int head_dim, int max_model_len, Tensor(a!) topk_indices_buffer) -> Tensor(a!)")
ops._lib_def.impl("sm70_sparse_indexer", _sm70_sparse_indexer_impl, "CUDA")
torch.library.register_fake(f"{ops.NAMESPACE}::sm70_sparse_indexer")(_sm70_sparse_indexer_fake)


def sm70_sparse_indexer(k_cache_prefix: str, kv_cache: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                        weights: torch.Tensor, topk_tokens: int, head_dim: int, max_model_len: int,
                        topk_indices_buffer: torch.Tensor) -> torch.Tensor:
    """The reference's Python entry (sai.py:1098-1119), dispatching through
    the registered op."""
    return getattr(torch.ops, ops.NAMESPACE).sm70_sparse_indexer(k_cache_prefix, kv_cache, q, k, weights, topk_tokens,
                                                                 head_dim, max_model_len, topk_indices_buffer)
