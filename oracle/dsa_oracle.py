"""CPU oracle for the DSA sparse-attention hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy (float64 where arithmetic matters), the
algorithms of the reference's DSA path so that tests can check the CUDA
kernels. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it; the product path never calls it.

Parity pins (see ``tests/golden/make_golden.py``):
  * ``sparse_mla_decode`` is pinned against the reference's own torch path
    ``TritonMLAImpl._forward_mqa_torch`` (reference/triton_mla.py:494-554),
    run through a page-size-1 block table over the selected rows, and
    against ``_varlen_attention``
    (vllm/v1/attention/backends/mla/prefill/sm70_triton.py:54-187).
  * ``shard_merge`` is pinned against the reference's torch.topk epilogue
    (reference/sparse_attn_indexer.py:1007-1030), executed from the
    reference source text.
  * ``indexer_logits`` / ``topk_rows`` / ``decode_topk`` have no CPU
    implementation in the reference (only SM70 CUDA kernels), so their
    restatement is pinned by the formula of
    csrc/attention/sm70_mla_decode.cu:132-149, :309-319 and by the
    reference's stated invariants (sparse == dense below top-k;
    global top-k subset of the union of shard top-ks).

Paths in citations are relative to the bayley/glm5-on-v100 project:
``dsa.cu`` = csrc/attention/sm70_mla_decode.cu.
"""
from __future__ import annotations

import numpy as np

FLT_MIN = np.float32(1.1754943508222875e-38)
E4M3_MAX = 448.0
DSMLA_ROW_BYTES = 656  # dsa.cu:81
IDXK_FP8_ROW_BYTES = 132  # dsa.cu:107
D_K = 576
D_V = 512
TOPK_NBIN = 4096  # dsa.cu:41


# ---------------------------------------------------------------------------
# OCP fp8 E4M3 (bias 7, no infinities, S.1111.111 = NaN, max 448).
# ---------------------------------------------------------------------------
def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * m * 2.0 ** -9
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()
_POS_VALUES = E4M3_VALUES[:0x7F]  # codes 0x00..0x7E, ascending


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """uint8 codes -> float64 values."""
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode_satfinite(x: np.ndarray) -> np.ndarray:
    """float -> e4m3 code, round-to-nearest-even, saturating to +-448.

    Same rounding as the hardware ``cvt.rn.satfinite.e4m3x2.f32`` and as
    ``__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)`` used by the
    reference's fp8 indexer-K store (dsa.cu:703).
    """
    x = np.asarray(x, dtype=np.float64)
    neg = np.signbit(x)
    a = np.minimum(np.abs(x), E4M3_MAX)
    # quantum of the e4m3 grid at |a|: 2^(e-3) for normals, 2^-9 below 2^-6
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)
    quantum = np.exp2(e - 3.0)
    q = np.rint(a / quantum) * quantum  # rint = half-to-even
    q = np.minimum(q, E4M3_MAX)
    code = np.searchsorted(_POS_VALUES, q).astype(np.uint8)
    nan = np.isnan(x)
    code = np.where(neg & (q > 0), code | 0x80, code)
    code = np.where(neg & (q == 0), np.uint8(0x80), code)
    code = np.where(nan, np.uint8(0x7F), code)
    return code.astype(np.uint8)


# ---------------------------------------------------------------------------
# Cache row formats.
# ---------------------------------------------------------------------------
def dsmla_encode_rows(latent: np.ndarray) -> np.ndarray:
    """[n, 576] float -> [n, 656] uint8 fp8_ds_mla rows (dsa.cu:74-100).

    Bytes [0,512): e4m3 of latent[:512] / scale_t per 128-wide tile t;
    bytes [512,528): the four f32 scales scale_t = max(amax_t / 448, FLT_MIN)
    (the per-token rule of the indexer-K store, dsa.cu:699-703, applied per
    tile); bytes [528,656): latent[512:576] as IEEE half, verbatim.
    All divisions are single-precision, as on the GPU.
    """
    latent = np.asarray(latent, dtype=np.float32)
    n = latent.shape[0]
    out = np.zeros((n, DSMLA_ROW_BYTES), dtype=np.uint8)
    nope = latent[:, :512].reshape(n, 4, 128)
    amax = np.abs(nope).max(axis=2)
    scale = np.maximum(amax / np.float32(448.0), FLT_MIN).astype(np.float32)
    codes = e4m3_encode_satfinite((nope / scale[:, :, None]).astype(np.float32))
    out[:, :512] = codes.reshape(n, 512)
    out[:, 512:528] = scale.view(np.uint8).reshape(n, 16)
    out[:, 528:656] = latent[:, 512:576].astype(np.float16).view(np.uint8).reshape(n, 128)
    return out


def dsmla_decode_rows(rows: np.ndarray, as_fp16: bool = True) -> np.ndarray:
    """[n, 656] uint8 -> [n, 576] float64 dequantised latent (dsa.cu:83-100).

    The reference's attention kernels gather each value as e4m3 * scale in
    f32 and store it as IEEE half before the tensor-core products
    (dsa.cu:983-1004, :1632-1677), so by default the dequantised values are
    rounded to fp16 here too; as_fp16=False keeps the f32 products.
    """
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n = rows.shape[0]
    vals = e4m3_decode(rows[:, :512]).reshape(n, 4, 128)
    scale = rows[:, 512:528].copy().view(np.float32).reshape(n, 4).astype(np.float64)
    nope = (vals * scale[:, :, None]).astype(np.float32)
    if as_fp16:
        nope = nope.astype(np.float16)
    nope = nope.astype(np.float64)
    rope = rows[:, 528:656].copy().view(np.float16).reshape(n, 64).astype(np.float64)
    return np.concatenate([nope.reshape(n, 512), rope], axis=1)


def idxk_encode_rows(k: np.ndarray) -> np.ndarray:
    """[n, 128] float -> [n, 132] uint8 fp8 indexer-K rows (dsa.cu:681-706)."""
    k = np.asarray(k, dtype=np.float32)
    n = k.shape[0]
    amax = np.abs(k).max(axis=1)
    scale = np.maximum(amax / np.float32(448.0), FLT_MIN).astype(np.float32)
    out = np.zeros((n, IDXK_FP8_ROW_BYTES), dtype=np.uint8)
    out[:, :128] = e4m3_encode_satfinite((k / scale[:, None]).astype(np.float32))
    out[:, 128:132] = scale.view(np.uint8).reshape(n, 4)
    return out


def idxk_decode_rows(rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    n = rows.shape[0]
    vals = e4m3_decode(rows[:, :128])
    scale = rows[:, 128:132].copy().view(np.float32).reshape(n).astype(np.float64)
    return vals * scale[:, None]


def indexer_k_store(cache_rows: np.ndarray, k: np.ndarray, slot: np.ndarray,
                    fmt: str) -> np.ndarray:
    """Indexer-K scatter (dsa.cu:662-706): row slot[t] <- k[t]; slot<0/OOB skipped.

    cache_rows: [n_rows, 128] float16/bfloat16-as-uint16 or [n_rows, 132] uint8.
    fmt: 'f16' | 'bf16' | 'fp8'. k is float32 holding the exact input values.
    Later tokens win when two tokens share a slot (the GPU's order is then
    unspecified; tests use distinct slots).
    """
    out = cache_rows.copy()
    n_rows = out.shape[0]
    for t in range(k.shape[0]):
        s = int(slot[t])
        if s < 0 or s >= n_rows:
            continue
        if fmt == "fp8":
            out[s] = idxk_encode_rows(k[t:t + 1])[0]
        elif fmt == "f16":
            out[s] = k[t].astype(np.float16)
        elif fmt == "bf16":
            out[s] = f32_to_bf16_bits(k[t])
        else:
            raise ValueError(fmt)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), round-to-nearest-even."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# Paged addressing (dsa.cu:976-981, tmla.py:524-535).
# ---------------------------------------------------------------------------
def resolve_rows(pos: np.ndarray, bt_row: np.ndarray, page: int) -> np.ndarray:
    """logical positions -> physical cache rows via one block-table row."""
    pos = np.asarray(pos, dtype=np.int64)
    blk = np.asarray(bt_row, dtype=np.int64)[pos // page]
    return blk * page + pos % page


# ---------------------------------------------------------------------------
# Sparse MLA decode (dsa.cu:918-1184 split + merge; tmla.py:494-554 math).
# ---------------------------------------------------------------------------
def sparse_mla_decode(q: np.ndarray, kv_rows: np.ndarray, idx: np.ndarray,
                      block_table: np.ndarray, seq_lens: np.ndarray,
                      page: int, scale: float):
    """Exact (float64) sparse MLA attention over the selected latent rows.

    q [B,H,576] float; kv_rows [n_rows,576] float (dequantised cache rows);
    idx [B,topk] int; block_table [B,max_blocks]; seq_lens [B].
    Column j of row b is used iff 0 <= idx[b,j] < seq_lens[b] (dsa.cu:978-979,
    :1052-1053); a resolved row outside [0, n_rows) contributes a zero key and
    value but is still counted (dsa.cu:980-981 loads zeros, the softmax mask
    only checks the position). No valid column gives o = 0 and lse = -inf
    (the merge rule, dsa.cu:1170-1183).
    Returns o [B,H,512] float64, lse [B,H] float64.
    """
    q = np.asarray(q, dtype=np.float64)
    B, H, _ = q.shape
    n_rows = kv_rows.shape[0]
    o = np.zeros((B, H, D_V), dtype=np.float64)
    lse = np.full((B, H), -np.inf, dtype=np.float64)
    for b in range(B):
        sl = int(seq_lens[b])
        pos = np.asarray(idx[b], dtype=np.int64)
        pos = pos[(pos >= 0) & (pos < sl)]
        if pos.size == 0:
            continue
        rows = resolve_rows(pos, block_table[b], page)
        ok = (rows >= 0) & (rows < n_rows)
        kv = np.zeros((pos.size, D_K), dtype=np.float64)
        kv[ok] = kv_rows[rows[ok]]
        s = (q[b] @ kv.T) * scale  # [H, n]
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        l = p.sum(axis=1, keepdims=True)
        o[b] = (p @ kv[:, :D_V]) / l
        lse[b] = (m + np.log(l))[:, 0]
    return o, lse


# ---------------------------------------------------------------------------
# Lightning-indexer logits (dsa.cu:132-149, :264-265, :309-319).
# ---------------------------------------------------------------------------
def indexer_logits(q: np.ndarray, k_rows: np.ndarray, w: np.ndarray,
                   block_table: np.ndarray, seq_lens: np.ndarray, page: int,
                   max_kv: int) -> np.ndarray:
    """score[b,p] = sum_h w[b,h] * relu(q[b,h] . k_p) for p < seq_len, else -inf.

    q [B,Hi,128]; k_rows [n_rows,128] float (dequantised); w [B,Hi].
    Rows outside [0, n_rows) read as zeros (score 0), as dsa.cu:242-263 does.
    Returns float64 [B, max_kv].
    """
    q = np.asarray(q, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    B = q.shape[0]
    n_rows = k_rows.shape[0]
    out = np.full((B, max_kv), -np.inf, dtype=np.float64)
    for b in range(B):
        n = min(int(seq_lens[b]), max_kv)
        if n <= 0:
            continue
        rows = resolve_rows(np.arange(n), block_table[b], page)
        ok = (rows >= 0) & (rows < n_rows)
        k = np.zeros((n, k_rows.shape[1]), dtype=np.float64)
        k[ok] = k_rows[rows[ok]]
        dots = q[b] @ k.T  # [Hi, n]
        out[b, :n] = (np.maximum(dots, 0.0) * w[b][:, None]).sum(axis=0)
    return out


def monotone32(x: np.ndarray) -> np.ndarray:
    """f32 -> uint32 key whose unsigned order is the float order (dsa.cu:43-46)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    return np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)


def level1_hist(score: np.ndarray, lens: np.ndarray) -> np.ndarray:
    """The 4096-bin histogram of monotone32(score) >> 20 over p < len (dsa.cu:315-319)."""
    score = np.asarray(score, dtype=np.float32)
    B, max_kv = score.shape
    hist = np.zeros((B, TOPK_NBIN), dtype=np.int32)
    for b in range(B):
        n = min(int(lens[b]), max_kv)
        if n > 0:
            np.add.at(hist[b], monotone32(score[b, :n]) >> 20, 1)
    return hist


def topk_rows(score: np.ndarray, lens: np.ndarray, K: int) -> np.ndarray:
    """Exact per-row top-K positions of f32 scores over p < len.

    Keys are the 32-bit monotone images of the f32 scores; equal keys are
    taken lowest position first. Output ascending, -1 padded. This is the
    selection contract of dsa_decode_topk / dsa_topk_rows; the reference's
    K12 (dsa.cu:1187-1469) is exact to 24 key bits with the same
    lowest-position tie rule.
    """
    score = np.asarray(score, dtype=np.float32)
    B, max_kv = score.shape
    out = np.full((B, K), -1, dtype=np.int32)
    for b in range(B):
        n = min(int(lens[b]), max_kv)
        if n <= 0:
            continue
        key = monotone32(score[b, :n]).astype(np.int64)
        order = np.lexsort((np.arange(n), -key))  # key desc, position asc
        sel = np.sort(order[:K])
        out[b, :sel.size] = sel
    return out


# ---------------------------------------------------------------------------
# Shard merge (dsa.cu:2054-2182; torch epilogue sai.py:1007-1030).
# ---------------------------------------------------------------------------
def shard_merge(allf: np.ndarray, K: int) -> np.ndarray:
    """Exact top-K over tp*K candidates per row, positions ascending.

    allf f32 [tp, R, 2K]: K values then K positions bit-cast to f32.
    Key(col) = (monotone32(val) << 32) | (tp*K - 1 - col), col = s*K + c, so
    keys are distinct and the lower column wins ties (dsa.cu:2058-2063).
    Selected -inf values (monotone key <= 0x007FFFFF) emit -1 (dsa.cu:2146-2151).
    Returns int32 [R, K] sorted ascending (-1 first, dsa.cu:2159-2160).
    """
    allf = np.ascontiguousarray(allf, dtype=np.float32)
    tp, R, twoK = allf.shape
    assert twoK == 2 * K
    vals = allf[:, :, :K].transpose(1, 0, 2).reshape(R, tp * K)
    pos = allf[:, :, K:].copy().view(np.int32).transpose(1, 0, 2).reshape(R, tp * K)
    ncand = tp * K
    mono = monotone32(vals).astype(np.uint64)
    col = np.arange(ncand, dtype=np.uint64)
    key = (mono << np.uint64(32)) | (np.uint64(ncand - 1) - col)
    out = np.empty((R, K), dtype=np.int32)
    for r in range(R):
        top = np.argsort(key[r])[::-1][:K]
        sel = np.where(mono[r, top] > 0x007FFFFF, pos[r, top], -1)
        out[r] = np.sort(sel)
    return out


def shard_merge_torch_epilogue(allf, K):
    """Restatement of the torch.topk epilogue (sai.py:1007-1030), sorted
    ascending for comparison with the fused merge (same set, sai.py:969-976)."""
    import torch

    allf = torch.as_tensor(np.ascontiguousarray(allf, dtype=np.float32))
    tp, R, _ = allf.shape
    av = allf[:, :, :K].permute(1, 0, 2).reshape(R, tp * K)
    ai = allf[:, :, K:].permute(1, 0, 2).reshape(R, tp * K).contiguous().view(torch.int32)
    mv, mp = torch.topk(av, K, dim=1)
    mi = ai.gather(1, mp)
    mi = torch.where(torch.isinf(mv), torch.full_like(mi, -1), mi).to(torch.int32)
    return np.sort(mi.numpy(), axis=1)


# ---------------------------------------------------------------------------
# Key-sharded indexer (sai.py:796-857): per-rank spans and local top-k.
# ---------------------------------------------------------------------------
def shard_span(max_kv: int, tp: int, rank: int, page: int, kt: int = 64):
    """(off, span) of rank's contiguous key span (sai.py:797-806)."""
    unit = max(kt, page)
    per = ((max_kv + tp - 1) // tp + unit - 1) // unit * unit
    off = rank * per
    span = min(per, max(max_kv - off, 0))
    span = max(span, page)
    return off, span


def sharded_local_candidates(score_full: np.ndarray, lens: np.ndarray, K: int,
                             off: int, span: int, rank: int):
    """One rank's [R, 2K] payload from full-row scores (sai.py:818-856).

    The rank scores keys [off, off+span) with local causal length
    clamp(len - off, 1, span); rows whose reach ends before the span force
    their single candidate to -inf (sai.py:833-835). Local positions are
    shifted by off. Returns (vals f32 [R,K], gidx int32 [R,K]).
    """
    R = score_full.shape[0]
    local = np.full((R, span), -np.inf, dtype=np.float32)
    w = min(span, score_full.shape[1] - off)
    if w > 0:
        local[:, :w] = score_full[:, off:off + w]
    sl_raw = np.asarray(lens, dtype=np.int64) - off
    sl_local = np.clip(sl_raw, 1, span)
    if rank > 0:
        local[sl_raw <= 0, 0] = -np.inf
    loc_idx = topk_rows(local, sl_local, K)
    neg = loc_idx < 0
    vals = np.take_along_axis(local, np.maximum(loc_idx, 0), axis=1)
    vals[neg] = -np.inf
    gidx = np.where(neg, loc_idx, loc_idx + off).astype(np.int32)
    return vals.astype(np.float32), gidx


# ---------------------------------------------------------------------------
# Cache writers: the fp8_ds_mla latent writer (upstream concat_and_cache_mla,
# amax fix full.patch:3209-3230, row dsa.cu:74-100) and the indexer's
# q / k / weights producer (full.patch:6404-6425) with the K store.
# ---------------------------------------------------------------------------
def rope_f32(x: np.ndarray, pos: np.ndarray, cos_sin: np.ndarray, neox: bool) -> np.ndarray:
    """Rotary embedding of the first 64 dims of x [n, >=64] at positions pos,
    cos_sin [max_pos, 64] = 32 cos | 32 sin (vLLM's RotaryEmbedding: NeoX
    pairs (i, i+32) or GPT-J pairs (2i, 2i+1)); every product and sum is
    rounded in f32, as the writer kernels compute it."""
    x = np.array(x, dtype=np.float32, copy=True)
    p = np.clip(np.asarray(pos, dtype=np.int64), 0, cos_sin.shape[0] - 1)
    c = cos_sin[p, :32].astype(np.float32)
    s = cos_sin[p, 32:64].astype(np.float32)
    i1, i2 = (np.arange(32), np.arange(32) + 32) if neox else (np.arange(0, 64, 2), np.arange(1, 64, 2))
    x1, x2 = x[:, i1], x[:, i2]
    x[:, i1] = (x1 * c).astype(np.float32) - (x2 * s).astype(np.float32)
    x[:, i2] = (x2 * c).astype(np.float32) + (x1 * s).astype(np.float32)
    return x


def dsmla_write_rows(kv_c, k_pe, pos=None, cos_sin=None, neox=False) -> np.ndarray:
    """Rows the latent writer stores for kv_c [n, 512] and k_pe [n, 64]
    (rotated first when pos is given): the per-tile encoding of
    dsmla_encode_rows over [kv_c | rope(k_pe)]."""
    kv = np.asarray(kv_c, dtype=np.float32)
    kp = np.asarray(k_pe, dtype=np.float32).reshape(kv.shape[0], 64)
    if pos is not None:
        kp = rope_f32(kp, pos, cos_sin, neox)
    return dsmla_encode_rows(np.concatenate([kv, kp], axis=1))


def indexer_qk_produce(q, kw, ln_w, ln_b, eps, pos, cos_sin, neox, w_scale):
    """(q_out [T, H, 128], k [T, 128], weights [T, H]) of the indexer's producer
    in float64: k = LayerNorm(kw[:, :128]) (biased variance, eps inside the
    root), rotary on dims [0, 64) of k and of every q head, weights =
    kw[:, 128:] * w_scale (full.patch:6406-6425)."""
    q = np.asarray(q, dtype=np.float64)
    kw = np.asarray(kw, dtype=np.float64)
    T, H, _ = q.shape
    k = kw[:, :128]
    mu = k.mean(axis=1, keepdims=True)
    var = ((k - mu) ** 2).mean(axis=1, keepdims=True)
    k = (k - mu) / np.sqrt(var + eps)
    if ln_w is not None:
        k = k * np.asarray(ln_w, dtype=np.float64)
    if ln_b is not None:
        k = k + np.asarray(ln_b, dtype=np.float64)
    qo = q.copy()
    if pos is not None:
        p = np.clip(np.asarray(pos, dtype=np.int64), 0, cos_sin.shape[0] - 1)
        c = np.asarray(cos_sin, dtype=np.float64)[p, :32]
        s = np.asarray(cos_sin, dtype=np.float64)[p, 32:64]
        i1, i2 = (np.arange(32), np.arange(32) + 32) if neox else (np.arange(0, 64, 2), np.arange(1, 64, 2))

        def rot(x, c, s):
            x1, x2 = x[..., i1].copy(), x[..., i2].copy()
            x[..., i1] = x1 * c - x2 * s
            x[..., i2] = x2 * c + x1 * s

        rot(k, c, s)
        rot(qo, c[:, None, :], s[:, None, :])
    return qo, k, kw[:, 128:] * w_scale
