/*
 * dsa_b200.h — C ABI of the B200 (sm_100a) DSA sparse-attention hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches on that stream, never synchronises the host,
 * and returns an int status (DSA_OK on success). On failure the message is
 * available from dsa_last_error() (thread-local). Outputs are caller-owned
 * out-parameters, as in the reference's torch ops (`Tensor!` arguments).
 *
 * Each function names the reference interface it replaces (paths relative
 * to the bayley/glm5-on-v100 project):
 *   dsa.cu   = csrc/attention/sm70_mla_decode.cu
 *   ops.py   = reference/_sm70_ops.py
 *   sai.py   = reference/sparse_attn_indexer.py
 *   tmla.py  = reference/triton_mla.py
 *   binds    = patches/glm5-v100-sm70-full.patch (csrc/torch_bindings.cpp hunk)
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
enum {
  DSA_OK = 0,
  DSA_ERR_INVALID = 1,     /* bad argument: shape, dtype, pointer, size   */
  DSA_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. head_dim)   */
  DSA_ERR_TIMEOUT = 3,     /* a bounded device wait expired (P2P flags)   */
  DSA_ERR_CUDA = 4,        /* a CUDA runtime call failed                  */
  DSA_ERR_WORKSPACE = 5    /* caller workspace too small                  */
};

/* ---- element / cache formats --------------------------------------- */
enum {
  DSA_F16 = 0,  /* IEEE half                                             */
  DSA_BF16 = 1, /* bfloat16                                              */
  DSA_F32 = 2,  /* float                                                 */
  /* fp8_ds_mla latent row, 656 B: 512 e4m3 | 4 x f32 tile scale | 64 f16
   * rope (dsa.cu:74-100). Used only as a latent-cache format.           */
  DSA_FP8_DS_MLA = 3,
  /* fp8 indexer-K row, 132 B: 128 e4m3 | f32 per-token scale
   * (dsa.cu:102-115). Used only as an indexer-cache format.             */
  DSA_FP8_IDXK = 4
};

/* Thread-local text of the last failure ("" when none). */
const char* dsa_last_error(void);
/* ABI version: (major << 16) | minor. */
int dsa_version(void);
/* Sticky device-side status of the current device's tensor-core attention
 * kernel: DSA_ERR_TIMEOUT after one of its bounded pipeline waits expired
 * (the launch then returned without finishing its output), else DSA_OK.
 * Synchronises with the device; reset != 0 clears it. A negative value is
 * -DSA_ERR_CUDA. No counterpart in the reference, whose waits never expire. */
int dsa_device_error(int reset);

/* Test entry for the bounded waits: one block whose mbarrier wait can never
 * complete runs for timeout_ns (1 us .. 1 s) of device time, then records
 * DSA_ERR_TIMEOUT in the status word that dsa_device_error reads and returns,
 * leaving the context usable. No reference counterpart. */
int dsa_selftest_wait_timeout(int64_t timeout_ns, void* stream);

/* =====================================================================
 * Sparse MLA decode / prefill attention.
 * Replaces sm70_sparse_mla_decode (dsa.cu:2457-2616; schema binds
 * "sm70_sparse_mla_decode(Tensor! o, Tensor! lse, Tensor q, Tensor kv_cache,
 * Tensor idx, Tensor block_table, Tensor seq_lens, float scale) -> ()";
 * Python wrapper ops.py:1848-1866; callers tmla.py:292-301, :476-485).
 *
 *   o[b,h,:512]  = sum_j softmax_j(scale * q[b,h,:] . kv_j[:576]) kv_j[:512]
 *   lse[b,h]     = log-sum-exp of the scaled scores (-inf when no j is valid)
 * over j in idx[b, 0:topk] with 0 <= idx < seq_lens[b]; the logical position
 * p resolves to cache row block_table[b, p / page] * page + p % page. A row
 * outside [0, n_kv_rows) reads as zeros (still counted), as in dsa.cu:976-981.
 *
 * q      [B, n_head, 576]  f16 or bf16, contiguous
 * kv     [n_kv_rows / page, page, 576] f16/bf16, or [.., page, 656] u8
 *        (kv_format DSA_FP8_DS_MLA)
 * idx    int32, row stride idx_stride (elements)
 * block_table int32 [B, max_blocks], row stride bt_stride
 * seq_lens int32 [B]
 * o      [B, n_head, 512] f16 or bf16 (o_dtype), contiguous
 * lse    [B, n_head] f32
 * workspace: device scratch of at least
 *   dsa_sparse_mla_decode_workspace_bytes(B, n_head, topk) bytes
 *   (may be NULL when that size is 0).
 * ===================================================================== */
size_t dsa_sparse_mla_decode_workspace_bytes(int B, int n_head, int topk);

/* How dsa_sparse_mla_decode runs a problem with this cache format: the
 * slices of the top-k axis per row (n_splits), how many of them merge inside
 * one thread-block cluster (cluster_size; 1 = partial states merged by a
 * second kernel), the workspace that needs (0 when none) and the kernel
 * launches per call. No reference counterpart (the reference picks its split
 * count and allocates the partial buffers inside the op, dsa.cu:2579-2590);
 * any output pointer may be NULL. */
int dsa_sparse_mla_decode_plan(int B, int n_head, int topk, int kv_format,
                               int* n_splits, int* cluster_size,
                               size_t* workspace_bytes, int* launches);

int dsa_sparse_mla_decode(void* o, int o_dtype, float* lse, const void* q,
                          int q_dtype, const void* kv_cache, int kv_format,
                          int64_t n_kv_rows, int page_size,
                          const int32_t* idx, int64_t idx_stride,
                          const int32_t* block_table, int64_t bt_stride,
                          int max_blocks, const int32_t* seq_lens, int B,
                          int n_head, int topk, double scale,
                          void* workspace, size_t workspace_bytes,
                          void* stream);

/* dsa_sparse_mla_decode without the workspace: it allocates nothing. It has
 * no counterpart in the reference. It is for callers that cannot allocate
 * device memory when they decode, such as an engine whose pool allocator owns
 * the GPU, or a plugin host that passes only input and output buffers. The
 * split partial states live in one static 32 MiB array in this library's
 * device memory, which every GPU that loads the library reserves until the
 * process exits. A call that needs more than that returns DSA_ERR_WORKSPACE
 * before it launches anything. All calls share the array. Nothing in it needs
 * to start at zero, but calls that overlap on the GPU race on it. The first
 * call on a device looks up the array's address, so make it before any stream
 * capture begins. Arguments, outputs and status codes are otherwise those of
 * dsa_sparse_mla_decode. */
int dsa_sparse_mla_decode_noalloc(void* o, int o_dtype, float* lse,
                                  const void* q, int q_dtype,
                                  const void* kv_cache, int kv_format,
                                  int64_t n_kv_rows, int page_size,
                                  const int32_t* idx, int64_t idx_stride,
                                  const int32_t* block_table,
                                  int64_t bt_stride, int max_blocks,
                                  const int32_t* seq_lens, int B, int n_head,
                                  int topk, double scale, void* stream);

/* =====================================================================
 * Lightning-indexer logits.
 * Replaces sm70_indexer_logits (dsa.cu:2626-2764; schema binds
 * "sm70_indexer_logits(Tensor! score, Tensor q, Tensor k_cache,
 * Tensor weights, Tensor block_table, Tensor seq_lens, Tensor!? hist)";
 * wrapper ops.py:1880-1896; callers sai.py:605-613, :622-629, :146-151).
 *
 *   score[b,p] = sum_h w[b,h] * relu(q[b,h,:] . k_p)   for p < seq_lens[b]
 *   score[b,p] = -inf                                 for seq_lens[b] <= p < max_kv
 * k_p is cache row block_table[b, p/page]*page + p%page (zeros when the row
 * is outside [0, n_kv_rows)). page_size must be a power of two.
 *
 * q        [B, n_ihead, 128] f16 or bf16, contiguous (n_ihead 1..64)
 * weights  [B, n_ihead] f16, bf16 or f32, contiguous
 * k_cache  [.., page, 128] f16/bf16 (k_format) or [.., page, 132] u8
 *          (DSA_FP8_IDXK)
 * score    f32 [B, max_kv], row stride score_stride
 * hist     optional (NULL) int32 [B, 4096], pre-zeroed by the caller: each
 *          valid score adds 1 to bin (monotone32(score) >> 20), the level-1
 *          histogram dsa_decode_topk consumes (dsa.cu:315-319).
 * ===================================================================== */
int dsa_indexer_logits(float* score, int64_t score_stride, int max_kv,
                       const void* q, int q_dtype, const void* k_cache,
                       int k_format, int64_t n_kv_rows, int page_size,
                       const void* weights, int w_dtype,
                       const int32_t* block_table, int64_t bt_stride,
                       int max_blocks, const int32_t* seq_lens, int B,
                       int n_ihead, int32_t* hist, void* stream);

/* Packed-Q variant. Replaces sm70_indexer_logits_packed (dsa.cu:2771-2836;
 * schema binds "sm70_indexer_logits_packed(Tensor! score, Tensor q_packed,
 * ...)"; wrapper ops.py:1899-1915; packing sai.py:131-148). q_packed is
 * [32, ceil(B/16), 8, 16, 16] f16/bf16: element (h, t, c, r, d) holds
 * q[16t + r, h, 16c + d] (zero rows past B). Same scores as
 * dsa_indexer_logits on the unpacked q. */
int dsa_indexer_logits_packed(float* score, int64_t score_stride, int max_kv,
                              const void* q_packed, int q_dtype,
                              const void* k_cache, int k_format,
                              int64_t n_kv_rows, int page_size,
                              const void* weights, int w_dtype,
                              const int32_t* block_table, int64_t bt_stride,
                              int max_blocks, const int32_t* seq_lens, int B,
                              void* stream);

/* =====================================================================
 * Top-k selection over score rows.
 * dsa_decode_topk replaces sm70_decode_topk (dsa.cu:2844-2905; schema binds
 * "sm70_decode_topk(Tensor! idx, Tensor score, Tensor seq_lens, Tensor hist,
 * int k)"; wrapper ops.py:1918-1928; caller sai.py:614-620).
 * dsa_topk_rows replaces the upstream persistent_topk op the SM70 indexer
 * calls (sai.py:632-639, :841-848, :873-880; vLLM fork v1.2.1, not vendored).
 *
 * idx[b, 0:K] = positions of the K largest score[b, p] over p < len[b],
 * exact on the 32-bit keys, ties broken towards the LOWER position, written
 * in ASCENDING position order and padded with -1 when len[b] < K.
 * hist (optional for dsa_decode_topk): the level-1 histogram built by
 * dsa_indexer_logits for the same rows; NULL recomputes it.
 * score  f32, row stride score_stride; lens int32 [B]; idx int32, row
 * stride idx_stride. K <= 4096. Reads only p < min(len[b], max_kv).
 * ===================================================================== */
int dsa_decode_topk(int32_t* idx, int64_t idx_stride, const float* score,
                    int64_t score_stride, int max_kv, const int32_t* lens,
                    const int32_t* hist, int B, int K, void* stream);

int dsa_topk_rows(int32_t* idx, int64_t idx_stride, const float* score,
                  int64_t score_stride, int max_kv, const int32_t* lens,
                  int B, int K, void* stream);

/* The same selection written as shard payload rows: pay[b, 0:K] = the
 * selected scores, pay[b, K:2K] = their positions + pos_off bit-cast to f32
 * (-inf / -1 for pads), row stride pay_stride floats (>= 2K). This is the
 * local top-K, the value gather and the global-id shift of a key-sharded
 * rank (sai.py:841-856) in one launch. hist (may be NULL) is consumed and
 * zeroed. */
int dsa_topk_rows_payload(float* pay, int64_t pay_stride, const float* score,
                          int64_t score_stride, int max_kv,
                          const int32_t* lens, int32_t* hist, int B, int K,
                          int pos_off, void* stream);

/* =====================================================================
 * Indexer-K cache scatter.
 * Replaces sm70_indexer_k_store (dsa.cu:2910-2939, kernels :662-706; schema
 * binds "sm70_indexer_k_store(Tensor! kv_cache, Tensor k, Tensor
 * slot_mapping)"; wrapper ops.py:1944-1951; caller sai.py:552-555).
 *
 * For t < n_tok with 0 <= slot[t] < n_rows: cache row slot[t] = k[t].
 * cache_format DSA_F16 / DSA_BF16: plain copy of head_dim elements (k is
 * converted when its dtype differs). DSA_FP8_IDXK (head_dim 128): 128 e4m3
 * (round-to-nearest-even, saturating) of k/scale then the f32 scale
 * max(amax/448, FLT_MIN). Rows with slot < 0 or >= n_rows are skipped.
 * k [n_tok, head_dim] f16/bf16 contiguous; slot int32 [n_tok].
 * ===================================================================== */
int dsa_indexer_k_store(void* kv_cache, int cache_format, int64_t n_rows,
                        const void* k, int k_dtype, int head_dim,
                        const int32_t* slot, int n_tok, void* stream);

/* =====================================================================
 * Cache writers.
 *
 * dsa_concat_and_cache_ds_mla: the fp8_ds_mla latent-cache writer, the
 * upstream concat_and_cache_mla with kv_cache_dtype "fp8_ds_mla" that the
 * reference patches (full.patch:3183-3242; row layout dsa.cu:74-100), with
 * the rotary embedding of k_pe fused in. For t < n_tok with
 * 0 <= slot[t] < n_rows, cache row slot[t] (656 B) =
 *   e4m3(kv_c[t, 128j + i] / s_j)  for the four 128-wide tiles j
 *     (round to nearest even, saturating), s_j = max(amax_j / 448, FLT_MIN)
 *   | s_0..s_3 as f32
 *   | fp16 of rope(k_pe[t], positions[t]) (64 values).
 * Rows with slot < 0 or >= n_rows are skipped. kv_c [n_tok, >= 512] and
 * k_pe [n_tok, >= 64] in in_dtype (f16 or bf16), row strides in elements;
 * kv_c rows 16-byte aligned. positions (int64, may be NULL for no rotation)
 * index cos_sin [max_pos, 64] f32 = 32 cos | 32 sin (vLLM's cos_sin_cache);
 * rope_neox selects pairs (i, i + 32) instead of (2i, 2i + 1). The
 * rotation is computed in f32 without fused multiply-adds.
 * ===================================================================== */
int dsa_concat_and_cache_ds_mla(void* kv_cache, int64_t n_rows,
                                const void* kv_c, int64_t kv_c_stride,
                                const void* k_pe, int64_t k_pe_stride,
                                int in_dtype, const int32_t* slot, int n_tok,
                                const int64_t* positions, const float* cos_sin,
                                int64_t max_pos, int rope_neox, void* stream);

/* dsa_indexer_qk_store: the lightning indexer's q / k / weights producer
 * (the post-GEMM part of Indexer.forward's SM70 branch,
 * full.patch:6404-6425) fused into the indexer-K store (dsa.cu:662-706).
 * Per token t (kw = [k | weight logits], [n_tok, 128 + n_head]):
 *   k = LayerNorm(kw[t, :128]; ln_weight, ln_bias, ln_eps) (NULL weight /
 *       bias = 1 / 0), rotated on dims [0, 64), written to cache row slot[t]
 *       as cache_format (f16, bf16, or DSA_FP8_IDXK with the K store's
 *       quantisation) unless slot[t] < 0 or >= n_rows;
 *   q_out[t, h] = q[t, h] rotated on dims [0, 64) (q [n_tok, n_head, 128],
 *       token stride q_stride elements), in q_out_dtype (f16 / bf16);
 *   w_out[t, h] = kw[t, 128 + h] * w_scale (the reference's
 *       softmax_scale * n_head^-0.5), in w_out_dtype (f16 / bf16 / f32).
 * Rotary pairs and cos_sin as for dsa_concat_and_cache_ds_mla. All
 * arithmetic in f32, each output rounded once. n_head in [1, 256].
 * ===================================================================== */
int dsa_indexer_qk_store(void* q_out, int q_out_dtype, void* w_out,
                         int w_out_dtype, void* k_cache, int cache_format,
                         int64_t n_rows, const void* q, int64_t q_stride,
                         const void* kw, int64_t kw_stride, int in_dtype,
                         const float* ln_weight, const float* ln_bias,
                         float ln_eps, const int64_t* positions,
                         const float* cos_sin, int64_t max_pos, int rope_neox,
                         float w_scale, const int32_t* slot, int n_tok,
                         int n_head, void* stream);

/* =====================================================================
 * Exact shard merge of key-sharded indexer top-k candidates.
 * Replaces sm70_indexer_shard_merge (dsa.cu:2411-2434, kernel :2054-2182;
 * schema binds "sm70_indexer_shard_merge(Tensor! out, Tensor allf, Tensor
 * dst_rows, int dst_base, int topk)"; caller sai.py:987-1006) and the
 * torch.topk epilogue it fuses (sai.py:1007-1030).
 *
 * allf f32 [tp, R, 2K]: per shard s and row r, K values then K int32
 * positions bit-cast to f32 (-1 / -inf = empty). Candidate column
 * col = s*K + c is keyed by (monotone32(val) << 32) | (tp*K - 1 - col), so
 * keys are distinct and ties go to the lower column (torch.topk order on the
 * [R, tp*K] layout). The top K keys' positions (-1 for -inf values) are
 * written ASCENDING to out row (dst_base >= 0 ? dst_base + r : dst_rows[r]).
 * tp in [1, 8], K in [1, 2048]; out row stride out_stride.
 * ===================================================================== */
int dsa_indexer_shard_merge(int32_t* out, int64_t out_stride,
                            const float* allf, const int32_t* dst_rows,
                            int dst_base, int tp, int R, int K, void* stream);

/* Same merge reading each shard's [R, 2K] slab directly from peer memory
 * (CUDA IPC / peer mappings: shard s at data_ptrs[s] + slot_off bytes),
 * after a bounded acquire-wait until every peer's staged flag
 * (flag_ptrs[s][0]) >= seq. Replaces sm70_indexer_shard_merge_p2p
 * (dsa.cu:2394-2409, kernel :2214-2329; caller sai.py:942-947). The wait
 * gives up after timeout_ns of device time and sets *err_flag (device int,
 * caller-zeroed) to DSA_ERR_TIMEOUT; the merge output is then undefined.
 * data_ptrs / flag_ptrs are HOST arrays of tp device addresses. */
int dsa_indexer_shard_merge_p2p(int32_t* out, int64_t out_stride,
                                const uint64_t* data_ptrs,
                                const uint64_t* flag_ptrs,
                                const int32_t* dst_rows, int dst_base, int K,
                                int tp, int R, int seq, int64_t slot_off,
                                int64_t timeout_ns, int32_t* err_flag,
                                void* stream);

/* =====================================================================
 * CUDA IPC helpers for the P2P shard exchange.
 * Replace sm70_ipc_alloc / sm70_ipc_open / sm70_ipc_flag_set /
 * sm70_ipc_slot_wait (dsa.cu:2331-2392; schemas binds; caller
 * sai.py:44-106, :893-952).
 * ===================================================================== */
/* cudaMalloc + zero + cudaIpcGetMemHandle; handle_out gets 64 bytes. */
int dsa_ipc_alloc(int64_t bytes, void** dev_ptr, uint8_t* handle_out);
int dsa_ipc_free(void* dev_ptr);
/* cudaIpcOpenMemHandle(LazyEnablePeerAccess) of a 64-byte handle. */
int dsa_ipc_open(const uint8_t* handle, void** dev_ptr);
int dsa_ipc_close(void* dev_ptr);
/* Stream-ordered release store: ((int*)flag_ptr)[which] = seq after a
 * system-scope fence. When err_flag (device int, may be NULL) is non-zero at
 * that point, nothing is published: a wait before this call failed, and a
 * peer must not read this rank's slot. */
int dsa_ipc_flag_set(uint64_t flag_ptr, int which, int seq,
                     const int32_t* err_flag, void* stream);
/* Stream-ordered bounded wait until every ((int*)flag_ptrs[s])[1] >=
 * min_seq (s < tp). On expiry (timeout_ns of device time) sets *err_flag
 * to DSA_ERR_TIMEOUT and returns on the device; the host reads err_flag. */
int dsa_ipc_slot_wait(const uint64_t* flag_ptrs, int tp, int min_seq,
                      int64_t timeout_ns, int32_t* err_flag, void* stream);

/* Stages a shard payload: slot row r = [vals[r, 0:K] | idx[r, 0:K] as f32
 * bits], r < R (the staging the reference does with two tensor copies,
 * sai.py:905-913). Returns on the device without writing when *err_flag is
 * set (a slot wait before it failed, so a peer may still read the slot);
 * err_flag may be NULL. */
int dsa_indexer_shard_stage(float* slot, const float* vals,
                            int64_t vals_stride, const int32_t* idx,
                            int64_t idx_stride, int R, int K,
                            const int32_t* err_flag, void* stream);

/* =====================================================================
 * Key-sharded decode indexer exchange with a device-side sequence counter.
 * No reference counterpart: the reference shards only prefill scoring and
 * sequences its exchange from the host (sai.py:885-952); here the decode
 * step of every rank is stream-ordered device work that a CUDA graph can
 * replay. Per rank: an IPC buffer of two slots (slot_bytes each, [R, 2K] f32
 * payload rows), the IPC flag pair {staged, merged} of every rank (flag_ptrs,
 * HOST array of tp device addresses, this rank's at index rank) and a local
 * control block ctl (device int32[4], zeroed once: [0] last completed
 * sequence number, [1] and [2] CTA arrival counters).
 *
 * Step seq = ctl[0] + 1:
 *   dsa_shard_exchange_topk: the exact top-K of each score row (as
 *     dsa_decode_topk; hist, if given, is consumed and zeroed for the next
 *     step) is written as a payload row of slot (seq & 1) of slot_base: K
 *     values then K positions + pos_off (-inf / -1 pads); the last CTA
 *     publishes staged = seq unless *err_flag is set. The slot needs no
 *     wait: this rank's merge of step seq - 1 saw every peer's staged
 *     flag of seq - 1, which a peer publishes only after its merge of step
 *     seq - 2 (the slot's last reader) has completed in stream order; the
 *     merged flags stay published for callers that check them.
 *   dsa_shard_exchange_merge: every peer's staged flag >= seq (bounded), the
 *     merge of dsa_indexer_shard_merge over the tp peer slots (plain
 *     relaxed system-scope peer loads) into out rows 0..R-1; the last CTA
 *     publishes merged = seq and sets ctl[0] = seq.
 * Every rank calls stage then merge, step after step, on one stream (the
 * slot reuse above relies on that order). A wait that expires sets
 * *err_flag = DSA_ERR_TIMEOUT; later calls then publish nothing and the host
 * must rebuild the exchange.
 * ===================================================================== */
int dsa_shard_exchange_topk(const float* score, int64_t score_stride,
                            int max_kv, const int32_t* lens, int32_t* hist,
                            int B, int K, int pos_off, void* slot_base,
                            int64_t slot_bytes, const uint64_t* flag_ptrs,
                            int tp, int rank, int32_t* ctl,
                            int64_t timeout_ns, int32_t* err_flag,
                            void* stream);
int dsa_shard_exchange_merge(int32_t* out, int64_t out_stride,
                             const uint64_t* data_ptrs,
                             const uint64_t* flag_ptrs, int tp, int rank,
                             int R, int K, int64_t slot_bytes, int32_t* ctl,
                             int64_t timeout_ns, int32_t* err_flag,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
