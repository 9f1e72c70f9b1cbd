// Exact per-row top-k over f32 score rows (decode and prefill).
//
// Replaces sm70_decode_topk (csrc/attention/sm70_mla_decode.cu:2844-2905,
// kernel :1187-1469) and the upstream persistent_topk op the SM70 indexer
// calls for prefill (reference/sparse_attn_indexer.py:632-639, :841-848,
// :873-880).
//
// One CTA of 1024 threads owns one row, so no cross-CTA arrival counters or
// spin-waits are needed (the reference's decode kernel spins on co-resident
// CTAs, dsa.cu:1372-1375). Selection is an exact MSB-first radix select on
// the 32-bit monotone image of each score: 12 bits (4096 bins, or the
// level-1 histogram the logits kernel already built), then 12 bits, then 8
// bits; the K-th key is exact, so the selected set is exact. Keys equal to
// the K-th key are taken lowest position first. The final compaction walks
// positions in order with block-wide prefix sums, so the output is in
// ascending position order (coalesced gathers downstream), -1 padded.
#include "common.cuh"

namespace dsa {
namespace {

constexpr int NT = 1024;
constexpr int NWARP = NT / 32;
constexpr int NBIN1 = 4096;

struct TopkParams {
  int32_t* idx;
  const float* score;
  const int32_t* lens;
  const int32_t* hist;  // optional level-1 histogram [B, 4096]
  int64_t idx_stride;
  int64_t score_stride;
  int max_kv;
  int K;
};

// Block-wide: find the largest bin T with count(bins >= T) >= need, scanning
// `nbins` (<= 4 * NT) bins. Writes T and count(bins > T) to shared memory.
__device__ void find_threshold(const uint32_t* hist, int nbins, uint32_t need, uint32_t* s_warp,
                               int* s_T, uint32_t* s_above) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (nbins + NT - 1) / NT;  // bins per thread (contiguous)
  if (tid == 0) {  // defined result even for an inconsistent caller histogram
    *s_T = 0;
    *s_above = 0;
  }
  uint32_t cs = 0;
  for (int i = 0; i < per; ++i) {
    const int bin = tid * per + i;
    if (bin < nbins) cs += hist[bin];
  }
  // inclusive suffix scan: sum over threads >= tid
  uint32_t suf = cs;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_down_sync(0xffffffffu, suf, off);
    if (lane + off < 32) suf += v;
  }
  if (lane == 0) s_warp[warp] = suf;  // warp total
  __syncthreads();
  if (warp == 0) {
    uint32_t wt = s_warp[lane];
    uint32_t ws = wt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_down_sync(0xffffffffu, ws, off);
      if (lane + off < 32) ws += v;
    }
    s_warp[32 + lane] = ws - wt;  // total of warps strictly after this one
  }
  __syncthreads();
  suf += s_warp[32 + warp];
  const uint32_t above_chunk = suf - cs;  // count in bins of later threads
  if (above_chunk < need && suf >= need) {
    uint32_t above = above_chunk;
    for (int i = per - 1; i >= 0; --i) {
      const int bin = tid * per + i;
      if (bin >= nbins) continue;
      const uint32_t c = hist[bin];
      if (above + c >= need) {
        *s_T = bin;
        *s_above = above;
        break;
      }
      above += c;
    }
  }
  __syncthreads();
}

// Block-wide exclusive prefix of a 0/1 flag in thread order; returns the
// prefix and writes the block total to *s_total.
__device__ __forceinline__ uint32_t block_prefix(bool flag, uint32_t* s_warp, uint32_t* s_total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, flag);
  const uint32_t in_warp = __popc(bal & ((1u << lane) - 1u));
  if (lane == 0) s_warp[warp] = __popc(bal);
  __syncthreads();
  if (warp == 0) {
    const uint32_t v = s_warp[lane];
    uint32_t inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += u;
    }
    s_warp[32 + lane] = inc - v;
    if (lane == 31) *s_total = inc;
  }
  __syncthreads();
  const uint32_t r = s_warp[32 + warp] + in_warp;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(NT) topk_rows_kernel(const TopkParams p) {
  __shared__ uint32_t s_hist[NBIN1];
  __shared__ uint32_t s_warp[64];
  __shared__ int s_T;
  __shared__ uint32_t s_above, s_total;

  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int K = p.K;
  int32_t* out = p.idx + (int64_t)b * p.idx_stride;
  const float* row = p.score + (int64_t)b * p.score_stride;
  const int n = max(0, min(p.lens[b], p.max_kv));

  if (n <= K) {  // everything valid is selected
    for (int i = tid; i < K; i += NT) out[i] = i < n ? i : -1;
    return;
  }
  // ---- level 1: bits 31..20
  if (p.hist) {
    for (int i = tid; i < NBIN1; i += NT) s_hist[i] = (uint32_t)p.hist[(int64_t)b * NBIN1 + i];
  } else {
    for (int i = tid; i < NBIN1; i += NT) s_hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += NT) atomicAdd(&s_hist[monotone32(__ldg(row + i)) >> 20], 1u);
  }
  __syncthreads();
  find_threshold(s_hist, NBIN1, (uint32_t)K, s_warp, &s_T, &s_above);
  const uint32_t T1 = (uint32_t)s_T;
  const uint32_t need2 = (uint32_t)K - s_above;
  // ---- level 2: bits 19..8 among keys with the level-1 prefix
  for (int i = tid; i < NBIN1; i += NT) s_hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const uint32_t key = monotone32(__ldg(row + i));
    if ((key >> 20) == T1) atomicAdd(&s_hist[(key >> 8) & 0xFFFu], 1u);
  }
  __syncthreads();
  find_threshold(s_hist, NBIN1, need2, s_warp, &s_T, &s_above);
  const uint32_t pre2 = (T1 << 12) | (uint32_t)s_T;
  const uint32_t need3 = need2 - s_above;
  // ---- level 3: bits 7..0
  for (int i = tid; i < 256; i += NT) s_hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const uint32_t key = monotone32(__ldg(row + i));
    if ((key >> 8) == pre2) atomicAdd(&s_hist[key & 0xFFu], 1u);
  }
  __syncthreads();
  find_threshold(s_hist, 256, need3, s_warp, &s_T, &s_above);
  const uint32_t kth = (pre2 << 8) | (uint32_t)s_T;
  const uint32_t n_ties = need3 - s_above;  // keys == kth to take, lowest positions first

  // ---- ordered compaction
  uint32_t out_base = 0, tie_base = 0;
  for (int base = 0; base < n; base += NT) {
    const int i = base + tid;
    uint32_t key = 0;
    bool in = i < n;
    if (in) key = monotone32(__ldg(row + i));
    const bool eq = in && key == kth;
    const uint32_t tie_rank = tie_base + block_prefix(eq, s_warp, &s_total);
    const uint32_t n_eq = s_total;
    const bool sel = in && (key > kth || (eq && tie_rank < n_ties));
    const uint32_t pos = out_base + block_prefix(sel, s_warp, &s_total);
    if (sel) out[pos] = i;
    out_base += s_total;
    tie_base += n_eq;
  }
}

int run_topk(const TopkParams& p, int B, cudaStream_t s) {
  DSA_REQUIRE(B >= 0 && p.max_kv >= 0, DSA_ERR_INVALID, "topk: negative size");
  DSA_REQUIRE(p.K >= 1 && p.K <= 4096, DSA_ERR_UNSUPPORTED, "topk: K must be in [1, 4096] (got %d)", p.K);
  if (B == 0) return DSA_OK;
  DSA_REQUIRE(p.idx && p.lens && (p.score || p.max_kv == 0), DSA_ERR_INVALID, "topk: null pointer");
  DSA_REQUIRE(p.idx_stride >= p.K && p.score_stride >= p.max_kv, DSA_ERR_INVALID,
              "topk: row stride smaller than the row");
  topk_rows_kernel<<<B, NT, 0, s>>>(p);
  return check_launch("topk_rows_kernel");
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_decode_topk(int32_t* idx, int64_t idx_stride, const float* score, int64_t score_stride,
                               int max_kv, const int32_t* lens, const int32_t* hist, int B, int K,
                               void* stream) {
  clear_error();
  TopkParams p{idx, score, lens, hist, idx_stride, score_stride, max_kv, K};
  return run_topk(p, B, as_stream(stream));
}

extern "C" int dsa_topk_rows(int32_t* idx, int64_t idx_stride, const float* score, int64_t score_stride,
                             int max_kv, const int32_t* lens, int B, int K, void* stream) {
  clear_error();
  TopkParams p{idx, score, lens, nullptr, idx_stride, score_stride, max_kv, K};
  return run_topk(p, B, as_stream(stream));
}
