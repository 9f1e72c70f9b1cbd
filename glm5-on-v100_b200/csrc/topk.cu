// Exact per-row top-k over f32 score rows (decode and prefill).
//
// Replaces sm70_decode_topk (csrc/attention/sm70_mla_decode.cu:2844-2905,
// kernel :1187-1469) and the upstream persistent_topk op the SM70 indexer
// calls for prefill (reference/sparse_attn_indexer.py:632-639, :841-848,
// :873-880).
//
// One CTA owns one row (512 threads when the rows fill the GPU, 1024 when
// there are fewer rows than half the SMs), so no cross-CTA arrival counters or
// spin-waits are needed (the reference's decode kernel spins on co-resident
// CTAs, dsa.cu:1372-1375). Keys are the 32-bit monotone images of the
// scores; the K-th largest key is found exactly, keys equal to it are taken
// lowest position first, and the output lists positions in ascending order
// (coalesced gathers downstream), -1 padded.
//
//   1. Level-1 histogram of the top 12 key bits (or the one the logits kernel
//      built) gives the bin T1 holding the K-th key.
//   2. One ordered sweep (each warp owns a contiguous run of positions, read
//      with 16-byte coalesced loads) writes every position of a bin above T1
//      to a "sure" list and every key of bin T1 with its position to a
//      candidate list, both in position order, in shared memory.
//   3. The remaining 20 bits are resolved among the candidates in shared
//      memory (12 + 8 bit radix levels), the selected candidates compacted in
//      order, and the two ascending lists merged into the output.
// When bin T1 holds more keys than the candidate buffer, the row is resolved
// by radix levels over global memory and an ordered block-wide compaction.
#include <cooperative_groups.h>

#include "common.cuh"
#include "sparse_mla.cuh"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace dsa {
namespace {

// Threads per row: 512 (two CTAs per SM) when rows fill the GPU, 1024 when
// there are fewer rows than half the SMs (decode batches).
constexpr int NT_SMALL = 512;
constexpr int NT_LARGE = 1024;
constexpr int NBIN1 = 4096;
constexpr int CAP = 8192;  // candidates of the threshold bin kept in shared memory
constexpr int KMAX = 4096;
constexpr int SWEEP_U = 4;  // 128-position steps whose loads a warp issues together

constexpr int MAX_TP = 8;

struct TopkParams {
  int32_t* idx;
  const float* score;
  const int32_t* lens;
  const int32_t* hist;  // optional level-1 histogram [B, 4096]
  int64_t idx_stride;
  int64_t score_stride;
  int max_kv;
  int K;
  // payload mode (pay != null): row b is written to pay + b * pay_stride as
  // K f32 values then K int32 positions + pos_off (bit-cast), -inf / -1 pads
  float* pay;
  int64_t pay_stride;
  int pos_off;
  int32_t* hist_clear;  // when set (== hist): each hist row is zeroed once read
  // exchange staging (ctl != null): the payload goes to slot (seq & 1) of
  // this rank's exchange buffer, seq = ctl[0] + 1; the last CTA publishes
  // staged = seq on my_flags[0] unless the error word is set. Slot seq & 1
  // is free without a wait: this rank's merge of step seq - 1 saw every
  // peer's staged(seq - 1), which each peer publishes only after its merge of
  // step seq - 2, the last reader of this slot, has completed (stream order).
  int* ctl;
  int* my_flags;
  int tp;
  int64_t slot_bytes;
  int64_t timeout_ns;
  int32_t* err;
  int32_t* dev_err;  // the library's sticky device status word (staging waits)
};

// Where the selected positions of one row go.
struct Emit {
  int32_t* idx;        // index mode
  float* val;          // payload mode: values ...
  int32_t* pos;        // ... and shifted positions
  const float* row;
  int off;
  __device__ __forceinline__ void operator()(int o, int P) const {
    if (val) {
      val[o] = P >= 0 ? row[P] : __int_as_float(0xff800000);
      pos[o] = P >= 0 ? P + off : -1;
    } else {
      idx[o] = P;
    }
  }
};

struct TopkSmem {
  uint32_t hist[NBIN1];
  uint32_t cand_key[CAP];
  int32_t cand_pos[CAP];
  int32_t sure[KMAX];
  int32_t sel[KMAX];
  uint32_t warp[64];
  uint32_t warp_off[32];
  int T;
  uint32_t above, total;
  int ok;
  uint32_t cl_cnt[8];  // cluster mode: every CTA's (sure | candidates << 16) counts
  int cl_ok[8];        // cluster mode: every CTA's staging waits succeeded
  uint32_t cl_lo;      // cluster mode: selected candidates before this CTA's range
  uint32_t cl_nsel;    // cluster mode: selected candidates in this CTA's range
  uint32_t cl_total;   // cluster mode: selected candidates of the row
};

// Block-wide: find the largest bin T with count(bins >= T) >= need, scanning
// `nbins` bins (contiguous runs per thread). Writes T and count(bins > T).
template <int NT>
__device__ void find_threshold(const uint32_t* hist, int nbins, uint32_t need, uint32_t* s_warp, int* s_T,
                               uint32_t* s_above) {
  constexpr int NWARP = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (nbins + NT - 1) / NT;
  if (tid == 0) {  // defined result even for an inconsistent caller histogram
    *s_T = 0;
    *s_above = 0;
  }
  uint32_t cs = 0;
  for (int i = 0; i < per; ++i) {
    const int bin = tid * per + i;
    if (bin < nbins) cs += hist[bin];
  }
  uint32_t suf = cs;  // inclusive suffix sum within the warp
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_down_sync(0xffffffffu, suf, off);
    if (lane + off < 32) suf += v;
  }
  if (lane == 0) s_warp[warp] = suf;
  __syncthreads();
  if (warp == 0) {
    const uint32_t wt = lane < NWARP ? s_warp[lane] : 0u;
    uint32_t ws = wt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_down_sync(0xffffffffu, ws, off);
      if (lane + off < 32) ws += v;
    }
    s_warp[32 + lane] = ws - wt;  // total of the warps after this one
  }
  __syncthreads();
  suf += s_warp[32 + warp];
  const uint32_t above_chunk = suf - cs;
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

// Block-wide exclusive prefix of v in thread order; *s_total gets the sum.
template <int NT>
__device__ __forceinline__ uint32_t block_exclusive(uint32_t v, uint32_t* s_warp, uint32_t* s_total) {
  constexpr int NWARP = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += u;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const uint32_t wv = lane < NWARP ? s_warp[lane] : 0u;
    uint32_t wi = wv;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += u;
    }
    s_warp[32 + lane] = wi - wv;
    if (lane == 31) *s_total = wi;
  }
  __syncthreads();
  const uint32_t r = s_warp[32 + warp] + inc - v;
  __syncthreads();
  return r;
}

// Four consecutive keys at positions i..i+3 (missing ones, past n, as 0).
__device__ __forceinline__ void load4(const float* row, int i, int n, bool vec, uint32_t (&k)[4]) {
  if (vec && i + 4 <= n) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(row + i));
    k[0] = monotone32(v.x);
    k[1] = monotone32(v.y);
    k[2] = monotone32(v.z);
    k[3] = monotone32(v.w);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) k[e] = i + e < n ? monotone32(__ldg(row + i + e)) : 0u;
  }
}

// Lower bound: number of entries of the ascending list a[0..m) below x.
__device__ __forceinline__ int count_below(const int32_t* a, int m, int32_t x) {
  int lo = 0, hi = m;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Rows whose threshold bin overflows the candidate buffer: two more radix
// levels and an ordered compaction, all over global memory.
template <int NT>
__device__ void select_global(const float* row, int n, int K, uint32_t T1, uint32_t need2, const Emit& out,
                              TopkSmem& s) {
  const int tid = threadIdx.x;
  for (int i = tid; i < NBIN1; i += NT) s.hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const uint32_t key = monotone32(__ldg(row + i));
    if ((key >> 20) == T1) atomicAdd(&s.hist[(key >> 8) & 0xFFFu], 1u);
  }
  __syncthreads();
  find_threshold<NT>(s.hist, NBIN1, need2, s.warp, &s.T, &s.above);
  const uint32_t pre2 = (T1 << 12) | (uint32_t)s.T;
  const uint32_t need3 = need2 - s.above;
  for (int i = tid; i < 256; i += NT) s.hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const uint32_t key = monotone32(__ldg(row + i));
    if ((key >> 8) == pre2) atomicAdd(&s.hist[key & 0xFFu], 1u);
  }
  __syncthreads();
  find_threshold<NT>(s.hist, 256, need3, s.warp, &s.T, &s.above);
  const uint32_t kth = (pre2 << 8) | (uint32_t)s.T;
  const uint32_t n_ties = need3 - s.above;
  uint32_t out_base = 0, tie_base = 0;
  for (int base = 0; base < n; base += NT) {
    const int i = base + tid;
    const bool in = i < n;
    const uint32_t key = in ? monotone32(__ldg(row + i)) : 0u;
    const bool eq = in && key == kth;
    const uint32_t tie_rank = tie_base + block_exclusive<NT>(eq ? 1u : 0u, s.warp, &s.total);
    const uint32_t n_eq = s.total;
    const bool sel = in && (key > kth || (eq && tie_rank < n_ties));
    const uint32_t pos = out_base + block_exclusive<NT>(sel ? 1u : 0u, s.warp, &s.total);
    if (sel && pos < (uint32_t)K) out((int)pos, i);
    out_base += s.total;
    tie_base += n_eq;
  }
}

// The K-th key among the n_cand candidates of level-1 bin T1 (held in
// position order in s.cand_key / s.cand_pos): two more radix levels (12 + 8
// bits), then the selected candidates (key > kth, or == kth among the first
// such keys) compacted in position order into s.sel. Returns their count.
// With have_hist2, s.hist already holds the candidates' level-2 histogram
// (bits 19..8), built by the caller.
template <int NT>
__device__ uint32_t resolve_candidates(TopkSmem& s, uint32_t n_cand, uint32_t need2, uint32_t T1,
                                       bool have_hist2 = false) {
  const int tid = threadIdx.x;
  if (!have_hist2) {
    for (int i = tid; i < NBIN1; i += NT) s.hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < (int)n_cand; i += NT) atomicAdd(&s.hist[(s.cand_key[i] >> 8) & 0xFFFu], 1u);
    __syncthreads();
  }
  find_threshold<NT>(s.hist, NBIN1, need2, s.warp, &s.T, &s.above);
  const uint32_t T2 = (uint32_t)s.T;
  const uint32_t need3 = need2 - s.above;
  __syncthreads();
  for (int i = tid; i < 256; i += NT) s.hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < (int)n_cand; i += NT) {
    const uint32_t key = s.cand_key[i];
    if (((key >> 8) & 0xFFFu) == T2) atomicAdd(&s.hist[key & 0xFFu], 1u);
  }
  __syncthreads();
  find_threshold<NT>(s.hist, 256, need3, s.warp, &s.T, &s.above);
  const uint32_t kth = (T1 << 20) | (T2 << 8) | (uint32_t)s.T;
  const uint32_t n_ties = need3 - s.above;
  __syncthreads();

  const int per = (int)((n_cand + NT - 1) / NT);
  const int c0 = min((int)n_cand, tid * per), c1 = min((int)n_cand, c0 + per);
  uint32_t my_eq = 0;
  for (int i = c0; i < c1; ++i) my_eq += s.cand_key[i] == kth;
  uint32_t tie = block_exclusive<NT>(my_eq, s.warp, &s.total);
  uint32_t my_sel = 0;
  for (int i = c0; i < c1; ++i) {
    const uint32_t key = s.cand_key[i];
    if (key > kth || (key == kth && tie < n_ties)) ++my_sel;
    tie += key == kth;
  }
  uint32_t sp = block_exclusive<NT>(my_sel, s.warp, &s.total);
  const uint32_t n_sel = min(s.total, (uint32_t)KMAX);
  tie -= my_eq;
  for (int i = c0; i < c1; ++i) {
    const uint32_t key = s.cand_key[i];
    if (key > kth || (key == kth && tie < n_ties)) {
      if (sp < (uint32_t)KMAX) s.sel[sp] = s.cand_pos[i];
      ++sp;
    }
    tie += key == kth;
  }
  __syncthreads();
  return n_sel;
}

template <int NT>
__device__ void topk_row(const TopkParams& p, int b, const Emit& out, TopkSmem& s) {
  constexpr int NWARP = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.K;
  const float* row = out.row;
  const int n = max(0, min(p.lens[b], p.max_kv));

  if (n <= K) {  // everything valid is selected
    for (int i = tid; i < K; i += NT) out(i, i < n ? i : -1);
    if (p.hist_clear)
      for (int i = tid; i < NBIN1; i += NT) p.hist_clear[(int64_t)b * NBIN1 + i] = 0;
    return;
  }
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  // each warp owns a contiguous run of positions, 128 per step (16-byte loads)
  const int run = ((n + NWARP * 128 - 1) / (NWARP * 128)) * 128;
  const int w0 = warp * run, w1 = min(n, w0 + run);

  // ---- 1. level-1 histogram: bits 31..20
  if (p.hist) {
    for (int i = tid; i < NBIN1; i += NT) {
      s.hist[i] = (uint32_t)p.hist[(int64_t)b * NBIN1 + i];
      if (p.hist_clear) p.hist_clear[(int64_t)b * NBIN1 + i] = 0;
    }
  } else {
    for (int i = tid; i < NBIN1; i += NT) s.hist[i] = 0;
    __syncthreads();
    for (int i0 = w0; i0 < w1; i0 += 128 * SWEEP_U) {
      uint32_t kq[SWEEP_U][4];
#pragma unroll
      for (int u = 0; u < SWEEP_U; ++u) load4(row, i0 + 128 * u + 4 * lane, w1, vec, kq[u]);
#pragma unroll
      for (int u = 0; u < SWEEP_U; ++u) {
        const int i = i0 + 128 * u + 4 * lane;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (i + e < w1) atomicAdd(&s.hist[kq[u][e] >> 20], 1u);
      }
    }
  }
  __syncthreads();
  find_threshold<NT>(s.hist, NBIN1, (uint32_t)K, s.warp, &s.T, &s.above);
  const uint32_t T1 = (uint32_t)s.T;
  const uint32_t n_above1 = s.above;
  const uint32_t need2 = (uint32_t)K - n_above1;
  const uint32_t cnt1 = s.hist[T1];
  __syncthreads();
  if (cnt1 > (uint32_t)CAP || n_above1 > (uint32_t)KMAX) {
    select_global<NT>(row, n, K, T1, need2, out, s);
    return;
  }

  // ---- 2. ordered sweep: sure positions (bin > T1) and candidates (bin == T1)
  uint32_t ns = 0, nc = 0;
  for (int i0 = w0; i0 < w1; i0 += 128 * SWEEP_U) {
    uint32_t kq[SWEEP_U][4];
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) load4(row, i0 + 128 * u + 4 * lane, w1, vec, kq[u]);
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) {
      const int i = i0 + 128 * u + 4 * lane;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        const uint32_t bin = kq[u][e] >> 20;
        ns += bin > T1;
        nc += bin == T1;
      }
    }
  }
  // per-warp totals -> warp offsets (sure in the low half, candidates high)
  uint32_t packed = ns | (nc << 16);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) packed += __shfl_xor_sync(0xffffffffu, packed, off);
  if (lane == 0) s.warp_off[warp] = packed;
  __syncthreads();
  if (warp == 0) {
    const uint32_t v = lane < NWARP ? s.warp_off[lane] : 0u;
    uint32_t inc_s = v & 0xFFFFu, inc_c = v >> 16;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t us = __shfl_up_sync(0xffffffffu, inc_s, off);
      const uint32_t uc = __shfl_up_sync(0xffffffffu, inc_c, off);
      if (lane >= off) {
        inc_s += us;
        inc_c += uc;
      }
    }
    if (lane < NWARP) s.warp[lane] = (inc_s - (v & 0xFFFFu)) | ((inc_c - (v >> 16)) << 16);
    if (lane == NWARP - 1) s.total = inc_s | (inc_c << 16);
  }
  __syncthreads();
  uint32_t off_s = s.warp[warp] & 0xFFFFu, off_c = s.warp[warp] >> 16;
  const uint32_t n_sure = min(s.total & 0xFFFFu, (uint32_t)KMAX);
  const uint32_t n_cand = min(s.total >> 16, (uint32_t)CAP);
  // every lane takes the same number of steps (the shuffles below need the
  // whole warp); positions past w1 count as absent
  for (int i0 = w0; i0 < w1; i0 += 128 * SWEEP_U) {
    uint32_t kq[SWEEP_U][4];
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) load4(row, i0 + 128 * u + 4 * lane, w1, vec, kq[u]);
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) {
      const int i = i0 + 128 * u + 4 * lane;
      const uint32_t* k = kq[u];
      uint32_t cs = 0, cc = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        cs += (k[e] >> 20) > T1;
        cc += (k[e] >> 20) == T1;
      }
      uint32_t inc = cs | (cc << 16);
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t up = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += up;
      }
      const uint32_t tot = __shfl_sync(0xffffffffu, inc, 31);
      const uint32_t ex = inc - (cs | (cc << 16));
      uint32_t ps = off_s + (ex & 0xFFFFu), pc = off_c + (ex >> 16);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        const uint32_t bin = k[e] >> 20;
        if (bin > T1) {
          if (ps < (uint32_t)KMAX) s.sure[ps] = i + e;
          ++ps;
        } else if (bin == T1) {
          if (pc < (uint32_t)CAP) {
            s.cand_key[pc] = k[e];
            s.cand_pos[pc] = i + e;
          }
          ++pc;
        }
      }
      off_s += tot & 0xFFFFu;
      off_c += tot >> 16;
    }
  }
  __syncthreads();

  // ---- 3. resolve the low 20 bits among the candidates
  const uint32_t n_sel = resolve_candidates<NT>(s, n_cand, need2, T1);

  // ---- merge the two ascending lists
  for (int i = tid; i < (int)n_sure; i += NT) {
    const int32_t P = s.sure[i];
    const int o = i + count_below(s.sel, (int)n_sel, P);
    if (o < K) out(o, P);
  }
  for (int i = tid; i < (int)n_sel; i += NT) {
    const int32_t P = s.sel[i];
    const int o = i + count_below(s.sure, (int)n_sure, P);
    if (o < K) out(o, P);
  }
  for (int i = (int)(n_sure + n_sel) + tid; i < K; i += NT) out(i, -1);  // only for an inconsistent histogram
}

// Exchange staging: the last CTA of the grid publishes staged = seq (nothing
// once the error word is set). Every CTA orders its payload writes at GPU
// scope before its arrival; the last one, having seen every arrival, orders
// them all at system scope before the release store peers acquire.
__device__ __forceinline__ void publish_staged(const TopkParams& p, int seq, int n_ctas) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence();
  if (atomicAdd(p.ctl + 1, 1) == n_ctas - 1) {
    p.ctl[1] = 0;
    __threadfence_system();
    if (read_err_word(p.err) == 0) st_release_sys_s32(p.my_flags, seq);
  }
}

template <int NT>
__global__ void __launch_bounds__(NT, 1024 / NT) topk_rows_kernel(const TopkParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem& s = *reinterpret_cast<TopkSmem*>(smem_raw);
  const int b = blockIdx.x;
  Emit e{};
  e.row = p.score + (int64_t)b * p.score_stride;
  float* pay = p.pay;
  int seq = 0;
  if (p.ctl) {  // exchange staging into slot seq & 1 (free, see TopkParams)
    seq = *reinterpret_cast<const volatile int*>(p.ctl) + 1;
    pay += (int64_t)(seq & 1) * (p.slot_bytes / 4);
  }
  if (pay) {
    e.val = pay + (int64_t)b * p.pay_stride;
    e.pos = reinterpret_cast<int32_t*>(e.val + p.K);
    e.off = p.pos_off;
  } else {
    e.idx = p.idx + (int64_t)b * p.idx_stride;
  }
  topk_row<NT>(p, b, e, s);
  if (p.ctl) publish_staged(p, seq, (int)gridDim.x);
}

// ---------------------------------------------------------- cluster mode
// Few long rows (decode batches with the logits kernel's histogram): the CL
// CTAs of one thread-block cluster share a row, each owning a contiguous
// CL-th of it, so a batch of 8 rows keeps 64 SMs busy instead of 8.
//   * At entry every CTA starts bulk copies of the row's histogram and of its
//     own range of scores into shared memory (when the range fits STAGE_F
//     floats and the row is 16-byte aligned; else both passes below read
//     global memory), so the scores are read from global memory once, with
//     all of the CTA's loads in flight together.
//   * Every CTA derives the same threshold bin T1 from the histogram; a count
//     pass gives each CTA its sure (bin > T1) and candidate (bin == T1)
//     counts, exchanged through distributed shared memory.
//   * The write pass keeps the sure positions in the CTA's own shared memory
//     and writes the candidates into rank 0's candidate lists at their
//     prefix offsets, in position order, adding each to rank 0's level-2
//     histogram (bits 19..8) with a distributed shared-memory atomic.
//   * Rank 0 resolves the K-th key among the candidates, then pushes to every
//     CTA the selected candidates of its range (and their offset); every CTA
//     then emits its sure and selected positions from its own shared memory.
// Rows whose bin T1 overflows the candidate buffer are done by rank 0 alone
// with the one-CTA path. Every CTA of a cluster takes the same sequence of
// cluster barriers on every path (no CTA waits on a barrier another skips).
constexpr int CL = 8;
constexpr int NT_CL = 512;
constexpr int STAGE_F = 28672;                  // staged scores per CTA (112 KB)
constexpr int STAGE_CHUNK = 4096;               // floats per bulk copy
constexpr int NCHUNK = STAGE_F / STAGE_CHUNK;   // 7
constexpr uint64_t kStageTimeoutNs = 2000000000ull;

struct ClusterStage {
  uint64_t mbar[NCHUNK + 1];  // score chunks, histogram
  int abort;
  int pad[3];
  float sc[STAGE_F];
};
constexpr size_t CLUSTER_SMEM = (sizeof(TopkSmem) + 15) / 16 * 16 + sizeof(ClusterStage);

__device__ __forceinline__ ClusterStage& cluster_stage(unsigned char* smem_raw) {
  return *reinterpret_cast<ClusterStage*>(smem_raw + (sizeof(TopkSmem) + 15) / 16 * 16);
}

template <int NT>
__device__ void topk_row_cluster(const TopkParams& p, int b, const Emit& out, TopkSmem& s, ClusterStage& cs,
                                 cg::cluster_group& cl, int rank) {
  constexpr int NWARP = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.K;
  const float* row = out.row;
  const int n = max(0, min(p.lens[b], p.max_kv));
  if (n <= K) {  // uniform over the cluster: rank 0 emits the row
    if (rank == 0) {
      for (int i = tid; i < K; i += NT) out(i, i < n ? i : -1);
      if (p.hist_clear)
        for (int i = tid; i < NBIN1; i += NT) p.hist_clear[(int64_t)b * NBIN1 + i] = 0;
    }
    return;
  }
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int per = ((n + CL * 128 - 1) / (CL * 128)) * 128;  // positions per CTA, 128-aligned
  const int r0 = min(n, rank * per), r1 = min(n, r0 + per);
  const int r1v = r0 + ((r1 - r0) & ~3);          // staged part [r0, r1v); the tail < 4 from global
  const bool staged = vec && (r1 - r0) <= STAGE_F;  // same for every CTA of the row (n, per, row)
  const int nchunk = staged ? (r1v - r0 + STAGE_CHUNK - 1) / STAGE_CHUNK : 0;

  // ---- bulk copies: histogram row and this CTA's scores
  const uint32_t mb = smem_u32(&cs.mbar[0]);
  if (tid == 0) {
    for (int c = 0; c <= NCHUNK; ++c) tc::mbar_init(mb + 8u * c, 1);
    tc::mbar_init_fence();
    cs.abort = 0;
    tc::mbar_arrive_expect_tx(mb + 8u * NCHUNK, NBIN1 * 4);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(s.hist)),
                 "l"(p.hist + (int64_t)b * NBIN1), "r"((uint32_t)(NBIN1 * 4)), "r"(mb + 8u * NCHUNK)
                 : "memory");
    for (int c = 0; c < nchunk; ++c) {
      const int c0 = r0 + c * STAGE_CHUNK, c1 = min(r1v, c0 + STAGE_CHUNK);
      const uint32_t bytes = (uint32_t)(c1 - c0) * 4u;
      tc::mbar_arrive_expect_tx(mb + 8u * c, bytes);
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       smem_u32(cs.sc + (c0 - r0))),
                   "l"(row + c0), "r"(bytes), "r"(mb + 8u * c)
                   : "memory");
    }
  }
  __syncthreads();  // barriers initialised before anyone waits on them
  bool ok = tc::mbar_wait(mb + 8u * NCHUNK, 0, &cs.abort, p.dev_err, kStageTimeoutNs);
  find_threshold<NT>(s.hist, NBIN1, (uint32_t)K, s.warp, &s.T, &s.above);
  const uint32_t T1 = (uint32_t)s.T;
  const uint32_t need2 = (uint32_t)K - s.above;
  const uint32_t cnt1 = s.hist[T1];
  const bool overflow = cnt1 > (uint32_t)CAP || s.above > (uint32_t)KMAX;
  for (int c = 0; c < nchunk; ++c) ok = tc::mbar_wait(mb + 8u * c, 0, &cs.abort, p.dev_err, kStageTimeoutNs) && ok;
  __syncthreads();
  if (rank == 0 && !overflow)  // rank 0's histogram becomes the candidates' level-2 histogram
    for (int i = tid; i < NBIN1; i += NT) s.hist[i] = 0;
  const int run = ((r1 - r0 + NWARP * 128 - 1) / (NWARP * 128)) * 128;
  const int w0 = r0 + warp * run, w1 = min(r1, w0 + run);
  // four keys at positions i..i+3 of this CTA's range (staged or global)
  auto keys4 = [&](int i, uint32_t (&k)[4]) {
    if (staged && i + 4 <= r1v) {
      const float4 v = *reinterpret_cast<const float4*>(cs.sc + (i - r0));
      k[0] = monotone32(v.x);
      k[1] = monotone32(v.y);
      k[2] = monotone32(v.z);
      k[3] = monotone32(v.w);
    } else {
      load4(row, i, w1, vec, k);
    }
  };

  // count pass
  uint32_t ns = 0, nc = 0;
  for (int i0 = w0; i0 < w1; i0 += 128 * SWEEP_U) {
    uint32_t kq[SWEEP_U][4];
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) keys4(i0 + 128 * u + 4 * lane, kq[u]);
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) {
      const int i = i0 + 128 * u + 4 * lane;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        const uint32_t bin = kq[u][e] >> 20;
        ns += bin > T1;
        nc += bin == T1;
      }
    }
  }
  uint32_t packed = ns | (nc << 16);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) packed += __shfl_xor_sync(0xffffffffu, packed, off);
  if (lane == 0) s.warp_off[warp] = packed;
  const int cta_ok = __syncthreads_and(ok ? 1 : 0);
  if (warp == 0) {
    const uint32_t v = lane < NWARP ? s.warp_off[lane] : 0u;
    uint32_t inc_s = v & 0xFFFFu, inc_c = v >> 16;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t us = __shfl_up_sync(0xffffffffu, inc_s, off);
      const uint32_t uc = __shfl_up_sync(0xffffffffu, inc_c, off);
      if (lane >= off) {
        inc_s += us;
        inc_c += uc;
      }
    }
    if (lane < NWARP) s.warp[lane] = (inc_s - (v & 0xFFFFu)) | ((inc_c - (v >> 16)) << 16);
    if (lane == NWARP - 1) {
      const uint32_t tot = inc_s | (inc_c << 16);
      for (int r = 0; r < CL; ++r) {
        *cl.map_shared_rank(&s.cl_cnt[rank], r) = tot;
        *cl.map_shared_rank(&s.cl_ok[rank], r) = cta_ok;
      }
    }
  }
  cl.sync();  // counts and staging verdicts exchanged; every CTA has read the histogram
  // From here every branch is uniform over the cluster: the verdicts are the
  // same everywhere, and with every copy complete so is the histogram.
  bool row_ok = true;
#pragma unroll
  for (int r = 0; r < CL; ++r) row_ok = row_ok && s.cl_ok[r] != 0;
  if (!row_ok) {  // a staging wait expired (recorded in the status word): nothing is emitted
    if (tid == 0 && !ok)  // this CTA's copies may still be in flight: drain them (bounded) first
      for (int c = 0; c <= NCHUNK; ++c)
        if (c < nchunk || c == NCHUNK) tc::mbar_wait_drain(mb + 8u * c, 0, kStageTimeoutNs);
    __syncthreads();
    return;
  }
  if (overflow) {       // rank 0 alone, from global memory (it reads the histogram, then clears it)
    if (rank == 0) topk_row<NT>(p, b, out, s);
    return;
  }
  if (rank == 0 && p.hist_clear)
    for (int i = tid; i < NBIN1; i += NT) p.hist_clear[(int64_t)b * NBIN1 + i] = 0;
  uint32_t sure_base = 0, cand_base = 0, n_cand = 0;
#pragma unroll
  for (int r = 0; r < CL; ++r) {
    const uint32_t c = s.cl_cnt[r];
    if (r < rank) {
      sure_base += c & 0xFFFFu;
      cand_base += c >> 16;
    }
    n_cand += c >> 16;
  }
  const uint32_t my_sure = s.cl_cnt[rank] & 0xFFFFu;
  n_cand = min(n_cand, (uint32_t)CAP);
  uint32_t* key0 = cl.map_shared_rank(s.cand_key, 0);
  int32_t* pos0 = cl.map_shared_rank(s.cand_pos, 0);
  uint32_t* hist0 = cl.map_shared_rank(s.hist, 0);

  // write pass: sure positions here, candidates into rank 0, in order
  uint32_t off_s = s.warp[warp] & 0xFFFFu, off_c = cand_base + (s.warp[warp] >> 16);
  for (int i0 = w0; i0 < w1; i0 += 128 * SWEEP_U) {
    uint32_t kq[SWEEP_U][4];
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) keys4(i0 + 128 * u + 4 * lane, kq[u]);
#pragma unroll
    for (int u = 0; u < SWEEP_U; ++u) {
      const int i = i0 + 128 * u + 4 * lane;
      const uint32_t* k = kq[u];
      uint32_t cs4 = 0, cc = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        cs4 += (k[e] >> 20) > T1;
        cc += (k[e] >> 20) == T1;
      }
      uint32_t inc = cs4 | (cc << 16);
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t up = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += up;
      }
      const uint32_t tot = __shfl_sync(0xffffffffu, inc, 31);
      const uint32_t ex = inc - (cs4 | (cc << 16));
      uint32_t ps = off_s + (ex & 0xFFFFu), pc = off_c + (ex >> 16);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (i + e >= w1) continue;
        const uint32_t bin = k[e] >> 20;
        if (bin > T1) {
          if (ps < (uint32_t)KMAX) s.sure[ps] = i + e;
          ++ps;
        } else if (bin == T1) {
          if (pc < (uint32_t)CAP) {
            key0[pc] = k[e];
            pos0[pc] = i + e;
            atomicAdd(hist0 + ((k[e] >> 8) & 0xFFFu), 1u);
          }
          ++pc;
        }
      }
      off_s += tot & 0xFFFFu;
      off_c += tot >> 16;
    }
  }
  cl.sync();  // all candidates and the level-2 histogram have landed in rank 0
  if (rank == 0) {
    const uint32_t n_sel = resolve_candidates<NT>(s, n_cand, need2, T1, true);
    // push every CTA its selected candidates (ascending) and their offset
    for (int q = warp; q < CL; q += NWARP) {
      const int q0 = min(n, q * per), q1 = min(n, q0 + per);
      const int lo = count_below(s.sel, (int)n_sel, q0), hi = count_below(s.sel, (int)n_sel, q1);
      TopkSmem* d = cl.map_shared_rank(&s, q);
      for (int j = lane; j < hi - lo; j += 32) d->cand_pos[j] = s.sel[lo + j];
      if (lane == 0) {
        d->cl_lo = (uint32_t)lo;
        d->cl_nsel = (uint32_t)(hi - lo);
        d->cl_total = n_sel;
      }
    }
  }
  cl.sync();  // every CTA holds its selected candidates; no shared memory of another CTA is used after this
  const int lo = (int)s.cl_lo, nm = (int)s.cl_nsel;
  const int32_t* mine = s.cand_pos;
  const int n_my_sure = (int)min(my_sure, (uint32_t)KMAX);
  for (int i = tid; i < n_my_sure; i += NT) {
    const int32_t P = s.sure[i];
    const int o = (int)sure_base + i + lo + count_below(mine, nm, P);
    if (o < K) out(o, P);
  }
  for (int j = tid; j < nm; j += NT) {
    const int32_t P = mine[j];
    const int o = (int)sure_base + lo + j + count_below(s.sure, n_my_sure, P);
    if (o < K) out(o, P);
  }
  if (rank == CL - 1) {  // only for an inconsistent histogram: pad the tail
    int total = (int)s.cl_total;
    for (int r = 0; r < CL; ++r) total += (int)(s.cl_cnt[r] & 0xFFFFu);
    for (int i = total + tid; i < K; i += NT) out(i, -1);
  }
}

__global__ void __launch_bounds__(NT_CL, 1) topk_cluster_kernel(const TopkParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopkSmem& s = *reinterpret_cast<TopkSmem*>(smem_raw);
  ClusterStage& cs = cluster_stage(smem_raw);
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int b = blockIdx.y;
  Emit e{};
  e.row = p.score + (int64_t)b * p.score_stride;
  float* pay = p.pay;
  int seq = 0;
  if (p.ctl) {  // exchange staging into slot seq & 1 (free, see TopkParams)
    seq = *reinterpret_cast<const volatile int*>(p.ctl) + 1;
    pay += (int64_t)(seq & 1) * (p.slot_bytes / 4);
  }
  if (pay) {
    e.val = pay + (int64_t)b * p.pay_stride;
    e.pos = reinterpret_cast<int32_t*>(e.val + p.K);
    e.off = p.pos_off;
  } else {
    e.idx = p.idx + (int64_t)b * p.idx_stride;
  }
  topk_row_cluster<NT_CL>(p, b, e, s, cs, cl, rank);
  if (p.ctl) publish_staged(p, seq, (int)(gridDim.x * gridDim.y));
}

std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];
int g_cluster_ok[kMaxDevices];  // clusters of CL topk CTAs can be resident

int run_topk(const TopkParams& p, int B, cudaStream_t s) {
  DSA_REQUIRE(B >= 0 && p.max_kv >= 0, DSA_ERR_INVALID, "topk: negative size");
  DSA_REQUIRE(p.K >= 1 && p.K <= KMAX, DSA_ERR_UNSUPPORTED, "topk: K must be in [1, %d] (got %d)", KMAX, p.K);
  if (B == 0) return DSA_OK;
  DSA_REQUIRE((p.idx || p.pay) && p.lens && (p.score || p.max_kv == 0), DSA_ERR_INVALID, "topk: null pointer");
  DSA_REQUIRE((p.pay ? p.pay_stride >= 2 * (int64_t)p.K : p.idx_stride >= p.K) && p.score_stride >= p.max_kv,
              DSA_ERR_INVALID, "topk: row stride smaller than the row");
  const int dev = current_device();
  DSA_REQUIRE(dev >= 0 && dev < kMaxDevices, DSA_ERR_UNSUPPORTED, "topk: device %d out of range", dev);
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(topk_rows_kernel<NT_SMALL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(TopkSmem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(topk_rows_kernel<NT_LARGE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(TopkSmem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(topk_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)CLUSTER_SMEM);
    g_status[dev] = (int)e;
    if (e == cudaSuccess) {  // can clusters of CL such CTAs be resident at all?
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(CL, 1, 1);
      cfg.blockDim = dim3(NT_CL);
      cfg.dynamicSmemBytes = CLUSTER_SMEM;
      cudaLaunchAttribute attr{};
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = CL;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, topk_cluster_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        nc = 0;
      }
      g_cluster_ok[dev] = nc > 0;
    }
  });
  if (g_status[dev] != 0) {
    set_error("cudaFuncSetAttribute(topk): %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  // few long rows with the logits kernel's histogram: a cluster of CL CTAs per row
  if (p.hist && (reinterpret_cast<uintptr_t>(p.hist) & 15) == 0 && g_cluster_ok[dev] && B < sm_count(dev) &&
      p.max_kv >= CL * 1024 && p.K <= KMAX) {
    TopkParams q = p;
    const int st = tc_error_word(dev, &q.dev_err);
    if (st != DSA_OK) return st;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(CL, B, 1);
    cfg.blockDim = dim3(NT_CL);
    cfg.dynamicSmemBytes = CLUSTER_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = CL;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_cluster_kernel, q);
    if (e != cudaSuccess) {
      set_error("topk_cluster_kernel launch: %s", cudaGetErrorString(e));
      return DSA_ERR_CUDA;
    }
    return DSA_OK;
  }
  if (2 * B < sm_count(dev))
    topk_rows_kernel<NT_LARGE><<<B, NT_LARGE, sizeof(TopkSmem), s>>>(p);
  else
    topk_rows_kernel<NT_SMALL><<<B, NT_SMALL, sizeof(TopkSmem), s>>>(p);
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

extern "C" int dsa_topk_rows_payload(float* pay, int64_t pay_stride, const float* score, int64_t score_stride,
                                     int max_kv, const int32_t* lens, int32_t* hist, int B, int K, int pos_off,
                                     void* stream) {
  clear_error();
  TopkParams p{};
  p.score = score;
  p.lens = lens;
  p.hist = hist;
  p.hist_clear = hist;
  p.score_stride = score_stride;
  p.max_kv = max_kv;
  p.K = K;
  p.pay = pay;
  p.pay_stride = pay_stride;
  p.pos_off = pos_off;
  return run_topk(p, B, as_stream(stream));
}

extern "C" int dsa_shard_exchange_topk(const float* score, int64_t score_stride, int max_kv, const int32_t* lens,
                                       int32_t* hist, int B, int K, int pos_off, void* slot_base,
                                       int64_t slot_bytes, const uint64_t* flag_ptrs, int tp, int rank,
                                       int32_t* ctl, int64_t timeout_ns, int32_t* err_flag, void* stream) {
  clear_error();
  DSA_REQUIRE(tp >= 1 && tp <= MAX_TP && rank >= 0 && rank < tp, DSA_ERR_UNSUPPORTED,
              "shard_exchange_topk: tp must be in [1, %d] and rank < tp", MAX_TP);
  DSA_REQUIRE(K >= 1 && K <= 2048, DSA_ERR_UNSUPPORTED, "shard_exchange_topk: K must be in [1, 2048]");
  DSA_REQUIRE(B >= 1 && slot_base && flag_ptrs && ctl && err_flag && timeout_ns > 0 &&
                  slot_bytes >= (int64_t)B * 2 * K * 4 && slot_bytes % 16 == 0,
              DSA_ERR_INVALID, "shard_exchange_topk: bad arguments");
  TopkParams p{};
  p.score = score;
  p.lens = lens;
  p.hist = hist;
  p.hist_clear = hist;
  p.score_stride = score_stride;
  p.max_kv = max_kv;
  p.K = K;
  p.pay = reinterpret_cast<float*>(slot_base);
  p.pay_stride = 2 * (int64_t)K;
  p.pos_off = pos_off;
  p.ctl = ctl;
  p.tp = tp;
  p.slot_bytes = slot_bytes;
  p.timeout_ns = timeout_ns;
  p.err = err_flag;
  for (int s = 0; s < tp; ++s)
    DSA_REQUIRE(flag_ptrs[s] != 0, DSA_ERR_INVALID, "shard_exchange_topk: null flag pointer %d", s);
  p.my_flags = reinterpret_cast<int*>(flag_ptrs[rank]);
  return run_topk(p, B, as_stream(stream));
}
