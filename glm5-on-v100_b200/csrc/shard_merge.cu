// Exact merge of key-sharded indexer top-k candidates (local buffers or peer
// memory) and the CUDA IPC helpers of the P2P shard exchange.
//
// Replaces sm70_indexer_shard_merge / sm70_indexer_shard_merge_p2p and the
// IPC helpers (csrc/attention/sm70_mla_decode.cu:2184-2434) and the torch.topk
// epilogue they fuse (reference/sparse_attn_indexer.py:1007-1030). The
// selection contract is the reference's: candidate column col = s*K + c is
// ordered by (float value, then lower column first), so the result equals
// torch.topk over the [R, tp*K] layout; -inf picks emit -1; the K positions
// are written ascending with the -1s first.
//
// Design (one 512-thread CTA per row, thread t owns columns c = 4t..4t+3 of
// every shard, loaded as one 16-byte vector per shard):
//   1. Values become 32-bit order-preserving keys. Keys at or below the -inf
//      key all emit -1, so only the "high" keys are ranked; when there are at
//      most K of them they are all taken.
//   2. Otherwise a radix select over the high keys finds the K-th largest
//      key. Its digits are 11 bits wide and start at the highest bit in which
//      the block's min and max high keys differ, so real score distributions
//      spread over the first pass's 2048 bins instead of piling into a few;
//      each further pass only sees the keys of the chosen bin, and the walk
//      stops as soon as a whole bin is taken.
//   3. Keys equal to the K-th key are ranked in column order with one
//      block-wide scan of per-shard counts packed 16 bits per shard, so the
//      lower-column rule costs O(candidates), whatever the number of ties.
//   4. The selected positions are compacted per shard, in column order, into
//      shared memory. When every shard's run is ascending (always so for lists
//      the top-k kernels write), the output rank of a position is its index in
//      its run plus, per other run, a count found from the run's first/last
//      entries (disjoint key shards) or a binary search. When a run is not
//      ascending, all selected positions are sorted instead (a bitonic
//      network over 2048 entries, mostly in registers and shuffles).
// The P2P variant checks the error word once, waits (bounded) on every peer's
// staged flag with acquire loads, and then reads the peers' slots with
// relaxed system-scope loads (plain peer loads; no TMA, no multicast).
#include <climits>

#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dsa {
namespace {

constexpr int MT = 512;               // threads per row
constexpr int NW = MT / 32;
constexpr int PER = 4;                // columns per thread per shard
constexpr int MAX_TP = 8;
constexpr int MAX_K = MT * PER;       // 2048
constexpr int DIGIT = 11;
constexpr int NBIN = 1 << DIGIT;      // 2048
constexpr uint32_t NEG_KEY = 0x007FFFFFu;  // monotone32(-inf); keys <= it emit -1

struct MergeArgs {
  const uint8_t* base[MAX_TP];  // shard s, row 0 of the slab, before slot_off
  const int* staged[MAX_TP];    // P2P: &flags_s[0]
  int32_t* out;
  const int32_t* dst_rows;
  int32_t* err;                 // P2P: error word (DSA_ERR_TIMEOUT on an expired wait)
  int* ctl;                     // exchange mode: [0] last completed seq, [2] CTA done counter
  int* my_flags;                // exchange mode: this rank's {staged, merged}
  int64_t out_stride;
  int64_t shard_stride;         // bytes between shards (local [tp, R, 2K] layout)
  int64_t slot_off;             // bytes added to every base (P2P slot)
  int64_t slot_bytes;           // exchange mode: slot (seq & 1) starts at base + (seq & 1) * slot_bytes
  int64_t timeout_ns;
  int R, tp, K, dst_base, seq;
  int p2p, vec;
};

struct MergeSmem {
  uint32_t hist[NBIN];
  int32_t pos[MAX_K];
  uint32_t red[3][NW];
  unsigned long long scan[2][NW];
  int seg[MAX_TP + 1];          // run s of pos[] is [seg[s], seg[s+1])
  uint32_t bin, above, cnt;
  int ok;
};

__device__ __forceinline__ float4 ld_sys_f4(const float* p) {
  float4 v;
  asm volatile("ld.relaxed.sys.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ float ld_sys_f32(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// 16-bit field s of a pair of packed per-shard counters.
__device__ __forceinline__ uint32_t field(unsigned long long lo, unsigned long long hi, int s) {
  return (uint32_t)(((s < 4 ? lo : hi) >> (16 * (s & 3))) & 0xFFFFull);
}

// Block-wide exclusive scan of two packed 64-bit counters in thread order;
// the block totals are returned through tot_lo / tot_hi.
__device__ __forceinline__ void scan_packed(unsigned long long& lo, unsigned long long& hi,
                                            unsigned long long& tot_lo, unsigned long long& tot_hi,
                                            MergeSmem& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long il = lo, ih = hi;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const unsigned long long ul = __shfl_up_sync(0xffffffffu, il, d);
    const unsigned long long uh = __shfl_up_sync(0xffffffffu, ih, d);
    if (lane >= d) {
      il += ul;
      ih += uh;
    }
  }
  if (lane == 31) {
    s.scan[0][warp] = il;
    s.scan[1][warp] = ih;
  }
  __syncthreads();
  unsigned long long pl = 0, ph = 0, tl = 0, th = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const unsigned long long a = s.scan[0][w], b = s.scan[1][w];
    if (w < warp) {
      pl += a;
      ph += b;
    }
    tl += a;
    th += b;
  }
  __syncthreads();
  lo = pl + il - lo;
  hi = ph + ih - hi;
  tot_lo = tl;
  tot_hi = th;
}

// The bin of the K-th largest key: with bins counted in s.hist[0..nbins),
// the largest bin b with count(bins >= b) >= need. Thread t owns bins
// [4t, 4t + 4). Leaves b, count(bins > b) and count(b) in s.bin/above/cnt.
__device__ __forceinline__ void pick_bin(int nbins, uint32_t need, MergeSmem& s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t h[4], c = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = 4 * tid + j;
    h[j] = b < nbins ? s.hist[b] : 0u;
    c += h[j];
  }
  uint32_t suf = c;  // inclusive suffix over the lanes of this warp
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t v = __shfl_down_sync(0xffffffffu, suf, d);
    if (lane + d < 32) suf += v;
  }
  if (lane == 0) s.red[0][warp] = suf;
  __syncthreads();
  uint32_t later = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w)
    if (w > warp) later += s.red[0][w];
  suf += later;
  uint32_t above = suf - c;
  if (above < need && suf >= need) {
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      if (above + h[j] >= need) {
        s.bin = 4 * tid + j;
        s.above = above;
        s.cnt = h[j];
        break;
      }
      above += h[j];
    }
  }
  __syncthreads();
}

// Number of entries of the ascending run a[0..n) that are < x (strict) or
// <= x (!strict).
__device__ __forceinline__ int count_run(const int32_t* a, int n, int32_t x, bool strict) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    const bool left = strict ? a[mid] < x : a[mid] <= x;
    if (left)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Ascending sort of a[0, n), n <= MAX_K = 4 * MT, in shared memory, by the MT
// threads of the block: a bitonic network over MAX_K entries (the padding is
// INT_MAX) with thread t holding entries 4t..4t+3 in registers. Partners at
// distance 1 or 2 are in the same thread, up to 64 in the same warp
// (shuffles); only the ten steps at distance >= 128 go through shared memory.
// Used when a shard's positions do not arrive ascending (the output lists
// positions in order; equal positions are the same value, so their relative
// order does not show).
__device__ __noinline__ void sort_positions(int32_t* a, int n) {
  static_assert(MAX_K == 4 * MT, "four entries per thread");
  const int t = threadIdx.x;
  int32_t v[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = 4 * t + e < n ? a[4 * t + e] : INT_MAX;
  __syncthreads();  // every entry is in registers before shared memory is reused
  for (int k = 2; k <= MAX_K; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      int32_t w[4];  // the partners' values
      if (j >= 128) {
#pragma unroll
        for (int e = 0; e < 4; ++e) a[4 * t + e] = v[e];
        __syncthreads();
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = a[(4 * t + e) ^ j];
        __syncthreads();
      } else if (j >= 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = __shfl_xor_sync(0xffffffffu, v[e], j >> 2);
      } else if (j == 2) {
        w[0] = v[2];
        w[1] = v[3];
        w[2] = v[0];
        w[3] = v[1];
      } else {
        w[0] = v[1];
        w[1] = v[0];
        w[2] = v[3];
        w[3] = v[2];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * t + e;
        const bool keep_min = ((i & j) == 0) == ((i & k) == 0);
        v[e] = keep_min ? min(v[e], w[e]) : max(v[e], w[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (4 * t + e < n) a[4 * t + e] = v[e];
  __syncthreads();
}

__device__ void merge_row(const MergeArgs& a, int r, int64_t soff, MergeSmem& s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.K, tp = a.tp;
  const int c0 = tid * PER;
  const int64_t row_off = (int64_t)r * 2 * K;  // floats

  // ---- 1. keys of this thread's columns
  uint32_t key[MAX_TP][PER];
  uint32_t vmask = 0;  // bit 4*s + e: column exists
#pragma unroll
  for (int sh = 0; sh < MAX_TP; ++sh) {
#pragma unroll
    for (int e = 0; e < PER; ++e) key[sh][e] = 0;
    if (sh < tp && c0 < K) {
      const float* v = reinterpret_cast<const float*>(a.base[sh] + soff + (int64_t)sh * a.shard_stride) + row_off + c0;
      float f[PER];
      if (a.vec) {
        const float4 q = a.p2p ? ld_sys_f4(v) : __ldg(reinterpret_cast<const float4*>(v));
        f[0] = q.x;
        f[1] = q.y;
        f[2] = q.z;
        f[3] = q.w;
      } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) f[e] = c0 + e < K ? (a.p2p ? ld_sys_f32(v + e) : __ldg(v + e)) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        if (c0 + e < K) {
          key[sh][e] = monotone32(f[e]);
          vmask |= 1u << (PER * sh + e);
        }
      }
    }
  }

  // ---- 2. high keys: count, min, max
  uint32_t nh = 0, kmin = 0xFFFFFFFFu, kmax = 0;
#pragma unroll
  for (int sh = 0; sh < MAX_TP; ++sh)
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if ((vmask >> (PER * sh + e)) & 1u) {
        const uint32_t k = key[sh][e];
        if (k > NEG_KEY) {
          ++nh;
          kmin = min(kmin, k);
          kmax = max(kmax, k);
        }
      }
  nh = __reduce_add_sync(0xffffffffu, nh);
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    s.red[0][warp] = nh;
    s.red[1][warp] = kmin;
    s.red[2][warp] = kmax;
  }
  __syncthreads();
  nh = 0;
  kmin = 0xFFFFFFFFu;
  kmax = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    nh += s.red[0][w];
    kmin = min(kmin, s.red[1][w]);
    kmax = max(kmax, s.red[2][w]);
  }
  __syncthreads();

  // ---- 3. the selection rule: key >= thr, or (tie) key > thr plus the
  // first need_eq keys == thr in column order
  uint32_t thr = NEG_KEY + 1;
  uint32_t need_eq = 0;
  bool tie = false;
  int n_neg = 0;
  if (nh <= (uint32_t)K) {
    n_neg = K - (int)nh;
  } else {
    uint32_t base = kmin, need = (uint32_t)K;
    const uint32_t span = kmax - kmin;
    int bits = span ? 32 - __clz(span) : 0;
    bool first = true;
    while (true) {
      if (bits == 0) {  // every remaining key equals base
        thr = base;
        need_eq = need;
        tie = true;
        break;
      }
      const int shift = max(bits - DIGIT, 0);
      const int nbins = 1 << (bits - shift);
      for (int i = tid; i < nbins; i += MT) s.hist[i] = 0;
      __syncthreads();
#pragma unroll
      for (int sh = 0; sh < MAX_TP; ++sh)
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const uint32_t k = key[sh][e];
          if (!((vmask >> (PER * sh + e)) & 1u) || k <= NEG_KEY || k < base) continue;
          const uint32_t d = k - base;
          if (!first && (d >> bits) != 0) continue;
          atomicAdd(&s.hist[d >> shift], 1u);
        }
      __syncthreads();
      pick_bin(nbins, need, s);
      const uint32_t b = s.bin, above = s.above, cnt = s.cnt;
      __syncthreads();
      need -= above;
      base += b << shift;
      bits = shift;
      first = false;
      if (cnt == need) {  // the whole bin is taken: every key >= base
        thr = base;
        break;
      }
    }
  }

  // ---- 4. which columns are selected (ties ranked in column order)
  uint32_t selm = 0;  // bit 4*s + e
  if (tie) {
    unsigned long long lo = 0, hi = 0;
#pragma unroll
    for (int sh = 0; sh < MAX_TP; ++sh) {
      uint32_t c = 0;
#pragma unroll
      for (int e = 0; e < PER; ++e) c += ((vmask >> (PER * sh + e)) & 1u) && key[sh][e] == thr;
      if (sh < 4)
        lo += (unsigned long long)c << (16 * sh);
      else
        hi += (unsigned long long)c << (16 * (sh - 4));
    }
    unsigned long long tl, th;
    scan_packed(lo, hi, tl, th, s);
    uint32_t before = 0;  // ties of the shards before this one
#pragma unroll
    for (int sh = 0; sh < MAX_TP; ++sh) {
      uint32_t rank = before + field(lo, hi, sh);
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        if (!((vmask >> (PER * sh + e)) & 1u)) continue;
        const uint32_t k = key[sh][e];
        if (k > thr) {
          selm |= 1u << (PER * sh + e);
        } else if (k == thr) {
          if (rank < need_eq) selm |= 1u << (PER * sh + e);
          ++rank;
        }
      }
      before += field(tl, th, sh);
    }
  } else {
#pragma unroll
    for (int sh = 0; sh < MAX_TP; ++sh)
#pragma unroll
      for (int e = 0; e < PER; ++e)
        if (((vmask >> (PER * sh + e)) & 1u) && key[sh][e] >= thr && key[sh][e] > NEG_KEY)
          selm |= 1u << (PER * sh + e);
  }

  // ---- 5. compact the selected positions per shard, in column order
  {
    unsigned long long lo = 0, hi = 0;
#pragma unroll
    for (int sh = 0; sh < MAX_TP; ++sh) {
      const uint32_t c = __popc((selm >> (PER * sh)) & 0xFu);
      if (sh < 4)
        lo += (unsigned long long)c << (16 * sh);
      else
        hi += (unsigned long long)c << (16 * (sh - 4));
    }
    unsigned long long tl, th;
    scan_packed(lo, hi, tl, th, s);
    if (tid == 0) {
      int acc = 0;
      for (int sh = 0; sh < MAX_TP; ++sh) {
        s.seg[sh] = acc;
        acc += sh < tp ? (int)field(tl, th, sh) : 0;
      }
      s.seg[MAX_TP] = acc;
    }
    uint32_t run0 = 0;
#pragma unroll
    for (int sh = 0; sh < MAX_TP; ++sh) {
      const uint32_t m = (selm >> (PER * sh)) & 0xFu;
      if (m) {
        const float* pv =
            reinterpret_cast<const float*>(a.base[sh] + soff + (int64_t)sh * a.shard_stride) + row_off + K + c0;
        int32_t pp[PER];
        if (a.vec) {
          const float4 q = a.p2p ? ld_sys_f4(pv) : __ldg(reinterpret_cast<const float4*>(pv));
          pp[0] = __float_as_int(q.x);
          pp[1] = __float_as_int(q.y);
          pp[2] = __float_as_int(q.z);
          pp[3] = __float_as_int(q.w);
        } else {
#pragma unroll
          for (int e = 0; e < PER; ++e)
            pp[e] = ((m >> e) & 1u) ? __float_as_int(a.p2p ? ld_sys_f32(pv + e) : __ldg(pv + e)) : 0;
        }
        uint32_t slot = run0 + field(lo, hi, sh);
#pragma unroll
        for (int e = 0; e < PER; ++e)
          if ((m >> e) & 1u) {
            if (slot < (uint32_t)MAX_K) s.pos[slot] = pp[e];
            ++slot;
          }
      }
      run0 += field(tl, th, sh);
    }
  }
  __syncthreads();

  // ---- 6. ascending output: -1s first, then the merged runs
  const int n_sel = min(s.seg[MAX_TP], K - n_neg);  // == K - n_neg by construction
  int32_t* out = a.out + (a.dst_base >= 0 ? (int64_t)a.dst_base + r : (int64_t)a.dst_rows[r]) * a.out_stride;
  for (int i = tid; i < n_neg; i += MT) out[i] = -1;
  bool unsorted = false;
  for (int i = tid; i + 1 < n_sel; i += MT) {
    int sh = 0;
    while (s.seg[sh + 1] <= i) ++sh;
    if (i + 1 < s.seg[sh + 1] && s.pos[i] > s.pos[i + 1]) unsorted = true;
  }
  if (!__syncthreads_or(unsorted)) {
    for (int i = tid; i < n_sel; i += MT) {
      const int32_t p = s.pos[i];
      int own = 0;
      while (s.seg[own + 1] <= i) ++own;
      int rank = i - s.seg[own];
      for (int sh = 0; sh < tp; ++sh) {
        const int lo = s.seg[sh], n = s.seg[sh + 1] - lo;
        if (sh == own || n == 0) continue;
        const bool strict = sh > own;  // equal positions: the lower shard goes first
        const int32_t f = s.pos[lo], l = s.pos[lo + n - 1];
        if (strict ? l < p : l <= p)
          rank += n;
        else if (strict ? f < p : f <= p)
          rank += count_run(s.pos + lo, n, p, strict);
      }
      out[n_neg + rank] = p;
    }
  } else {
    // a run out of order: sort all selected positions
    sort_positions(s.pos, n_sel);
    for (int i = tid; i < n_sel; i += MT) out[n_neg + i] = s.pos[i];
  }
}

// Exchange mode: the last CTA to finish publishes merged = seq and advances
// the rank's sequence counter (every CTA arrives, even after an error). Each
// CTA orders its work at GPU scope before its arrival; the last one orders
// them all at system scope before the release store.
__device__ void finish_exchange(const MergeArgs& a, int seq) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence();
  if (atomicAdd(a.ctl + 2, 1) == (int)(gridDim.x * gridDim.y) - 1) {
    a.ctl[2] = 0;
    __threadfence_system();
    if (read_err_word(a.err) == 0) st_release_sys_s32(a.my_flags + 1, seq);
    a.ctl[0] = seq;
  }
}

__global__ void __launch_bounds__(MT, 2) shard_merge_kernel(const MergeArgs a) {
  __shared__ MergeSmem s;
  const int r = blockIdx.x;
  int seq = a.seq;
  int64_t soff = a.slot_off;
  if (a.ctl) {
    seq = *reinterpret_cast<const volatile int*>(a.ctl) + 1;
    soff = (int64_t)(seq & 1) * a.slot_bytes;
  }
  bool ok = true;
  if (a.p2p) {
    if (threadIdx.x == 0) s.ok = read_err_word(a.err) == 0;
    __syncthreads();
    if (s.ok && (int)threadIdx.x < a.tp && !wait_flag_geq(a.staged[threadIdx.x], seq, a.timeout_ns, a.err)) s.ok = 0;
    __syncthreads();
    ok = s.ok != 0;
  }
  if (ok && r < a.R) merge_row(a, r, soff, s);
  if (a.ctl) finish_exchange(a, seq);
}

// ---------------------------------------------------------- cluster mode
// Few rows (a decode batch): the tp CTAs of one thread-block cluster share a
// row, CTA s owning shard s's K candidates (its peer's slot in P2P mode), so
// 8 rows x 8 shards keep 64 SMs busy instead of 8. The same steps as
// merge_row, with the block-wide reductions made cluster-wide through
// distributed shared memory:
//   * every CTA publishes (high count, min, max) to all CTAs;
//   * a radix pass: local histogram, flushed into rank 0's (DSMEM atomics);
//     rank 0 picks the bin and writes it to every CTA; two cluster barriers;
//   * tie counts, run lengths and run bounds are exchanged per shard, which
//     is also column order;
//   * each CTA ranks the positions of its own run against the other runs
//     (bounds first, a binary search over DSMEM otherwise) and writes them;
//     runs that are not ascending are gathered into rank 0, which sorts
//     them all.
struct ClusterMergeSmem {
  uint32_t hist[NBIN];
  int32_t pos[MAX_K];        // this CTA's run; rank 0: all runs in the unsorted fallback
  uint32_t red[3][NW];
  unsigned long long scan[2][NW];
  uint32_t x_nh[MAX_TP], x_min[MAX_TP], x_max[MAX_TP];  // per-CTA values, published to all
  uint32_t x_eq[MAX_TP], x_len[MAX_TP];
  int32_t x_first[MAX_TP], x_last[MAX_TP];
  int x_sorted[MAX_TP], x_ok[MAX_TP];
  uint32_t bin, above, cnt;  // rank 0 -> all: the chosen bin of a pass
  uint32_t total;
};

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint32_t t = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) t += red[w];
  __syncthreads();
  return t;
}

// Block-wide exclusive prefix of v in thread order (one counter).
__device__ __forceinline__ uint32_t block_excl_u32(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += u;
  }
  if (lane == 31) red[warp] = inc;
  __syncthreads();
  uint32_t pre = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w)
    if (w < warp) pre += red[w];
  __syncthreads();
  return pre + inc - v;
}

// The same pick as pick_bin, on the cluster smem layout.
__device__ __forceinline__ void pick_bin_cl(int nbins, uint32_t need, ClusterMergeSmem& s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t h[4], c = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int b = 4 * tid + j;
    h[j] = b < nbins ? s.hist[b] : 0u;
    c += h[j];
  }
  uint32_t suf = c;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t v = __shfl_down_sync(0xffffffffu, suf, d);
    if (lane + d < 32) suf += v;
  }
  if (lane == 0) s.red[0][warp] = suf;
  __syncthreads();
  uint32_t later = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w)
    if (w > warp) later += s.red[0][w];
  suf += later;
  uint32_t above = suf - c;
  if (above < need && suf >= need) {
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      if (above + h[j] >= need) {
        s.bin = 4 * tid + j;
        s.above = above;
        s.cnt = h[j];
        break;
      }
      above += h[j];
    }
  }
  __syncthreads();
}

__device__ void merge_row_cluster(const MergeArgs& a, int r, int64_t soff, ClusterMergeSmem& s,
                                  cg::cluster_group& cl, int rank) {
  const int tid = threadIdx.x;
  const int K = a.K, tp = a.tp;
  const int c0 = tid * PER;
  const int64_t row_off = (int64_t)r * 2 * K;
  const float* slab = reinterpret_cast<const float*>(a.base[rank] + soff + (int64_t)rank * a.shard_stride) + row_off;
  ClusterMergeSmem* s0 = cl.map_shared_rank(&s, 0);

  // ---- 1. this shard's keys
  uint32_t key[PER];
  uint32_t vmask = 0;
  if (c0 < K) {
    float f[PER];
    if (a.vec) {
      const float4 q = a.p2p ? ld_sys_f4(slab + c0) : __ldg(reinterpret_cast<const float4*>(slab + c0));
      f[0] = q.x;
      f[1] = q.y;
      f[2] = q.z;
      f[3] = q.w;
    } else {
#pragma unroll
      for (int e = 0; e < PER; ++e)
        f[e] = c0 + e < K ? (a.p2p ? ld_sys_f32(slab + c0 + e) : __ldg(slab + c0 + e)) : 0.f;
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      key[e] = monotone32(f[e]);
      if (c0 + e < K) vmask |= 1u << e;
    }
  }
  uint32_t nh = 0, kmin = 0xFFFFFFFFu, kmax = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e)
    if (((vmask >> e) & 1u) && key[e] > NEG_KEY) {
      ++nh;
      kmin = min(kmin, key[e]);
      kmax = max(kmax, key[e]);
    }
  nh = block_sum_u32(nh, s.red[0]);
  {
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t wmin = __reduce_min_sync(0xffffffffu, kmin), wmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) {
      s.red[1][warp] = wmin;
      s.red[2][warp] = wmax;
    }
    __syncthreads();
    kmin = 0xFFFFFFFFu;
    kmax = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      kmin = min(kmin, s.red[1][w]);
      kmax = max(kmax, s.red[2][w]);
    }
  }
  if (tid < tp) {  // publish this CTA's values to every CTA
    ClusterMergeSmem* d = cl.map_shared_rank(&s, tid);
    d->x_nh[rank] = nh;
    d->x_min[rank] = kmin;
    d->x_max[rank] = kmax;
  }
  if (rank == 0)
    for (int i = tid; i < NBIN; i += MT) s.hist[i] = 0;
  cl.sync();
  nh = 0;
  kmin = 0xFFFFFFFFu;
  kmax = 0;
  for (int q = 0; q < tp; ++q) {
    nh += s.x_nh[q];
    kmin = min(kmin, s.x_min[q]);
    kmax = max(kmax, s.x_max[q]);
  }

  // ---- 2. selection rule (cluster-wide radix select over the high keys)
  uint32_t thr = NEG_KEY + 1, need_eq = 0;
  bool tie = false;
  int n_neg = 0;
  if (nh <= (uint32_t)K) {
    n_neg = K - (int)nh;
  } else {
    uint32_t base = kmin, need = (uint32_t)K;
    const uint32_t span = kmax - kmin;
    int bits = span ? 32 - __clz(span) : 0;
    bool first = true;
    while (true) {
      if (bits == 0) {
        thr = base;
        need_eq = need;
        tie = true;
        break;
      }
      const int shift = max(bits - DIGIT, 0);
      const int nbins = 1 << (bits - shift);
      if (rank != 0)  // rank 0's histogram was cleared before the last cluster barrier
        for (int i = tid; i < nbins; i += MT) s.hist[i] = 0;
      __syncthreads();
      // local counts (rank 0 counts straight into the row's histogram)
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const uint32_t k = key[e];
        if (!((vmask >> e) & 1u) || k <= NEG_KEY || k < base) continue;
        const uint32_t d = k - base;
        if (!first && (d >> bits) != 0) continue;
        atomicAdd(&s.hist[d >> shift], 1u);
      }
      __syncthreads();
      if (rank != 0)
        for (int i = tid; i < nbins; i += MT) {
          const uint32_t c = s.hist[i];
          if (c) atomicAdd(&s0->hist[i], c);
        }
      cl.sync();  // rank 0 holds the row's histogram
      if (rank == 0) {
        pick_bin_cl(nbins, need, s);
        for (int i = tid; i < nbins; i += MT) s.hist[i] = 0;  // cleared for the next pass
        if (tid > 0 && tid < tp) {
          ClusterMergeSmem* d = cl.map_shared_rank(&s, tid);
          d->bin = s.bin;
          d->above = s.above;
          d->cnt = s.cnt;
        }
      }
      cl.sync();  // every CTA has the pass's bin
      const uint32_t b = s.bin, above = s.above, cnt = s.cnt;
      need -= above;
      base += b << shift;
      bits = shift;
      first = false;
      if (cnt == need) {
        thr = base;
        break;
      }
    }
  }

  // ---- 3. selected columns of this shard (ties ranked in column order)
  uint32_t selm = 0;
  if (tie) {
    uint32_t my_eq = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) my_eq += ((vmask >> e) & 1u) && key[e] == thr;
    uint32_t rank_eq = block_excl_u32(my_eq, s.red[0]);
    const uint32_t tot_eq = block_sum_u32(my_eq, s.red[1]);
    if (tid < tp) cl.map_shared_rank(&s, tid)->x_eq[rank] = tot_eq;
    cl.sync();
    for (int q = 0; q < rank; ++q) rank_eq += s.x_eq[q];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      if (!((vmask >> e) & 1u)) continue;
      if (key[e] > thr) {
        selm |= 1u << e;
      } else if (key[e] == thr) {
        if (rank_eq < need_eq) selm |= 1u << e;
        ++rank_eq;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if (((vmask >> e) & 1u) && key[e] >= thr && key[e] > NEG_KEY) selm |= 1u << e;
  }

  // ---- 4. this CTA's run of selected positions, in column order
  const uint32_t my_n = __popc(selm);
  uint32_t slot = block_excl_u32(my_n, s.red[0]);
  const uint32_t run_len = block_sum_u32(my_n, s.red[1]);
  if (selm) {
    const float* pv = slab + K + c0;
    int32_t pp[PER];
    if (a.vec) {
      const float4 q = a.p2p ? ld_sys_f4(pv) : __ldg(reinterpret_cast<const float4*>(pv));
      pp[0] = __float_as_int(q.x);
      pp[1] = __float_as_int(q.y);
      pp[2] = __float_as_int(q.z);
      pp[3] = __float_as_int(q.w);
    } else {
#pragma unroll
      for (int e = 0; e < PER; ++e)
        pp[e] = ((selm >> e) & 1u) ? __float_as_int(a.p2p ? ld_sys_f32(pv + e) : __ldg(pv + e)) : 0;
    }
#pragma unroll
    for (int e = 0; e < PER; ++e)
      if ((selm >> e) & 1u) {
        if (slot < (uint32_t)MAX_K) s.pos[slot] = pp[e];
        ++slot;
      }
  }
  __syncthreads();
  const int n_run = (int)min(run_len, (uint32_t)MAX_K);
  bool unsorted = false;
  for (int i = tid; i + 1 < n_run; i += MT)
    if (s.pos[i] > s.pos[i + 1]) unsorted = true;
  const int my_sorted = !__syncthreads_or(unsorted);
  if (tid < tp) {
    ClusterMergeSmem* d = cl.map_shared_rank(&s, tid);
    d->x_len[rank] = (uint32_t)n_run;
    d->x_first[rank] = n_run ? s.pos[0] : 0;
    d->x_last[rank] = n_run ? s.pos[n_run - 1] : 0;
    d->x_sorted[rank] = my_sorted;
  }
  cl.sync();
  int all_sorted = 1, total = 0, seg0 = 0;
  for (int q = 0; q < tp; ++q) {
    all_sorted &= s.x_sorted[q];
    if (q < rank) seg0 += (int)s.x_len[q];
    total += (int)s.x_len[q];
  }
  total = min(total, K - n_neg);
  int32_t* out = a.out + (a.dst_base >= 0 ? (int64_t)a.dst_base + r : (int64_t)a.dst_rows[r]) * a.out_stride;
  if (rank == 0)
    for (int i = tid; i < n_neg; i += MT) out[i] = -1;

  // ---- 5. ascending output
  if (all_sorted) {
    for (int i = tid; i < n_run; i += MT) {
      const int32_t p = s.pos[i];
      int rk = i;
      for (int q = 0; q < tp; ++q) {
        const int n = (int)s.x_len[q];
        if (q == rank || n == 0) continue;
        const bool strict = q > rank;  // equal positions: the lower shard goes first
        const int32_t f = s.x_first[q], l = s.x_last[q];
        if (strict ? l < p : l <= p)
          rk += n;
        else if (strict ? f < p : f <= p)
          rk += count_run(cl.map_shared_rank(s.pos, q), n, p, strict);
      }
      if (n_neg + rk < K) out[n_neg + rk] = p;
    }
  } else {
    // gather every run into rank 0 (its own run moves to its segment too)
    int32_t* pos0 = cl.map_shared_rank(s.pos, 0);
    __syncthreads();
    int32_t mine[PER];
    int nm = 0;
    for (int i = tid; i < n_run && nm < PER; i += MT) mine[nm++] = s.pos[i];
    cl.sync();  // rank 0's own run is read by its threads before it is overwritten
    for (int k = 0; k < nm; ++k) {
      const int i = tid + k * MT;
      if (seg0 + i < MAX_K) pos0[seg0 + i] = mine[k];
    }
    cl.sync();
    if (rank == 0) {
      const int n = min(total, MAX_K);
      sort_positions(s.pos, n);
      for (int i = tid; i < n; i += MT)
        if (n_neg + i < K) out[n_neg + i] = s.pos[i];
    }
  }
  cl.sync();  // no CTA leaves while another reads its run
}

__global__ void __launch_bounds__(MT, 1) shard_merge_cluster_kernel(const MergeArgs a) {
  __shared__ ClusterMergeSmem s;
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int r = blockIdx.y;
  int seq = a.seq;
  int64_t soff = a.slot_off;
  if (a.ctl) {
    seq = *reinterpret_cast<const volatile int*>(a.ctl) + 1;
    soff = (int64_t)(seq & 1) * a.slot_bytes;
  }
  bool ok = true;
  if (a.p2p) {  // each CTA waits for its own shard's peer, the cluster agrees
    if (threadIdx.x == 0) {
      int mine = read_err_word(a.err) == 0;
      if (mine) mine = wait_flag_geq(a.staged[rank], seq, a.timeout_ns, a.err);
      for (int q = 0; q < a.tp; ++q) cl.map_shared_rank(&s, q)->x_ok[rank] = mine;
    }
    cl.sync();
    for (int q = 0; q < a.tp; ++q) ok = ok && s.x_ok[q] != 0;
  }
  if (ok && r < a.R) merge_row_cluster(a, r, soff, s, cl, rank);
  if (a.ctl) finish_exchange(a, seq);
}

__global__ void ipc_flag_set_kernel(int* flag, int seq, const int32_t* err) {
  if (read_err_word(err) != 0) return;  // a failed wait before this point: publish nothing
  __threadfence_system();
  st_release_sys_s32(flag, seq);
}

struct FlagPtrs {
  const int* merged[MAX_TP];  // &flags[s][1]
};

__global__ void ipc_slot_wait_kernel(FlagPtrs f, int tp, int min_seq, int64_t timeout_ns, int32_t* err) {
  if ((int)threadIdx.x < tp) wait_flag_geq(f.merged[threadIdx.x], min_seq, timeout_ns, err);
  __syncthreads();
  __threadfence_system();
}

// Stages [R, K] values and [R, K] positions as the [R, 2K] f32 payload;
// returns at once when the error word is set (a slot wait before it failed,
// so a peer may still be reading the slot).
__global__ void shard_stage_kernel(float* slot, const float* vals, int64_t vals_stride, const int32_t* idx,
                                   int64_t idx_stride, int K, const int32_t* err) {
  if (read_err_word(err) != 0) return;
  const int r = blockIdx.x;
  float* dst = slot + (int64_t)r * 2 * K;
  for (int c = threadIdx.x; c < K; c += blockDim.x) {
    dst[c] = vals[(int64_t)r * vals_stride + c];
    dst[K + c] = __int_as_float(idx[(int64_t)r * idx_stride + c]);
  }
}

int check_merge_args(int tp, int R, int K, int dst_base, const int32_t* dst_rows, const int32_t* out) {
  DSA_REQUIRE(tp >= 1 && tp <= MAX_TP, DSA_ERR_UNSUPPORTED, "shard_merge: tp must be in [1, %d] (got %d)",
              MAX_TP, tp);
  DSA_REQUIRE(K >= 1 && K <= MAX_K, DSA_ERR_UNSUPPORTED, "shard_merge: K must be in [1, %d] (got %d)", MAX_K, K);
  DSA_REQUIRE(R >= 0, DSA_ERR_INVALID, "shard_merge: negative R");
  DSA_REQUIRE(dst_base >= 0 || dst_rows != nullptr, DSA_ERR_INVALID, "shard_merge: need dst_rows when dst_base < 0");
  DSA_REQUIRE(out != nullptr, DSA_ERR_INVALID, "shard_merge: null out");
  return DSA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

std::once_flag g_cl_once[kMaxDevices];
int g_cl_ok[kMaxDevices];  // clusters of 8 merge CTAs can be resident

// One CTA per row, or, for few rows, a cluster of tp CTAs per row. rows = R
// (at least one CTA runs, so the exchange mode always publishes its flag).
int launch_merge(const MergeArgs& a, int rows, cudaStream_t s, const char* what) {
  const int dev = current_device();
  bool cluster = false;
  if (a.tp >= 2 && a.R > 0 && a.R <= 32 && dev >= 0 && dev < kMaxDevices) {
    std::call_once(g_cl_once[dev], [dev] {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(MAX_TP, 1, 1);
      cfg.blockDim = dim3(MT);
      cudaLaunchAttribute attr{};
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = MAX_TP;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, shard_merge_cluster_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      g_cl_ok[dev] = n > 0;
    });
    cluster = g_cl_ok[dev] != 0;
  }
  if (!cluster) {
    shard_merge_kernel<<<rows, MT, 0, s>>>(a);
    return check_launch(what);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.tp, a.R, 1);
  cfg.blockDim = dim3(MT);
  cfg.stream = s;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = a.tp;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, shard_merge_cluster_kernel, a);
  if (e != cudaSuccess) {
    set_error("%s (cluster) launch: %s", what, cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_indexer_shard_merge(int32_t* out, int64_t out_stride, const float* allf,
                                       const int32_t* dst_rows, int dst_base, int tp, int R, int K,
                                       void* stream) {
  clear_error();
  int st = check_merge_args(tp, R, K, dst_base, dst_rows, out);
  if (st != DSA_OK) return st;
  if (R == 0) return DSA_OK;
  DSA_REQUIRE(allf != nullptr && out_stride >= K, DSA_ERR_INVALID, "shard_merge: null allf or short out rows");
  MergeArgs a{};
  for (int s = 0; s < MAX_TP; ++s) a.base[s] = reinterpret_cast<const uint8_t*>(allf);
  a.shard_stride = (int64_t)R * 2 * K * sizeof(float);
  a.out = out;
  a.dst_rows = dst_rows;
  a.out_stride = out_stride;
  a.R = R;
  a.tp = tp;
  a.K = K;
  a.dst_base = dst_base;
  a.vec = (K % 4 == 0) && aligned16(allf);
  return launch_merge(a, R, as_stream(stream), "shard_merge_kernel");
}

extern "C" int dsa_indexer_shard_merge_p2p(int32_t* out, int64_t out_stride, const uint64_t* data_ptrs,
                                           const uint64_t* flag_ptrs, const int32_t* dst_rows, int dst_base,
                                           int K, int tp, int R, int seq, int64_t slot_off, int64_t timeout_ns,
                                           int32_t* err_flag, void* stream) {
  clear_error();
  int st = check_merge_args(tp, R, K, dst_base, dst_rows, out);
  if (st != DSA_OK) return st;
  if (R == 0) return DSA_OK;
  DSA_REQUIRE(data_ptrs && flag_ptrs && out_stride >= K && timeout_ns > 0, DSA_ERR_INVALID,
              "shard_merge_p2p: null pointer arrays, short out rows or non-positive timeout");
  MergeArgs a{};
  a.vec = K % 4 == 0 && slot_off % 16 == 0;
  for (int s = 0; s < tp; ++s) {
    DSA_REQUIRE(data_ptrs[s] != 0 && flag_ptrs[s] != 0, DSA_ERR_INVALID, "shard_merge_p2p: null peer pointer %d", s);
    a.base[s] = reinterpret_cast<const uint8_t*>(data_ptrs[s]);
    a.staged[s] = reinterpret_cast<const int*>(flag_ptrs[s]);
    a.vec = a.vec && aligned16(a.base[s]);
  }
  a.slot_off = slot_off;
  a.out = out;
  a.dst_rows = dst_rows;
  a.err = err_flag;
  a.out_stride = out_stride;
  a.timeout_ns = timeout_ns;
  a.R = R;
  a.tp = tp;
  a.K = K;
  a.dst_base = dst_base;
  a.seq = seq;
  a.p2p = 1;
  return launch_merge(a, R, as_stream(stream), "shard_merge_kernel(p2p)");
}

extern "C" int dsa_shard_exchange_merge(int32_t* out, int64_t out_stride, const uint64_t* data_ptrs,
                                        const uint64_t* flag_ptrs, int tp, int rank, int R, int K,
                                        int64_t slot_bytes, int32_t* ctl, int64_t timeout_ns, int32_t* err_flag,
                                        void* stream) {
  clear_error();
  int st = check_merge_args(tp, R, K, 0, nullptr, out);
  if (st != DSA_OK) return st;
  DSA_REQUIRE(data_ptrs && flag_ptrs && ctl && err_flag && out_stride >= K && timeout_ns > 0 && rank >= 0 &&
                  rank < tp && slot_bytes >= (int64_t)R * 2 * K * 4 && slot_bytes % 16 == 0,
              DSA_ERR_INVALID, "shard_exchange_merge: bad arguments");
  MergeArgs a{};
  a.vec = K % 4 == 0;
  for (int s = 0; s < tp; ++s) {
    DSA_REQUIRE(data_ptrs[s] != 0 && flag_ptrs[s] != 0, DSA_ERR_INVALID,
                "shard_exchange_merge: null peer pointer %d", s);
    a.base[s] = reinterpret_cast<const uint8_t*>(data_ptrs[s]);
    a.staged[s] = reinterpret_cast<const int*>(flag_ptrs[s]);
    a.vec = a.vec && aligned16(a.base[s]);
  }
  a.my_flags = reinterpret_cast<int*>(flag_ptrs[rank]);
  a.ctl = ctl;
  a.slot_bytes = slot_bytes;
  a.out = out;
  a.err = err_flag;
  a.out_stride = out_stride;
  a.timeout_ns = timeout_ns;
  a.R = R;
  a.tp = tp;
  a.K = K;
  a.p2p = 1;
  // at least one CTA, so the merged flag is published even for R == 0
  return launch_merge(a, R > 0 ? R : 1, as_stream(stream), "shard_merge_kernel(exchange)");
}

extern "C" int dsa_indexer_shard_stage(float* slot, const float* vals, int64_t vals_stride, const int32_t* idx,
                                       int64_t idx_stride, int R, int K, const int32_t* err_flag, void* stream) {
  clear_error();
  DSA_REQUIRE(R >= 0 && K >= 1 && vals_stride >= K && idx_stride >= K, DSA_ERR_INVALID,
              "shard_stage: bad sizes");
  if (R == 0) return DSA_OK;
  DSA_REQUIRE(slot && vals && idx, DSA_ERR_INVALID, "shard_stage: null pointer");
  shard_stage_kernel<<<R, 256, 0, as_stream(stream)>>>(slot, vals, vals_stride, idx, idx_stride, K, err_flag);
  return check_launch("shard_stage_kernel");
}

extern "C" int dsa_ipc_alloc(int64_t bytes, void** dev_ptr, uint8_t* handle_out) {
  clear_error();
  DSA_REQUIRE(bytes > 0 && dev_ptr && handle_out, DSA_ERR_INVALID, "ipc_alloc: bad arguments");
  void* ptr = nullptr;
  DSA_CUDA_TRY(cudaMalloc(&ptr, (size_t)bytes), "ipc_alloc cudaMalloc");
  cudaError_t e = cudaMemset(ptr, 0, (size_t)bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    cudaFree(ptr);
    set_error("ipc_alloc: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = ptr;
  return DSA_OK;
}

extern "C" int dsa_ipc_free(void* dev_ptr) {
  clear_error();
  if (!dev_ptr) return DSA_OK;
  DSA_CUDA_TRY(cudaFree(dev_ptr), "ipc_free");
  return DSA_OK;
}

extern "C" int dsa_ipc_open(const uint8_t* handle, void** dev_ptr) {
  clear_error();
  DSA_REQUIRE(handle && dev_ptr, DSA_ERR_INVALID, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* ptr = nullptr;
  DSA_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open cudaIpcOpenMemHandle");
  *dev_ptr = ptr;
  return DSA_OK;
}

extern "C" int dsa_ipc_close(void* dev_ptr) {
  clear_error();
  if (!dev_ptr) return DSA_OK;
  DSA_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr), "ipc_close");
  return DSA_OK;
}

extern "C" int dsa_ipc_flag_set(uint64_t flag_ptr, int which, int seq, const int32_t* err_flag, void* stream) {
  clear_error();
  DSA_REQUIRE(flag_ptr != 0 && (which == 0 || which == 1), DSA_ERR_INVALID, "ipc_flag_set: bad arguments");
  ipc_flag_set_kernel<<<1, 1, 0, as_stream(stream)>>>(reinterpret_cast<int*>(flag_ptr) + which, seq, err_flag);
  return check_launch("ipc_flag_set_kernel");
}

extern "C" int dsa_ipc_slot_wait(const uint64_t* flag_ptrs, int tp, int min_seq, int64_t timeout_ns,
                                 int32_t* err_flag, void* stream) {
  clear_error();
  DSA_REQUIRE(flag_ptrs && tp >= 1 && tp <= MAX_TP && timeout_ns > 0, DSA_ERR_INVALID,
              "ipc_slot_wait: bad arguments");
  FlagPtrs f{};
  for (int s = 0; s < tp; ++s) {
    DSA_REQUIRE(flag_ptrs[s] != 0, DSA_ERR_INVALID, "ipc_slot_wait: null flag pointer %d", s);
    f.merged[s] = reinterpret_cast<const int*>(flag_ptrs[s]) + 1;
  }
  ipc_slot_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(f, tp, min_seq, timeout_ns, err_flag);
  return check_launch("ipc_slot_wait_kernel");
}
