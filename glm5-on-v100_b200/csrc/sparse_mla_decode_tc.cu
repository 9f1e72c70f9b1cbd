// Sparse MLA decode / prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), for the fp8_ds_mla latent cache.
//
// Same function as the reference's split decode + merge
// (csrc/attention/sm70_mla_decode.cu:918-1184) and prefill kernels
// (:1563-2051); see sparse_mla_decode.cu for the semantics.
//
// One CTA = one query row x 64 heads x one slice of the top-k axis, processed
// in tiles of 64 selected latent rows that alternate between two shared-memory
// buffers, so that one tile is stored while the previous one is in QK, softmax
// and PV. The MMAs are "transposed" so that latent rows are the M side and the
// 64 heads are N:
//   S^T[64 x 64]   = KV[64 x 576] . Q^T          (M = 64; A = KV tile,
//                                                 K-major; B = Q, K-major)
//   O^T[512 x 64] += V^T[512 x 64] . P^T         (M = 128 per value tile;
//                                                 A = same KV tile read
//                                                 MN-major; B = P^T, MN-major)
// O^T (256 columns) and one S^T per buffer (64 columns each) live in tensor
// memory. A KV tile is stored once as fp16 in 128-byte-swizzled rows that serve
// both as K-major A of QK and MN-major A of PV; P^T (fp16) overwrites the
// tile's rope columns after QK has consumed them. Q (72 KB) + two tiles
// (2 x 72 KB) + the slice's row table (8 KB) fill one SM's shared memory.
//
// Warp roles (32 warps, 64 registers each):
//   * warps 0-15, producers: 4 rows of every tile each; the 656-byte rows are
//     read with 16-byte coalesced loads into registers, and as soon as a
//     128-wide scale group of tile t is stored (dequantised: e4m3 bits
//     expanded to fp16 with integer ops, times the per-group scale, rounded
//     once) the same registers receive that group of tile t+1; tile t+2's
//     rows are prefetched into L2 with bulk prefetches.
//   * warp 24, lane 0: issues QK(t) when tile t is stored and PV(t-1) when its
//     P^T is written, committing mbarriers that release S, the tile buffer
//     and (for the softmax) the accumulated O^T.
//   * warps 16-23, softmax: two per TMEM sub-partition, each thread one tile
//     row and 16 heads of S^T (tcgen05.ld 16x64b). Probabilities use a lazily
//     updated running max per head, moved (with an in-TMEM rescale of O^T
//     after PV(t-1) completes) only when a score exceeds it by more than 2^8,
//     so P <= 256 in fp16 while o and lse stay exact; row sums accumulate in
//     registers.
//   * the other warps join the block barriers and the epilogue.
// Setup overlaps its two dependent chains: the producers resolve the slice's
// selected positions through the block table into a row table in shared
// memory and issue tile 0's loads while the other warps stage Q (cp.async).
// When a row's top-k axis is split in 2 or 4 slices, the slices form one
// thread-block cluster and merge on chip (one DSMEM bulk copy per receiver,
// see the epilogue); other slice counts write partial states for the merge
// kernel. Every wait on another role or the tensor core is an mbarrier wait
// bounded by a device-time limit that reports DSA_ERR_TIMEOUT instead of
// hanging.
#include "sparse_mla.cuh"
#include "tc_common.cuh"

namespace dsa {
namespace {

using namespace tc;

constexpr int TM = kTcTileRows;             // 64 latent rows per tile
constexpr int NH = 64;                      // heads per CTA (MMA N)
constexpr int NWARPS = 32;
constexpr int NTHREADS = 32 * NWARPS;
constexpr int PRODUCERS = 16;               // warps 0-15
constexpr int SOFTMAX0 = 16;                // warps 16-23: two per TMEM sub-partition
constexpr int SOFTMAX_WARPS = 8;
constexpr int MMA_WARP = 24;                // warps 25-31 only join the block barriers
constexpr int ROWS_PER_WARP = TM / PRODUCERS;  // 4
constexpr int RS = ROWS_PER_WARP / 4;          // rows per group of 8 lanes
constexpr int DV = 512;
constexpr int TABLE_ROWS = 2048;            // resolved rows held at a time
constexpr uint32_t KV_REGION = TM * 128;    // one 64-wide K block of a tile: 8 KB
constexpr uint32_t KV_BUF = 9 * KV_REGION;  // one tile: 72 KB
constexpr uint32_t Q_REGION = NH * 128;     // one 64-wide K block of Q: 8 KB
constexpr uint32_t SM_KV = 0;               // two tile buffers
constexpr uint32_t SM_Q = 2 * KV_BUF;
constexpr uint32_t SM_TABLE = SM_Q + 9 * Q_REGION;
constexpr uint32_t SM_MISC = SM_TABLE + TABLE_ROWS * 4;
constexpr uint32_t MISC_BYTES = 2048;
constexpr uint32_t SMEM_BYTES = SM_MISC + MISC_BYTES + 1024;  // + alignment slack = 232,448
constexpr uint32_t S_COL = 256;             // S^T of buffer x at [256 + 64x, +64); O^T tile j at [64j, 64j+64)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t kSendOff = 112 * 1024;   // epilogue: outgoing rows after received rows + staged output
constexpr int ROW_BYTES = 656;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kRescaleThreshold = 8.0f;   // log2 units: P stays <= 256
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;
// row table codes
constexpr int kRowSkip = -1;   // position not selected / out of range: not counted
constexpr int kRowZero = -2;   // counted position whose row lies outside the cache: zeros

constexpr uint32_t IDESC_QK = idesc_f16(TM, NH, false, false);
constexpr uint32_t IDESC_PV = idesc_f16(128, NH, true, true);

static_assert(TM == 64, "M = 64 QK tiles");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// cluster epilogue (csize 2 or 4): received (csize-1) x W x 256 B + output 128 W B
// below kSendOff; (csize-1) x W x 256 B to send above it, below the misc block
static_assert(3 * 128 * 256 + 128 * 128 <= kSendOff && kSendOff + 3 * 128 * 256 <= SM_MISC, "epilogue layout");

__device__ int32_t g_tc_error;  // sticky: DSA_ERR_TIMEOUT when a bounded wait expired

__device__ __forceinline__ float unmono(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(a), "r"(sel));
  return d;
}

// Four e4m3 bytes -> two half2 words holding value/256 each, exactly: each
// byte is placed in a 16-bit lane with its sign replicated above it (prmt
// sign-extension selectors), shifted so exponent+mantissa fill fp16 bits
// 7..13 and the sign lands on bit 15; bit 14 is cleared. e4m3's exponent bias
// (7) vs fp16's (15) is the 2^-8 factor; e4m3 subnormals become fp16
// subnormals. Integer ops only (no conversion-pipe instructions).
__device__ __forceinline__ void e4m3x4_div256(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = (prmt(w, 0x9180u) << 7) & 0xBF80BF80u;
  hi = (prmt(w, 0xB3A2u) << 7) & 0xBF80BF80u;
}

// 16 e4m3 (uint4) times scale -> 16 fp16 (two uint4).
__device__ __forceinline__ void dequant16(const uint4& r, float sc, uint4& o0, uint4& o1) {
  uint32_t q[8];
  e4m3x4_div256(r.x, q[0], q[1]);
  e4m3x4_div256(r.y, q[2], q[3]);
  e4m3x4_div256(r.z, q[4], q[5]);
  e4m3x4_div256(r.w, q[6], q[7]);
  const float s256 = sc * 256.0f;
  if (s256 >= 0.0078125f && s256 <= 32768.0f) {  // hi, lo and every product stay normal in fp16
    // scale = hi + lo with hi cut to 7 significant bits: x (an e4m3 value,
    // 4 significant bits) times hi fits fp16's 11 bits exactly, so
    // fma(x, lo, x*hi) rounds once, like the f32 product rounded to fp16
    // (lo carries the rest of the scale to ~2^-18 relative)
    const float hi7 = __uint_as_float(__float_as_uint(s256) & 0xFFFE0000u);
    const __half2 s_hi = __float2half2_rn(hi7);
    const __half2 s_lo = __float2half2_rn(s256 - hi7);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half2 x = *reinterpret_cast<const __half2*>(&q[e]);
      const __half2 v = __hfma2(x, s_lo, __hmul2(x, s_hi));
      q[e] = *reinterpret_cast<const uint32_t*>(&v);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[e]));
      q[e] = pack_half2(f.x * s256, f.y * s256);
    }
  }
  o0 = make_uint4(q[0], q[1], q[2], q[3]);
  o1 = make_uint4(q[4], q[5], q[6], q[7]);
}

__device__ __forceinline__ float pick(const float4& s, int j) {
  return j == 0 ? s.x : (j == 1 ? s.y : (j == 2 ? s.z : s.w));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One producer warp's share of a tile: rows 8*w + (lane >> 3) + 4*rs (rs = 0,
// 1). Lane l holds, for each of its 2 rows, nope chunk (l & 7) + 8*j of every
// 128-wide scale group j (16 e4m3 per chunk), the row's four scales, and rope
// chunk (l & 7); eight consecutive lanes read 128 contiguous bytes of a row.
struct Tile {
  uint4 nope[RS][4];  // [rs][j]
  float4 sc[RS];
  uint4 rope[RS];
};

__device__ __forceinline__ int64_t row_offset(const int* table, int i) {
  const int code = table[i];
  return code >= 0 ? (int64_t)code * ROW_BYTES : -1;
}

__device__ __forceinline__ void load_group(Tile& T, const uint8_t* kv, const int* table, int tbase, int j, int w,
                                           int lane) {
#pragma unroll
  for (int rs = 0; rs < RS; ++rs) {
    const int64_t off = row_offset(table, tbase + ROWS_PER_WARP * w + (lane >> 3) + 4 * rs);
    T.nope[rs][j] = off >= 0 ? ldg_nc16(kv + off + 16 * ((lane & 7) + 8 * j)) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void load_tail(Tile& T, const uint8_t* kv, const int* table, int tbase, int w, int lane) {
#pragma unroll
  for (int rs = 0; rs < RS; ++rs) {
    const int64_t off = row_offset(table, tbase + ROWS_PER_WARP * w + (lane >> 3) + 4 * rs);
    if (off >= 0) {
      const uint4 s = ldg_nc16(kv + off + 512);
      T.sc[rs] = make_float4(__uint_as_float(s.x), __uint_as_float(s.y), __uint_as_float(s.z), __uint_as_float(s.w));
      T.rope[rs] = ldg_nc16(kv + off + 528 + 16 * (lane & 7));
    } else {
      T.sc[rs] = make_float4(0.f, 0.f, 0.f, 0.f);
      T.rope[rs] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Store scale group j (K blocks 2j, 2j+1) of this warp's rows into tile buffer `buf`.
__device__ __forceinline__ void store_group(const Tile& T, uint8_t* buf, int j, int w, int lane) {
  const int c = (lane & 7) + 8 * j;  // nope chunk: e4m3 values [16c, 16c+16)
  uint8_t* region = buf + (c >> 2) * KV_REGION;
  const int c0 = 2 * (c & 3);
#pragma unroll
  for (int rs = 0; rs < RS; ++rs) {
    const int i = ROWS_PER_WARP * w + (lane >> 3) + 4 * rs;
    uint4 o0, o1;
    dequant16(T.nope[rs][j], pick(T.sc[rs], j), o0, o1);
    *reinterpret_cast<uint4*>(region + sw128_off(i, c0)) = o0;
    *reinterpret_cast<uint4*>(region + sw128_off(i, c0 + 1)) = o1;
  }
}

__device__ __forceinline__ void store_rope(const Tile& T, uint8_t* buf, int w, int lane) {
#pragma unroll
  for (int rs = 0; rs < RS; ++rs)
    *reinterpret_cast<uint4*>(buf + 8 * KV_REGION +
                              sw128_off(ROWS_PER_WARP * w + (lane >> 3) + 4 * rs, lane & 7)) = T.rope[rs];
}

// Row table for slice rows [r0, r0 + n): physical row, kRowZero or kRowSkip;
// written by threads [0, nthreads) of the block. Each thread takes four rows
// at a time and issues their four index loads, then their four block-table
// loads, so a batch costs two dependent memory round trips.
__device__ __forceinline__ void resolve_rows_batched(const SparseMlaArgs& p, int b, int seq_len, int r0, int n,
                                                     int* table, int nthreads) {
  const int* idx = p.idx + (int64_t)b * p.idx_stride + r0;
  const int* bt = p.bt + (int64_t)b * p.bt_stride;
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * nthreads) {
    int pos[4], blk[4], code[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * nthreads;
      pos[k] = i < n ? idx[i] : -1;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      code[k] = kRowSkip;
      blk[k] = 0;
      if (pos[k] >= 0 && pos[k] < seq_len) {
        code[k] = kRowZero;
        const int blk_i = pos[k] / p.page_size;
        if (blk_i < p.max_blocks) {
          blk[k] = bt[blk_i];
          pos[k] -= blk_i * p.page_size;  // offset in the page
          code[k] = 0;                    // resolved below
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i0 + k * nthreads;
      if (i >= n) break;
      if (code[k] == 0) {
        const int64_t r = (int64_t)blk[k] * p.page_size + pos[k];
        code[k] = (r >= 0 && r < p.n_kv_rows) ? (int)r : kRowZero;
      }
      table[i] = code[k];
    }
  }
}

// Row table for slice rows [r0, r0 + n) (a later window of a long slice), one
// row per thread at a time.
__device__ __forceinline__ void resolve_rows(const SparseMlaArgs& p, int b, int seq_len, int r0, int n, int* table,
                                             int nthreads) {
  for (int i = threadIdx.x; i < n; i += nthreads) {
    int code = kRowSkip;
    const int pos = p.idx[(int64_t)b * p.idx_stride + r0 + i];
    if (pos >= 0 && pos < seq_len) {
      code = kRowZero;
      const int blk_i = pos / p.page_size;
      if (blk_i < p.max_blocks) {
        const int64_t r = (int64_t)p.bt[(int64_t)b * p.bt_stride + blk_i] * p.page_size + (pos - blk_i * p.page_size);
        if (r >= 0 && r < p.n_kv_rows) code = (int)r;
      }
    }
    table[i] = code;
  }
}

__global__ void __launch_bounds__(NTHREADS, 1) sparse_mla_decode_tc_kernel(const SparseMlaArgs p, int32_t* err,
                                                                                  int csize) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw_base);
  int* table = reinterpret_cast<int*>(sm + SM_TABLE);
  uint8_t* misc = sm + SM_MISC;
  // misc: [0, 80) 10 mbarriers | 80 TMEM base | 84 abort | 88 any_rescale |
  // 92 q_bits | [96, 160) ovf | [160, 288) s_valid | [288, 1824) per-head floats
  uint64_t* mbar = reinterpret_cast<uint64_t*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 80);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 84);
  int* any_rescale = reinterpret_cast<int*>(misc + 88);
  uint32_t* q_bits = reinterpret_cast<uint32_t*>(misc + 92);  // largest |q| bf16 bit pattern of this CTA
  int* ovf = reinterpret_cast<int*>(misc + 96);           // [2 parities][8 softmax warps] overflow votes
  uint8_t* s_valid = misc + 160;                          // [2 buffers][64 rows] row counted
  float* m_ref = reinterpret_cast<float*>(misc + 288);    // [64] running max (log2 units)
  float* alpha = m_ref + 64;                              // [64] this tile's rescale factors
  float* tmax = alpha + 64;                               // [4][64] tile maxima; then row-sum partials
  float* l_sum = alpha;                                   // [64] in the epilogue (alpha is dead)
  const uint32_t mb0 = smem_u32(&mbar[0]);
  auto mb_kv_full = [&](int x) { return mb0 + 8u * (uint32_t)x; };         // producers: tile stored
  auto mb_s_full = [&](int x) { return mb0 + 16u + 8u * (uint32_t)x; };    // QK done
  auto mb_p_full = [&](int x) { return mb0 + 32u + 8u * (uint32_t)x; };    // softmax: P^T written
  auto mb_kv_free = [&](int x) { return mb0 + 48u + 8u * (uint32_t)x; };   // PV done: buffer and O^T released
  const uint32_t mb_done = mb0 + 64u;
  const uint32_t mb_recv = mb0 + 72u;  // rows sent by the other CTAs of the cluster have landed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int h0 = blockIdx.y * NH;
  const int split = blockIdx.z;
  const int seq_len = p.seq_lens[b];
  const int lo = split * p.span;
  const int hi = min(lo + p.span, p.topk);
  const int nrows = max(hi - lo, 0);
  const int ntiles = (nrows + TM - 1) / TM;
  constexpr int kTilesPerTable = TABLE_ROWS / TM;

  if (warp == 0) {
    if (lane == 0) {
      for (int x = 0; x < 2; ++x) {
        mbar_init(mb_kv_full(x), PRODUCERS);
        mbar_init(mb_s_full(x), 1);
        mbar_init(mb_p_full(x), SOFTMAX_WARPS);
        mbar_init(mb_kv_free(x), 1);
      }
      mbar_init(mb_done, 1);
      mbar_init(mb_recv, 1);
      mbar_init_fence();
      *abort_flag = 0;
      *any_rescale = 0;
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
  }
  // Setup in two halves that overlap: the producers resolve the first table
  // window and issue tile 0's loads (held in registers across the barrier)
  // while warps 16-31 stage Q.
  Tile T;
  if (warp < PRODUCERS) {
    // pad the table so that reads for rows past the slice are "not counted"
    resolve_rows_batched(p, b, seq_len, lo, min(nrows, TABLE_ROWS), table, PRODUCERS * 32);
    for (int i = min(nrows, TABLE_ROWS) + threadIdx.x; i < min(ntiles * TM, TABLE_ROWS); i += PRODUCERS * 32)
      table[i] = kRowSkip;
    named_bar(2, PRODUCERS * 32);
    if (ntiles > 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) load_group(T, p.kv, table, 0, j, warp, lane);
      load_tail(T, p.kv, table, 0, warp, lane);
    }
  } else {
    // Q: every 16-byte chunk this thread owns is copied at once (cp.async)
    // into the second tile buffer, idle until tile 1, then converted to fp16
    // into the swizzled Q operand; a thread converts only its own chunks
    const int nheads = min(NH, p.n_head - h0);
    const int tid = threadIdx.x - PRODUCERS * 32;
    constexpr int kQThreads = NTHREADS - PRODUCERS * 32;
    uint8_t* qraw = sm + SM_KV + KV_BUF;
    const uint8_t* qg = reinterpret_cast<const uint8_t*>(p.q) + ((int64_t)b * p.n_head + h0) * 576 * 2;
    for (int i = tid; i < nheads * 72; i += kQThreads) cp_async16(smem_u32(qraw + 16 * i), qg + 16 * i);
    cp_async_commit();
    cp_async_wait<0>();
    // bf16 q may exceed the fp16 range of the MMA operand: this CTA's Q is
    // then scaled by 2^-qe and the softmax scale by 2^qe (both exact), so
    // every score * scale is unchanged
    int qe = 0;
    if (p.q_bf16) {
      uint32_t bits = 0;
      for (int i = tid; i < nheads * 72; i += kQThreads)
        bits = max(bits, bf16x8_max_abs_bits(*reinterpret_cast<const uint4*>(qraw + 16 * i)));
      bits = __reduce_max_sync(0xffffffffu, bits);
      if (tid == 0) *q_bits = 0;
      named_bar(3, kQThreads);
      if (lane == 0) atomicMax(q_bits, bits);
      named_bar(3, kQThreads);
      qe = bf16_fp16_shift(*q_bits);
    }
    for (int i = tid; i < NH * 72; i += kQThreads) {
      const int h = i / 72, c = i % 72;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h < nheads) {
        v = *reinterpret_cast<const uint4*>(qraw + 16 * i);
        if (p.q_bf16) v = bf16x8_to_half8_scaled(v, qe);
      }
      *reinterpret_cast<uint4*>(sm + SM_Q + (c >> 3) * Q_REGION + sw128_off(h, c & 7)) = v;
    }
    if (tid < NH) {
      m_ref[tid] = -1e30f;
      alpha[tid] = 1.f;
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // softmax scale in log2 units, times 2^qe when this CTA's bf16 Q was scaled down
  const float scale_log2 = p.q_bf16 ? p.scale_log2 * exp2f((float)bf16_fp16_shift(*q_bits)) : p.scale_log2;
  // Base descriptors; a start-address advance of X bytes adds X >> 4.
  const uint64_t desc_kv = sw128_desc(base + SM_KV, 16, 1024);                       // tile buffer 0, K-major
  const uint64_t desc_q = sw128_desc(base + SM_Q, 16, 1024);                         // Q, K-major
  const uint64_t desc_v = sw128_desc(base + SM_KV, KV_REGION, 1024);                 // tile buffer 0, MN-major
  const uint64_t desc_p = sw128_desc(base + SM_KV + 8 * KV_REGION, KV_REGION, 1024);  // P^T of buffer 0, MN-major
  constexpr uint64_t kBufStep = KV_BUF >> 4;                                         // descriptor step per buffer

  bool ok = true;
  bool issued = false;  // the MMA thread issued at least one MMA
  // Control flow is uniform within each role: after a timed-out wait (`ok`
  // false, abort flag set) every thread still executes its role's barriers
  // and arrivals, and every later wait returns at once.
  if (warp < PRODUCERS) {
    // ------------------------------------------------------------- producers
    const int w = warp;
    bool have_next = true;  // tile t's data is in registers (tile 0: loaded during setup)
    for (int t = 0; t < ntiles; ++t) {
      const int x = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      const int tbase = (t % kTilesPerTable) * TM;  // tile rows in the row table
      if (!have_next) {
        if (t > 0) {  // a new table window: every producer has read its last entries
          named_bar(2, PRODUCERS * 32);
          const int r0 = t * TM;
          resolve_rows(p, b, seq_len, lo + r0, min(nrows - r0, TABLE_ROWS), table, PRODUCERS * 32);
          for (int i = min(nrows - r0, TABLE_ROWS) + threadIdx.x; i < min((ntiles - t) * TM, TABLE_ROWS);
               i += PRODUCERS * 32)
            table[i] = kRowSkip;
          named_bar(2, PRODUCERS * 32);
        }
        if (ok) {
#pragma unroll
          for (int j = 0; j < 4; ++j) load_group(T, p.kv, table, tbase, j, w, lane);
          load_tail(T, p.kv, table, tbase, w, lane);
        }
      }
      // buffer x is free once PV(t-2) has completed
      if (t >= 2) ok = ok && mbar_wait(mb_kv_free(x), ph ^ 1, abort_flag, err, kWaitTimeoutNs);
      const bool prefetch = (t + 1 < ntiles) && ((t + 1) % kTilesPerTable != 0);
      const int nbase = ((t + 1) % kTilesPerTable) * TM;
      uint8_t* buf = sm + SM_KV + x * KV_BUF;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (ok) store_group(T, buf, j, w, lane);
        if (ok && prefetch) load_group(T, p.kv, table, nbase, j, w, lane);
      }
      if (ok) store_rope(T, buf, w, lane);
      if (ok && prefetch) load_tail(T, p.kv, table, nbase, w, lane);
      // tile t+2's rows into L2 (bulk prefetch: no registers held), so that
      // next iteration's register loads of them return quickly
      if (ok && t + 2 < ntiles && (t + 2) / kTilesPerTable == t / kTilesPerTable && (lane & 7) == 0) {
        const int pb = ((t + 2) % kTilesPerTable) * TM;
#pragma unroll
        for (int rs = 0; rs < RS; ++rs) {
          const int code = table[pb + ROWS_PER_WARP * w + (lane >> 3) + 4 * rs];
          if (code >= 0) prefetch_l2(p.kv + (int64_t)code * ROW_BYTES, ROW_BYTES);
        }
      }
      if ((lane & 7) == 0) {  // which of this warp's rows count, for the softmax
#pragma unroll
        for (int rs = 0; rs < RS; ++rs) {
          const int row = ROWS_PER_WARP * w + (lane >> 3) + 4 * rs;
          s_valid[x * TM + row] = table[tbase + row] != kRowSkip ? 1 : 0;
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(mb_kv_full(x));
      have_next = prefetch;
    }
  } else if (warp == MMA_WARP) {
    // --------------------------------------------------------- MMA issue
    // Lane 0 issues QK(t) as soon as tile t is stored and PV(u) as soon as
    // P^T(u) is written, whichever comes first (the two touch different
    // buffers), so PV(t-1), which frees the buffer of tile t+1, never waits
    // for tile t. Polling is bounded: no progress for kWaitTimeoutNs aborts.
    if (lane == 0 && ntiles > 0) {
      int tq = 0, tp = 0;  // next tile to issue QK / PV for
      uint64_t t_idle = globaltimer_ns();
      uint32_t spins = 0;
      while (tp < ntiles) {
        bool progress = false;
        if (tq < ntiles && mbar_test(mb_kv_full(tq & 1), (tq >> 1) & 1)) {  // S^T(x) = KV(tq) . Q^T
          const int x = tq & 1;
          fence_after_sync();
          const uint64_t dk = desc_kv + x * kBufStep;
#pragma unroll
          for (int kb = 0; kb < 9; ++kb)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16_ss(tmem + S_COL + 64 * x, dk + ((kb * KV_REGION + 32 * k) >> 4),
                         desc_q + ((kb * Q_REGION + 32 * k) >> 4), IDESC_QK, (kb | k) != 0);
          mma_commit(mb_s_full(x));
          issued = true;
          ++tq;
          progress = true;
        }
        if (tp < tq && mbar_test(mb_p_full(tp & 1), (tp >> 1) & 1)) {  // O^T += V^T(tp) . P^T(tp)
          const int y = tp & 1;
          fence_after_sync();
          const uint64_t dv = desc_v + y * kBufStep, dp = desc_p + y * kBufStep;
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int s = 0; s < TM / 16; ++s)
              mma_f16_ss(tmem + 64 * j, dv + ((2 * j * KV_REGION + 2048 * s) >> 4), dp + ((2048 * s) >> 4), IDESC_PV,
                         (tp > 0 || s > 0) ? 1u : 0u);
          mma_commit(mb_kv_free(y));
          ++tp;
          progress = true;
        }
        if (progress) {
          t_idle = globaltimer_ns();
          spins = 0;
        } else if ((++spins & 255u) == 0) {
          if (*abort_flag) {
            ok = false;
            break;
          }
          if (globaltimer_ns() - t_idle > kWaitTimeoutNs) {
            *abort_flag = 1;
            if (err) atomicExch(err, (int32_t)DSA_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
    }
    __syncwarp();
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    issued = __shfl_sync(0xffffffffu, issued ? 1 : 0, 0) != 0;
  } else if (warp >= SOFTMAX0 && warp < SOFTMAX0 + SOFTMAX_WARPS) {
    // ---------------------------------------------------------- softmax
    const int s8 = warp - SOFTMAX0;                    // softmax warp 0..7
    const int sp = warp & 3;                           // TMEM sub-partition: lanes [32sp, 32sp + 16)
    const int hh = s8 >> 2;                            // heads [32hh, 32hh + 32)
    const int row = 16 * sp + (lane >> 2) + 8 * (lane & 1);  // tile row of this thread (16x64b layout)
    const int par = (lane >> 1) & 1;
    const int hbase = 32 * hh + par;                   // this thread's heads: hbase + 2i, i < 16
    const bool head_row = ((lane >> 2) + 8 * (lane & 1)) == 0;  // lanes 0 and 2: first row of the group
    const uint32_t t_sp = tmem + ((uint32_t)(32 * sp) << 16);
    float L[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) L[i] = 0.f;
    for (int t = 0; t < ntiles; ++t) {
      const int x = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      ok = ok && mbar_wait(mb_s_full(x), ph, abort_flag, err, kWaitTimeoutNs) &&
           mbar_wait(mb_kv_full(x), ph, abort_flag, err, kWaitTimeoutNs);
      ok = __all_sync(0xffffffffu, ok);
      fence_after_sync();
      uint32_t s[16];
      if (ok) {
        tmem_ld16x32(t_sp + S_COL + 64 * x + 32 * hh, s);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) s[i] = 0u;
      }
      const bool vrow = s_valid[x * TM + row] != 0;
      // in place: score (log2 units) - running max
      bool over = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float v = (vrow ? __uint_as_float(s[i]) * scale_log2 : -INFINITY) - m_ref[hbase + 2 * i];
        s[i] = __float_as_uint(v);
        over |= v > kRescaleThreshold;
      }
      const unsigned vote = __ballot_sync(0xffffffffu, over);
      if (lane == 0) ovf[x * 8 + s8] = vote != 0u;
      named_bar(1, SOFTMAX_WARPS * 32);
      int any_ovf = 0;
#pragma unroll
      for (int k = 0; k < SOFTMAX_WARPS; ++k) any_ovf |= ovf[x * 8 + k];
      if (any_ovf) {
        // exact tile maxima per head (S^T read again); heads whose max grew by
        // more than 2^8 move their running max and rescale what was accumulated
        if (ok) {
          tmem_ld16x32(t_sp + S_COL + 64 * x + 32 * hh, s);
          tmem_wait_ld();
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float v = vrow ? __uint_as_float(s[i]) * scale_log2 : -INFINITY;
          s[i] = __float_as_uint(v);
          uint32_t m = monotone32(v);
          m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
          m = max(m, __shfl_xor_sync(0xffffffffu, m, 4));
          m = max(m, __shfl_xor_sync(0xffffffffu, m, 8));
          m = max(m, __shfl_xor_sync(0xffffffffu, m, 16));
          if (head_row) tmax[sp * 64 + hbase + 2 * i] = unmono(m);
        }
        named_bar(1, SOFTMAX_WARPS * 32);
        if (s8 == 0) {
          bool moved = false;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int head = lane + 32 * k;
            const float tm = fmaxf(fmaxf(tmax[head], tmax[64 + head]), fmaxf(tmax[128 + head], tmax[192 + head]));
            const float m_old = m_ref[head];
            float a = 1.f;
            if (tm > m_old + kRescaleThreshold) {
              a = ex2(m_old - tm);
              m_ref[head] = tm;
              moved = true;
            }
            alpha[head] = a;
          }
          const unsigned any = __ballot_sync(0xffffffffu, moved);
          if (lane == 0) *any_rescale = any != 0u;
        }
        named_bar(1, SOFTMAX_WARPS * 32);
        if (*any_rescale && t > 0) {
          // O^T holds PV(0..t-1): rescale after PV(t-1) has completed; this
          // warp takes columns [128hh, 128hh + 128) of its sub-partition's lanes
          const int u = t - 1;
          ok = ok && mbar_wait(mb_kv_free(u & 1), (u >> 1) & 1, abort_flag, err, kWaitTimeoutNs);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            fence_after_sync();
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
              const int col = 128 * hh + 16 * c;  // heads (col % 64) ..
              uint32_t o[16];
              tmem_ld16(t_sp + col, o);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[(col + h) & 63]);
              tmem_st16(t_sp + col, o);
            }
            tmem_wait_st();
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          s[i] = __float_as_uint(__uint_as_float(s[i]) - m_ref[hbase + 2 * i]);
          L[i] *= alpha[hbase + 2 * i];
        }
      }
      // probabilities and row sums
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float pe = ex2(__uint_as_float(s[i]));
        s[i] = __float_as_uint(pe);
        L[i] += pe;
      }
      // P^T row `row`, heads [32hh, 32hh + 32): the even-parity thread writes
      // the first 16, its partner (lane ^ 2) the last 16, each pairing its
      // values with the partner's; 16-byte chunks of 8 heads
      uint8_t* preg = sm + SM_KV + x * KV_BUF + 8 * KV_REGION;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 4 * c + e;
          const float lo_v = __uint_as_float(s[j]), hi_v = __uint_as_float(s[8 + j]);
          const float recv = __shfl_xor_sync(0xffffffffu, par ? lo_v : hi_v, 2);
          pk[e] = par ? pack_half2(recv, hi_v) : pack_half2(lo_v, recv);
        }
        if (ok)
          *reinterpret_cast<uint4*>(preg + sw128_off(row, 4 * hh + 2 * par + c)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      fence_proxy_async();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(mb_p_full(x));
    }
    // per-head sums over this sub-partition's rows (threads of one parity)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v = L[i];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      L[i] = v;
    }
    named_bar(1, SOFTMAX_WARPS * 32);  // every warp is past its last use of tmax as tile maxima
    if (head_row) {
#pragma unroll
      for (int i = 0; i < 16; ++i) tmax[sp * 64 + hbase + 2 * i] = L[i];
    }
  }
  // -------------------------------------------------------------- epilogue
  __syncthreads();
  if (ok && ntiles > 0)  // the last PV has completed
    ok = mbar_wait(mb_kv_free((ntiles - 1) & 1), ((ntiles - 1) >> 1) & 1, abort_flag, err, kWaitTimeoutNs);
  __syncthreads();
  // A thread whose wait failed set the abort flag before this barrier, so
  // every thread reads the same decision; nothing sets it after this point.
  const bool live = *abort_flag == 0;
  const bool have_o = live && ntiles > 0;  // O^T holds this slice's accumulation
  const int sp = warp & 3;                 // TMEM sub-partition: lanes [32*sp, 32*sp+32)
  const uint32_t t_lane = (uint32_t)(32 * sp) << 16;
  if (threadIdx.x < NH)
    l_sum[threadIdx.x] =
        have_o ? (tmax[threadIdx.x] + tmax[64 + threadIdx.x]) + (tmax[128 + threadIdx.x] + tmax[192 + threadIdx.x])
               : 0.f;
  fence_after_sync();
  if (csize == 1 && p.n_splits > 1) {
    // ------------------------------------------- partial state of this slice
    // O^T is staged as [64 heads][512 dims] f32 (128 KB) in the free tile
    // buffers, then each head's 2 KB row leaves with one bulk copy.
    __syncthreads();
    float* stg = reinterpret_cast<float*>(sm + SM_KV);
    const int hb = 16 * ((warp >> 2) & 3);  // heads [hb, hb + 16), for warps 0-15
#pragma unroll 1
    for (int j = 0; j < 4 && warp < 16; ++j) {
      uint32_t o[16];
      if (have_o) {
        tmem_ld16(tmem + t_lane + 64 * j + hb, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = 0u;
      }
      const int d = 128 * j + 32 * sp + lane;
#pragma unroll
      for (int h = 0; h < 16; ++h) stg[(hb + h) * DV + d] = __uint_as_float(o[h]);
    }
    fence_proxy_async();  // the staged rows are read by the bulk copies
    __syncthreads();
    if ((int)threadIdx.x < min(NH, p.n_head - h0)) {
      float* dst = p.part_o + (((int64_t)b * p.n_head + h0 + threadIdx.x) * p.n_splits + split) * DV;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                   "r"(smem_u32(stg + threadIdx.x * DV)), "r"((uint32_t)(DV * 4))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // written before the CTA moves on
    }
    if (threadIdx.x < NH && h0 + (int)threadIdx.x < p.n_head) {
      const int64_t bh = (int64_t)b * p.n_head + h0 + threadIdx.x;
      p.part_ml[(bh * p.n_splits + split) * 2] = m_ref[threadIdx.x];
      p.part_ml[(bh * p.n_splits + split) * 2 + 1] = l_sum[threadIdx.x];
    }
  } else {
    // ------------------------------------------------- final o and lse
    // The csize slices of this row form one cluster; CTA `rank` owns value
    // dims [rank*W, rank*W + W). Each CTA sends the raw O^T rows that other
    // CTAs own into their shared memory (the tile buffers are free by now),
    // then combines its own rows with what it received: the flash-decode
    // reduction o = sum_s w_s o_s / sum_s w_s l_s, w_s = 2^(m_s - max m) over
    // slices with l_s > 0 (dsa.cu:1136-1184), with lse = -inf and o = 0 when
    // nothing was counted.
    const int W = DV / csize;
    const uint32_t rank = csize > 1 ? cluster_rank() : 0u;
    const uint32_t xbytes = (uint32_t)W * 256;  // one sender's rows: [W dims][64 heads] f32, 16-byte chunks XOR-swizzled by dim
    uint8_t* xbuf = sm + SM_KV;                   // [csize - 1 senders] received rows
    uint8_t* ybuf = xbuf + (csize - 1) * xbytes;  // [64 heads][W dims] in o's type
    uint8_t* gbuf = sm + SM_KV + kSendOff;        // [csize - 1 receivers] rows to send
    float* fac = tmax;                            // [csize][64] w_s / sum (tmax is dead once l_sum is formed)
    const int g = warp >> 2;  // 8 warps per sub-partition: chunks g and g + 8 of its 16 (tile j, 16 heads)
    if (csize > 1) {
      // stage the rows other CTAs own, one contiguous block per receiver
#pragma unroll 1
      for (int c = g; c < 16; c += 8) {
        const int j = c >> 2, cb = c & 3;
        const int dv0 = 128 * j + 32 * sp;  // this warp's 32 dims
        const int owner = dv0 / W;
        if (owner == (int)rank) continue;
        uint32_t o[16];
        if (have_o) {
          tmem_ld16(tmem + t_lane + 64 * j + 16 * cb, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int h = 0; h < 16; ++h) o[h] = 0u;
        }
        const int oi = owner < (int)rank ? owner : owner - 1;
        const int dl = dv0 + lane - owner * W;
        uint8_t* row = gbuf + oi * xbytes + dl * 256;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          *reinterpret_cast<uint4*>(row + (((4 * cb + e) ^ (dl & 15)) << 4)) =
              make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
      }
      fence_proxy_async();  // the staged rows are read by the bulk copies
      if (threadIdx.x == 0) mbar_arrive_expect_tx(mb_recv, (uint32_t)(csize - 1) * xbytes);
      cluster_sync();  // every CTA of the cluster is past its tile loop, its m, l published and rows staged
      if (threadIdx.x < (unsigned)(csize - 1)) {
        const int oi = threadIdx.x;
        const int owner = oi < (int)rank ? oi : oi + 1;
        const int slot = (int)rank < owner ? (int)rank : (int)rank - 1;
        const uint32_t dst = cluster_map(smem_u32(xbuf + slot * xbytes), owner);
        const uint32_t mb = cluster_map(mb_recv, owner);
        for (uint32_t off = 0; off < xbytes; off += 16384u)
          bulk_copy_to_peer(dst + off, smem_u32(gbuf + oi * xbytes) + off, 16384u, mb);
      }
    } else {
      __syncthreads();
    }
    if (threadIdx.x < NH) {
      const int h = threadIdx.x;
      auto m_of = [&](int q) { return csize > 1 ? ld_cluster_f32(cluster_map(smem_u32(&m_ref[h]), q)) : m_ref[h]; };
      auto l_of = [&](int q) { return csize > 1 ? ld_cluster_f32(cluster_map(smem_u32(&l_sum[h]), q)) : l_sum[h]; };
      float M = -INFINITY;
      for (int q = 0; q < csize; ++q)
        if (l_of(q) > 0.f) M = fmaxf(M, m_of(q));
      float L = 0.f;
      for (int q = 0; q < csize; ++q) {
        const float l = l_of(q);
        const float w = l > 0.f ? exp2f(m_of(q) - M) : 0.f;
        fac[q * 64 + h] = w;
        L += l * w;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      for (int q = 0; q < csize; ++q) fac[q * 64 + h] *= inv;
      if (rank == 0 && h0 + h < p.n_head)
        p.lse[(int64_t)b * p.n_head + h0 + h] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
    __syncthreads();  // fac visible
    if (csize > 1) mbar_wait(mb_recv, 0, abort_flag, err, kWaitTimeoutNs);  // received rows landed
    const int ybytes = W * 2;  // one head's row of ybuf
#pragma unroll 1
    for (int c = g; c < 16; c += 8) {
      const int j = c >> 2, cb = c & 3;
      const int dv0 = 128 * j + 32 * sp;
      if (dv0 / W != (int)rank) continue;
      uint32_t o[16];
      if (have_o) {
        tmem_ld16(tmem + t_lane + 64 * j + 16 * cb, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) o[h] = 0u;
      }
      // o[] becomes the combined value in place (f32 bits)
#pragma unroll
      for (int h = 0; h < 16; ++h) o[h] = __float_as_uint(fac[rank * 64 + 16 * cb + h] * __uint_as_float(o[h]));
      const int dl = dv0 + lane - (int)rank * W;
      for (int q = 0; q < csize; ++q) {
        if (q == (int)rank) continue;
        const int slot = q < (int)rank ? q : q - 1;
        const uint8_t* row = xbuf + ((size_t)slot * W + dl) * 256;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 v = *reinterpret_cast<const float4*>(row + (((4 * cb + e) ^ (dl & 15)) << 4));
          const float* f = fac + q * 64 + 16 * cb + 4 * e;
          o[4 * e] = __float_as_uint(fmaf(f[0], v.x, __uint_as_float(o[4 * e])));
          o[4 * e + 1] = __float_as_uint(fmaf(f[1], v.y, __uint_as_float(o[4 * e + 1])));
          o[4 * e + 2] = __float_as_uint(fmaf(f[2], v.z, __uint_as_float(o[4 * e + 2])));
          o[4 * e + 3] = __float_as_uint(fmaf(f[3], v.w, __uint_as_float(o[4 * e + 3])));
        }
      }
      uint8_t* y = ybuf + 16 * cb * ybytes + dl * 2;
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        if (p.o_bf16)
          *reinterpret_cast<__nv_bfloat16*>(y + h * ybytes) = __float2bfloat16_rn(__uint_as_float(o[h]));
        else
          *reinterpret_cast<__half*>(y + h * ybytes) = __float2half_rn(__uint_as_float(o[h]));
      }
    }
    __syncthreads();
    // 16-byte coalesced stores of this CTA's W dims of every head
    const int cpr = W / 8;  // 16-byte chunks per head
    for (int i = threadIdx.x; i < NH * cpr; i += NTHREADS) {
      const int h = i / cpr, c8 = i % cpr;
      if (h0 + h >= p.n_head) continue;
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.o) +
                                (((int64_t)b * p.n_head + h0 + h) * DV + (int)rank * W + 8 * c8) * 2) =
          *reinterpret_cast<const uint4*>(ybuf + h * ybytes + c8 * 16);
    }
    if (csize > 1) cluster_sync();  // every copy out of this CTA's memory has landed before it exits
  }
  // every MMA of this CTA has completed before TMEM is released (a commit
  // tracks the MMAs of the thread that issues it: lane 0 of the MMA warp
  // issued all)
  if (warp == MMA_WARP && issued && !live) {
    if (lane == 0) mma_commit(mb_done);
    __syncwarp();
    mbar_wait_drain(mb_done, 0, kWaitTimeoutNs);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];
int32_t* g_err_ptr[kMaxDevices];
int g_cluster_ctas[kMaxDevices][3];  // [log2 csize]: CTAs resident at once in clusters of csize (0: unusable)

int ensure_setup(int dev) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("sparse_mla_decode_tc: device index %d out of range", dev);
    return DSA_ERR_UNSUPPORTED;
  }
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(sparse_mla_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES);
    void* ptr = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&ptr, g_tc_error);
    g_err_ptr[dev] = reinterpret_cast<int32_t*>(ptr);
    g_status[dev] = (int)e;
    g_cluster_ctas[dev][0] = sm_count(dev);
    for (int l = 1; l < 3 && e == cudaSuccess; ++l) {
      const int c = 1 << l;
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(1, 1, 16 * c);
      cfg.blockDim = dim3(NTHREADS);
      cfg.dynamicSmemBytes = SMEM_BYTES;
      cudaLaunchAttribute attr{};
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 1;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = c;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, sparse_mla_decode_tc_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();  // a refused size only disables that size
        n = 0;
      }
      g_cluster_ctas[dev][l] = n * c;
    }
  });
  if (g_status[dev] != 0) {
    set_error("sparse_mla_decode_tc setup: %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

int log2_csize(int n_splits) { return n_splits == 2 ? 1 : n_splits == 4 ? 2 : -1; }  // the epilogue layout holds 4

}  // namespace

int tc_cluster_size(int n_splits) {
  const int l = log2_csize(n_splits);
  if (l < 0) return 1;
  const int dev = current_device();
  if (ensure_setup(dev) != DSA_OK) return 1;
  return g_cluster_ctas[dev][l] > 0 ? n_splits : 1;
}

int tc_choose_splits(int B, int head_tiles, int topk, int nsm) {
  const int ntiles = (topk + TM - 1) / TM;
  if (ntiles <= 1) return 1;
  const double units = (double)B * head_tiles;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 32 && s <= ntiles; ++s) {
    const int per = (ntiles + s - 1) / s;
    if ((ntiles + per - 1) / per != s) continue;
    // slices of a row merge in a cluster (s = 2, 4, 8, when clusters of s
    // fit) or through partial states that a second kernel re-reads
    const bool cl = s > 1 && tc_cluster_size(s) == s;
    int cap = nsm;
    if (cl) cap = g_cluster_ctas[current_device()][log2_csize(s)];
    const double waves = std::ceil(units * s / std::max(cap, 1));
    // cost in tile times: a tile of TM fp8 rows moves TM x 656 B; each wave
    // adds about one tile of setup and epilogue; a partial state is written
    // (one bulk copy per head) and merged (2 x 128 KB), which streams at
    // about twice the rate of a gathered tile (B = 8, 64 heads: 16 slices
    // 24.5 us, 8 slices 27.4 us, 4 slices in clusters 39.4 us)
    double cost = waves * (per + 1.0);
    if (s > 1 && !cl) cost += 0.5 * units * s * 2.0 * NH * DV * 4.0 / ((double)nsm * TM * ROW_BYTES);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

int launch_sparse_mla_tc(const SparseMlaArgs& a, cudaStream_t s) {
  const int dev = current_device();
  int st = ensure_setup(dev);
  if (st != DSA_OK) return st;
  const int csize = a.n_splits > 1 ? tc_cluster_size(a.n_splits) : 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.B, (a.n_head + NH - 1) / NH, a.n_splits);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = csize;
  cfg.attrs = &attr;
  cfg.numAttrs = csize > 1 ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, sparse_mla_decode_tc_kernel, a, g_err_ptr[dev], csize);
  if (e != cudaSuccess) {
    set_error("sparse_mla_decode_tc_kernel launch: %s", cudaGetErrorString(e));
    return DSA_ERR_CUDA;
  }
  return check_launch("sparse_mla_decode_tc_kernel");
}

int tc_error_word(int dev, int32_t** out) {
  const int st = ensure_setup(dev);
  if (st != DSA_OK) return st;
  *out = g_err_ptr[dev];
  return DSA_OK;
}

}  // namespace dsa

namespace dsa {
namespace {
// One mbarrier whose phase needs two arrivals and gets one: every thread's
// bounded wait runs out, records DSA_ERR_TIMEOUT in the status word and
// returns (the same wait every tensor-core kernel of the library uses).
__global__ void selftest_wait_kernel(int32_t* err, int64_t timeout_ns) {
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int abort_flag;
  const uint32_t mb = smem_u32(&mbar);
  if (threadIdx.x == 0) {
    tc::mbar_init(mb, 2);
    tc::mbar_init_fence();
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) tc::mbar_arrive(mb);
  tc::mbar_wait(mb, 0, &abort_flag, err, (uint64_t)timeout_ns);
}
}  // namespace
}  // namespace dsa

extern "C" int dsa_selftest_wait_timeout(int64_t timeout_ns, void* stream) {
  dsa::clear_error();
  DSA_REQUIRE(timeout_ns >= 1000 && timeout_ns <= 1000000000LL, DSA_ERR_INVALID,
              "selftest_wait_timeout: timeout must be in [1 us, 1 s]");
  const int dev = dsa::current_device();
  int32_t* err = nullptr;
  const int st = dsa::tc_error_word(dev, &err);
  if (st != DSA_OK) return st;
  dsa::selftest_wait_kernel<<<1, 32, 0, dsa::as_stream(stream)>>>(err, timeout_ns);
  return dsa::check_launch("selftest_wait_kernel");
}

extern "C" int dsa_device_error(int reset) {
  dsa::clear_error();
  int32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, dsa::g_tc_error, sizeof(v));
  if (e != cudaSuccess) {
    dsa::set_error("dsa_device_error: %s", cudaGetErrorString(e));
    return -DSA_ERR_CUDA;
  }
  if (reset && v != 0) {
    const int32_t z = 0;
    cudaMemcpyToSymbol(dsa::g_tc_error, &z, sizeof(z));
  }
  return v;
}
