// Sparse MLA decode / prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), for the fp8_ds_mla latent cache.
//
// Same function as the reference's split decode + merge
// (csrc/attention/sm70_mla_decode.cu:918-1184) and prefill kernels
// (:1563-2051); see sparse_mla_decode.cu for the semantics.
//
// One CTA = one query row x 64 heads x one slice of the top-k axis, processed
// in tiles of 128 selected latent rows. The MMAs are "transposed" so that the
// 128 latent rows are the M side (full-rate M = 128 tcgen05 tiles) and the 64
// heads are N:
//   S^T[128 x 64]  = KV[128 x 576] . Q^T        (A = KV tile, K-major smem;
//                                                 B = Q, K-major smem)
//   O^T[512 x 64] += V^T[512 x 128] . P^T        (A = same KV tile read
//                                                 MN-major; B = P^T, MN-major)
// S^T and O^T live in tensor memory (64 + 256 columns). The KV tile is stored
// once as fp16 in 128-byte-swizzled rows that serve both as K-major A of QK
// and MN-major A of PV; P^T (fp16) overwrites the tile's rope columns after QK
// has consumed them, which keeps Q (72 KB) + tile (144 KB) within one SM.
//
// Block of 8 warps (256 threads, so up to 255 registers per thread). Warp 0
// allocates TMEM and its lane 0 issues the MMAs between block barriers. As
// producers, all warps gather the next tile's 656-B rows with coalesced
// 16-byte loads into registers while the current tile is in the tensor core,
// then dequantise (e4m3 x per-128 scale -> fp16) into the swizzled tile. As
// softmax warps, each thread owns one latent row and 32 heads of S^T
// (tcgen05.ld), computes per-head tile maxima with warp reductions, and keeps
// a lazily-updated running max: O^T is rescaled in TMEM only when a head's max
// grows by more than 2^8, which keeps P <= 256 in fp16 while leaving o and lse
// exact. Row sums accumulate per thread in spare TMEM columns and are reduced
// once at the end. Every wait on the tensor core is an mbarrier wait bounded
// by a device-time limit that reports DSA_ERR_TIMEOUT instead of hanging.
#include "sparse_mla.cuh"
#include "tc_common.cuh"

namespace dsa {
namespace {

using namespace tc;

constexpr int TM = kTcTileRows;   // 128 latent rows per tile (MMA M)
constexpr int NH = 64;            // heads per CTA (MMA N)
constexpr int NWORK = 8;          // warps; all of them produce tiles and run the softmax
constexpr int NTHREADS = 32 * NWORK;
constexpr int DV = 512;
constexpr uint32_t KV_REGION = TM * 128;   // one 64-wide K block of the tile: 16 KB
constexpr uint32_t Q_REGION = NH * 128;    // one 64-wide K block of Q: 8 KB
constexpr uint32_t SM_KV = 0;
constexpr uint32_t SM_Q = 9 * KV_REGION;
constexpr uint32_t SM_MISC = SM_Q + 9 * Q_REGION;
constexpr uint32_t MISC_BYTES = 4096;
constexpr uint32_t SMEM_BYTES = SM_MISC + MISC_BYTES + 1024;  // + alignment slack
constexpr uint32_t S_COL = 256;            // S^T columns [256, 320); O^T tile j at [64j, 64j+64)
constexpr uint32_t L_COL = 320;            // running row sums of P: columns [320, 384)
constexpr uint32_t TMEM_COLS = 512;
constexpr int ROW_BYTES = 656;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

constexpr uint32_t IDESC_QK = idesc_f16(128, NH, false, false);
constexpr uint32_t IDESC_PV = idesc_f16(128, NH, true, true);

__device__ int32_t g_tc_error;  // sticky: DSA_ERR_TIMEOUT when a bounded wait expired

__device__ __forceinline__ float unmono(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

// One warp's share of a tile: rows 16*w + (lane >> 3) + 4*rs (rs = 0..3).
// Lane l holds, for each of its 4 rows, the nope chunk (l & 7) + 8*j of every
// 128-wide scale group j (one 16-byte chunk = 16 e4m3 per group), the row's
// four tile scales, and rope chunk (l & 7). Loads of 8 consecutive lanes cover
// 128 contiguous bytes of a row.
struct Tile {
  uint4 nope[4][4];  // [rs][j]
  float4 sc[4];      // [rs] scales of groups 0..3
  uint4 rope[4];     // [rs]
  int my_valid;      // lanes 0-15: row 16*w + lane is a counted position
};

__device__ __forceinline__ float sc_of(const float4& s, int j) {
  return j == 0 ? s.x : (j == 1 ? s.y : (j == 2 ? s.z : s.w));
}

// Resolve + issue the global loads of this warp's 16 rows of a tile.
__device__ __forceinline__ void load_tile(Tile& T, const SparseMlaArgs& p, int b, int j0, int hi, int seq_len,
                                          int w, int lane) {
  int64_t my_row = -1;
  T.my_valid = 0;
  if (lane < 16) {
    const int j = j0 + 16 * w + lane;
    if (j < hi) {
      const int pos = p.idx[(int64_t)b * p.idx_stride + j];
      if (pos >= 0 && pos < seq_len) {
        T.my_valid = 1;
        const int blk_i = pos / p.page_size;
        if (blk_i < p.max_blocks) {
          const int64_t r = (int64_t)p.bt[(int64_t)b * p.bt_stride + blk_i] * p.page_size + (pos - blk_i * p.page_size);
          if (r >= 0 && r < p.n_kv_rows) my_row = r * ROW_BYTES;
        }
      }
    }
  }
#pragma unroll
  for (int rs = 0; rs < 4; ++rs) {
    const int64_t off = __shfl_sync(0xffffffffu, my_row, (lane >> 3) + 4 * rs);
    if (off >= 0) {
      const uint8_t* row = p.kv + off;
#pragma unroll
      for (int j = 0; j < 4; ++j) T.nope[rs][j] = ldg_nc16(row + 16 * ((lane & 7) + 8 * j));
      const uint4 s = ldg_nc16(row + 512);
      T.sc[rs] = make_float4(__uint_as_float(s.x), __uint_as_float(s.y), __uint_as_float(s.z), __uint_as_float(s.w));
      T.rope[rs] = ldg_nc16(row + 528 + 16 * (lane & 7));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) T.nope[rs][j] = make_uint4(0, 0, 0, 0);
      T.sc[rs] = make_float4(0.f, 0.f, 0.f, 0.f);
      T.rope[rs] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Two e4m3 bytes (in the low byte of each 16-bit half of x) -> half2 holding
// value/256 exactly: sign to bit 15, exponent+mantissa shifted into the fp16
// field (e4m3 bias 7 vs fp16 bias 15 is the 2^8 factor; e4m3 subnormals land
// on fp16 subnormals). Integer ops only, so the conversion stays off the
// (narrow) conversion pipe.
__device__ __forceinline__ uint32_t e4m3x2_div256(uint32_t x) {
  return ((x << 8) & 0x80008000u) | ((x << 7) & 0x3F803F80u);
}

// e4m3 x 8 (two words) times scale -> 8 fp16 (uint4).
__device__ __forceinline__ uint4 dequant8(uint32_t w0, uint32_t w1, float sc) {
  const uint32_t q[4] = {e4m3x2_div256(__byte_perm(w0, 0, 0x4140)), e4m3x2_div256(__byte_perm(w0, 0, 0x4342)),
                         e4m3x2_div256(__byte_perm(w1, 0, 0x4140)), e4m3x2_div256(__byte_perm(w1, 0, 0x4342))};
  uint4 o;
  const float s256 = sc * 256.0f;
  if (s256 >= 6.2e-5f && s256 <= 32768.0f) {  // scale*256 and every product stay normal in fp16
    const __half2 s2 = __float2half2_rn(s256);
    __half2 r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = __hmul2(*reinterpret_cast<const __half2*>(&q[e]), s2);
    o = make_uint4(*reinterpret_cast<uint32_t*>(&r[0]), *reinterpret_cast<uint32_t*>(&r[1]),
                   *reinterpret_cast<uint32_t*>(&r[2]), *reinterpret_cast<uint32_t*>(&r[3]));
  } else {
    uint32_t r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[e]));
      r[e] = pack_half2(f.x * s256, f.y * s256);
    }
    o = make_uint4(r[0], r[1], r[2], r[3]);
  }
  return o;
}

// Store scale group j (K blocks 2j, 2j+1) of this warp's rows.
__device__ __forceinline__ void store_group(const Tile& T, uint8_t* sm, int j, int w, int lane) {
  const int c = (lane & 7) + 8 * j;  // nope chunk: e4m3 values [16c, 16c+16)
  uint8_t* region = sm + SM_KV + (c >> 2) * KV_REGION;
  const int c0 = 2 * (c & 3);
#pragma unroll
  for (int rs = 0; rs < 4; ++rs) {
    const int i = 16 * w + (lane >> 3) + 4 * rs;
    const float sc = sc_of(T.sc[rs], j);
    *reinterpret_cast<uint4*>(region + sw128_off(i, c0)) = dequant8(T.nope[rs][j].x, T.nope[rs][j].y, sc);
    *reinterpret_cast<uint4*>(region + sw128_off(i, c0 + 1)) = dequant8(T.nope[rs][j].z, T.nope[rs][j].w, sc);
  }
}

__device__ __forceinline__ void store_rope(const Tile& T, uint8_t* sm, uint8_t* valid, int w, int lane) {
#pragma unroll
  for (int rs = 0; rs < 4; ++rs)
    *reinterpret_cast<uint4*>(sm + SM_KV + 8 * KV_REGION + sw128_off(16 * w + (lane >> 3) + 4 * rs, lane & 7)) =
        T.rope[rs];
  if (lane < 16) valid[16 * w + lane] = (uint8_t)T.my_valid;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(NTHREADS, 1) sparse_mla_decode_tc_kernel(const SparseMlaArgs p, int32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw_base);
  uint8_t* misc = sm + SM_MISC;
  // mbarriers: [0..4] kv_full (groups 0..3, rope), [5..8] kv_free (PV tile j), [9] s_full, [10] done
  uint64_t* mbar = reinterpret_cast<uint64_t*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 96);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 100);
  int* ovf = reinterpret_cast<int*>(misc + 104);           // [2][4] per-warp "score above running max" votes
  int* any_rescale = reinterpret_cast<int*>(misc + 136);   // [2]
  float* m_ref = reinterpret_cast<float*>(misc + 256);     // [64] running max (log2 units)
  float* alpha = m_ref + 64;                               // [64] this tile's rescale factors
  float* tmax = alpha + 64;                                // [2][4][32] per-warp tile maxima
  float* l_sum = tmax + 256;                               // [64]
  uint8_t* valid = reinterpret_cast<uint8_t*>(l_sum + 64); // [128]
  const uint32_t mb0 = smem_u32(&mbar[0]);
  auto mb_kv_full = [&](int j) { return mb0 + 8u * (uint32_t)j; };
  auto mb_kv_free = [&](int j) { return mb0 + 8u * (uint32_t)(5 + j); };
  const uint32_t mb_s_full = mb0 + 8u * 9, mb_done = mb0 + 8u * 10;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int h0 = blockIdx.y * NH;
  const int split = blockIdx.z;
  const int seq_len = p.seq_lens[b];
  const int lo = split * p.span;
  const int hi = min(lo + p.span, p.topk);
  const int ntiles = hi > lo ? (hi - lo + TM - 1) / TM : 0;
  const bool issuer = threadIdx.x == 0;  // lane 0 of warp 0 issues every MMA

  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < 5; ++j) mbar_init(mb_kv_full(j), NWORK);
      for (int j = 0; j < 4; ++j) mbar_init(mb_kv_free(j), 1);
      mbar_init(mb_s_full, 1);
      mbar_init(mb_done, 1);
      mbar_init_fence();
      *abort_flag = 0;
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
  }
  {
    const int nheads = min(NH, p.n_head - h0);
    for (int i = threadIdx.x; i < NH * 72; i += NTHREADS) {
      const int h = i / 72, c = i % 72;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h < nheads) {
        v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.q) +
                                            (((int64_t)b * p.n_head + h0 + h) * 576 + 8 * c) * 2);
        if (p.q_bf16) v = bf16x8_to_half8(v);
      }
      *reinterpret_cast<uint4*>(sm + SM_Q + (c >> 3) * Q_REGION + sw128_off(h, c & 7)) = v;
    }
    if (threadIdx.x < NH) {
      m_ref[threadIdx.x] = -1e30f;
      alpha[threadIdx.x] = 1.f;
    }
  }
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  const int w = warp;                // producer: rows 16*w .. 16*w + 15 of a tile
  const int sp = warp & 3;           // TMEM sub-partition: lanes [32*sp, 32*sp+32)
  const int hh = warp >> 2;          // softmax head half: heads [32*hh, 32*hh+32)
  const int row_s = 32 * sp + lane;  // the tile row this thread owns in the softmax
  const uint32_t t_lane = (uint32_t)(32 * sp) << 16;
  // The running row sums of P live in TMEM columns [L_COL + 32*hh, +32) of
  // this thread's lane (one latent-row slot x 32 heads), not in registers.
  Tile T;
  if (ntiles > 0) load_tile(T, p, b, lo, hi, seq_len, w, lane);
  // Control flow is uniform across the block: after a timed-out wait (`ok`
  // false, abort flag set) every warp still executes the same sequence of
  // barriers and arrivals, and every later wait returns at once.
  bool ok = true;
  bool issued = false;
  for (int t = 0; t < ntiles; ++t) {
    const uint32_t ph = t & 1;
    // ---- store tile t group by group as PV(t-1) releases it; QK(t) follows each group
    // (unrolled: the tile registers are indexed by the group)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (t > 0) ok = ok && mbar_wait(mb_kv_free(j), ph ^ 1, abort_flag, err, kWaitTimeoutNs);
      if (ok) store_group(T, sm, j, w, lane);
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(mb_kv_full(j));
      if (issuer) {
        ok = ok && mbar_wait(mb_kv_full(j), ph, abort_flag, err, kWaitTimeoutNs);
        if (ok) {
          fence_after_sync();
#pragma unroll
          for (int kb = 2 * j; kb < 2 * j + 2; ++kb)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t a = sw128_desc(base + SM_KV + kb * KV_REGION + 32 * k, 16, 1024);
              const uint64_t bq = sw128_desc(base + SM_Q + kb * Q_REGION + 32 * k, 16, 1024);
              mma_f16_ss(tmem + S_COL, a, bq, IDESC_QK, (kb | k) != 0);
            }
          issued = true;
        }
      }
      __syncwarp();
    }
    // rope group: its region held P^T(t-1), released when all of PV(t-1) is done (kv_free[3])
    if (ok) store_rope(T, sm, valid, w, lane);
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(mb_kv_full(4));
    if (issuer) {
      ok = ok && mbar_wait(mb_kv_full(4), ph, abort_flag, err, kWaitTimeoutNs);
      if (ok) {
        fence_after_sync();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = sw128_desc(base + SM_KV + 8 * KV_REGION + 32 * k, 16, 1024);
          const uint64_t bq = sw128_desc(base + SM_Q + 8 * Q_REGION + 32 * k, 16, 1024);
          mma_f16_ss(tmem + S_COL, a, bq, IDESC_QK, 1u);
        }
        mma_commit(mb_s_full);
      }
    }
    __syncwarp();
    // ---- next tile's loads stay in flight through softmax(t) and PV(t)
    if (ok && t + 1 < ntiles) load_tile(T, p, b, lo + (t + 1) * TM, hi, seq_len, w, lane);

    // ---- softmax(t)
    ok = ok && mbar_wait(mb_s_full, ph, abort_flag, err, kWaitTimeoutNs);
    __syncthreads();  // validity bytes of tile t (written with the rope group) are visible
    fence_after_sync();
    float v[32];
    {
      uint32_t sreg[32];
      if (ok) {
        tmem_ld32(tmem + t_lane + S_COL + 32 * hh, sreg);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int h = 0; h < 32; ++h) sreg[h] = 0u;
      }
      const bool vrow = valid[row_s] != 0;
      bool over = false;
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        v[h] = vrow ? __uint_as_float(sreg[h]) * p.scale_log2 : -INFINITY;
        over |= v[h] > m_ref[32 * hh + h] + kRescaleThreshold;
      }
      const unsigned vote = __ballot_sync(0xffffffffu, over);
      if (lane == 0) ovf[hh * 4 + sp] = vote != 0u;
    }
    named_bar(1 + hh, 128);
    const bool slow = ovf[hh * 4] | ovf[hh * 4 + 1] | ovf[hh * 4 + 2] | ovf[hh * 4 + 3];
    if (slow) {
      // exact tile maxima of this head half; heads whose max grew by more than
      // 2^8 move their running max and rescale what was accumulated
      uint32_t my_max = 0;
#pragma unroll
      for (int h = 0; h < 32; ++h) {
        const uint32_t wm = __reduce_max_sync(0xffffffffu, monotone32(v[h]));
        if (lane == h) my_max = wm;
      }
      tmax[(hh * 4 + sp) * 32 + lane] = unmono(my_max);
      named_bar(1 + hh, 128);
      if (sp == 0) {
        const int head = 32 * hh + lane;
        float tm = tmax[(hh * 4) * 32 + lane];
#pragma unroll
        for (int s = 1; s < 4; ++s) tm = fmaxf(tm, tmax[(hh * 4 + s) * 32 + lane]);
        const float m_old = m_ref[head];
        float a = 1.f;
        if (tm > m_old + kRescaleThreshold) {
          a = ex2(m_old - tm);
          m_ref[head] = tm;
        }
        alpha[head] = a;
        const unsigned any = __ballot_sync(0xffffffffu, a != 1.f);
        if (lane == 0) any_rescale[hh] = any != 0u;
      }
      named_bar(1 + hh, 128);
      if (ok && any_rescale[hh] && t > 0) {  // O^T columns of this head half, lanes of this sub-partition
#pragma unroll 1
        for (int jj = 0; jj < 8; ++jj) {  // 4 value tiles x 2 groups of 16 head columns
          uint32_t o[16];
          const uint32_t col = 64 * (jj >> 1) + 32 * hh + 16 * (jj & 1);
          tmem_ld16(tmem + t_lane + col, o);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 16; ++h)
            o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[32 * hh + 16 * (jj & 1) + h]);
          tmem_st16(tmem + t_lane + col, o);
        }
        tmem_wait_st();
      }
    }
    // P = 2^(v - m) in fp16 into the P^T rows (the rope region, consumed by QK(t));
    // row sums updated in TMEM
    uint8_t* preg = sm + SM_KV + 8 * KV_REGION;
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      const int hb = 32 * hh + 16 * c2;  // first head of this group
      uint32_t l16[16];
      if (ok && t > 0) {
        tmem_ld16(tmem + t_lane + L_COL + hb, l16);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) l16[h] = 0u;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 8 heads per 16-byte chunk of the P^T row
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const int h = 16 * c2 + 8 * c + e;  // head index within the half
          const float p0 = ex2(v[h] - m_ref[32 * hh + h]);
          const float p1 = ex2(v[h + 1] - m_ref[32 * hh + h + 1]);
          const int hl = 8 * c + e;
          const float a0 = slow ? alpha[32 * hh + h] : 1.f, a1 = slow ? alpha[32 * hh + h + 1] : 1.f;
          l16[hl] = __float_as_uint(__uint_as_float(l16[hl]) * a0 + p0);
          l16[hl + 1] = __float_as_uint(__uint_as_float(l16[hl + 1]) * a1 + p1);
          pk[e >> 1] = pack_half2(p0, p1);
        }
        *reinterpret_cast<uint4*>(preg + sw128_off(row_s, 4 * hh + 2 * c2 + c)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      if (ok) tmem_st16(tmem + t_lane + L_COL + hb, l16);
    }
    tmem_wait_st();
    fence_proxy_async();
    fence_before_sync();
    __syncthreads();
    // ---- O^T += V^T . P^T, one commit per 128-wide value tile
    if (issuer && ok) {
      fence_after_sync();
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int s = 0; s < TM / 16; ++s) {
          const uint64_t a = sw128_desc(base + SM_KV + 2 * j * KV_REGION + 2048 * s, KV_REGION, 1024);
          const uint64_t bp = sw128_desc(base + SM_KV + 8 * KV_REGION + 2048 * s, KV_REGION, 1024);
          mma_f16_ss(tmem + 64 * j, a, bp, IDESC_PV, (t > 0 || s > 0) ? 1u : 0u);
        }
        mma_commit(mb_kv_free(j));
      }
    }
    __syncwarp();
  }
  // -------------------------------------------------------------- epilogue
  if (ok && ntiles > 0) ok = mbar_wait(mb_kv_free(3), (ntiles - 1) & 1, abort_flag, err, kWaitTimeoutNs);
  __syncthreads();
  // A thread whose wait failed set the abort flag before this barrier, so
  // every thread reads the same decision.
  const bool live = *abort_flag == 0;
  __syncthreads();
  if (ntiles > 0 && live) {
    fence_after_sync();
    float* lbuf = reinterpret_cast<float*>(sm + SM_KV);  // [64 heads][128 rows]; the tile is dead now
    {
      uint32_t lr[32];
      tmem_ld32(tmem + t_lane + L_COL + 32 * hh, lr);
      tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 32; ++h) lbuf[(32 * hh + h) * TM + row_s] = __uint_as_float(lr[h]);
    }
    __syncthreads();
    {
      const int head = threadIdx.x >> 2, q4 = threadIdx.x & 3;
      float s = 0.f;
#pragma unroll 8
      for (int r = 0; r < 32; ++r) s += lbuf[head * TM + 32 * q4 + r];
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (q4 == 0) l_sum[head] = s;
    }
    __syncthreads();
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint32_t o[32];
      tmem_ld32(tmem + t_lane + 64 * j + 32 * hh, o);
      tmem_wait_ld();
      const int d = 128 * j + 32 * sp + lane;
#pragma unroll 4
      for (int h = 0; h < 32; ++h) {
        const int hl = 32 * hh + h;
        const int head = h0 + hl;
        if (head >= p.n_head) break;
        const float val = __uint_as_float(o[h]);
        if (p.n_splits == 1) {
          const float l = l_sum[hl];
          const float out = l > 0.f ? val / l : 0.f;
          const int64_t off = ((int64_t)b * p.n_head + head) * DV + d;
          if (p.o_bf16)
            reinterpret_cast<__nv_bfloat16*>(p.o)[off] = __float2bfloat16_rn(out);
          else
            reinterpret_cast<__half*>(p.o)[off] = __float2half_rn(out);
        } else {
          p.part_o[(((int64_t)b * p.n_head + head) * p.n_splits + split) * DV + d] = val;
        }
      }
    }
    if (threadIdx.x < NH && h0 + (int)threadIdx.x < p.n_head) {
      const float l = l_sum[threadIdx.x], m = m_ref[threadIdx.x];
      const int64_t bh = (int64_t)b * p.n_head + h0 + threadIdx.x;
      if (p.n_splits == 1) {
        p.lse[bh] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
      } else {
        p.part_ml[(bh * p.n_splits + split) * 2] = m;
        p.part_ml[(bh * p.n_splits + split) * 2 + 1] = l;
      }
    }
  } else if (ntiles == 0) {
    // empty slice: o = 0 / lse = -inf, or an empty partial state
    for (int i = threadIdx.x; i < NH * DV; i += NTHREADS) {
      const int head = h0 + i / DV, d = i % DV;
      if (head >= p.n_head) continue;
      const int64_t bh = (int64_t)b * p.n_head + head;
      if (p.n_splits == 1) {
        if (p.o_bf16)
          reinterpret_cast<__nv_bfloat16*>(p.o)[bh * DV + d] = __float2bfloat16_rn(0.f);
        else
          reinterpret_cast<__half*>(p.o)[bh * DV + d] = __float2half_rn(0.f);
        if (d == 0) p.lse[bh] = -INFINITY;
      } else {
        p.part_o[(bh * p.n_splits + split) * DV + d] = 0.f;
        if (d == 0) {
          p.part_ml[(bh * p.n_splits + split) * 2] = -1e30f;
          p.part_ml[(bh * p.n_splits + split) * 2 + 1] = 0.f;
        }
      }
    }
  }
  // every MMA of this CTA has completed before TMEM is released
  if (issuer && issued && !live) {
    mma_commit(mb_done);
    mbar_wait(mb_done, 0, abort_flag, err, kWaitTimeoutNs);
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
  });
  if (g_status[dev] != 0) {
    set_error("sparse_mla_decode_tc setup: %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

}  // namespace

int tc_choose_splits(int B, int head_tiles, int topk, int nsm) {
  const int ntiles = (topk + TM - 1) / TM;
  if (ntiles <= 1) return 1;
  const double units = (double)B * head_tiles;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 32 && s <= ntiles; ++s) {
    const int per = (ntiles + s - 1) / s;
    if ((ntiles + per - 1) / per != s) continue;
    const double waves = std::ceil(units * s / nsm);
    // one tile of 128 fp8 rows moves 84 KB; a slice's partial state 2 x 128 KB
    double cost = waves * per + (s > 1 ? units * s * 2.0 * NH * DV * 4.0 / ((double)nsm * TM * ROW_BYTES) : 0.0);
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
  const dim3 grid(a.B, (a.n_head + NH - 1) / NH, a.n_splits);
  sparse_mla_decode_tc_kernel<<<grid, NTHREADS, SMEM_BYTES, s>>>(a, g_err_ptr[dev]);
  return check_launch("sparse_mla_decode_tc_kernel");
}

}  // namespace dsa

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
