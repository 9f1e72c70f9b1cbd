// Lightning-indexer logits: score[b,p] = sum_h w[b,h] * relu(q[b,h,:] . k_p).
//
// Replaces sm70_indexer_logits (csrc/attention/sm70_mla_decode.cu:2626-2764;
// decode kernel :150-329, staged prefill kernel :345-458) and
// sm70_indexer_logits_packed (:2771-2836, kernel :542-653).
//
// Two kernels here, both on the tensor cores (m16n8k16, fp32 accumulate),
// beside the tcgen05 kernels of indexer_logits_tc.cu (prefill, 16-bit caches)
// and indexer_decode_tc.cu (decode, fp8 cache in 64-token pages):
//   * rows kernel (decode rows of the other caches, or whenever the caller
//     asks for the fused histogram): one CTA = one query row x 128 key
//     positions; every row uses
//     its own block-table row. The q rows of all heads are the MMA's M side,
//     the key tile the N side; relu * w and the head sum are done on the
//     accumulators in registers, and the level-1 top-k histogram is built
//     from the final scores.
//   * tiles kernel (prefill): one CTA = 64 query rows x 128 keys, looping
//     over the indexer heads with the per-head q tile double-buffered by
//     cp.async; the key tile is gathered once through the block table of the
//     tile's FIRST row (the same contract as the reference's WMMA kernels,
//     which the caller satisfies by launching per request segment,
//     reference/sparse_attn_indexer.py:750-760). Per-row causal lengths mask
//     p >= seq_len[row] to -inf.
// fp8 key rows (128 e4m3 | f32 scale) are expanded exactly to fp16 and the
// per-key scale is applied to the dot product (scale > 0 commutes with relu).
#include "common.cuh"
#include "indexer_tc.cuh"

namespace dsa {
namespace {

constexpr int HD = 128;
constexpr int KSTR = HD + 8;  // 272 B rows (17 x 16 B): conflict-free ldmatrix
constexpr int IDXK_ROW = 132;
constexpr int NBIN = 4096;

enum KFmt { K_F16 = 0, K_BF16 = 1, K_FP8 = 2 };

struct LogitsParams {
  float* score;
  const void* q;
  const uint8_t* k;
  const void* w;
  const int32_t* bt;
  const int32_t* seq_lens;
  int32_t* hist;
  int64_t score_stride;
  int64_t n_kv_rows;
  int64_t bt_stride;
  int max_kv;
  int page_shift;
  int max_blocks;
  int B;
  int n_ihead;
  int q_bf16;     // q element type
  int w_dtype;    // DSA_F16 / DSA_BF16 / DSA_F32
  int packed;     // q in the [32, ceil(B/16), 8, 16, 16] layout
  int nqt;        // ceil(B/16) for the packed layout
};

__device__ __forceinline__ float load_w(const LogitsParams& p, int64_t i) {
  if (p.w_dtype == DSA_F32) return reinterpret_cast<const float*>(p.w)[i];
  if (p.w_dtype == DSA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.w)[i]);
  return __half2float(reinterpret_cast<const __half*>(p.w)[i]);
}

// Byte offset of q[row, head, 8*c .. 8*c+8) (a 16-byte chunk).
__device__ __forceinline__ int64_t q_chunk_offset(const LogitsParams& p, int row, int head, int c) {
  if (p.packed) {
    const int d = 8 * c;
    const int64_t e = ((((int64_t)head * p.nqt + (row >> 4)) * 8 + (d >> 4)) * 16 + (row & 15)) * 16 + (d & 15);
    return e * 2;
  }
  return (((int64_t)row * p.n_ihead + head) * HD + 8 * c) * 2;
}

// Convert a 16-byte chunk of q to the MMA element type.
template <bool MMA_BF16>
__device__ __forceinline__ uint4 q_to_mma(uint4 v, int q_bf16) {
  if (!MMA_BF16 && q_bf16) return bf16x8_to_half8(v);
  return v;
}

// Physical row of logical key position pos for block-table row `bt_row`.
__device__ __forceinline__ int64_t key_row(const LogitsParams& p, const int32_t* bt_row, int pos) {
  const int blk_i = pos >> p.page_shift;
  if (blk_i >= p.max_blocks) return -1;
  const int64_t r = ((int64_t)bt_row[blk_i] << p.page_shift) + (pos & ((1 << p.page_shift) - 1));
  return (r >= 0 && r < p.n_kv_rows) ? r : -1;
}

// Gather NKEYS key rows (fp16/bf16 expanded) into sK[NKEYS][KSTR]; per-key
// fp8 scale into sScale (1 for plain rows, 0 for missing rows).
template <int KF, bool MMA_BF16, int NKEYS, int NT>
__device__ __forceinline__ void gather_keys(const LogitsParams& p, const int64_t* sRow,
                                            __half* sK, float* sScale) {
  if constexpr (KF == K_FP8) {
    // 132-byte rows are only 4-byte aligned: 32 words per row.
    for (int i = threadIdx.x; i < NKEYS * 32; i += NT) {
      const int r = i >> 5, wd = i & 31;
      const int64_t row = sRow[r];
      uint32_t v = 0;
      if (row >= 0) v = __ldg(reinterpret_cast<const uint32_t*>(p.k + row * IDXK_ROW) + wd);
      __half2 lo, hi;
      e4m3x4_to_half2x2(v, lo, hi);
      uint2 out;
      if (MMA_BF16) {
        const float2 a = __half22float2(lo), b = __half22float2(hi);
        __nv_bfloat162 x = __floats2bfloat162_rn(a.x, a.y), y = __floats2bfloat162_rn(b.x, b.y);
        out = make_uint2(*reinterpret_cast<uint32_t*>(&x), *reinterpret_cast<uint32_t*>(&y));
      } else {
        out = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
      }
      *reinterpret_cast<uint2*>(sK + r * KSTR + 4 * wd) = out;
      if (wd == 0)
        sScale[r] = row >= 0 ? __ldg(reinterpret_cast<const float*>(p.k + row * IDXK_ROW + 128)) : 0.f;
    }
  } else {
    for (int i = threadIdx.x; i < NKEYS * 16; i += NT) {
      const int r = i >> 4, c = i & 15;
      const int64_t row = sRow[r];
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row >= 0) v = ldg_nc16(p.k + (row * HD + 8 * c) * 2);
      if (KF == K_BF16 && !MMA_BF16) v = bf16x8_to_half8(v);
      *reinterpret_cast<uint4*>(sK + r * KSTR + 8 * c) = v;
      if (c == 0) sScale[r] = 1.f;
    }
  }
}

template <bool MMA_BF16>
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (MMA_BF16)
    mma_bf16_16816(d, a0, a1, a2, a3, b0, b1);
  else
    mma_f16_16816(d, a0, a1, a2, a3, b0, b1);
}

// ------------------------------------------------------------------ rows
constexpr int ROWS_KEYS = 128;
constexpr int ROWS_NT = 128;  // 4 warps x 32 keys

template <int KF, bool MMA_BF16, int MT>
__global__ void __launch_bounds__(ROWS_NT) indexer_rows_kernel(const LogitsParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sQ = reinterpret_cast<__half*>(smem);                       // [16*MT][KSTR]
  __half* sK = sQ + 16 * MT * KSTR;                                    // [128][KSTR]
  float* sW = reinterpret_cast<float*>(sK + ROWS_KEYS * KSTR);         // [16*MT]
  float* sScale = sW + 16 * MT;                                        // [128]
  int64_t* sRow = reinterpret_cast<int64_t*>(sScale + ROWS_KEYS);      // [128]

  const int b = blockIdx.x;
  const int p0 = blockIdx.y * ROWS_KEYS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* score_row = p.score + (int64_t)b * p.score_stride;
  const int p_hi = min(p0 + ROWS_KEYS, p.max_kv);
  const int valid_len = min(p.seq_lens[b], p.max_kv);
  if (p0 >= valid_len) {
    for (int i = p0 + tid; i < p_hi; i += ROWS_NT) score_row[i] = -INFINITY;
    return;
  }
  // q rows of all heads (zero padding up to 16*MT), weights
  for (int i = tid; i < 16 * MT * 16; i += ROWS_NT) {
    const int h = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < p.n_ihead)
      v = q_to_mma<MMA_BF16>(
          *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.q) + q_chunk_offset(p, b, h, c)),
          p.q_bf16);
    *reinterpret_cast<uint4*>(sQ + h * KSTR + 8 * c) = v;
  }
  for (int h = tid; h < 16 * MT; h += ROWS_NT)
    sW[h] = h < p.n_ihead ? load_w(p, (int64_t)b * p.n_ihead + h) : 0.f;
  {
    const int pos = p0 + tid;
    sRow[tid] = pos < valid_len ? key_row(p, p.bt + (int64_t)b * p.bt_stride, pos) : -1;
  }
  __syncthreads();
  gather_keys<KF, MMA_BF16, ROWS_KEYS, ROWS_NT>(p, sRow, sK, sScale);
  __syncthreads();

  float acc[MT][4][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
    uint32_t bfr[2][4];
#pragma unroll
    for (int np = 0; np < 2; ++np)
      ldmatrix_x4(smem_u32(sK + (32 * warp + 16 * np + (lane & 7) + 8 * (lane >> 4)) * KSTR + 16 * ks +
                           8 * ((lane >> 3) & 1)),
                  bfr[np][0], bfr[np][1], bfr[np][2], bfr[np][3]);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(smem_u32(sQ + (16 * m + (lane & 15)) * KSTR + 16 * ks + 8 * (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        mma16816<MMA_BF16>(acc[m][2 * np], a0, a1, a2, a3, bfr[np][0], bfr[np][1]);
        mma16816<MMA_BF16>(acc[m][2 * np + 1], a0, a1, a2, a3, bfr[np][2], bfr[np][3]);
      }
    }
  }
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    const int c0 = 32 * warp + 8 * n + 2 * t4;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float w0 = sW[16 * m + g], w1 = sW[16 * m + g + 8];
      s0 += w0 * fmaxf(acc[m][n][0], 0.f) + w1 * fmaxf(acc[m][n][2], 0.f);
      s1 += w0 * fmaxf(acc[m][n][1], 0.f) + w1 * fmaxf(acc[m][n][3], 0.f);
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, off);
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    }
    if (g == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int pos = p0 + c0 + e;
        if (pos < p_hi) {
          float v = -INFINITY;
          if (pos < valid_len) {
            v = (e == 0 ? s0 : s1) * sScale[c0 + e];
            if (p.hist) atomicAdd(p.hist + (int64_t)b * NBIN + (monotone32(v) >> 20), 1);
          }
          score_row[pos] = v;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ tiles
constexpr int TQ = 64;        // query rows per CTA
constexpr int TK = 128;       // keys per CTA
constexpr int TILES_NT = 256; // 8 warps: 4 row groups x 2 key halves

template <int KF, bool MMA_BF16>
__global__ void __launch_bounds__(TILES_NT) indexer_tiles_kernel(const LogitsParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sQ = reinterpret_cast<__half*>(smem);                  // [2][TQ][KSTR]
  __half* sK = sQ + 2 * TQ * KSTR;                                 // [TK][KSTR]
  float* sW = reinterpret_cast<float*>(sK + TK * KSTR);           // [TQ][n_ihead]
  float* sScale = sW + TQ * 64;                                    // [TK]
  int* sLen = reinterpret_cast<int*>(sScale + TK);                 // [TQ]
  int64_t* sRow = reinterpret_cast<int64_t*>(sLen + TQ);           // [TK]
  __shared__ int sMaxLen;

  const int q0 = blockIdx.x * TQ;
  const int p0 = blockIdx.y * TK;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nrows = min(TQ, p.B - q0);

  if (tid == 0) sMaxLen = 0;
  __syncthreads();
  if (tid < TQ) {
    const int len = tid < nrows ? min(p.seq_lens[q0 + tid], p.max_kv) : 0;
    sLen[tid] = len;
    atomicMax(&sMaxLen, len);
  }
  __syncthreads();
  const int p_hi = min(p0 + TK, p.max_kv);
  if (p0 >= sMaxLen) {  // every row of the tile is causal-masked here
    for (int i = tid; i < nrows * TK; i += TILES_NT) {
      const int r = i / TK, c = i % TK;
      if (p0 + c < p_hi) p.score[(int64_t)(q0 + r) * p.score_stride + p0 + c] = -INFINITY;
    }
    return;
  }
  const bool direct_q = (MMA_BF16 == (p.q_bf16 != 0));
  auto load_q_tile = [&](int head, int buf) {
    __half* dst = sQ + buf * TQ * KSTR;
    for (int i = tid; i < TQ * 16; i += TILES_NT) {
      const int r = i >> 4, c = i & 15;
      __half* d = dst + r * KSTR + 8 * c;
      if (r < nrows) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.q) + q_chunk_offset(p, q0 + r, head, c);
        if (direct_q)
          cp_async16(smem_u32(d), src);
        else
          *reinterpret_cast<uint4*>(d) = q_to_mma<MMA_BF16>(*reinterpret_cast<const uint4*>(src), p.q_bf16);
      } else {
        *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  load_q_tile(0, 0);
  for (int i = tid; i < TQ * p.n_ihead; i += TILES_NT) {
    const int r = i / p.n_ihead, h = i % p.n_ihead;
    sW[r * 64 + h] = r < nrows ? load_w(p, (int64_t)(q0 + r) * p.n_ihead + h) : 0.f;
  }
  if (tid < TK) {
    const int pos = p0 + tid;
    sRow[tid] = pos < sMaxLen ? key_row(p, p.bt + (int64_t)q0 * p.bt_stride, pos) : -1;
  }
  __syncthreads();
  gather_keys<KF, MMA_BF16, TK, TILES_NT>(p, sRow, sK, sScale);

  const int rg = warp & 3;   // rows 16*rg ..
  const int kh = warp >> 2;  // keys 64*kh ..
  const int g = lane >> 2, t4 = lane & 3;
  float sc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;

  for (int h = 0; h < p.n_ihead; ++h) {
    const int buf = h & 1;
    if (h + 1 < p.n_ihead) {
      load_q_tile(h + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float acc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    const __half* qt = sQ + buf * TQ * KSTR;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(smem_u32(qt + (16 * rg + (lane & 15)) * KSTR + 16 * ks + 8 * (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(sK + (64 * kh + 16 * np + (lane & 7) + 8 * (lane >> 4)) * KSTR + 16 * ks +
                             8 * ((lane >> 3) & 1)),
                    b0, b1, b2, b3);
        mma16816<MMA_BF16>(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816<MMA_BF16>(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    const float w0 = sW[(16 * rg + g) * 64 + h];
    const float w1 = sW[(16 * rg + g + 8) * 64 + h];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sc[n][0] += w0 * fmaxf(acc[n][0], 0.f);
      sc[n][1] += w0 * fmaxf(acc[n][1], 0.f);
      sc[n][2] += w1 * fmaxf(acc[n][2], 0.f);
      sc[n][3] += w1 * fmaxf(acc[n][3], 0.f);
    }
    __syncthreads();  // q buffer `buf` is refilled by the next iteration's prefetch
  }
  const int r0 = 16 * rg + g, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int c = 64 * kh + 8 * n + 2 * t4;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int pos = p0 + c + e;
      if (pos >= p_hi) continue;
      const float ks = sScale[c + e];
      if (r0 < nrows)
        p.score[(int64_t)(q0 + r0) * p.score_stride + pos] = pos < sLen[r0] ? sc[n][e] * ks : -INFINITY;
      if (r1 < nrows)
        p.score[(int64_t)(q0 + r1) * p.score_stride + pos] = pos < sLen[r1] ? sc[n][2 + e] * ks : -INFINITY;
    }
  }
}

size_t rows_smem(int mt) {
  return (size_t)16 * mt * KSTR * 2 + (size_t)ROWS_KEYS * KSTR * 2 + (size_t)16 * mt * 4 +
         (size_t)ROWS_KEYS * 4 + (size_t)ROWS_KEYS * 8;
}
constexpr size_t kTilesSmem = (size_t)2 * TQ * KSTR * 2 + (size_t)TK * KSTR * 2 + (size_t)TQ * 64 * 4 +
                              (size_t)TK * 4 + (size_t)TQ * 4 + (size_t)TK * 8;

template <typename K>
cudaError_t set_smem(K kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];

int ensure_attrs(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return DSA_OK;
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaSuccess;
#define DSA_SET_TILES(KF, BF)                                                  \
  if (e == cudaSuccess) e = set_smem(indexer_tiles_kernel<KF, BF>, kTilesSmem);
    DSA_SET_TILES(K_F16, false)
    DSA_SET_TILES(K_BF16, false)
    DSA_SET_TILES(K_BF16, true)
    DSA_SET_TILES(K_FP8, false)
#undef DSA_SET_TILES
#define DSA_SET_ROWS(KF, BF, MT)                                               \
  if (e == cudaSuccess) e = set_smem(indexer_rows_kernel<KF, BF, MT>, rows_smem(MT));
    DSA_SET_ROWS(K_F16, false, 1) DSA_SET_ROWS(K_F16, false, 2) DSA_SET_ROWS(K_F16, false, 4)
    DSA_SET_ROWS(K_BF16, false, 1) DSA_SET_ROWS(K_BF16, false, 2) DSA_SET_ROWS(K_BF16, false, 4)
    DSA_SET_ROWS(K_BF16, true, 1) DSA_SET_ROWS(K_BF16, true, 2) DSA_SET_ROWS(K_BF16, true, 4)
    DSA_SET_ROWS(K_FP8, false, 1) DSA_SET_ROWS(K_FP8, false, 2) DSA_SET_ROWS(K_FP8, false, 4)
#undef DSA_SET_ROWS
    g_status[dev] = (int)e;
  });
  if (g_status[dev] != 0) {
    set_error("cudaFuncSetAttribute(indexer): %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

template <int KF, bool BF>
void launch_rows(const LogitsParams& p, int mt, cudaStream_t s) {
  const dim3 grid(p.B, (p.max_kv + ROWS_KEYS - 1) / ROWS_KEYS);
  if (mt == 1)
    indexer_rows_kernel<KF, BF, 1><<<grid, ROWS_NT, rows_smem(1), s>>>(p);
  else if (mt == 2)
    indexer_rows_kernel<KF, BF, 2><<<grid, ROWS_NT, rows_smem(2), s>>>(p);
  else
    indexer_rows_kernel<KF, BF, 4><<<grid, ROWS_NT, rows_smem(4), s>>>(p);
}

template <int KF, bool BF>
void launch_tiles(const LogitsParams& p, cudaStream_t s) {
  const dim3 grid((p.B + TQ - 1) / TQ, (p.max_kv + TK - 1) / TK);
  indexer_tiles_kernel<KF, BF><<<grid, TILES_NT, kTilesSmem, s>>>(p);
}

int run_logits(LogitsParams p, int k_format, int page_size, bool use_rows, cudaStream_t s) {
  DSA_REQUIRE(p.B >= 0 && p.max_kv >= 0, DSA_ERR_INVALID, "indexer_logits: negative size");
  if (p.B == 0 || p.max_kv == 0) return DSA_OK;
  DSA_REQUIRE(p.score && p.q && p.w && p.seq_lens && p.bt && p.k, DSA_ERR_INVALID,
              "indexer_logits: null pointer");
  DSA_REQUIRE(p.n_ihead >= 1 && p.n_ihead <= 64, DSA_ERR_UNSUPPORTED,
              "indexer_logits: n_ihead must be in [1, 64] (got %d)", p.n_ihead);
  DSA_REQUIRE(page_size > 0 && (page_size & (page_size - 1)) == 0, DSA_ERR_INVALID,
              "indexer_logits: page size must be a power of two (got %d)", page_size);
  DSA_REQUIRE(k_format == DSA_F16 || k_format == DSA_BF16 || k_format == DSA_FP8_IDXK, DSA_ERR_INVALID,
              "indexer_logits: k_cache must be f16, bf16 or fp8 (u8 132)");
  DSA_REQUIRE(p.w_dtype == DSA_F16 || p.w_dtype == DSA_BF16 || p.w_dtype == DSA_F32, DSA_ERR_INVALID,
              "indexer_logits: weights must be f16, bf16 or f32");
  DSA_REQUIRE(p.score_stride >= p.max_kv && p.bt_stride >= p.max_blocks, DSA_ERR_INVALID,
              "indexer_logits: row stride smaller than the row");
  DSA_REQUIRE(((uintptr_t)p.q & 15) == 0 && ((uintptr_t)p.k & 15) == 0, DSA_ERR_INVALID,
              "indexer_logits: q and k_cache must be 16-byte aligned");
  DSA_REQUIRE((p.max_kv + ROWS_KEYS - 1) / ROWS_KEYS <= 65535, DSA_ERR_UNSUPPORTED,
              "indexer_logits: max_kv too large");
  int st = ensure_attrs(current_device());
  if (st != DSA_OK) return st;
  p.page_shift = 31 - __builtin_clz((unsigned)page_size);
  const bool bf = p.q_bf16 && k_format == DSA_BF16;
  if (use_rows) {
    const int mt = p.n_ihead <= 16 ? 1 : (p.n_ihead <= 32 ? 2 : 4);
    if (indexer_decode_tc_eligible(k_format, page_size, p.n_ihead, p.packed)) {
      IndexerDecodeTcArgs t{};
      t.score = p.score;
      t.score_stride = p.score_stride;
      t.max_kv = p.max_kv;
      t.q = p.q;
      t.q_bf16 = p.q_bf16;
      t.n_ihead = p.n_ihead;
      t.B = p.B;
      t.k = p.k;
      t.n_kv_rows = p.n_kv_rows;
      t.w = p.w;
      t.w_dtype = p.w_dtype;
      t.bt = p.bt;
      t.bt_stride = p.bt_stride;
      t.max_blocks = p.max_blocks;
      t.seq_lens = p.seq_lens;
      t.hist = p.hist;
      return launch_indexer_decode_tc(t, s);
    }
    if (k_format == DSA_FP8_IDXK)
      launch_rows<K_FP8, false>(p, mt, s);
    else if (k_format == DSA_BF16)
      bf ? launch_rows<K_BF16, true>(p, mt, s) : launch_rows<K_BF16, false>(p, mt, s);
    else
      launch_rows<K_F16, false>(p, mt, s);
    return check_launch("indexer_rows_kernel");
  }
  if ((!p.packed || p.n_ihead == 32) &&
      indexer_tc_eligible(k_format, p.q_bf16, page_size, p.n_ihead, p.n_kv_rows, p.B, p.max_kv)) {
    IndexerTcArgs t{};
    t.score = p.score;
    t.score_stride = p.score_stride;
    t.max_kv = p.max_kv;
    t.q = p.q;
    t.q_bf16 = p.q_bf16;
    t.n_ihead = p.n_ihead;
    t.B = p.B;
    t.k = p.k;
    t.n_kv_rows = p.n_kv_rows;
    t.page_size = page_size;
    t.w = p.w;
    t.w_dtype = p.w_dtype;
    t.bt = p.bt;
    t.bt_stride = p.bt_stride;
    t.max_blocks = p.max_blocks;
    t.seq_lens = p.seq_lens;
    t.packed = p.packed;
    return launch_indexer_logits_tc(t, s);
  }
  if (k_format == DSA_FP8_IDXK)
    launch_tiles<K_FP8, false>(p, s);
  else if (k_format == DSA_BF16)
    bf ? launch_tiles<K_BF16, true>(p, s) : launch_tiles<K_BF16, false>(p, s);
  else
    launch_tiles<K_F16, false>(p, s);
  return check_launch("indexer_tiles_kernel");
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_indexer_logits(float* score, int64_t score_stride, int max_kv, const void* q, int q_dtype,
                                  const void* k_cache, int k_format, int64_t n_kv_rows, int page_size,
                                  const void* weights, int w_dtype, const int32_t* block_table,
                                  int64_t bt_stride, int max_blocks, const int32_t* seq_lens, int B,
                                  int n_ihead, int32_t* hist, void* stream) {
  clear_error();
  DSA_REQUIRE(q_dtype == DSA_F16 || q_dtype == DSA_BF16, DSA_ERR_INVALID, "indexer_logits: q must be f16 or bf16");
  LogitsParams p{};
  p.score = score;
  p.q = q;
  p.k = reinterpret_cast<const uint8_t*>(k_cache);
  p.w = weights;
  p.bt = block_table;
  p.seq_lens = seq_lens;
  p.hist = hist;
  p.score_stride = score_stride;
  p.n_kv_rows = n_kv_rows;
  p.bt_stride = bt_stride;
  p.max_kv = max_kv;
  p.max_blocks = max_blocks;
  p.B = B;
  p.n_ihead = n_ihead;
  p.q_bf16 = q_dtype == DSA_BF16;
  p.w_dtype = w_dtype;
  // Per-row block tables for decode batches and whenever the fused histogram
  // is requested; the tiled prefill kernel otherwise (dsa.cu:2667 uses B >= 8).
  const bool use_rows = hist != nullptr || B < 8;
  return run_logits(p, k_format, page_size, use_rows, as_stream(stream));
}

extern "C" int dsa_indexer_logits_packed(float* score, int64_t score_stride, int max_kv, const void* q_packed,
                                         int q_dtype, const void* k_cache, int k_format, int64_t n_kv_rows,
                                         int page_size, const void* weights, int w_dtype,
                                         const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                         const int32_t* seq_lens, int B, void* stream) {
  clear_error();
  DSA_REQUIRE(q_dtype == DSA_F16 || q_dtype == DSA_BF16, DSA_ERR_INVALID,
              "indexer_logits_packed: q_packed must be f16 or bf16");
  LogitsParams p{};
  p.score = score;
  p.q = q_packed;
  p.k = reinterpret_cast<const uint8_t*>(k_cache);
  p.w = weights;
  p.bt = block_table;
  p.seq_lens = seq_lens;
  p.hist = nullptr;
  p.score_stride = score_stride;
  p.n_kv_rows = n_kv_rows;
  p.bt_stride = bt_stride;
  p.max_kv = max_kv;
  p.max_blocks = max_blocks;
  p.B = B;
  p.n_ihead = 32;  // the packed layout is defined for 32 heads (dsa.cu:2796-2801)
  p.q_bf16 = q_dtype == DSA_BF16;
  p.w_dtype = w_dtype;
  p.packed = 1;
  p.nqt = (B + 15) / 16;
  return run_logits(p, k_format, page_size, B < 8, as_stream(stream));
}
