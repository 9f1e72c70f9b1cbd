// Sparse MLA decode / prefill attention over the paged latent cache.
//
// Replaces the reference's split decode kernel + flash-decode merge
// (csrc/attention/sm70_mla_decode.cu:918-1184, launcher :2457-2616) and its
// prefill kernels (:1563-2051), which compute the same function.
//
// Design (one CTA = one query row x 64 heads x one slice of the top-k axis):
//   * Q for the 64 heads stays resident in shared memory as fp16.
//   * The selected latent rows of a 32-row tile are gathered with 16-byte
//     non-allocating loads straight into registers one tile AHEAD of the
//     compute (register double buffer), then dequantised (fp8_ds_mla: e4m3 x
//     per-128-tile f32 scale, rounded once to fp16) into shared memory.
//   * S = Q K^T and O += P V run on the tensor cores (m16n8k16, fp16 in,
//     fp32 accumulate); O lives in registers for the whole slice, so PV never
//     round-trips shared memory. Softmax is online in base 2 (scale*log2e is
//     folded into S).
//   * With one slice per row the CTA normalises and writes o / lse directly;
//     otherwise it writes an unnormalised partial (o, m, l) and a small merge
//     kernel combines the slices.
#include <algorithm>
#include <cmath>

#include "sparse_mla.cuh"

namespace dsa {
namespace {

constexpr int DK = 576;
constexpr int DV = 512;
constexpr int HT = 64;         // heads per CTA
constexpr int TN = 32;         // latent rows per tile
constexpr int NTHR = 256;      // 8 warps
constexpr int QSTR = DK + 8;   // fp16 elements per smem row (1168 B = 73 x 16 B)
constexpr int PSTR = TN + 8;   // 80 B rows
constexpr int SSTR = TN + 1;
constexpr int DSMLA_ROW = 656;
constexpr float kLn2 = 0.69314718055994530942f;

enum KvFmt { KV_F16 = 0, KV_BF16 = 1, KV_FP8 = 2 };

using DecodeParams = SparseMlaArgs;

constexpr size_t kSmemQ = (size_t)HT * QSTR * 2;
constexpr size_t kSmemK = (size_t)TN * QSTR * 2;
constexpr size_t kSmemS = (size_t)HT * SSTR * 4;
constexpr size_t kSmemP = (size_t)HT * PSTR * 2;
constexpr size_t kSmemStats = (size_t)3 * HT * 4;
constexpr size_t kSmemRows = (size_t)2 * TN * 8 + (size_t)2 * TN * 4;
constexpr size_t kSmemDecode = kSmemQ + kSmemK + kSmemS + kSmemP + kSmemStats + kSmemRows;

template <int KVF>
struct KvTraits;
template <>
struct KvTraits<KV_FP8> {
  static constexpr int kChunks = 40;  // 32 nope chunks (16 e4m3) + 8 rope chunks (8 f16)
  static constexpr int kRowBytes = DSMLA_ROW;
};
template <>
struct KvTraits<KV_F16> {
  static constexpr int kChunks = 72;  // 576 halves / 8
  static constexpr int kRowBytes = DK * 2;
};
template <>
struct KvTraits<KV_BF16> {
  static constexpr int kChunks = 72;
  static constexpr int kRowBytes = DK * 2;
};

// Resolve tile rows [base, base+TN) of row b: validity and physical row.
__device__ __forceinline__ void resolve_rows(const DecodeParams& p, int b, int base, int hi,
                                             int seq_len, int64_t* s_row, int* s_valid) {
  const int t = threadIdx.x;
  if (t < TN) {
    const int j = base + t;
    int valid = 0;
    int64_t row = -1;
    if (j < hi) {
      const int pos = p.idx[(int64_t)b * p.idx_stride + j];
      if (pos >= 0 && pos < seq_len) {
        valid = 1;
        const int blk_i = pos / p.page_size;
        if (blk_i < p.max_blocks) {
          const int64_t blk = p.bt[(int64_t)b * p.bt_stride + blk_i];
          const int64_t r = blk * p.page_size + (pos - blk_i * p.page_size);
          if (r >= 0 && r < p.n_kv_rows) row = r;
        }
      }
    }
    s_row[t] = row;
    s_valid[t] = valid;
  }
}

template <int KVF>
struct Prefetch {
  static constexpr int kItems = TN * KvTraits<KVF>::kChunks / NTHR;
  static_assert(TN * KvTraits<KVF>::kChunks % NTHR == 0, "items must divide");
  uint4 raw[kItems];
  float sc[KVF == KV_FP8 ? kItems : 1];

  __device__ __forceinline__ void load(const DecodeParams& p, const int64_t* s_row) {
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int i = threadIdx.x + k * NTHR;
      const int r = i / KvTraits<KVF>::kChunks;
      const int c = i % KvTraits<KVF>::kChunks;
      const int64_t row = s_row[r];
      raw[k] = make_uint4(0, 0, 0, 0);
      if constexpr (KVF == KV_FP8) sc[k] = 0.f;
      if (row >= 0) {
        const uint8_t* rp = p.kv + row * KvTraits<KVF>::kRowBytes;
        if constexpr (KVF == KV_FP8) {
          if (c < 32) {
            raw[k] = ldg_nc16(rp + 16 * c);
            sc[k] = __ldg(reinterpret_cast<const float*>(rp + 512) + (c >> 3));
          } else {
            raw[k] = ldg_nc16(rp + 528 + 16 * (c - 32));
          }
        } else {
          raw[k] = ldg_nc16(rp + 16 * c);
        }
      }
    }
  }

  // Dequantise into the fp16 tile sK[TN][QSTR].
  __device__ __forceinline__ void store(__half* sK) const {
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int i = threadIdx.x + k * NTHR;
      const int r = i / KvTraits<KVF>::kChunks;
      const int c = i % KvTraits<KVF>::kChunks;
      if constexpr (KVF == KV_FP8) {
        if (c < 32) {
          const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
          uint32_t out[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __half2 lo, hi;
            e4m3x4_to_half2x2(w[e], lo, hi);
            const float2 flo = __half22float2(lo);
            const float2 fhi = __half22float2(hi);
            out[2 * e] = pack_half2(flo.x * sc[k], flo.y * sc[k]);
            out[2 * e + 1] = pack_half2(fhi.x * sc[k], fhi.y * sc[k]);
          }
          uint4* dst = reinterpret_cast<uint4*>(sK + r * QSTR + 16 * c);
          dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
          dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
        } else {
          *reinterpret_cast<uint4*>(sK + r * QSTR + 512 + 8 * (c - 32)) = raw[k];
        }
      } else if constexpr (KVF == KV_BF16) {
        *reinterpret_cast<uint4*>(sK + r * QSTR + 8 * c) = bf16x8_to_half8(raw[k]);
      } else {
        *reinterpret_cast<uint4*>(sK + r * QSTR + 8 * c) = raw[k];
      }
    }
  }
};

template <int KVF>
__global__ void __launch_bounds__(NTHR, 1) sparse_mla_decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* sQ = reinterpret_cast<__half*>(smem);
  __half* sK = reinterpret_cast<__half*>(smem + kSmemQ);
  float* sS = reinterpret_cast<float*>(smem + kSmemQ + kSmemK);
  __half* sP = reinterpret_cast<__half*>(smem + kSmemQ + kSmemK + kSmemS);
  float* sM = reinterpret_cast<float*>(smem + kSmemQ + kSmemK + kSmemS + kSmemP);
  float* sL = sM + HT;
  float* sAlpha = sL + HT;
  int64_t* sRow = reinterpret_cast<int64_t*>(sAlpha + HT);  // [2][TN]
  int* sValid = reinterpret_cast<int*>(sRow + 2 * TN);       // [2][TN]

  const int b = blockIdx.x;
  const int h0 = blockIdx.y * HT;
  const int split = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int t4 = lane & 3;

  const int seq_len = p.seq_lens[b];
  const int lo = split * p.span;
  const int hi = min(lo + p.span, p.topk);
  const int ntiles = hi > lo ? (hi - lo + TN - 1) / TN : 0;

  // ---- Q tile (fp16) and softmax state
  {
    const int nheads = min(HT, p.n_head - h0);
    for (int i = tid; i < HT * (DK / 8); i += NTHR) {
      const int h = i / (DK / 8);
      const int c = i % (DK / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h < nheads) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.q) +
                             (((int64_t)b * p.n_head + h0 + h) * DK + 8 * c) * 2;
        v = *reinterpret_cast<const uint4*>(src);
        if (p.q_bf16) v = bf16x8_to_half8(v);
      }
      *reinterpret_cast<uint4*>(sQ + h * QSTR + 8 * c) = v;
    }
    for (int i = tid; i < HT; i += NTHR) {
      sM[i] = -1e30f;
      sL[i] = 0.f;
      sAlpha[i] = 1.f;
    }
  }
  if (ntiles > 0) resolve_rows(p, b, lo, hi, seq_len, sRow, sValid);
  __syncthreads();

  Prefetch<KVF> pf;
  if (ntiles > 0) pf.load(p, sRow);

  float oacc[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;

  const int hg = warp & 3;
  const int half_id = warp >> 2;

  for (int t = 0; t < ntiles; ++t) {
    const int cur = t & 1;
    pf.store(sK);
    if (t + 1 < ntiles)
      resolve_rows(p, b, lo + (t + 1) * TN, hi, seq_len, sRow + (cur ^ 1) * TN,
                   sValid + (cur ^ 1) * TN);
    __syncthreads();
    if (t + 1 < ntiles) pf.load(p, sRow + (cur ^ 1) * TN);

    // ---- S = Q K^T (warp: 16 heads x 16 rows)
    {
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint32_t a_base =
          smem_u32(sQ + (16 * hg + (lane & 15)) * QSTR + 8 * (lane >> 4));
      const uint32_t b_base = smem_u32(sK + (16 * half_id + (lane & 7) + 8 * (lane >> 4)) * QSTR +
                                       8 * ((lane >> 3) & 1));
#pragma unroll 6
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldmatrix_x4(a_base + ks * 32, a0, a1, a2, a3);
        ldmatrix_x4(b_base + ks * 32, b0, b1, b2, b3);
        mma_f16_16816(acc[0], a0, a1, a2, a3, b0, b1);
        mma_f16_16816(acc[1], a0, a1, a2, a3, b2, b3);
      }
      const int* valid = sValid + cur * TN;
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int col = 16 * half_id + 8 * n + 2 * t4;
        const bool v0 = valid[col] != 0, v1 = valid[col + 1] != 0;
        float* r0 = sS + (16 * hg + g) * SSTR + col;
        float* r1 = sS + (16 * hg + g + 8) * SSTR + col;
        r0[0] = v0 ? acc[n][0] * p.scale_log2 : -INFINITY;
        r0[1] = v1 ? acc[n][1] * p.scale_log2 : -INFINITY;
        r1[0] = v0 ? acc[n][2] * p.scale_log2 : -INFINITY;
        r1[1] = v1 ? acc[n][3] * p.scale_log2 : -INFINITY;
      }
    }
    __syncthreads();

    // ---- online softmax (warp: 8 heads, lane = tile column)
#pragma unroll
    for (int hh = 0; hh < HT / 8; ++hh) {
      const int h = warp * (HT / 8) + hh;
      const float v = sS[h * SSTR + lane];
      float mx = v;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = sM[h];
      const float m_new = fmaxf(m_old, mx);
      const float pr = exp2f(v - m_new);
      float sum = pr;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      sP[h * PSTR + lane] = __float2half_rn(pr);
      __syncwarp();
      if (lane == 0) {
        const float alpha = exp2f(m_old - m_new);
        sM[h] = m_new;
        sL[h] = sL[h] * alpha + sum;
        sAlpha[h] = alpha;
      }
    }
    __syncthreads();

    // ---- O += P V (warp: 16 heads x 256 value dims, accumulators in registers)
    {
      const float al0 = sAlpha[16 * hg + g];
      const float al1 = sAlpha[16 * hg + g + 8];
#pragma unroll
      for (int n = 0; n < 32; ++n) {
        oacc[n][0] *= al0;
        oacc[n][1] *= al0;
        oacc[n][2] *= al1;
        oacc[n][3] *= al1;
      }
#pragma unroll
      for (int kk = 0; kk < TN / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(smem_u32(sP + (16 * hg + (lane & 15)) * PSTR + 16 * kk + 8 * (lane >> 4)), a0,
                    a1, a2, a3);
        const uint32_t vb = smem_u32(sK + (16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1)) * QSTR +
                                     256 * half_id + 8 * (lane >> 4));
#pragma unroll
        for (int np = 0; np < 16; ++np) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vb + np * 32, b0, b1, b2, b3);
          mma_f16_16816(oacc[2 * np], a0, a1, a2, a3, b0, b1);
          mma_f16_16816(oacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  // ---- epilogue
  const int hr0 = h0 + 16 * hg + g;
  const int hr1 = hr0 + 8;
  if (p.n_splits == 1) {
    const float l0 = sL[16 * hg + g], l1 = sL[16 * hg + g + 8];
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
    const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int d = 256 * half_id + 8 * n + 2 * t4;
      if (hr0 < p.n_head) {
        const int64_t off = ((int64_t)b * p.n_head + hr0) * DV + d;
        if (p.o_bf16)
          *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.o) + off) =
              __floats2bfloat162_rn(oacc[n][0] * inv0, oacc[n][1] * inv0);
        else
          *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(p.o) + off) =
              __floats2half2_rn(oacc[n][0] * inv0, oacc[n][1] * inv0);
      }
      if (hr1 < p.n_head) {
        const int64_t off = ((int64_t)b * p.n_head + hr1) * DV + d;
        if (p.o_bf16)
          *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.o) + off) =
              __floats2bfloat162_rn(oacc[n][2] * inv1, oacc[n][3] * inv1);
        else
          *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(p.o) + off) =
              __floats2half2_rn(oacc[n][2] * inv1, oacc[n][3] * inv1);
      }
    }
    for (int h = tid; h < HT; h += NTHR) {
      if (h0 + h < p.n_head) {
        const float l = sL[h];
        p.lse[(int64_t)b * p.n_head + h0 + h] = l > 0.f ? (sM[h] + log2f(l)) * kLn2 : -INFINITY;
      }
    }
  } else {
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int d = 256 * half_id + 8 * n + 2 * t4;
      if (hr0 < p.n_head) {
        float* dst = p.part_o + (((int64_t)b * p.n_head + hr0) * p.n_splits + split) * DV + d;
        *reinterpret_cast<float2*>(dst) = make_float2(oacc[n][0], oacc[n][1]);
      }
      if (hr1 < p.n_head) {
        float* dst = p.part_o + (((int64_t)b * p.n_head + hr1) * p.n_splits + split) * DV + d;
        *reinterpret_cast<float2*>(dst) = make_float2(oacc[n][2], oacc[n][3]);
      }
    }
    for (int h = tid; h < HT; h += NTHR) {
      if (h0 + h < p.n_head) {
        float* dst = p.part_ml + (((int64_t)b * p.n_head + h0 + h) * p.n_splits + split) * 2;
        dst[0] = sM[h];
        dst[1] = sL[h];
      }
    }
  }
}

// Combine per-slice partial states: o = sum_s w_s o_s / sum_s w_s l_s with
// w_s = 2^(m_s - max m) over slices with l_s > 0 (the flash-decode reduction
// of the reference's merge, dsa.cu:1136-1184); lse = -inf when nothing was
// valid. One CTA per (row, head), 128 threads x 4 value dims.
__global__ void __launch_bounds__(128) sparse_mla_merge_kernel(const float* __restrict__ part_o,
                                                               const float* __restrict__ part_ml,
                                                               void* __restrict__ o, int o_bf16,
                                                               float* __restrict__ lse,
                                                               int n_splits) {
  const int64_t bh = blockIdx.x;
  const float* ml = part_ml + bh * n_splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s)
    if (ml[2 * s + 1] > 0.f) M = fmaxf(M, ml[2 * s]);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int d = threadIdx.x * 4;
  // eight slices' loads in flight at a time, all inside the workspace; a
  // slice that counted nothing (l = 0) is loaded but not used
  constexpr int U = 8;
  for (int s0 = 0; s0 < n_splits; s0 += U) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      v[u] = s0 + u < n_splits ? *reinterpret_cast<const float4*>(part_o + (bh * n_splits + s0 + u) * DV + d)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int s = s0 + u;
      const float l = s < n_splits ? ml[2 * s + 1] : 0.f;
      if (l > 0.f) {
        const float w = exp2f(ml[2 * s] - M);
        L += l * w;
        acc.x += w * v[u].x;
        acc.y += w * v[u].y;
        acc.z += w * v[u].z;
        acc.w += w * v[u].w;
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int64_t off = bh * DV + d;
  if (o_bf16) {
    __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(o) + off);
    dst[0] = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    dst[1] = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
  } else {
    __half2* dst = reinterpret_cast<__half2*>(reinterpret_cast<__half*>(o) + off);
    dst[0] = __floats2half2_rn(acc.x * inv, acc.y * inv);
    dst[1] = __floats2half2_rn(acc.z * inv, acc.w * inv);
  }
  if (threadIdx.x == 0) lse[bh] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
}

// Slice count for the top-k axis: balance waves of CTAs (one resident CTA
// per SM) against the traffic of the partial states the merge re-reads.
int choose_splits(int B, int head_tiles, int topk, int nsm) {
  const int ntiles = (topk + TN - 1) / TN;
  if (ntiles <= 1) return 1;
  const double units = (double)B * head_tiles;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 32 && s <= ntiles; ++s) {
    const int per = (ntiles + s - 1) / s;
    const int s_eff = (ntiles + per - 1) / per;
    if (s_eff != s) continue;
    const double waves = std::ceil(units * s / nsm);
    double cost = waves * per;
    if (s > 1) cost += units * HT * DV * 8.0 * s / ((double)nsm * TN * DSMLA_ROW);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

std::once_flag g_attr_once[kMaxDevices];
int g_attr_status[kMaxDevices];

int ensure_attrs(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return DSA_OK;
  std::call_once(g_attr_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(sparse_mla_decode_kernel<KV_F16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemDecode);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(sparse_mla_decode_kernel<KV_BF16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemDecode);
    g_attr_status[dev] = (e == cudaSuccess) ? 0 : (int)e;
  });
  if (g_attr_status[dev] != 0) {
    set_error("cudaFuncSetAttribute(sparse_mla_decode): %s",
              cudaGetErrorString((cudaError_t)g_attr_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

}  // namespace
}  // namespace dsa

using namespace dsa;

namespace dsa {
int launch_sparse_mla_merge(const SparseMlaArgs& a, cudaStream_t s) {
  sparse_mla_merge_kernel<<<(unsigned)((int64_t)a.B * a.n_head), 128, 0, s>>>(a.part_o, a.part_ml, a.o, a.o_bf16,
                                                                               a.lse, a.n_splits);
  return check_launch("sparse_mla_merge_kernel");
}
}  // namespace dsa

// Slice count of the kernel that serves kv_format (the workspace holds the
// partial states of every slice).
static int splits_for(int kv_format, int B, int n_head, int topk, int nsm) {
  const int head_tiles = (n_head + HT - 1) / HT;
  if (kv_format == DSA_FP8_DS_MLA) return tc_choose_splits(B, head_tiles, topk, nsm);
  return choose_splits(B, head_tiles, topk, nsm);
}

extern "C" size_t dsa_sparse_mla_decode_workspace_bytes(int B, int n_head, int topk) {
  if (B <= 0 || n_head <= 0 || topk <= 0) return 0;
  const int nsm = sm_count(current_device());
  int s = 1;
  for (int fmt : {DSA_FP8_DS_MLA, DSA_F16}) s = std::max(s, splits_for(fmt, B, n_head, topk, nsm));
  if (s <= 1) return 0;
  return (size_t)B * n_head * s * (DV + 2) * sizeof(float);
}

extern "C" int dsa_sparse_mla_decode_plan(int B, int n_head, int topk, int kv_format, int* n_splits,
                                          int* cluster_size, size_t* workspace_bytes, int* launches) {
  clear_error();
  DSA_REQUIRE(B >= 0 && n_head >= 0 && topk >= 0, DSA_ERR_INVALID,
              "sparse_mla_decode_plan: negative size (B=%d n_head=%d topk=%d)", B, n_head, topk);
  DSA_REQUIRE(kv_format == DSA_F16 || kv_format == DSA_BF16 || kv_format == DSA_FP8_DS_MLA, DSA_ERR_INVALID,
              "sparse_mla_decode_plan: kv_format must be f16, bf16 or fp8_ds_mla");
  int s = 1, c = 1;
  size_t ws = 0;
  int n = 0;
  if (B > 0 && n_head > 0) {
    s = splits_for(kv_format, B, n_head, std::max(topk, 1), sm_count(current_device()));
    if (topk == 0) s = 1;
    if (kv_format == DSA_FP8_DS_MLA && s > 1) c = tc_cluster_size(s);
    const bool partials = s > 1 && c == 1;
    if (partials) ws = (size_t)B * n_head * s * (DV + 2) * sizeof(float);
    n = partials ? 2 : 1;
  }
  if (n_splits) *n_splits = s;
  if (cluster_size) *cluster_size = c;
  if (workspace_bytes) *workspace_bytes = ws;
  if (launches) *launches = n;
  return DSA_OK;
}

extern "C" int dsa_sparse_mla_decode(void* o, int o_dtype, float* lse, const void* q, int q_dtype,
                                     const void* kv_cache, int kv_format, int64_t n_kv_rows,
                                     int page_size, const int32_t* idx, int64_t idx_stride,
                                     const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                     const int32_t* seq_lens, int B, int n_head, int topk,
                                     double scale, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  clear_error();
  DSA_REQUIRE(B >= 0 && n_head >= 0 && topk >= 0, DSA_ERR_INVALID,
              "sparse_mla_decode: negative size (B=%d n_head=%d topk=%d)", B, n_head, topk);
  if (B == 0 || n_head == 0) return DSA_OK;
  DSA_REQUIRE(o && lse && q && seq_lens, DSA_ERR_INVALID, "sparse_mla_decode: null pointer");
  DSA_REQUIRE(topk == 0 || (idx && block_table && kv_cache), DSA_ERR_INVALID,
              "sparse_mla_decode: null idx/block_table/kv_cache");
  DSA_REQUIRE(q_dtype == DSA_F16 || q_dtype == DSA_BF16, DSA_ERR_INVALID,
              "sparse_mla_decode: q must be f16 or bf16");
  DSA_REQUIRE(o_dtype == DSA_F16 || o_dtype == DSA_BF16, DSA_ERR_INVALID,
              "sparse_mla_decode: o must be f16 or bf16");
  DSA_REQUIRE(kv_format == DSA_F16 || kv_format == DSA_BF16 || kv_format == DSA_FP8_DS_MLA,
              DSA_ERR_INVALID, "sparse_mla_decode: kv_cache must be f16, bf16 or fp8_ds_mla (u8 656)");
  DSA_REQUIRE(page_size > 0 && max_blocks >= 0 && n_kv_rows >= 0, DSA_ERR_INVALID,
              "sparse_mla_decode: bad cache geometry (page=%d max_blocks=%d rows=%lld)", page_size,
              max_blocks, (long long)n_kv_rows);
  DSA_REQUIRE(idx_stride >= topk && bt_stride >= max_blocks, DSA_ERR_INVALID,
              "sparse_mla_decode: idx/block_table row stride smaller than the row");
  DSA_REQUIRE(((uintptr_t)q & 15) == 0 && ((uintptr_t)kv_cache & 15) == 0 &&
                  ((uintptr_t)o & 15) == 0,
              DSA_ERR_INVALID, "sparse_mla_decode: q, kv_cache and o must be 16-byte aligned");
  DSA_REQUIRE(B <= 0x7fffffff && ((n_head + HT - 1) / HT) <= 65535, DSA_ERR_UNSUPPORTED,
              "sparse_mla_decode: grid too large");
  const int dev = current_device();
  int st = ensure_attrs(dev);
  if (st != DSA_OK) return st;

  const int head_tiles = (n_head + HT - 1) / HT;
  const bool use_tc = kv_format == DSA_FP8_DS_MLA;
  const int tile = use_tc ? kTcTileRows : TN;
  const int n_splits = splits_for(kv_format, B, n_head, topk, sm_count(dev));
  const int ntiles = (topk + tile - 1) / tile;
  const int per = n_splits > 0 ? (ntiles + n_splits - 1) / n_splits : ntiles;

  DecodeParams p{};
  p.q = q;
  p.kv = reinterpret_cast<const uint8_t*>(kv_cache);
  p.idx = idx;
  p.bt = block_table;
  p.seq_lens = seq_lens;
  p.o = o;
  p.lse = lse;
  p.n_kv_rows = n_kv_rows;
  p.idx_stride = idx_stride;
  p.bt_stride = bt_stride;
  p.page_size = page_size;
  p.max_blocks = max_blocks;
  p.B = B;
  p.n_head = n_head;
  p.topk = topk;
  p.n_splits = n_splits;
  p.span = per * tile;
  p.q_bf16 = q_dtype == DSA_BF16;
  p.o_bf16 = o_dtype == DSA_BF16;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  // the tensor-core kernel merges the slices of a row inside a cluster when
  // it can; otherwise slices leave partial states for the merge kernel
  const bool partials = n_splits > 1 && !(use_tc && tc_cluster_size(n_splits) > 1);
  if (partials) {
    const size_t need = (size_t)B * n_head * n_splits * (DV + 2) * sizeof(float);
    DSA_REQUIRE(workspace != nullptr && workspace_bytes >= need, DSA_ERR_WORKSPACE,
                "sparse_mla_decode: workspace needs %zu bytes, got %zu", need, workspace_bytes);
    DSA_REQUIRE(((uintptr_t)workspace & 15) == 0, DSA_ERR_INVALID,
                "sparse_mla_decode: workspace must be 16-byte aligned");
    p.part_o = reinterpret_cast<float*>(workspace);
    p.part_ml = p.part_o + (size_t)B * n_head * n_splits * DV;
  }
  cudaStream_t s = as_stream(stream);
  const dim3 grid(B, head_tiles, n_splits);
  if (use_tc) {
    st = launch_sparse_mla_tc(p, s);
  } else {
    if (kv_format == DSA_BF16)
      sparse_mla_decode_kernel<KV_BF16><<<grid, NTHR, kSmemDecode, s>>>(p);
    else
      sparse_mla_decode_kernel<KV_F16><<<grid, NTHR, kSmemDecode, s>>>(p);
    st = check_launch("sparse_mla_decode_kernel");
  }
  if (st != DSA_OK) return st;
  if (partials) st = launch_sparse_mla_merge(p, s);
  return st;
}
