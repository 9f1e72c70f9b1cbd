// Indexer-K cache scatter: cache row slot[t] <- k[t] (slot < 0 / out of range skipped).
//
// Replaces sm70_indexer_k_store (csrc/attention/sm70_mla_decode.cu:2910-2939,
// kernels :662-706). One warp per token: 16-byte / 8-byte vector accesses,
// the fp8 row's amax by warp shuffle, e4m3 packing by the hardware
// round-to-nearest-even saturating converter. The quantisation rule is the
// reference's: scale = max(amax / 448, FLT_MIN), code = e4m3(v / scale), row
// = 128 codes | f32 scale (dsa.cu:692-705).
#include <cfloat>
#include <type_traits>

#include "common.cuh"

namespace dsa {
namespace {

constexpr int WARPS = 8;

template <typename TIn>
__device__ __forceinline__ float4 load4(const TIn* src);
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* src) {
  const uint2 v = *reinterpret_cast<const uint2*>(src);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* src) {
  const uint2 v = *reinterpret_cast<const uint2*>(src);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename TIn>
__global__ void __launch_bounds__(WARPS * 32) k_store_fp8_kernel(const TIn* __restrict__ k,
                                                                 const int32_t* __restrict__ slot,
                                                                 uint8_t* __restrict__ cache, int n_tok,
                                                                 int64_t n_rows) {
  const int t = blockIdx.x * WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n_tok) return;
  const int64_t row = slot[t];
  if (row < 0 || row >= n_rows) return;
  const float4 v = load4(k + (int64_t)t * 128 + 4 * lane);
  float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  const float scale = fmaxf(a / 448.0f, FLT_MIN);
  const uint32_t lo = f32x2_to_e4m3x2(v.x / scale, v.y / scale);
  const uint32_t hi = f32x2_to_e4m3x2(v.z / scale, v.w / scale);
  uint8_t* rp = cache + row * 132;
  *reinterpret_cast<uint32_t*>(rp + 4 * lane) = lo | (hi << 16);
  if (lane == 0) *reinterpret_cast<float*>(rp + 128) = scale;
}

template <typename TIn, typename TOut>
__device__ __forceinline__ TOut convert(TIn v);
template <>
__device__ __forceinline__ __half convert<__half, __half>(__half v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 convert<__nv_bfloat16, __nv_bfloat16>(__nv_bfloat16 v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 convert<__half, __nv_bfloat16>(__half v) {
  return __float2bfloat16_rn(__half2float(v));
}
template <>
__device__ __forceinline__ __half convert<__nv_bfloat16, __half>(__nv_bfloat16 v) {
  return __float2half_rn(__bfloat162float(v));
}

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(WARPS * 32) k_store_copy_kernel(const TIn* __restrict__ k,
                                                                  const int32_t* __restrict__ slot,
                                                                  TOut* __restrict__ cache, int n_tok,
                                                                  int head_dim, int64_t n_rows) {
  const int t = blockIdx.x * WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n_tok) return;
  const int64_t row = slot[t];
  if (row < 0 || row >= n_rows) return;
  const TIn* src = k + (int64_t)t * head_dim;
  TOut* dst = cache + row * head_dim;
  if (sizeof(TIn) == sizeof(TOut) && (head_dim & 7) == 0 && std::is_same<TIn, TOut>::value) {
    for (int c = lane; c < head_dim / 8; c += 32)
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
  } else {
    for (int d = lane; d < head_dim; d += 32) dst[d] = convert<TIn, TOut>(src[d]);
  }
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_indexer_k_store(void* kv_cache, int cache_format, int64_t n_rows, const void* k, int k_dtype,
                                   int head_dim, const int32_t* slot, int n_tok, void* stream) {
  clear_error();
  DSA_REQUIRE(n_tok >= 0 && n_rows >= 0 && head_dim > 0, DSA_ERR_INVALID,
              "indexer_k_store: bad sizes (n_tok=%d n_rows=%lld head_dim=%d)", n_tok, (long long)n_rows,
              head_dim);
  if (n_tok == 0) return DSA_OK;
  DSA_REQUIRE(kv_cache && k && slot, DSA_ERR_INVALID, "indexer_k_store: null pointer");
  DSA_REQUIRE(k_dtype == DSA_F16 || k_dtype == DSA_BF16, DSA_ERR_INVALID, "indexer_k_store: k must be f16 or bf16");
  cudaStream_t s = as_stream(stream);
  const int grid = (n_tok + WARPS - 1) / WARPS;
  if (cache_format == DSA_FP8_IDXK) {
    DSA_REQUIRE(head_dim == 128, DSA_ERR_UNSUPPORTED, "indexer_k_store: fp8 cache requires head_dim 128");
    DSA_REQUIRE(((uintptr_t)k & 7) == 0 && ((uintptr_t)kv_cache & 3) == 0, DSA_ERR_INVALID,
                "indexer_k_store: misaligned k or cache");
    if (k_dtype == DSA_BF16)
      k_store_fp8_kernel<__nv_bfloat16><<<grid, WARPS * 32, 0, s>>>(
          reinterpret_cast<const __nv_bfloat16*>(k), slot, reinterpret_cast<uint8_t*>(kv_cache), n_tok, n_rows);
    else
      k_store_fp8_kernel<__half><<<grid, WARPS * 32, 0, s>>>(reinterpret_cast<const __half*>(k), slot,
                                                             reinterpret_cast<uint8_t*>(kv_cache), n_tok, n_rows);
    return check_launch("k_store_fp8_kernel");
  }
  DSA_REQUIRE(cache_format == DSA_F16 || cache_format == DSA_BF16, DSA_ERR_INVALID,
              "indexer_k_store: cache must be f16, bf16 or fp8 (u8 132)");
  DSA_REQUIRE(((uintptr_t)k & 15) == 0 && ((uintptr_t)kv_cache & 15) == 0, DSA_ERR_INVALID,
              "indexer_k_store: k and cache must be 16-byte aligned");
  if (k_dtype == DSA_F16 && cache_format == DSA_F16)
    k_store_copy_kernel<__half, __half><<<grid, WARPS * 32, 0, s>>>(
        reinterpret_cast<const __half*>(k), slot, reinterpret_cast<__half*>(kv_cache), n_tok, head_dim, n_rows);
  else if (k_dtype == DSA_BF16 && cache_format == DSA_BF16)
    k_store_copy_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, WARPS * 32, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(k), slot, reinterpret_cast<__nv_bfloat16*>(kv_cache), n_tok,
        head_dim, n_rows);
  else if (k_dtype == DSA_F16)
    k_store_copy_kernel<__half, __nv_bfloat16><<<grid, WARPS * 32, 0, s>>>(
        reinterpret_cast<const __half*>(k), slot, reinterpret_cast<__nv_bfloat16*>(kv_cache), n_tok, head_dim,
        n_rows);
  else
    k_store_copy_kernel<__nv_bfloat16, __half><<<grid, WARPS * 32, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(k), slot, reinterpret_cast<__half*>(kv_cache), n_tok, head_dim,
        n_rows);
  return check_launch("k_store_copy_kernel");
}
