// Cache writers of the DSA path.
//
// 1. The fp8_ds_mla latent-cache writer (the upstream concat_and_cache_mla
//    with kv_cache_dtype "fp8_ds_mla", whose amax fix the reference carries in
//    patches/glm5-v100-sm70-full.patch:3183-3242; row format
//    csrc/attention/sm70_mla_decode.cu:74-100), with the rotary embedding of
//    k_pe fused in: row slot[t] = 512 e4m3 of kv_c[t] / scale_j per 128-wide
//    tile j | the four f32 scales max(amax_j / 448, FLT_MIN) | 64 fp16 of
//    rope(k_pe[t], positions[t]). One warp per token: lane l owns latent dims
//    [16 l, 16 l + 16) (tile l / 8, amax by three shuffles) and rope pair l.
// 2. The lightning indexer's q / k / weights producer fused into the
//    indexer-K store (the post-GEMM part of Indexer.forward's SM70 branch,
//    full.patch:6404-6425, then sm70_indexer_k_store, dsa.cu:662-706): k =
//    LayerNorm(kw[:, :128]) with the rotary embedding on its first 64 dims is
//    quantised straight into the cache row (no k tensor), q gets the same
//    rotary embedding per head, and weights = kw[:, 128:] * w_scale. One CTA
//    (8 warps) per token: warp 0 the key, all warps the q heads.
//
// Rotary embedding (vLLM's RotaryEmbedding): cos_sin[p] = 32 cos | 32 sin;
// pair i is (x[2i], x[2i+1]) (GPT-J order) or (x[i], x[i + 32]) (NeoX order);
// o1 = x1 cos - x2 sin, o2 = x2 cos + x1 sin, each product and sum rounded in
// f32 (no fused multiply-add), so the CPU check reproduces it bit for bit.
// Everything is computed in f32 from the inputs and rounded once into the
// stored format (the reference rounds to the model dtype after each torch op).
#include <cfloat>

#include "common.cuh"

namespace dsa {
namespace {

constexpr int HD = 128;      // indexer head dim
constexpr int ROPE = 64;     // rotary dims (latent k_pe; first dims of indexer q / k)
constexpr int WARPS = 8;

struct Rope {
  const int64_t* pos;   // null: no rotation (k_pe copied)
  const float* cos_sin; // [max_pos, 64]
  int64_t max_pos;
  int neox;
};

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int bf16) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
              : __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void rotate(float x1, float x2, float c, float s, float& o1, float& o2) {
  o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

// cos / sin of pair i at token t's position (clamped into the table).
__device__ __forceinline__ void cos_sin_of(const Rope& r, int t, int i, float& c, float& s) {
  int64_t p = r.pos[t];
  p = p < 0 ? 0 : (p >= r.max_pos ? r.max_pos - 1 : p);
  c = r.cos_sin[p * ROPE + i];
  s = r.cos_sin[p * ROPE + ROPE / 2 + i];
}

__device__ __forceinline__ void store_out(void* p, int64_t i, float v, int fmt) {
  if (fmt == DSA_F32)
    reinterpret_cast<float*>(p)[i] = v;
  else if (fmt == DSA_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

// --------------------------------------------------------- latent writer
__global__ void __launch_bounds__(WARPS * 32) ds_mla_write_kernel(uint8_t* __restrict__ cache, int64_t n_rows,
                                                                  const void* kv_c, int64_t kv_c_stride,
                                                                  const void* k_pe, int64_t k_pe_stride, int bf16,
                                                                  const int32_t* __restrict__ slot, int n_tok,
                                                                  Rope rope) {
  const int t = blockIdx.x * WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n_tok) return;
  const int64_t row = slot[t];
  if (row < 0 || row >= n_rows) return;
  uint8_t* rp = cache + row * 656;

  // latent: 16 dims per lane, tile = lane / 8
  float f[16];
  {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(kv_c) + ((int64_t)t * kv_c_stride + 16 * lane) * 2;
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint4 b = *reinterpret_cast<const uint4*>(src + 16);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 v;
      if (bf16)
        v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      else
        v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = fmaxf(amax / 448.0f, FLT_MIN);
  uint32_t code[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    code[i] = (uint32_t)f32x2_to_e4m3x2(f[4 * i] / scale, f[4 * i + 1] / scale) |
              ((uint32_t)f32x2_to_e4m3x2(f[4 * i + 2] / scale, f[4 * i + 3] / scale) << 16);
  *reinterpret_cast<uint4*>(rp + 16 * lane) = make_uint4(code[0], code[1], code[2], code[3]);
  if ((lane & 7) == 0) *reinterpret_cast<float*>(rp + 512 + 4 * (lane >> 3)) = scale;

  // rope part: pair `lane`
  const int d1 = rope.neox ? lane : 2 * lane;
  const int d2 = rope.neox ? lane + ROPE / 2 : 2 * lane + 1;
  float x1 = load_elem(k_pe, (int64_t)t * k_pe_stride + d1, bf16);
  float x2 = load_elem(k_pe, (int64_t)t * k_pe_stride + d2, bf16);
  if (rope.pos) {
    float c, s;
    cos_sin_of(rope, t, lane, c, s);
    rotate(x1, x2, c, s, x1, x2);
  }
  __half* rope_out = reinterpret_cast<__half*>(rp + 528);
  rope_out[d1] = __float2half_rn(x1);
  rope_out[d2] = __float2half_rn(x2);
}

// ----------------------------------------- indexer q / k / weights producer
struct ProducerArgs {
  const void* q;         // [T, H, 128] (rows of 128 contiguous, token stride q_stride)
  int64_t q_stride;
  const void* kw;        // [T, 128 + H]: k, then the weight logits
  int64_t kw_stride;
  int bf16;              // input dtype of q and kw
  const float* ln_w;     // [128] LayerNorm weight, or null (1)
  const float* ln_b;     // [128] LayerNorm bias, or null (0)
  float ln_eps;
  Rope rope;
  float w_scale;
  int n_head, n_tok;
  void* q_out;           // [T, H, 128]
  int q_fmt;
  void* w_out;           // [T, H]
  int w_fmt;
  uint8_t* cache;        // indexer-K cache rows
  int cache_fmt;         // DSA_F16, DSA_BF16 or DSA_FP8_IDXK
  int64_t n_rows;
  const int32_t* slot;
};

// Rotary embedding of a 128-dim row held 4 dims per lane (lane l: dims
// 4l..4l+3); only dims < 64 rotate.
__device__ __forceinline__ void rope_row(float (&x)[4], const Rope& r, int t, int lane) {
  if (!r.pos) return;
  if (r.neox) {  // pair i = (i, i + 32): lanes 0-7 hold i, lanes 8-15 hold i + 32
    float y[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = __shfl_xor_sync(0xffffffffu, x[e], 8);
    if (lane < 16) {
      const bool first = lane < 8;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * (lane & 7) + e;
        float c, s, o1, o2;
        cos_sin_of(r, t, i, c, s);
        if (first) {
          rotate(x[e], y[e], c, s, o1, o2);
          x[e] = o1;
        } else {
          rotate(y[e], x[e], c, s, o1, o2);
          x[e] = o2;
        }
      }
    }
  } else if (lane < 16) {  // pairs (2i, 2i+1) inside the lane
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = 2 * lane + e / 2;
      float c, s;
      cos_sin_of(r, t, i, c, s);
      rotate(x[e], x[e + 1], c, s, x[e], x[e + 1]);
    }
  }
}

__global__ void __launch_bounds__(WARPS * 32) indexer_qk_store_kernel(const ProducerArgs a) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == 0) {  // key: LayerNorm, rotary, store
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = load_elem(a.kw, (int64_t)t * a.kw_stride + 4 * lane + e, a.bf16);
    float sum = x[0] + x[1] + x[2] + x[3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const float mean = sum / (float)HD;
    float sq = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) sq += (x[e] - mean) * (x[e] - mean);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    const float rstd = rsqrtf(sq / (float)HD + a.ln_eps);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 4 * lane + e;
      x[e] = (x[e] - mean) * rstd * (a.ln_w ? a.ln_w[d] : 1.f) + (a.ln_b ? a.ln_b[d] : 0.f);
    }
    rope_row(x, a.rope, t, lane);
    const int64_t row = a.slot[t];
    if (row >= 0 && row < a.n_rows) {
      if (a.cache_fmt == DSA_FP8_IDXK) {
        float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        const float scale = fmaxf(amax / 448.0f, FLT_MIN);
        uint8_t* rp = a.cache + row * 132;
        *reinterpret_cast<uint32_t*>(rp + 4 * lane) =
            (uint32_t)f32x2_to_e4m3x2(x[0] / scale, x[1] / scale) |
            ((uint32_t)f32x2_to_e4m3x2(x[2] / scale, x[3] / scale) << 16);
        if (lane == 0) *reinterpret_cast<float*>(rp + 128) = scale;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) store_out(a.cache, row * HD + 4 * lane + e, x[e], a.cache_fmt);
      }
    }
  }
  // q heads: rotary on the first 64 dims
  for (int h = warp; h < a.n_head; h += WARPS) {
    float x[4];
    const int64_t base = (int64_t)t * a.q_stride + (int64_t)h * HD + 4 * lane;
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = load_elem(a.q, base + e, a.bf16);
    rope_row(x, a.rope, t, lane);
    const int64_t ob = ((int64_t)t * a.n_head + h) * HD + 4 * lane;
#pragma unroll
    for (int e = 0; e < 4; ++e) store_out(a.q_out, ob + e, x[e], a.q_fmt);
  }
  // weights
  for (int h = threadIdx.x; h < a.n_head; h += WARPS * 32)
    store_out(a.w_out, (int64_t)t * a.n_head + h,
              __fmul_rn(load_elem(a.kw, (int64_t)t * a.kw_stride + HD + h, a.bf16), a.w_scale), a.w_fmt);
}

bool aligned(const void* p, int b) { return (reinterpret_cast<uintptr_t>(p) % b) == 0; }

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_concat_and_cache_ds_mla(void* kv_cache, int64_t n_rows, const void* kv_c, int64_t kv_c_stride,
                                           const void* k_pe, int64_t k_pe_stride, int in_dtype,
                                           const int32_t* slot, int n_tok, const int64_t* positions,
                                           const float* cos_sin, int64_t max_pos, int rope_neox, void* stream) {
  clear_error();
  DSA_REQUIRE(in_dtype == DSA_F16 || in_dtype == DSA_BF16, DSA_ERR_INVALID,
              "concat_and_cache_ds_mla: kv_c / k_pe must be f16 or bf16");
  DSA_REQUIRE(n_tok >= 0 && n_rows >= 0 && kv_c_stride >= 512 && k_pe_stride >= ROPE, DSA_ERR_INVALID,
              "concat_and_cache_ds_mla: bad sizes or strides");
  if (n_tok == 0) return DSA_OK;
  DSA_REQUIRE(kv_cache && kv_c && k_pe && slot, DSA_ERR_INVALID, "concat_and_cache_ds_mla: null pointer");
  DSA_REQUIRE(aligned(kv_cache, 16) && aligned(kv_c, 16) && kv_c_stride % 8 == 0, DSA_ERR_INVALID,
              "concat_and_cache_ds_mla: kv_cache / kv_c rows must be 16-byte aligned");
  DSA_REQUIRE(!positions || (cos_sin && max_pos > 0), DSA_ERR_INVALID,
              "concat_and_cache_ds_mla: positions need a cos/sin table");
  Rope r{positions, cos_sin, max_pos, rope_neox};
  ds_mla_write_kernel<<<(n_tok + WARPS - 1) / WARPS, WARPS * 32, 0, as_stream(stream)>>>(
      reinterpret_cast<uint8_t*>(kv_cache), n_rows, kv_c, kv_c_stride, k_pe, k_pe_stride, in_dtype == DSA_BF16, slot,
      n_tok, r);
  return check_launch("ds_mla_write_kernel");
}

extern "C" int dsa_indexer_qk_store(void* q_out, int q_out_dtype, void* w_out, int w_out_dtype, void* k_cache,
                                    int cache_format, int64_t n_rows, const void* q, int64_t q_stride,
                                    const void* kw, int64_t kw_stride, int in_dtype, const float* ln_weight,
                                    const float* ln_bias, float ln_eps, const int64_t* positions,
                                    const float* cos_sin, int64_t max_pos, int rope_neox, float w_scale,
                                    const int32_t* slot, int n_tok, int n_head, void* stream) {
  clear_error();
  DSA_REQUIRE(in_dtype == DSA_F16 || in_dtype == DSA_BF16, DSA_ERR_INVALID, "indexer_qk_store: q / kw must be f16 or bf16");
  DSA_REQUIRE(q_out_dtype == DSA_F16 || q_out_dtype == DSA_BF16, DSA_ERR_INVALID,
              "indexer_qk_store: q_out must be f16 or bf16");
  DSA_REQUIRE(w_out_dtype == DSA_F16 || w_out_dtype == DSA_BF16 || w_out_dtype == DSA_F32, DSA_ERR_INVALID,
              "indexer_qk_store: weights out must be f16, bf16 or f32");
  DSA_REQUIRE(cache_format == DSA_F16 || cache_format == DSA_BF16 || cache_format == DSA_FP8_IDXK,
              DSA_ERR_INVALID, "indexer_qk_store: cache must be f16, bf16 or fp8 indexer-K");
  DSA_REQUIRE(n_tok >= 0 && n_head >= 1 && n_head <= 256 && q_stride >= (int64_t)n_head * HD &&
                  kw_stride >= HD + n_head,
              DSA_ERR_INVALID, "indexer_qk_store: bad sizes or strides");
  if (n_tok == 0) return DSA_OK;
  DSA_REQUIRE(q_out && w_out && k_cache && q && kw && slot, DSA_ERR_INVALID, "indexer_qk_store: null pointer");
  DSA_REQUIRE(!positions || (cos_sin && max_pos > 0), DSA_ERR_INVALID,
              "indexer_qk_store: positions need a cos/sin table");
  DSA_REQUIRE(cache_format != DSA_FP8_IDXK || aligned(k_cache, 4), DSA_ERR_INVALID,
              "indexer_qk_store: fp8 cache must be 4-byte aligned");
  ProducerArgs a{};
  a.q = q;
  a.q_stride = q_stride;
  a.kw = kw;
  a.kw_stride = kw_stride;
  a.bf16 = in_dtype == DSA_BF16;
  a.ln_w = ln_weight;
  a.ln_b = ln_bias;
  a.ln_eps = ln_eps;
  a.rope = Rope{positions, cos_sin, max_pos, rope_neox};
  a.w_scale = w_scale;
  a.n_head = n_head;
  a.n_tok = n_tok;
  a.q_out = q_out;
  a.q_fmt = q_out_dtype;
  a.w_out = w_out;
  a.w_fmt = w_out_dtype;
  a.cache = reinterpret_cast<uint8_t*>(k_cache);
  a.cache_fmt = cache_format;
  a.n_rows = n_rows;
  a.slot = slot;
  indexer_qk_store_kernel<<<n_tok, WARPS * 32, 0, as_stream(stream)>>>(a);
  return check_launch("indexer_qk_store_kernel");
}
