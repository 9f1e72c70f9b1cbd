// Shared helpers for the DSA B200 kernels: status reporting, dtype
// conversion, fp8 e4m3 handling, monotone float keys, warp MMA wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/dsa_b200.h"

namespace dsa {

// ---------------------------------------------------------------- status
// Thread-local last-error text (dsa_last_error()).
void set_error(const char* fmt, ...);
void clear_error();

// Returns DSA_ERR_CUDA (with text) when the last launch failed.
int check_launch(const char* what);

#define DSA_REQUIRE(cond, code, ...)        \
  do {                                      \
    if (!(cond)) {                          \
      ::dsa::set_error(__VA_ARGS__);        \
      return (code);                        \
    }                                       \
  } while (0)

#define DSA_CUDA_TRY(call, what)                                           \
  do {                                                                     \
    cudaError_t e_ = (call);                                               \
    if (e_ != cudaSuccess) {                                               \
      ::dsa::set_error("%s: %s", (what), cudaGetErrorString(e_));          \
      return DSA_ERR_CUDA;                                                 \
    }                                                                      \
  } while (0)

// Per-device one-time initialisation (function attributes are per device).
constexpr int kMaxDevices = 64;
int current_device();
int sm_count(int dev);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ----------------------------------------------------------- conversions
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

// Four consecutive e4m3 bytes (packed in a uint32) -> two half2, exact.
__device__ __forceinline__ void e4m3x4_to_half2x2(uint32_t v, __half2& lo, __half2& hi) {
  __half2_raw r0 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v & 0xFFFFu), __NV_E4M3);
  __half2_raw r1 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(v >> 16), __NV_E4M3);
  lo = *reinterpret_cast<__half2*>(&r0);
  hi = *reinterpret_cast<__half2*>(&r1);
}

// Four e4m3 bytes -> two half2 words holding value / 256 each, exactly, with
// integer operations only (no conversion-pipe instructions): each byte goes to
// a 16-bit lane with its sign replicated above it (prmt sign-extension
// selectors), and a shift puts exponent + mantissa in fp16 bits 7..13 and the
// sign on bit 15 (bit 14 cleared). e4m3's exponent bias (7) vs fp16's (15) is
// the 2^-8 factor; e4m3 subnormals become fp16 subnormals. lo holds bytes 0, 1
// and hi bytes 2, 3.
__device__ __forceinline__ void e4m3x4_to_half2x2_div256(uint32_t w, uint32_t& lo, uint32_t& hi) {
  uint32_t a, b;
  asm("prmt.b32 %0, %1, 0, 0x9180;" : "=r"(a) : "r"(w));
  asm("prmt.b32 %0, %1, 0, 0xB3A2;" : "=r"(b) : "r"(w));
  lo = (a << 7) & 0xBF80BF80u;
  hi = (b << 7) & 0xBF80BF80u;
}

// Two floats -> two e4m3 bytes (round-to-nearest-even, saturating to +-448).
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// f32 -> uint32 whose unsigned order is the float order.
__device__ __forceinline__ uint32_t monotone32(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// bf16 pair (as uint32) -> half2 (exact for values in the half normal range).
__device__ __forceinline__ uint32_t bf16x2_to_half2_bits(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  float2 f = __bfloat1622float2(b);
  return pack_half2(f.x, f.y);
}

__device__ __forceinline__ uint4 bf16x8_to_half8(uint4 v) {
  return make_uint4(bf16x2_to_half2_bits(v.x), bf16x2_to_half2_bits(v.y),
                    bf16x2_to_half2_bits(v.z), bf16x2_to_half2_bits(v.w));
}

// Largest |x| of eight bf16 values, as its 15-bit magnitude pattern (the
// unsigned order of these patterns is the order of |x|).
__device__ __forceinline__ uint32_t bf16x8_max_abs_bits(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) m = max(m, max(w[i] & 0x7FFFu, (w[i] >> 16) & 0x7FFFu));
  return m;
}

// Power-of-two shift qe such that x * 2^-qe puts the largest magnitude
// (pattern `bits`) in [2^14, 2^15): inside fp16's normal range with room to
// spare, whatever the bf16 exponent (small values are scaled up, so they do
// not fall into fp16 subnormals). Clamped so 2^+-qe stays a normal float.
__device__ __forceinline__ int bf16_fp16_shift(uint32_t bits) {
  return min(114, max(-100, (int)((bits >> 7) & 0xFFu) - 141));
}

// bf16 pair x 2^-qe -> half2 bits (exact while the scaled values stay in the
// half normal range; qe = 0 is a plain conversion).
__device__ __forceinline__ uint32_t bf16x2_to_half2_scaled(uint32_t v, float mul) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  float2 f = __bfloat1622float2(b);
  return pack_half2(f.x * mul, f.y * mul);
}

__device__ __forceinline__ uint4 bf16x8_to_half8_scaled(uint4 v, int qe) {
  const float mul = __int_as_float((127 - qe) << 23);  // 2^-qe, exact
  return make_uint4(bf16x2_to_half2_scaled(v.x, mul), bf16x2_to_half2_scaled(v.y, mul),
                    bf16x2_to_half2_scaled(v.z, mul), bf16x2_to_half2_scaled(v.w, mul));
}

// --------------------------------------------------------- shared memory
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D += A * B, m16n8k16, f16 inputs, f32 accumulators.
__device__ __forceinline__ void mma_f16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gptr));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Read-only 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Bulk prefetch of [p, p + bytes) into L2 (p and bytes multiples of 16);
// no registers or scoreboards are held while it is in flight.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------- cross-GPU flags (P2P exchange)
__device__ __forceinline__ int ld_acquire_sys_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_s32(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int read_err_word(const int32_t* err) {
  return err ? *reinterpret_cast<const volatile int32_t*>(err) : 0;
}

// Bounded wait until *flag >= target. Returns false after timeout_ns of
// device time (recording DSA_ERR_TIMEOUT in *err) or as soon as the error
// word is set by another wait.
__device__ __forceinline__ bool wait_flag_geq(const int* flag, int target, int64_t timeout_ns, int32_t* err) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (ld_acquire_sys_s32(flag) < target) {
    if ((++spins & 63u) == 0) {
      if (read_err_word(err) != 0) return false;
      if ((int64_t)(globaltimer_ns() - t0) > timeout_ns) {
        if (err) atomicExch(err, (int32_t)DSA_ERR_TIMEOUT);
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

}  // namespace dsa
