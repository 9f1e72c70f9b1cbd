// Sparse MLA decode that allocates nothing: the per-slice partial states,
// which dsa_sparse_mla_decode keeps in a caller workspace, live here in a
// fixed array of this library's own device memory.
//
// Who needs it: callers that cannot allocate device memory when they decode.
// Examples are an engine that gives the whole GPU to its own pool allocator
// at start-up (a later cudaMalloc fails or fragments that pool), a plugin
// host whose ABI passes only the input and output buffers, and plain C code
// that has no CUDA allocator of its own. They call
// dsa_sparse_mla_decode_noalloc and never see a workspace. This entry point
// calls no cudaMalloc, no cudaFree and no allocating library routine.
//
// Limits, which the header repeats:
//   * The array holds kScratchBytes (32 MiB). Every GPU that loads this
//     library keeps it reserved until the process exits.
//   * A call whose slices need more scratch than that is rejected with
//     DSA_ERR_WORKSPACE before anything is launched.
//   * Every call uses the same array, and it keeps whatever the last call
//     left there. Nothing in it has to start at zero: the decode kernels write
//     every partial state (o, running max, row sum) of each (row, head, slice)
//     before the merge reads it. Two calls that overlap on the GPU (on
//     different streams, or from different host threads without ordering)
//     race on the array and may corrupt each other's outputs.
//   * The first call on a device looks up the array's device address. Make
//     that first call before any stream capture begins.
#include <mutex>
#include <string>

#include "common.cuh"

namespace dsa {
namespace {

constexpr size_t kScratchBytes = (size_t)32 << 20;
constexpr int kMaxDevices = 64;

// Split partial states for dsa_sparse_mla_decode_noalloc. In host code this
// name is only a host-side stand-in for the array; kernels get the device
// address that cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device, looked up once
// per device with that device current.
int scratch_address(void** out) {
  int dev = -1;
  DSA_CUDA_TRY(cudaGetDevice(&dev), "sparse_mla_decode_noalloc: cudaGetDevice");
  DSA_REQUIRE(dev >= 0 && dev < kMaxDevices, DSA_ERR_UNSUPPORTED,
              "sparse_mla_decode_noalloc: device %d is beyond the %d devices it supports", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    DSA_CUDA_TRY(cudaGetSymbolAddress(&p, g_decode_scratch),
                 "sparse_mla_decode_noalloc: cudaGetSymbolAddress of the static scratch");
    DSA_REQUIRE(p != nullptr, DSA_ERR_CUDA, "sparse_mla_decode_noalloc: static scratch has no device address");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DSA_OK;
}

}  // namespace
}  // namespace dsa

extern "C" int dsa_sparse_mla_decode_noalloc(void* o, int o_dtype, float* lse, const void* q, int q_dtype,
                                             const void* kv_cache, int kv_format, int64_t n_kv_rows,
                                             int page_size, const int32_t* idx, int64_t idx_stride,
                                             const int32_t* block_table, int64_t bt_stride, int max_blocks,
                                             const int32_t* seq_lens, int B, int n_head, int topk,
                                             double scale, void* stream) {
  dsa::clear_error();
  void* scratch = nullptr;
  int st = dsa::scratch_address(&scratch);
  if (st != DSA_OK) return st;
  st = dsa_sparse_mla_decode(o, o_dtype, lse, q, q_dtype, kv_cache, kv_format, n_kv_rows, page_size, idx,
                             idx_stride, block_table, bt_stride, max_blocks, seq_lens, B, n_head, topk, scale,
                             scratch, dsa::kScratchBytes, stream);
  if (st == DSA_ERR_WORKSPACE) {
    // raised before any launch: this call's slices need more than the array
    const std::string inner = dsa_last_error();
    dsa::set_error(
        "sparse_mla_decode_noalloc: the call needs more scratch than the library's static %zu bytes (%s); "
        "decode fewer rows per call, or use dsa_sparse_mla_decode with a caller workspace",
        dsa::kScratchBytes, inner.c_str());
  }
  return st;
}
