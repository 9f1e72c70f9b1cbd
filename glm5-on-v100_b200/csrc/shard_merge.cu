// Exact merge of key-sharded indexer top-k candidates, local or over peer
// memory, and the CUDA IPC helpers of the P2P shard exchange.
//
// Replaces sm70_indexer_shard_merge / sm70_indexer_shard_merge_p2p and the
// IPC helpers (csrc/attention/sm70_mla_decode.cu:2054-2434) and the torch.topk
// epilogue they fuse (reference/sparse_attn_indexer.py:1007-1030).
//
// One CTA (512 threads) per row. Every candidate column col = s*K + c gets the
// distinct 64-bit key (monotone32(val) << 32) | (tp*K - 1 - col), so an
// MSB-first byte radix walk finds the exact K-th key and ties resolve to the
// lower column. Keys stay in registers (<= 32 per thread, tp <= 8); each pass
// only visits candidates still matching the prefix. The selected positions
// (-1 for -inf values) are sorted ascending with a bitonic network in shared
// memory. The P2P variant reads each shard straight from the peer's buffer
// with plain loads (no TMA) after a bounded acquire-wait on the
// peer's staged flag.
#include <climits>

#include "common.cuh"

namespace dsa {
namespace {

constexpr int MNT = 512;
constexpr int MAX_PER = 32;  // tp * K / MNT <= 32  (tp <= 8, K <= 2048)
constexpr int MAX_TP = 8;
constexpr int MAX_K = 2048;

struct ShardSrc {
  const uint8_t* base[MAX_TP];  // shard s slab: [R, 2K] f32 at base[s] (+ slot_off)
  const int* staged[MAX_TP];    // P2P only: &flags[s][0]
};

struct MergeParams {
  ShardSrc src;
  int32_t* out;
  const int32_t* dst_rows;
  int32_t* err;
  int64_t out_stride;
  int64_t shard_stride;  // bytes between shards for the local [tp, R, 2K] layout (0 for P2P)
  int64_t timeout_ns;
  int R, tp, K, dst_base, seq;
  int p2p;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait: returns false (and records DSA_ERR_TIMEOUT in *err) when
// flag < target after timeout_ns of device time, or when another wait of the
// same launch already gave up.
__device__ bool wait_flag_geq(const int* flag, int target, int64_t timeout_ns, int32_t* err) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (ld_acquire_sys(flag) < target) {
    if ((++spins & 63u) == 0) {
      if (err && *reinterpret_cast<volatile int32_t*>(err) != 0) return false;
      if ((int64_t)(globaltimer_ns() - t0) > timeout_ns) {
        if (err) atomicExch(err, (int32_t)DSA_ERR_TIMEOUT);
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

__global__ void __launch_bounds__(MNT) shard_merge_kernel(const MergeParams p) {
  __shared__ uint32_t s_hist[256];
  __shared__ int32_t s_sel[MAX_K];
  __shared__ uint32_t s_cnt;
  __shared__ unsigned long long s_prefix;
  __shared__ uint32_t s_target;
  __shared__ uint32_t s_eq;  // keys matching the new prefix
  __shared__ int s_ok;

  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const int K = p.K;
  const int ncand = p.tp * K;
  const int nper = (ncand + MNT - 1) / MNT;

  if (p.p2p) {
    if (tid == 0) s_ok = 1;
    __syncthreads();
    if (tid < p.tp) {
      if (!wait_flag_geq(p.src.staged[tid], p.seq, p.timeout_ns, p.err)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) return;  // output undefined; the host reads *err
    __threadfence_system();
  }

  auto slab = [&](int s) -> const float* {
    return reinterpret_cast<const float*>(p.src.base[s] + (p.p2p ? 0 : (int64_t)s * p.shard_stride)) +
           (int64_t)r * 2 * K;
  };

  // all of this thread's candidate values are loaded before any is used, so
  // the loads are in flight together
  float val[MAX_PER];
#pragma unroll
  for (int i = 0; i < MAX_PER; ++i) {
    const int col = tid + i * MNT;
    val[i] = 0.f;
    if (i < nper && col < ncand) {
      const int s = col / K, c = col - s * K;
      val[i] = __ldg(slab(s) + c);
    }
  }
  unsigned long long key[MAX_PER];
  uint32_t act = 0;
#pragma unroll
  for (int i = 0; i < MAX_PER; ++i) {
    key[i] = 0ull;
    const int col = tid + i * MNT;
    if (i < nper && col < ncand) {
      key[i] = ((unsigned long long)monotone32(val[i]) << 32) | (uint32_t)(ncand - 1 - col);
      act |= 1u << i;
    }
  }
  if (tid == 0) {
    s_prefix = 0ull;
    s_target = (uint32_t)K;
    s_cnt = 0;
  }
  const uint32_t valid_mask = act;
  for (int byte = 7; byte >= 0; --byte) {
    for (int i = tid; i < 256; i += MNT) s_hist[i] = 0;
    __syncthreads();
    const int sh = 8 * byte;
    const unsigned long long hi_mask = byte == 7 ? 0ull : (~0ull << (sh + 8));
    const unsigned long long pfx = s_prefix;
#pragma unroll
    for (int i = 0; i < MAX_PER; ++i) {
      if (!(act & (1u << i))) continue;
      if ((key[i] & hi_mask) != (pfx & hi_mask)) {
        act &= ~(1u << i);
        continue;
      }
      atomicAdd(&s_hist[(key[i] >> sh) & 0xFFu], 1u);
    }
    __syncthreads();
    if (tid < 32) {  // warp 0: lane owns bins [8*lane, 8*lane+8)
      const uint32_t tgt = s_target;
      __syncwarp();
      uint32_t cs = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) cs += s_hist[8 * tid + j];
      uint32_t suf = cs;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, suf, off);
        if (tid + off < 32) suf += v;
      }
      const uint32_t above = suf - cs;
      if (above < tgt && suf >= tgt) {
        uint32_t run = above;
        for (int j = 7; j >= 0; --j) {
          const uint32_t c = s_hist[8 * tid + j];
          if (run + c >= tgt) {
            s_prefix = pfx | ((unsigned long long)(8 * tid + j) << sh);
            s_target = tgt - run;
            s_eq = c;
            break;
          }
          run += c;
        }
      }
    }
    __syncthreads();
    // after the value bytes: when every key with the K-th value is needed the
    // column bytes (which only order equal values) cannot change the cut
    if (byte == 4 && s_target == s_eq) break;
  }
  const unsigned long long T = s_prefix;
#pragma unroll
  for (int i = 0; i < MAX_PER; ++i) {
    if (!(valid_mask & (1u << i))) continue;
    if (key[i] >= T) {
      const uint32_t slot = atomicAdd(&s_cnt, 1u);
      int32_t pos = -1;
      if ((uint32_t)(key[i] >> 32) > 0x007FFFFFu) {  // not -inf
        const int col = tid + i * MNT;
        const int s = col / K, c = col - s * K;
        pos = __float_as_int(slab(s)[K + c]);
      }
      if (slot < (uint32_t)K) s_sel[slot] = pos;
    }
  }
  __syncthreads();
  // ascending bitonic sort over the next power of two (padding sorts last)
  int np2 = 1;
  while (np2 < K) np2 <<= 1;
  for (int i = K + tid; i < np2; i += MNT) s_sel[i] = INT_MAX;
  __syncthreads();
  for (int k2 = 2; k2 <= np2; k2 <<= 1) {
    for (int j = k2 >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += MNT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const int32_t a = s_sel[i], c = s_sel[ixj];
          const bool up = (i & k2) == 0;
          if ((a > c) == up) {
            s_sel[i] = c;
            s_sel[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const int64_t dst = p.dst_base >= 0 ? (int64_t)p.dst_base + r : (int64_t)p.dst_rows[r];
  for (int i = tid; i < K; i += MNT) p.out[dst * p.out_stride + i] = s_sel[i];
}

__global__ void ipc_flag_set_kernel(int* flag, int seq) {
  __threadfence_system();
  st_release_sys(flag, seq);
}

struct FlagPtrs {
  const int* merged[MAX_TP];  // &flags[s][1]
};

__global__ void ipc_slot_wait_kernel(FlagPtrs f, int tp, int min_seq, int64_t timeout_ns, int32_t* err) {
  if ((int)threadIdx.x < tp) wait_flag_geq(f.merged[threadIdx.x], min_seq, timeout_ns, err);
  __syncthreads();
  __threadfence_system();
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
  MergeParams p{};
  for (int s = 0; s < MAX_TP; ++s) p.src.base[s] = reinterpret_cast<const uint8_t*>(allf);
  p.shard_stride = (int64_t)R * 2 * K * sizeof(float);
  p.out = out;
  p.dst_rows = dst_rows;
  p.out_stride = out_stride;
  p.R = R;
  p.tp = tp;
  p.K = K;
  p.dst_base = dst_base;
  shard_merge_kernel<<<R, MNT, 0, as_stream(stream)>>>(p);
  return check_launch("shard_merge_kernel");
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
  MergeParams p{};
  for (int s = 0; s < tp; ++s) {
    DSA_REQUIRE(data_ptrs[s] != 0 && flag_ptrs[s] != 0, DSA_ERR_INVALID, "shard_merge_p2p: null peer pointer %d", s);
    p.src.base[s] = reinterpret_cast<const uint8_t*>(data_ptrs[s]) + slot_off;
    p.src.staged[s] = reinterpret_cast<const int*>(flag_ptrs[s]);
  }
  p.out = out;
  p.dst_rows = dst_rows;
  p.err = err_flag;
  p.out_stride = out_stride;
  p.timeout_ns = timeout_ns;
  p.R = R;
  p.tp = tp;
  p.K = K;
  p.dst_base = dst_base;
  p.seq = seq;
  p.p2p = 1;
  shard_merge_kernel<<<R, MNT, 0, as_stream(stream)>>>(p);
  return check_launch("shard_merge_kernel(p2p)");
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

extern "C" int dsa_ipc_flag_set(uint64_t flag_ptr, int which, int seq, void* stream) {
  clear_error();
  DSA_REQUIRE(flag_ptr != 0 && (which == 0 || which == 1), DSA_ERR_INVALID, "ipc_flag_set: bad arguments");
  ipc_flag_set_kernel<<<1, 1, 0, as_stream(stream)>>>(reinterpret_cast<int*>(flag_ptr) + which, seq);
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
