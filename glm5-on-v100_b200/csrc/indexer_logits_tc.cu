// Lightning-indexer logits for prefill on the 5th-generation tensor cores:
//   score[r, p] = sum_h w[r,h] * relu(q[r,h,:] . k_p)   for p < seq_lens[r]
//   score[r, p] = -inf                                 for seq_lens[r] <= p < max_kv
// Same function as the reference's multi-row WMMA kernels
// (csrc/attention/sm70_mla_decode.cu:345-458, :542-653) under the same
// contract: the rows of one call belong to one request, and the first row of
// each tile supplies the block table that resolves the key positions
// (sm70_mla_decode.cu:372).
//
// One CTA = 128 query rows x 256 key positions, 16 warps:
//   * TMA brings the key tile (256 rows of the paged cache, one box per page
//     run, zero-filled where a block is missing) into 128-byte-swizzled
//     shared memory once, and the 128 x 128 query tile of every indexer head
//     through a 3-stage ring (a 3-D tensor map over q[B, heads, 128]).
//   * Lane 0 of warp 0 issues, per head, S_h[128 x 256] = Q_h . K^T as eight
//     M=128, N=256, K=16 tcgen05 MMAs (fp32 accumulation in TMEM). S is
//     double-buffered in TMEM (2 x 256 columns), so the MMAs of head h+1 run
//     while the warps read S_h.
//   * Each thread owns one query row and 64 key columns of S: it reads them
//     with tcgen05.ld and accumulates w[r,h] * relu(s) in registers; after
//     the last head it writes the row's 64 scores (masked to -inf past the
//     row's length).
// Every wait is bounded by device time; on expiry the CTA records
// DSA_ERR_TIMEOUT in the sticky status word, drains its own copies and MMAs,
// frees TMEM and returns without writing scores.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>

#include "indexer_tc.cuh"
#include "sparse_mla.cuh"
#include "tc_common.cuh"

namespace dsa {
namespace {

using namespace tc;

constexpr int QM = 128;  // query rows per tile (MMA M)
constexpr int KN = 256;  // key positions per tile (MMA N)
constexpr int HD = 128;
constexpr int NWARPS = 16;
constexpr int NTHREADS = NWARPS * 32;
constexpr int QSTAGES = 3;
constexpr int MAX_HEADS = 64;
constexpr uint32_t KTILE_BYTES = KN * HD * 2;   // 64 KB: two 64-dim regions of 256 x 128 B
constexpr uint32_t QSTAGE_BYTES = QM * HD * 2;  // 32 KB: two 64-dim regions of 128 x 128 B
constexpr uint32_t OFF_K = 0;
constexpr uint32_t OFF_Q = OFF_K + KTILE_BYTES;
constexpr uint32_t OFF_W = OFF_Q + QSTAGES * QSTAGE_BYTES;
constexpr uint32_t OFF_MISC = OFF_W + MAX_HEADS * QM * 4;
constexpr uint32_t MISC_BYTES = 1024;
constexpr uint32_t SMEM_BYTES = OFF_MISC + MISC_BYTES + 1024;  // + alignment slack
constexpr uint32_t TMEM_COLS = 512;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ float load_weight(const IndexerTcArgs& a, int64_t i) {
  if (a.w_dtype == DSA_F32) return reinterpret_cast<const float*>(a.w)[i];
  if (a.w_dtype == DSA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.w)[i]);
  return __half2float(reinterpret_cast<const __half*>(a.w)[i]);
}

template <bool BF16>
__global__ void __launch_bounds__(NTHREADS, 1)
    indexer_logits_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                             const IndexerTcArgs a, const int k_box_rows, int32_t* err) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;  // swizzled tiles need 1024-byte alignment
  unsigned char* smem = smem_raw + pad;
  const uint32_t sbase = raw + pad;
  float* s_w = reinterpret_cast<float*>(smem + OFF_W);  // [head][row]
  unsigned char* misc = smem + OFF_MISC;
  const uint32_t mb = sbase + OFF_MISC;
  const uint32_t mb_k = mb;                                       // key tile landed
  auto mb_q_full = [&](int s) { return mb + 8u + 8u * (uint32_t)s; };   // Q stage landed
  auto mb_s_full = [&](int b) { return mb + 32u + 8u * (uint32_t)b; };  // S buffer written
  auto mb_s_free = [&](int b) { return mb + 48u + 8u * (uint32_t)b; };  // S buffer read by all warps
  const uint32_t mb_done = mb + 64u;                              // drain after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 72);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 76);
  int* s_maxlen = reinterpret_cast<int*>(misc + 80);
  int* s_len = reinterpret_cast<int*>(misc + 128);  // [QM]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p0 = blockIdx.x * KN;
  const int q0 = blockIdx.y * QM;
  const int nrows = min(QM, a.B - q0);

  if (tid == 0) {
    *s_maxlen = 0;
    *abort_flag = 0;
  }
  __syncthreads();
  if (tid < QM) {
    const int len = tid < nrows ? min(a.seq_lens[q0 + tid], a.max_kv) : 0;
    s_len[tid] = len;
    if (len > 0) atomicMax(s_maxlen, len);
  }
  __syncthreads();
  const int maxlen = *s_maxlen;
  const int p_hi = min(p0 + KN, a.max_kv);
  if (p0 >= maxlen) {  // every row of the tile is past its length here
    const int cols = p_hi - p0;
    for (int i = tid; i < nrows * cols; i += NTHREADS) {
      const int r = i / cols, c = i - r * cols;
      a.score[(int64_t)(q0 + r) * a.score_stride + p0 + c] = -INFINITY;
    }
    return;
  }

  if (warp == 0) tmem_alloc(sbase + OFF_MISC + 72, TMEM_COLS);
  if (tid == 32) {
    mbar_init(mb_k, 1);
    for (int s = 0; s < QSTAGES; ++s) mbar_init(mb_q_full(s), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(mb_s_full(b), 1);
      mbar_init(mb_s_free(b), NWARPS);
    }
    mbar_init(mb_done, 1);
    mbar_init_fence();
  }
  const int H = a.n_ihead;
  for (int i = tid; i < QM * H; i += NTHREADS) {
    const int r = i / H, h = i - r * H;
    s_w[h * QM + r] = r < nrows ? load_weight(a, (int64_t)(q0 + r) * H + h) : 0.f;
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  const uint64_t tmq = reinterpret_cast<uint64_t>(&tm_q);
  const uint64_t tmk = reinterpret_cast<uint64_t>(&tm_k);
  constexpr uint32_t IDESC = idesc_f16(QM, KN, false, false, BF16);
  bool ok = true;
  int q_issued = 0;  // heads whose Q tile thread 0 has requested

  auto load_q = [&](int h) {  // thread 0
    const int s = h % QSTAGES;
    mbar_arrive_expect_tx(mb_q_full(s), QSTAGE_BYTES);
    if (a.packed) {  // one 32-byte-swizzled [128 rows x 16 dims] box per K-step (dims d, r, c, t, h)
      for (int kk = 0; kk < HD / 16; ++kk)
        tma_load_5d(sbase + OFF_Q + s * QSTAGE_BYTES + kk * (QM * 32), tmq, 0, 0, kk, q0 / 16, h, mb_q_full(s));
    } else {
      for (int rg = 0; rg < 2; ++rg)
        tma_load_3d(sbase + OFF_Q + s * QSTAGE_BYTES + rg * (QSTAGE_BYTES / 2), tmq, 64 * rg, h, q0, mb_q_full(s));
    }
  };
  auto issue_head = [&](int h) {  // thread 0: S_(h&1) = Q_h . K^T
    const uint32_t qa = sbase + OFF_Q + (h % QSTAGES) * QSTAGE_BYTES;
    const uint32_t kb = sbase + OFF_K;
    const uint32_t d = tmem + 256u * (uint32_t)(h & 1);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      const uint32_t off_a = (kk >> 2) * (QSTAGE_BYTES / 2) + (kk & 3) * 32;
      const uint32_t off_b = (kk >> 2) * (KTILE_BYTES / 2) + (kk & 3) * 32;
      const uint64_t da = a.packed ? sw32_desc(qa + kk * (QM * 32), 256) : sw128_desc(qa + off_a, 16, 1024);
      mma_f16_ss(d, da, sw128_desc(kb + off_b, 16, 1024), IDESC, kk > 0 ? 1u : 0u);
    }
    mma_commit(mb_s_full(h & 1));
  };

  if (tid == 0) {
    // key tile: boxes of k_box_rows positions per 64-dim half; a missing
    // block (outside the table or the cache) loads as zeros
    mbar_arrive_expect_tx(mb_k, KTILE_BYTES);
    const int nbox = KN / k_box_rows;
    const int oob_row = (int)min(a.n_kv_rows, (int64_t)INT_MAX);
    for (int j = 0; j < nbox; ++j) {
      const int pos = p0 + j * k_box_rows;
      int row = oob_row;
      const int blk_i = pos / a.page_size;
      if (pos < maxlen && blk_i < a.max_blocks) {
        const int64_t r = (int64_t)a.bt[(int64_t)q0 * a.bt_stride + blk_i] * a.page_size + (pos % a.page_size);
        if (r >= 0 && r < a.n_kv_rows) row = (int)r;
      }
#pragma unroll
      for (int rg = 0; rg < 2; ++rg)
        tma_load_2d(sbase + OFF_K + rg * (KTILE_BYTES / 2) + j * k_box_rows * 128, tmk, 64 * rg, row, mb_k);
    }
    for (; q_issued < min(QSTAGES, H); ++q_issued) load_q(q_issued);
    // two heads in flight from the start: S buffers 0 and 1 are both free
    ok = mbar_wait(mb_k, 0, abort_flag, err, kWaitTimeoutNs);
    for (int h = 0; h < 2 && h < H && ok; ++h) {
      ok = mbar_wait(mb_q_full(h), 0, abort_flag, err, kWaitTimeoutNs);
      if (ok) {
        fence_after_sync();
        issue_head(h);
      }
    }
  }
  __syncwarp();

  const int quad = warp & 3, cb = warp >> 2;
  const int row = 32 * quad + lane;
  const uint32_t t_lane = tmem + ((uint32_t)(32 * quad) << 16) + 64u * (uint32_t)cb;
  float acc[64];
#pragma unroll
  for (int j = 0; j < 64; ++j) acc[j] = 0.f;

#pragma unroll 1
  for (int h = 0; h < H; ++h) {
    const int b = h & 1;
    ok = ok && mbar_wait(mb_s_full(b), (uint32_t)((h >> 1) & 1), abort_flag, err, kWaitTimeoutNs);
    ok = __all_sync(0xffffffffu, ok);
    fence_after_sync();
    if (tid == 0 && ok && q_issued < H) {  // MMA h completed: its Q stage takes head h + QSTAGES
      load_q(q_issued);
      ++q_issued;
    }
    __syncwarp();
    const float wv = s_w[h * QM + row];
    // 64 columns in 4 chunks of 16: the next chunk's TMEM load is in flight
    // while the current one is accumulated
    uint32_t va[16], vb[16];
    if (ok) {
      const uint32_t ta = t_lane + 256u * (uint32_t)b;
      tmem_ld16(ta, va);
      tmem_wait_ld();
      tmem_ld16(ta + 16u, vb);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = fmaf(wv, fmaxf(__uint_as_float(va[j]), 0.f), acc[j]);
      tmem_wait_ld();
      tmem_ld16(ta + 32u, va);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[16 + j] = fmaf(wv, fmaxf(__uint_as_float(vb[j]), 0.f), acc[16 + j]);
      tmem_wait_ld();
      tmem_ld16(ta + 48u, vb);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[32 + j] = fmaf(wv, fmaxf(__uint_as_float(va[j]), 0.f), acc[32 + j]);
      tmem_wait_ld();
    }
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(mb_s_free(b));
    // every warp has read S_h: its buffer takes head h + 2
    if (tid == 0 && ok && h + 2 < H) {
      bool ok2 = mbar_wait(mb_s_free(b), (uint32_t)((h >> 1) & 1), abort_flag, err, kWaitTimeoutNs);
      ok2 = ok2 && mbar_wait(mb_q_full((h + 2) % QSTAGES), (uint32_t)(((h + 2) / QSTAGES) & 1), abort_flag, err,
                             kWaitTimeoutNs);
      if (ok2) {
        fence_after_sync();
        issue_head(h + 2);
      }
    }
    __syncwarp();
    if (ok) {
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[48 + j] = fmaf(wv, fmaxf(__uint_as_float(vb[j]), 0.f), acc[48 + j]);
    }
  }

  if (ok && row < nrows) {
    const int len = s_len[row];
    const int pc = p0 + 64 * cb;
    float* dst = a.score + (int64_t)(q0 + row) * a.score_stride + pc;
    const bool vec = ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) && pc + 64 <= a.max_kv;
    if (vec) {
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        float4 o;
        o.x = pc + j + 0 < len ? acc[j + 0] : -INFINITY;
        o.y = pc + j + 1 < len ? acc[j + 1] : -INFINITY;
        o.z = pc + j + 2 < len ? acc[j + 2] : -INFINITY;
        o.w = pc + j + 3 < len ? acc[j + 3] : -INFINITY;
        *reinterpret_cast<float4*>(dst + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (pc + j < a.max_kv) dst[j] = pc + j < len ? acc[j] : -INFINITY;
    }
  }

  // after an abort, wait (bounded) for this CTA's own copies and MMAs
  if (tid == 0 && *abort_flag) {
    mma_commit(mb_done);
    mbar_wait_drain(mb_done, 0, kWaitTimeoutNs);
    mbar_wait_drain(mb_k, 0, kWaitTimeoutNs);
    for (int s = 0; s < QSTAGES && s < q_issued; ++s) {
      const int last = s + QSTAGES * ((q_issued - 1 - s) / QSTAGES);  // last head loaded into stage s
      mbar_wait_drain(mb_q_full(s), (uint32_t)((last / QSTAGES) & 1), kWaitTimeoutNs);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];

int ensure_setup(int dev) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  DSA_REQUIRE(g_encode != nullptr, DSA_ERR_CUDA, "indexer_logits_tc: cuTensorMapEncodeTiled is unavailable");
  DSA_REQUIRE(dev >= 0 && dev < kMaxDevices, DSA_ERR_UNSUPPORTED, "indexer_logits_tc: device %d out of range", dev);
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(indexer_logits_tc_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(indexer_logits_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)SMEM_BYTES);
    g_status[dev] = (int)e;
  });
  if (g_status[dev] != 0) {
    set_error("indexer_logits_tc setup: %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

int encode(CUtensorMap* m, const void* base, bool bf16, cuuint32_t rank, const cuuint64_t* dims,
           const cuuint64_t* strides_bytes, const cuuint32_t* box, const char* what,
           CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  const CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank,
                              const_cast<void*>(base), dims, strides_bytes, box, elem_strides,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DSA_REQUIRE(r == CUDA_SUCCESS, DSA_ERR_CUDA, "indexer_logits_tc: tensor map for %s failed (CUresult %d)", what,
              (int)r);
  return DSA_OK;
}

}  // namespace

bool indexer_tc_eligible(int k_format, int q_bf16, int page_size, int n_ihead, int64_t n_kv_rows, int B,
                         int max_kv) {
  if (k_format != DSA_F16 && k_format != DSA_BF16) return false;
  if ((k_format == DSA_BF16) != (q_bf16 != 0)) return false;  // one MMA operand type
  return page_size >= 8 && n_ihead >= 1 && n_ihead <= MAX_HEADS && n_kv_rows > 0 && n_kv_rows < INT_MAX &&
         B > 0 && (B + QM - 1) / QM <= 65535 && max_kv > 0;
}

int launch_indexer_logits_tc(const IndexerTcArgs& a, cudaStream_t s) {
  const int dev = current_device();
  int st = ensure_setup(dev);
  if (st != DSA_OK) return st;
  int32_t* err = nullptr;
  st = tc_error_word(dev, &err);
  if (st != DSA_OK) return st;
  const bool bf16 = a.q_bf16 != 0;
  CUtensorMap tq, tk;
  if (a.packed) {
    // packed q [32, nqt, 8, 16, 16]: element (h, t, c, r, d) = q[16t + r, h, 16c + d]; a box is one
    // head's 16-dim chunk c of 128 rows (8 row groups t), 32 bytes per row
    const cuuint64_t nqt = (cuuint64_t)((a.B + 15) / 16);
    const cuuint64_t dims[5] = {16, 16, 8, nqt, (cuuint64_t)a.n_ihead};
    const cuuint64_t strides[4] = {32, 16 * 32, 8 * 16 * 32, nqt * 8 * 16 * 32};
    const cuuint32_t box[5] = {16, 16, 1, QM / 16, 1};
    st = encode(&tq, a.q, bf16, 5, dims, strides, box, "q_packed", CU_TENSOR_MAP_SWIZZLE_32B);
    if (st != DSA_OK) return st;
  } else {
    const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)a.n_ihead, (cuuint64_t)a.B};
    const cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)a.n_ihead * HD * 2};
    const cuuint32_t box[3] = {64, 1, QM};
    st = encode(&tq, a.q, bf16, 3, dims, strides, box, "q");
    if (st != DSA_OK) return st;
  }
  const int box_rows = a.page_size < KN ? a.page_size : KN;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)a.n_kv_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    st = encode(&tk, a.k, bf16, 2, dims, strides, box, "k_cache");
    if (st != DSA_OK) return st;
  }
  const dim3 grid((unsigned)((a.max_kv + KN - 1) / KN), (unsigned)((a.B + QM - 1) / QM));
  if (bf16)
    indexer_logits_tc_kernel<true><<<grid, NTHREADS, SMEM_BYTES, s>>>(tq, tk, a, box_rows, err);
  else
    indexer_logits_tc_kernel<false><<<grid, NTHREADS, SMEM_BYTES, s>>>(tq, tk, a, box_rows, err);
  return check_launch("indexer_logits_tc_kernel");
}

}  // namespace dsa
