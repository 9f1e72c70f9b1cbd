// Lightning-indexer logits for decode rows on the 5th-generation tensor cores,
// fp8 indexer-K cache (128 e4m3 + f32 scale per key) in 64-token pages:
//   score[b, p] = scale_p * sum_h w[b,h] * relu(q[b,h,:] . k_p)  for p < seq_lens[b]
//   score[b, p] = -inf                                         for seq_lens[b] <= p < max_kv
// plus the level-1 top-k histogram of the scores (4096 bins of
// monotone32(score) >> 20). Same function as the reference's decode kernel
// (csrc/attention/sm70_mla_decode.cu:150-329, histogram :309-319).
//
// One CTA = one query row x up to 4096 positions (fewer when the rows x keys
// would not fill whole waves of the GPU), in sub-tiles of 128 keys (two
// pages), two CTAs per SM, three roles that meet only at mbarriers, so none
// waits for another's instruction issue:
//   * copy thread (warp 9): a page is 64 x 132 = 8,448 contiguous bytes, so
//     each arrives with one bulk copy (cp.async.bulk, completing on a "stage
//     full" mbarrier), DSTAGES sub-tiles ahead, reissued into a stage as soon
//     as the workers mark it read; the page bases come from the block table
//     once per CTA;
//   * workers (warps 0-7): every thread expands half of one key's staged
//     e4m3 bytes exactly to fp16 and stores them with tcgen05.st straight
//     into the MMA's A operand in tensor memory (row = key, two fp16 per
//     32-bit column), double buffered, so the bytes cross shared memory once;
//     each warp then arrives on "A full" and "stage free";
//   * MMA thread (warp 8): on "A full" it issues S^T[128 keys x NQ heads] =
//     K . Q^T as eight M=128, N=NQ, K=16 tcgen05 MMAs (A from TMEM, q from
//     shared memory, fp32 accumulation into one of two TMEM accumulators);
//   * while sub-tile i's MMAs run, every worker reads sub-tile i-1's
//     accumulator for its key (half of the heads): w * relu(s) summed, the
//     second half parked in shared memory and added, times the key's scale,
//     one iteration later (after the workers' next named barrier).
// q and w are loaded once per CTA and the histogram is accumulated in shared
// memory and added to the global one once per CTA. Every wait is bounded by
// device time; on expiry the CTA records DSA_ERR_TIMEOUT in the sticky status
// word, drains its own copies and MMAs, frees TMEM and returns.
#include <algorithm>

#include "indexer_tc.cuh"
#include "sparse_mla.cuh"
#include "tc_common.cuh"

namespace dsa {
namespace {

using namespace tc;

constexpr int HD = 128;
constexpr int IDXK_ROW = 132;
constexpr int NBIN = 4096;
constexpr int DP = 64;                        // page size served
constexpr int DP_BYTES = DP * IDXK_ROW;       // 8,448
constexpr int DSUB = 128;                     // keys per sub-tile (MMA M)
constexpr int DSTAGES = 4;                    // staged sub-tiles
constexpr int DCTA_KEYS = 4096;               // most positions per CTA
constexpr int NWORK = 256;                    // warps 0-7: expansion and epilogue
constexpr int MMA_WARP = NWORK / 32;          // warp 8, lane 0: the MMAs
constexpr int COPY_WARP = MMA_WARP + 1;       // warp 9, lane 0: the page copies
constexpr int DNT = NWORK + 64;
constexpr uint32_t TMEM_COLS = 256;           // A0 | A1 | D0 | D1
constexpr uint32_t A_COLS = HD / 2;           // 128 fp16 per key: 64 columns
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

template <int NQ>
struct DecodeTcLayout {
  static constexpr uint32_t Q_REGION = NQ * 128;                 // one 64-dim region of q
  static constexpr uint32_t OFF_Q = 0;                           // q, 2 regions
  static constexpr uint32_t OFF_STAGE = OFF_Q + 2 * Q_REGION;    // [DSTAGES][2 pages]
  static constexpr uint32_t OFF_HIST = OFF_STAGE + DSTAGES * 2 * DP_BYTES;
  static constexpr uint32_t OFF_W = OFF_HIST + NBIN * 4;         // [NQ]
  static constexpr uint32_t OFF_PART = OFF_W + NQ * 4;           // [2][DSUB] second-half head sums
  static constexpr uint32_t OFF_BASE = OFF_PART + 2 * DSUB * 4;  // [DCTA_KEYS / DP] int64 page bases
  // mbarriers: [DSTAGES] stage full, [DSTAGES] stage free, [2] A full, [2] MMAs done, drain
  static constexpr uint32_t OFF_MBAR = OFF_BASE + (DCTA_KEYS / DP) * 8;
  static constexpr uint32_t OFF_SLOT = OFF_MBAR + (2 * DSTAGES + 5) * 8;
  static constexpr uint32_t BYTES = OFF_SLOT + 16 + 1024;        // + alignment slack
  static constexpr uint32_t D_COL = 2 * A_COLS;                  // accumulator p at D_COL + p * NQ
  static_assert(Q_REGION % 1024 == 0 && OFF_STAGE % 1024 == 0, "swizzled regions stay 1024-aligned");
  static_assert(D_COL + 2 * NQ <= TMEM_COLS, "two A tiles and two accumulators fit the allocation");
};

__device__ __forceinline__ float load_weight(const IndexerDecodeTcArgs& a, int64_t i) {
  if (a.w_dtype == DSA_F32) return reinterpret_cast<const float*>(a.w)[i];
  if (a.w_dtype == DSA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.w)[i]);
  return __half2float(reinterpret_cast<const __half*>(a.w)[i]);
}

// NQ/2 consecutive TMEM columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 32) {
    tmem_ld32(taddr, r);
  } else if constexpr (N == 16) {
    tmem_ld16(taddr, r);
  } else {
    static_assert(N == 8, "8, 16 or 32 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  }
}

template <int NQ>
__global__ void __launch_bounds__(DNT, 2) indexer_decode_tc_kernel(const IndexerDecodeTcArgs a, int32_t* err) {
  using Lay = DecodeTcLayout<NQ>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* sm = smem_raw + (base - raw_base);
  uint8_t* stage = sm + Lay::OFF_STAGE;
  uint32_t* sHist = reinterpret_cast<uint32_t*>(sm + Lay::OFF_HIST);
  float* sW = reinterpret_cast<float*>(sm + Lay::OFF_W);
  float* sPart = reinterpret_cast<float*>(sm + Lay::OFF_PART);
  int64_t* sBase = reinterpret_cast<int64_t*>(sm + Lay::OFF_BASE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Lay::OFF_SLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + Lay::OFF_SLOT + 4);
  uint32_t* q_bits = reinterpret_cast<uint32_t*>(sm + Lay::OFF_SLOT + 8);  // largest |q| bf16 pattern
  const uint32_t mb0 = base + Lay::OFF_MBAR;
  auto mb_full = [&](int st) { return mb0 + 8u * (uint32_t)st; };                  // stage's copies landed
  auto mb_free = [&](int st) { return mb0 + 8u * (uint32_t)(DSTAGES + st); };      // stage read by the workers
  auto mb_afull = [&](int x) { return mb0 + 8u * (uint32_t)(2 * DSTAGES + x); };  // A[x] written
  auto mb_mma = [&](int x) { return mb0 + 8u * (uint32_t)(2 * DSTAGES + 2 + x); }; // MMAs into D[x] done
  const uint32_t mb_done = mb0 + 8u * (2 * DSTAGES + 4);                           // drain on abort

  const int b = blockIdx.x;
  const int p0 = blockIdx.y * a.cta_keys;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* score_row = a.score + (int64_t)b * a.score_stride;
  const int p_end = min(p0 + a.cta_keys, a.max_kv);
  const int valid_len = min(a.seq_lens[b], a.max_kv);
  const int v_end = min(p_end, valid_len);  // positions [p0, v_end) are scored
  for (int i = max(p0, v_end) + tid; i < p_end; i += DNT) score_row[i] = -INFINITY;
  if (v_end <= p0) return;
  const int nsub = (v_end - p0 + DSUB - 1) / DSUB;
  const int32_t* bt_row = a.bt + (int64_t)b * a.bt_stride;

  // The copy thread: bulk copies of sub-tile i's two pages into stage
  // i % DSTAGES, from the page base codes in sBase.
  auto issue = [&](int i) {
    const int st = i % DSTAGES;
    const uint32_t mb = mb_full(st);
    uint32_t bytes = 0;
    int64_t pb[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      pb[j] = sBase[2 * i + j];
      if (pb[j] >= 0) bytes += DP_BYTES;
    }
    mbar_arrive_expect_tx(mb, bytes);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (pb[j] >= 0)
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(stage + (2 * st + j) * DP_BYTES)),
            "l"(a.k + pb[j] * IDXK_ROW), "r"((uint32_t)DP_BYTES), "r"(mb)
            : "memory");
  };

  if (warp == 0) {
    if (lane == 0) {
      for (int st = 0; st < DSTAGES; ++st) {
        mbar_init(mb_full(st), 1);
        mbar_init(mb_free(st), NWORK / 32);
      }
      for (int x = 0; x < 2; ++x) {
        mbar_init(mb_afull(x), NWORK / 32);
        mbar_init(mb_mma(x), 1);
      }
      mbar_init(mb_done, 1);
      mbar_init_fence();
      *abort_flag = 0;
      abort_flag[2] = 0;  // n_done below
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
  }
  for (int i = tid; i < NBIN; i += DNT) sHist[i] = 0;
  // Page base codes of the CTA's pages: row of the page's first key (whole
  // page in the cache); -1: no key of the page is read; -2: the page runs
  // past the cache end (keys read one by one).
  for (int j = tid; j < 2 * nsub; j += DNT) {
    const int pos = p0 + DP * j;
    int64_t pb = -1;
    if (pos < v_end) {
      const int blk_i = pos / DP;
      if (blk_i < a.max_blocks) {
        const int64_t r = (int64_t)bt_row[blk_i] * DP;
        if (r >= 0 && r + DP <= a.n_kv_rows)
          pb = r;
        else if (r >= 0 && r < a.n_kv_rows)
          pb = -2;
      }
    }
    sBase[j] = pb;
  }
  // bf16 q beyond fp16's range: the row's q is scaled by 2^-qe for the MMA
  // and every score by 2^qe after it (both exact; relu commutes with them)
  int qe = 0;
  if (a.q_bf16) {
    if (tid == 0) *q_bits = 0;
    __syncthreads();
    uint32_t bits = 0;
    for (int i = tid; i < a.n_ihead * 16; i += DNT)
      bits = max(bits, bf16x8_max_abs_bits(*reinterpret_cast<const uint4*>(
                           reinterpret_cast<const uint8_t*>(a.q) + ((int64_t)b * a.n_ihead * HD + 8 * i) * 2)));
    bits = __reduce_max_sync(0xffffffffu, bits);
    if (lane == 0) atomicMax(q_bits, bits);
    __syncthreads();
    qe = bf16_fp16_shift(*q_bits);
  }
  const float qmul = __int_as_float((127 + qe) << 23);  // 2^qe
  // q as the MMA's B operand: NQ rows (heads, zero past n_ihead) x 128 dims,
  // two 64-dim regions of 128-byte swizzled rows
  for (int i = tid; i < NQ * 16; i += DNT) {
    const int h = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < a.n_ihead) {
      v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.q) +
                                          (((int64_t)b * a.n_ihead + h) * HD + 8 * c) * 2);
      if (a.q_bf16) v = bf16x8_to_half8_scaled(v, qe);
    }
    *reinterpret_cast<uint4*>(sm + Lay::OFF_Q + (c >> 3) * Lay::Q_REGION + sw128_off(h, c & 7)) = v;
  }
  for (int h = tid; h < NQ; h += DNT) sW[h] = h < a.n_ihead ? load_weight(a, (int64_t)b * a.n_ihead + h) : 0.f;
  fence_proxy_async();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint64_t desc_q = sw128_desc(base + Lay::OFF_Q, 16, 1024);
  constexpr uint32_t IDESC = idesc_f16(DSUB, NQ, false, false);
  volatile int* n_done = abort_flag + 2;  // thread 0: sub-tiles whose copies were seen complete
  int n_issued = 0;                       // copy thread: sub-tiles whose copies were issued
  bool issued = false;                    // MMA thread: at least one MMA issued

  if (warp == COPY_WARP) {
    // ---- page copies, DSTAGES sub-tiles ahead of the workers
    if (lane == 0) {
      for (; n_issued < nsub; ++n_issued) {
        const int j = n_issued;
        if (j >= DSTAGES &&
            !mbar_wait(mb_free(j % DSTAGES), (uint32_t)(((j - DSTAGES) / DSTAGES) & 1), abort_flag, err,
                       kWaitTimeoutNs))
          break;
        if (*abort_flag) break;
        issue(j);
      }
    }
  } else if (warp == MMA_WARP) {
    // ---- S^T(it) = K(it) . Q^T as soon as the workers have written A[it & 1]
    if (lane == 0) {
      for (int it = 0; it < nsub; ++it) {
        if (!mbar_wait(mb_afull(it & 1), (uint32_t)((it >> 1) & 1), abort_flag, err, kWaitTimeoutNs)) break;
        if (*abort_flag) break;
        fence_after_sync();
        const uint32_t a_tm = tmem + (uint32_t)((it & 1) * A_COLS);
        const uint32_t d_tm = tmem + Lay::D_COL + (uint32_t)((it & 1) * NQ);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_f16_ts(d_tm, a_tm + 8u * kk, desc_q + (((kk >> 2) * Lay::Q_REGION + 32 * (kk & 3)) >> 4), IDESC,
                     kk != 0);
        mma_commit(mb_mma(it & 1));
        issued = true;
      }
    }
  } else {
    // ---- workers: key kq = 32 (warp & 3) + lane of every sub-tile (the TMEM
    // lane quarter its warp may access), dims / heads half hh
    const int kq = 32 * (warp & 3) + lane, hh = warp >> 2;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    bool ok = true;
    float sc_prev = 0.f, sc_cur = 0.f;  // hh == 0: the key's scale for sub-tiles i-1, i
    float s_prev = 0.f;                 // hh == 0: first-half head sum of sub-tile i-2 (finished at iteration i)
    for (int it = 0; it < nsub + 2; ++it) {
      // expand sub-tile it into A[it & 1] (free: this warp waited for MMA(it-2) last iteration)
      float sc_new = 0.f;
      if (it < nsub) {
        const int st = it % DSTAGES;
        ok = ok && mbar_wait(mb_full(st), (uint32_t)((it / DSTAGES) & 1), abort_flag, err, kWaitTimeoutNs);
        if (tid == 0 && ok) *n_done = it + 1;
        const int pos = p0 + DSUB * it + kq;
        const int j = kq >> 6;
        const int64_t pbase = sBase[2 * it + j];
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e] = 0u;
        if (ok && pos < v_end && pbase != -1) {
          if (pbase >= 0) {  // the staged page: 132-byte rows are only 4-byte aligned
            const uint32_t src = smem_u32(stage + (2 * st + j) * DP_BYTES + (kq & 63) * IDXK_ROW) + 64 * hh;
#pragma unroll
            for (int e = 0; e < 16; ++e) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w[e]) : "r"(src + 4 * e));
            if (hh == 0) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(sc_new) : "r"(src + 128));
          } else {  // a page that runs past the cache end: this key's own row, if inside
            const int64_t r = (int64_t)bt_row[pos / DP] * DP + (pos % DP);
            if (r < a.n_kv_rows) {
              const uint32_t* g = reinterpret_cast<const uint32_t*>(a.k + r * IDXK_ROW + 64 * hh);
#pragma unroll
              for (int e = 0; e < 16; ++e) w[e] = __ldg(g + e);
              if (hh == 0) sc_new = __ldg(reinterpret_cast<const float*>(a.k + r * IDXK_ROW + 128));
            }
          }
        }
        uint32_t hv[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) e4m3x4_to_half2x2_div256(w[e], hv[2 * e], hv[2 * e + 1]);  // keys / 256, exact
        tmem_st32(tmem + lane_base + (uint32_t)((it & 1) * A_COLS + 32 * hh), hv);
        tmem_wait_st();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) {  // A[it & 1] rows of this warp written; stage st read
          mbar_arrive(mb_afull(it & 1));
          mbar_arrive(mb_free(st));
        }
      }
      named_bar(1, NWORK);  // the workers' sPart of sub-tile it-2 visible
      // finish sub-tile it-2: both head halves, scale, histogram, store
      if (it >= 2 && hh == 0) {
        const int pos = p0 + DSUB * (it - 2) + kq;
        if (pos < v_end) {
          const float v = (s_prev + sPart[((it - 2) & 1) * DSUB + kq]) * (sc_prev * 256.0f) * qmul;
          atomicAdd(&sHist[monotone32(v) >> 20], 1u);
          score_row[pos] = v;
        }
      }
      // half-head sums of sub-tile it-1 from its accumulator
      if (it >= 1 && it <= nsub) {
        const int i1 = it - 1;
        ok = ok && mbar_wait(mb_mma(i1 & 1), (uint32_t)((i1 >> 1) & 1), abort_flag, err, kWaitTimeoutNs);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-wide
        fence_after_sync();
        float sum = 0.f;
        if (ok) {
          uint32_t acc[NQ / 2];
          tmem_ld_cols<NQ / 2>(tmem + lane_base + Lay::D_COL + (uint32_t)((i1 & 1) * NQ + hh * (NQ / 2)), acc);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < NQ / 2; ++h) sum += sW[hh * (NQ / 2) + h] * fmaxf(__uint_as_float(acc[h]), 0.f);
        }
        if (hh == 1)
          sPart[(i1 & 1) * DSUB + kq] = sum;
        else
          s_prev = sum;
      }
      if (hh == 0) {  // the scales ride along with the sub-tiles they belong to
        sc_prev = sc_cur;
        sc_cur = sc_new;
      }
    }
  }
  __syncthreads();  // every role is done; the last sub-tile's histogram counts are in
  for (int i = tid; i < NBIN; i += DNT) {
    const uint32_t c = sHist[i];
    if (c && a.hist) atomicAdd(a.hist + (int64_t)b * NBIN + i, (int)c);
  }
  if (*abort_flag) {  // drain this CTA's copies and MMAs before its memory is released
    if (warp == COPY_WARP && lane == 0)
      for (int j = *n_done; j < n_issued; ++j)
        mbar_wait_drain(mb_full(j % DSTAGES), (uint32_t)((j / DSTAGES) & 1), kWaitTimeoutNs);
    if (warp == MMA_WARP && lane == 0 && issued) {
      mma_commit(mb_done);
      mbar_wait_drain(mb_done, 0, kWaitTimeoutNs);
    }
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

int ensure_setup(int dev) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("indexer_decode_tc: device index %d out of range", dev);
    return DSA_ERR_UNSUPPORTED;
  }
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(indexer_decode_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)DecodeTcLayout<16>::BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(indexer_decode_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)DecodeTcLayout<32>::BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(indexer_decode_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)DecodeTcLayout<64>::BYTES);
    g_status[dev] = (int)e;
  });
  if (g_status[dev] != 0) {
    set_error("indexer_decode_tc setup: %s", cudaGetErrorString((cudaError_t)g_status[dev]));
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

}  // namespace

bool indexer_decode_tc_eligible(int k_format, int page_size, int n_ihead, int packed) {
  return k_format == DSA_FP8_IDXK && page_size == DP && n_ihead >= 1 && n_ihead <= 64 && !packed;
}

int launch_indexer_decode_tc(const IndexerDecodeTcArgs& a, cudaStream_t s) {
  const int dev = current_device();
  int st = ensure_setup(dev);
  if (st != DSA_OK) return st;
  int32_t* err = nullptr;
  st = tc_error_word(dev, &err);
  if (st != DSA_OK) return st;
  // Positions per CTA: whole waves of the resident CTAs (two per SM), at
  // most DCTA_KEYS each, so few rows or short key spans (a key-sharded rank)
  // still spread over every SM.
  IndexerDecodeTcArgs b = a;
  const int64_t resident = 2LL * sm_count(dev);
  const int64_t keys = (int64_t)a.B * a.max_kv;
  const int64_t waves = (keys + resident * DCTA_KEYS - 1) / (resident * DCTA_KEYS);
  int64_t per = (keys + waves * resident - 1) / std::max<int64_t>(waves * resident, 1);
  per = (per + DSUB - 1) / DSUB * DSUB;
  b.cta_keys = (int)std::min<int64_t>(std::max<int64_t>(per, 2 * DSUB), DCTA_KEYS);
  const dim3 grid(a.B, (a.max_kv + b.cta_keys - 1) / b.cta_keys);
  if (a.n_ihead <= 16)
    indexer_decode_tc_kernel<16><<<grid, DNT, DecodeTcLayout<16>::BYTES, s>>>(b, err);
  else if (a.n_ihead <= 32)
    indexer_decode_tc_kernel<32><<<grid, DNT, DecodeTcLayout<32>::BYTES, s>>>(b, err);
  else
    indexer_decode_tc_kernel<64><<<grid, DNT, DecodeTcLayout<64>::BYTES, s>>>(b, err);
  return check_launch("indexer_decode_tc_kernel");
}

}  // namespace dsa
