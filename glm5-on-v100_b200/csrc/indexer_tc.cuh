// Internal interface of the tensor-core (tcgen05) indexer-logits kernel.
#pragma once

#include "common.cuh"

namespace dsa {

struct IndexerTcArgs {
  float* score;
  int64_t score_stride;
  int max_kv;
  const void* q;       // [B, n_ihead, 128], same 16-bit type as the cache
  int q_bf16;
  int n_ihead;
  int B;
  const void* k;       // [n_kv_rows / page, page, 128] f16 / bf16
  int64_t n_kv_rows;
  int page_size;
  const void* w;       // [B, n_ihead]
  int w_dtype;
  const int32_t* bt;   // the first row of each 128-row tile serves the tile
  int64_t bt_stride;
  int max_blocks;
  const int32_t* seq_lens;
  int packed;          // q is the packed layout [32, ceil(B/16), 8, 16, 16] (sai.py:131-148)
};

// True when the tcgen05 kernel serves this call (16-bit cache of q's type,
// page >= 8; packed q needs 32 heads); the caller keeps the mma.sync kernel
// otherwise.
bool indexer_tc_eligible(int k_format, int q_bf16, int page_size, int n_ihead, int64_t n_kv_rows, int B,
                         int max_kv);
int launch_indexer_logits_tc(const IndexerTcArgs& a, cudaStream_t s);

// Decode rows over an fp8 indexer-K cache (132-byte keys) in 64-token pages:
// each row with its own block table; scores plus the fused level-1 histogram.
struct IndexerDecodeTcArgs {
  float* score;
  int64_t score_stride;
  int max_kv;
  const void* q;       // [B, n_ihead, 128] f16 or bf16
  int q_bf16;
  int n_ihead;
  int B;
  const uint8_t* k;    // [n_kv_rows / 64, 64, 132] u8
  int64_t n_kv_rows;
  const void* w;       // [B, n_ihead]
  int w_dtype;
  const int32_t* bt;   // [B, max_blocks]
  int64_t bt_stride;
  int max_blocks;
  const int32_t* seq_lens;
  int32_t* hist;       // [B, 4096] or null
  int cta_keys;        // positions per CTA (set by the launcher)
};

bool indexer_decode_tc_eligible(int k_format, int page_size, int n_ihead, int packed);
int launch_indexer_decode_tc(const IndexerDecodeTcArgs& a, cudaStream_t s);

}  // namespace dsa
