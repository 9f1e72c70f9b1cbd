// Internal interface between the sparse-MLA launcher and its kernels.
#pragma once

#include "common.cuh"

namespace dsa {

struct SparseMlaArgs {
  const void* q;
  const uint8_t* kv;
  const int32_t* idx;
  const int32_t* bt;
  const int32_t* seq_lens;
  void* o;
  float* lse;
  float* part_o;   // [B, n_head, n_splits, 512] f32 when n_splits > 1
  float* part_ml;  // [B, n_head, n_splits, 2]
  int64_t n_kv_rows;
  int64_t idx_stride;
  int64_t bt_stride;
  int page_size;
  int max_blocks;
  int B, n_head, topk, n_splits, span;
  int q_bf16, o_bf16;
  float scale_log2;  // softmax scale * log2(e)
};

// Tensor-core (tcgen05) kernel for the fp8_ds_mla cache: rows per tile and
// the slice count it would use for a problem.
constexpr int kTcTileRows = 64;
int tc_choose_splits(int B, int head_tiles, int topk, int nsm);
// Slices of one row that the tcgen05 kernel merges inside one thread-block
// cluster: n_splits when that cluster size (2 or 4) is resident on this
// device, else 1 (partial states + the merge kernel).
int tc_cluster_size(int n_splits);
// Launch the tcgen05 kernel; args.n_splits / args.span already chosen.
int launch_sparse_mla_tc(const SparseMlaArgs& a, cudaStream_t s);
// Merge per-slice partial states into o / lse (defined with the v1 kernel).
int launch_sparse_mla_merge(const SparseMlaArgs& a, cudaStream_t s);
// Device address of the sticky status word that every tensor-core kernel of
// this library sets on a timed-out wait (read by dsa_device_error).
int tc_error_word(int dev, int32_t** out);

}  // namespace dsa
