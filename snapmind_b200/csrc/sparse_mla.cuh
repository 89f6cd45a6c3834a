// Shared declarations of the sparse MLA decode kernels.
#pragma once

#include "paged_decode.cuh"

namespace snapmind {

struct SparseParams {
  const void* q_lat;   // [B][H][R]
  const void* q_pe;    // [B][H][P]
  const void* latent;  // layer base: [blocks][bs][R]
  const void* rope;    // layer base: [blocks][bs][P]
  const int32_t* tables;
  int64_t table_stride;
  int32_t table_width;
  const int32_t* seq_lens;
  const int32_t* selected;  // [B][k] chunk ids, -1 = empty
  int32_t k, sink, window;
  float scale;
  int32_t batch, n_heads, R, P, bs, num_blocks, n_splits;
  DecodeParams dp;  // output, partials and tickets in the paged-decode layout (group = 16 heads)
};

// tcgen05 path (sparse_mla_umma.cu): bf16/f16, 128 heads, R = 512, P = 64, block 64.
bool sparse_mla_umma_supported(const SparseParams& p, int dtype);
int launch_sparse_mla_umma(const SparseParams& p, int dtype, cudaStream_t stream);
int sparse_mla_umma_splits(int batch);

// mma.sync path (sparse_mla_tc.cu): bf16/f16, heads a multiple of 16, R = 512, P = 64, block 64.
bool sparse_mla_tc_supported(const SparseParams& p, int dtype);
int launch_sparse_mla_tc(const SparseParams& p, int dtype, cudaStream_t stream);

}  // namespace snapmind
