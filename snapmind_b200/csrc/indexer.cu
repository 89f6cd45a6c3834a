// Lookahead sparse indexer kernels for sm_100a.
//
// * indexer_pool_chunks: the frozen key of a chunk is the mean of its cached
//   latent rows (LookaheadSparseIndexer.build_frozen_keys,
//   snapmind/layers/indexer/lookahead.py:40-50); with block_size == chunk
//   size a chunk is one block of the paged latent pool.  Optionally the mean
//   is projected (out = P . mean, P row-major [out_dim][width]) in the same
//   kernel, so the latent is read from HBM once.
// * indexer_score_ref: the reference score of every chunk at once,
//   mean_n sigmoid(sum_h relu(q[n,h] . k) * w[n,h]) (lookahead.py:82-106).
// * indexer_topk: score = sigmoid(q . k * scale + bias) per chunk and the k
//   best chunks per sequence, ordered by score (descending) then chunk id
//   (ascending) — a stable descending sort, done as a bitonic sort of
//   (ordered score bits, inverted id) keys in shared memory.
#include <cfloat>

#include "common.cuh"

namespace snapmind {
namespace {

// ---------------------------------------------------------------------------
// chunk mean-pool (+ projection)
// ---------------------------------------------------------------------------
struct PoolParams {
  const char* pool;         // layer base, rows of row_width elements
  int64_t row_width;        // elements per pool row
  int32_t width;            // leading columns averaged
  const int32_t* tables;
  int64_t table_stride;
  int32_t table_width;
  const int32_t* seq_lens;
  int32_t batch, block_size, num_blocks;
  int32_t chunk_begin, chunk_count, max_chunks;
  const char* proj;         // [out_dim][width] or null
  int32_t out_dim;
  float* out;               // [batch][max_chunks][out_dim or width]
  int32_t* err;
};

template <typename T, typename TP>
__global__ void __launch_bounds__(256) indexer_pool_kernel(PoolParams p) {
  extern __shared__ float mean[];  // [width]
  const int c = p.chunk_begin + blockIdx.x;
  const int b = blockIdx.y;
  const int out_w = p.proj ? p.out_dim : p.width;
  float* out = p.out + ((int64_t)b * p.max_chunks + c) * out_w;
  // without lengths every chunk is full
  const int n = p.seq_lens ? min(p.block_size, p.seq_lens[b] - c * p.block_size) : p.block_size;
  if (c >= p.max_chunks) return;
  if (n <= 0 || c >= p.table_width) {
    for (int i = threadIdx.x; i < out_w; i += blockDim.x) out[i] = 0.f;
    return;
  }
  const int32_t phys = p.tables[(int64_t)b * p.table_stride + c];
  if (phys < 0 || phys >= p.num_blocks) {
    if (threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
    for (int i = threadIdx.x; i < out_w; i += blockDim.x) out[i] = 0.f;
    return;
  }
  const T* rows = reinterpret_cast<const T*>(p.pool) + (int64_t)phys * p.block_size * p.row_width;
  const float inv = 1.f / (float)n;
  for (int d = threadIdx.x; d < p.width; d += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < n; ++r) s += Conv<T>::to_f(rows[(int64_t)r * p.row_width + d]);
    mean[d] = s * inv;
  }
  __syncthreads();
  if (!p.proj) {
    for (int d = threadIdx.x; d < p.width; d += blockDim.x) out[d] = mean[d];
    return;
  }
  // projection: one warp per output, lanes over the width
  const TP* P = reinterpret_cast<const TP*>(p.proj);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int o = warp; o < p.out_dim; o += nw) {
    const TP* prow = P + (int64_t)o * p.width;
    float acc = 0.f;
    for (int d = lane; d < p.width; d += 32) acc = fmaf(Conv<TP>::to_f(prow[d]), mean[d], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[o] = acc;
  }
}

// ---------------------------------------------------------------------------
// reference score: one warp per chunk
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) indexer_score_ref_kernel(const float* q, const float* w, int n_rows,
                                                                int n_heads, const float* keys, int n_chunks,
                                                                int R, float* scores) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_chunks) return;
  const float* k = keys + (int64_t)warp * R;
  float total = 0.f;
  for (int n = 0; n < n_rows; ++n) {
    float fused = 0.f;
    for (int h = 0; h < n_heads; ++h) {
      const float* qh = q + ((int64_t)n * n_heads + h) * R;
      float dot = 0.f;
      for (int d = lane; d < R; d += 32) dot = fmaf(qh[d], k[d], dot);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      fused += fmaxf(dot, 0.f) * w[n * n_heads + h];
    }
    total += 1.f / (1.f + expf(-fused));
  }
  if (lane == 0) scores[warp] = total / (float)n_rows;
}

// ---------------------------------------------------------------------------
// sigmoid score + stable top-k, one CTA per sequence
// ---------------------------------------------------------------------------
constexpr int kTopkThreads = 512;

__device__ __forceinline__ uint32_t ordered_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads) indexer_topk_kernel(
    const T* q, const T* keys, const int32_t* n_chunks_arr, int n_chunks0, int max_chunks, int dim, float scale,
    float bias, int k, int sort_n, int32_t* out_idx, float* out_score, float* all_scores) {
  extern __shared__ unsigned long long skeys[];  // [sort_n]
  const int b = blockIdx.x;
  int nc = n_chunks_arr ? n_chunks_arr[b] : n_chunks0;
  nc = max(0, min(nc, max_chunks));
  const T* qb = q + (int64_t)b * dim;
  const T* kb = keys + (int64_t)b * max_chunks * dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  // scores: one warp per chunk
  for (int c = warp; c < sort_n; c += nw) {
    unsigned long long key = 0ull;  // below every real key
    if (c < nc) {
      float dot = 0.f;
      for (int d = lane; d < dim; d += 32) dot = fmaf(Conv<T>::to_f(qb[d]), Conv<T>::to_f(kb[(int64_t)c * dim + d]), dot);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float s = 1.f / (1.f + expf(-(dot * scale + bias)));
      if (lane == 0 && all_scores) all_scores[(int64_t)b * max_chunks + c] = s;
      key = ((unsigned long long)ordered_bits(s) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)c);
    }
    if (lane == 0) skeys[c] = key;
  }
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= sort_n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < sort_n; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = skeys[i], c2 = skeys[j];
          if (desc ? (a < c2) : (a > c2)) {
            skeys[i] = c2;
            skeys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const bool ok = i < nc;
    const unsigned long long key = skeys[i];
    out_idx[(int64_t)b * k + i] = ok ? (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : -1;
    if (out_score) {
      const uint32_t ob = (uint32_t)(key >> 32);
      const uint32_t u = (ob & 0x80000000u) ? (ob & 0x7FFFFFFFu) : ~ob;
      out_score[(int64_t)b * k + i] = ok ? __uint_as_float(u) : -INFINITY;
    }
  }
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_indexer_pool_chunks(const void* pool, int dtype, int64_t row_width, int32_t width,
                                 const int32_t* block_tables, int64_t table_stride, int32_t table_width,
                                 const int32_t* seq_lens, int32_t batch, int32_t block_size, int32_t num_blocks,
                                 int32_t chunk_begin, int32_t chunk_count, int32_t max_chunks, const void* proj,
                                 int proj_dtype, int32_t out_dim, float* out, int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(dtype_size(dtype) > 0, "indexer_pool_chunks: unknown dtype");
  SNAPMIND_CHECK_ARG(width > 0 && width <= row_width && width <= 16384 && batch >= 0 && batch <= 65535 &&
                         block_size > 0 && chunk_begin >= 0 && chunk_count >= 0 &&
                         chunk_begin + chunk_count <= max_chunks,
                     "indexer_pool_chunks: bad sizes");
  SNAPMIND_CHECK_ARG(!proj || (out_dim > 0 && dtype_size(proj_dtype) > 0), "indexer_pool_chunks: bad projection");
  if (batch == 0 || chunk_count == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(pool && block_tables && out, "indexer_pool_chunks: null pointer");
  PoolParams p{static_cast<const char*>(pool), row_width, width, block_tables, table_stride, table_width,
               seq_lens, batch, block_size, num_blocks, chunk_begin, chunk_count, max_chunks,
               static_cast<const char*>(proj), out_dim, out, err_word};
  dim3 grid(chunk_count, batch);
  const size_t smem = sizeof(float) * width;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kernel) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "indexer_pool smem attribute");
    }
    kernel<<<grid, 256, smem, st>>>(p);
    return cuda_status(cudaGetLastError(), "indexer_pool launch");
  };
  const int pd = proj ? proj_dtype : SNAPMIND_DTYPE_F32;
#define SNAPMIND_POOL_CASE(TT, TPP) return go(indexer_pool_kernel<TT, TPP>)
  if (dtype == SNAPMIND_DTYPE_F32) {
    if (pd == SNAPMIND_DTYPE_F32) SNAPMIND_POOL_CASE(float, float);
    if (pd == SNAPMIND_DTYPE_BF16) SNAPMIND_POOL_CASE(float, __nv_bfloat16);
    SNAPMIND_POOL_CASE(float, __half);
  }
  if (dtype == SNAPMIND_DTYPE_BF16) {
    if (pd == SNAPMIND_DTYPE_F32) SNAPMIND_POOL_CASE(__nv_bfloat16, float);
    if (pd == SNAPMIND_DTYPE_BF16) SNAPMIND_POOL_CASE(__nv_bfloat16, __nv_bfloat16);
    SNAPMIND_POOL_CASE(__nv_bfloat16, __half);
  }
  if (pd == SNAPMIND_DTYPE_F32) SNAPMIND_POOL_CASE(__half, float);
  if (pd == SNAPMIND_DTYPE_BF16) SNAPMIND_POOL_CASE(__half, __nv_bfloat16);
  SNAPMIND_POOL_CASE(__half, __half);
#undef SNAPMIND_POOL_CASE
}

int snapmind_indexer_score_ref(const float* q, const float* w, int32_t n_rows, int32_t n_heads,
                               const float* keys, int32_t n_chunks, int32_t dim, float* scores, void* stream) {
  SNAPMIND_CHECK_ARG(n_rows > 0 && n_heads > 0 && n_chunks >= 0 && dim > 0, "indexer_score_ref: bad sizes");
  if (n_chunks == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(q && w && keys && scores, "indexer_score_ref: null pointer");
  const int warps_per_block = 8;
  const int grid = (n_chunks + warps_per_block - 1) / warps_per_block;
  indexer_score_ref_kernel<<<grid, 32 * warps_per_block, 0, static_cast<cudaStream_t>(stream)>>>(
      q, w, n_rows, n_heads, keys, n_chunks, dim, scores);
  SNAPMIND_LAUNCH_CHECK("indexer_score_ref launch");
}

int snapmind_indexer_topk(const void* q, const void* keys, int dtype, const int32_t* n_chunks, int32_t n_chunks0,
                          int32_t batch, int32_t max_chunks, int32_t dim, float scale, float bias, int32_t k,
                          int32_t* out_idx, float* out_score, float* all_scores, void* stream) {
  SNAPMIND_CHECK_ARG(dtype_size(dtype) > 0, "indexer_topk: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && max_chunks > 0 && max_chunks <= 16384 && dim > 0 && k > 0 && k <= max_chunks,
                     "indexer_topk: bad sizes (max_chunks <= 16384, 0 < k <= max_chunks)");
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(q && keys && out_idx, "indexer_topk: null pointer");
  int sort_n = 1;
  while (sort_n < max_chunks) sort_n <<= 1;
  const size_t smem = sizeof(unsigned long long) * sort_n;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kernel, const auto* qq, const auto* kk) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "indexer_topk smem attribute");
    }
    kernel<<<batch, kTopkThreads, smem, st>>>(qq, kk, n_chunks, n_chunks0, max_chunks, dim, scale, bias, k, sort_n,
                                              out_idx, out_score, all_scores);
    return cuda_status(cudaGetLastError(), "indexer_topk launch");
  };
  switch (dtype) {
    case SNAPMIND_DTYPE_F32:
      return go(indexer_topk_kernel<float>, static_cast<const float*>(q), static_cast<const float*>(keys));
    case SNAPMIND_DTYPE_BF16:
      return go(indexer_topk_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(q),
                static_cast<const __nv_bfloat16*>(keys));
    default:
      return go(indexer_topk_kernel<__half>, static_cast<const __half*>(q), static_cast<const __half*>(keys));
  }
}

}  // extern "C"
