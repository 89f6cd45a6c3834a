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

constexpr int kPoolThreads = 512;
constexpr int kPoolUnroll = 8;

// Where item `it` (sequence b, chunk c) lives: its pool block and row count
// (phys < 0: nothing to read, the output is zero).  Out-of-range block ids
// are flagged and skipped.
__device__ __forceinline__ void pool_item(const PoolParams& p, int64_t it, int& b, int& c, int& n, int& phys) {
  b = (int)(it / p.chunk_count);
  c = p.chunk_begin + (int)(it - (int64_t)b * p.chunk_count);
  // without lengths every chunk is full
  n = p.seq_lens ? min(p.block_size, p.seq_lens[b] - c * p.block_size) : p.block_size;
  phys = -1;
  if (n > 0 && c < p.table_width) {
    phys = p.tables[(int64_t)b * p.table_stride + c];
    if (phys < 0 || phys >= p.num_blocks) {
      if (threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
      phys = -1;
    }
  }
}

// out[o] = P[o] . mean for o < out_dim.  4 threads per output, each over a
// quarter of the width.  Lane l of a warp takes quarter l / 8 of output
// (warp slot * 8 + l % 8): the 8 lanes of one shared-memory phase read 8
// padded projection rows at the same column (distinct bank groups) and the
// same mean elements (a broadcast).
template <typename TP>
__device__ __forceinline__ void project_mean(const TP* P, int w_stride, const float* mean, int W, int out_dim,
                                             float* out) {
  const int tid = threadIdx.x;
  const int qw = (W + 3) / 4;
  constexpr int EPP = 16 / (int)sizeof(TP);  // projection elements per 16-byte vector
  const bool pvec = (qw % EPP == 0) && (W % 4 == 0) && (w_stride % EPP == 0) &&
                    ((reinterpret_cast<uintptr_t>(P) & 15) == 0);
  for (int base = 0; base < out_dim * 4; base += kPoolThreads) {  // uniform trip count (shuffles)
    const int task = base + tid;
    const int lane = task & 31, qd = lane >> 3;
    const int o = (task >> 5) * 8 + (lane & 7);
    const bool active = o < out_dim;
    const int d_lo = qd * qw, d_hi = min(W, d_lo + qw), n_d = active ? max(0, d_hi - d_lo) : 0;
    const TP* prow = P + (int64_t)(active ? o : 0) * w_stride + d_lo;
    const float* mrow = mean + d_lo;
    float a0 = 0.f, a1 = 0.f;
    if (pvec) {
      const int nv = n_d / EPP;
      for (int v = 0; v < nv; ++v) {
        const uint4 wv = *reinterpret_cast<const uint4*>(prow + v * EPP);
        const TP* w = reinterpret_cast<const TP*>(&wv);
#pragma unroll
        for (int e = 0; e < EPP; e += 2) {
          a0 = fmaf(Conv<TP>::to_f(w[e]), mrow[v * EPP + e], a0);
          a1 = fmaf(Conv<TP>::to_f(w[e + 1]), mrow[v * EPP + e + 1], a1);
        }
      }
    } else {
      for (int i = 0; i < n_d; ++i) a0 = fmaf(Conv<TP>::to_f(prow[i]), mrow[i], a0);
    }
    float a = a0 + a1;
    a += __shfl_xor_sync(0xffffffffu, a, 8);
    a += __shfl_xor_sync(0xffffffffu, a, 16);
    if (active && qd == 0) out[o] = a;
  }
}

// out[o] = P[o] . mean, sliced: warp s takes columns [32 s, 32 s + 32) and
// lane l the outputs l, l + 32, l + 64, l + 96.  The slice of the mean is read
// once into registers (broadcast loads); projection rows are padded so their
// stride is an odd number of 16-byte granules, which puts the 8 lanes of a
// shared-memory phase (8 consecutive rows, one column) on 8 distinct bank
// groups.  Slice partials meet in `red` ([W / 32][out_dim] floats) and are
// summed in slice order.  Needs W % 32 == 0, W / 32 <= warps, out_dim <= 128.
template <typename TP>
__device__ __forceinline__ void project_mean_sliced(const TP* P, int w_stride, const float* mean, int W,
                                                    int out_dim, float* out, float* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_slices = W / 32;
  constexpr int EPP = 16 / (int)sizeof(TP);
  constexpr int NV = 32 / EPP;
  if (warp < n_slices) {
    float m[32];
    const float4* m4 = reinterpret_cast<const float4*>(mean + warp * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 t = m4[k];
      m[4 * k] = t.x;
      m[4 * k + 1] = t.y;
      m[4 * k + 2] = t.z;
      m[4 * k + 3] = t.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int o = lane + 32 * i;
      if (o < out_dim) {
        const uint4* row = reinterpret_cast<const uint4*>(P + (int64_t)o * w_stride + warp * 32);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          const uint4 wv = row[v];
          const TP* w = reinterpret_cast<const TP*>(&wv);
#pragma unroll
          for (int e = 0; e < EPP; e += 2) {
            a0 = fmaf(Conv<TP>::to_f(w[e]), m[v * EPP + e], a0);
            a1 = fmaf(Conv<TP>::to_f(w[e + 1]), m[v * EPP + e + 1], a1);
          }
        }
        red[warp * out_dim + o] = a0 + a1;
      }
    }
  }
  __syncthreads();
  for (int o = tid; o < out_dim; o += kPoolThreads) {
    float acc = 0.f;
    for (int w = 0; w < n_slices; ++w) acc += red[w * out_dim + o];
    out[o] = acc;
  }
}

// Persistent: each CTA loops over (sequence, chunk) items with a stride of
// the grid.  The projection matrix is staged once per CTA in shared memory
// (when it fits), its rows padded by 16 bytes.  A chunk's rows are summed by
// row groups of threads with 16-byte loads and the group partials reduced in
// shared memory.
//
// Pipelined path (16-byte rows, a chunk fits one batch of kPoolUnroll rows per
// thread): the loads of item i+1 are issued right after item i's registers
// were summed, and the block id of item i+2 is looked up at the same time, so
// HBM traffic of the next chunk overlaps the reduction and the projection of
// the current one.  Otherwise a plain loop does one item after another.
//
// smem: [proj cache (optional), out_dim rows of width + pad][mean: width][partials: groups x width]
template <typename T, typename TP>
__global__ void __launch_bounds__(kPoolThreads, 1) indexer_pool_kernel(PoolParams p, int cache_proj, int vec_ok) {
  extern __shared__ __align__(16) unsigned char pool_smem[];
  const int W = p.width;
  constexpr int kPad = 16 / (int)sizeof(TP);
  const int w_stride = cache_proj ? W + kPad : W;  // elements between projection rows
  const int64_t proj_elems = cache_proj ? (int64_t)p.out_dim * w_stride : 0;
  TP* wcache = reinterpret_cast<TP*>(pool_smem);
  float* mean = reinterpret_cast<float*>(pool_smem + ((proj_elems * (int64_t)sizeof(TP) + 15) / 16) * 16);
  float* part = mean + W;
  const int tid = threadIdx.x;
  if (cache_proj) {
    const TP* P = reinterpret_cast<const TP*>(p.proj);
    const int64_t n = (int64_t)p.out_dim * W;
    for (int64_t i = tid; i < n; i += kPoolThreads) wcache[(i / W) * w_stride + i % W] = P[i];
  }
  const TP* P = cache_proj ? wcache : reinterpret_cast<const TP*>(p.proj);
  constexpr int EPV = 16 / (int)sizeof(T);  // elements per 16-byte vector
  const int n_vec = W / EPV;
  const int groups = vec_ok ? kPoolThreads / n_vec : 1;
  const int out_w = p.proj ? p.out_dim : W;
  const int64_t items = (int64_t)p.batch * p.chunk_count;
  const int64_t stride = gridDim.x;
  // the sliced projection reuses the partials buffer (groups x W floats) for its slice sums
  constexpr int EPP = 16 / (int)sizeof(TP);
  const bool sliced = p.proj && W % 32 == 0 && W / 32 <= kPoolThreads / 32 && p.out_dim <= 128 &&
                      (W / 32) * p.out_dim <= groups * W && w_stride % EPP == 0 &&
                      (reinterpret_cast<uintptr_t>(P) & 15) == 0;
  auto project = [&](float* out) {
    if (sliced) project_mean_sliced(P, w_stride, mean, W, p.out_dim, out, part);
    else project_mean(P, w_stride, mean, W, p.out_dim, out);
  };

  if (vec_ok && p.block_size <= groups * kPoolUnroll) {
    const int j = tid % n_vec, g = tid / n_vec;
    const bool loader = g < groups;
    uint4 v[kPoolUnroll];
    auto issue = [&](int phys, int n) {
      const T* rows = reinterpret_cast<const T*>(p.pool) + (int64_t)(phys < 0 ? 0 : phys) * p.block_size * p.row_width;
#pragma unroll
      for (int u = 0; u < kPoolUnroll; ++u) {
        const int r = g + u * groups;
        v[u] = (loader && phys >= 0 && r < n) ? *reinterpret_cast<const uint4*>(rows + (int64_t)r * p.row_width + j * EPV)
                                             : make_uint4(0, 0, 0, 0);
      }
    };
    int64_t it = blockIdx.x;
    int b, c, n, phys, b1 = 0, c1 = 0, n1 = 0, phys1 = -1;
    if (it < items) {
      pool_item(p, it, b, c, n, phys);
      issue(phys, n);
      if (it + stride < items) pool_item(p, it + stride, b1, c1, n1, phys1);
    }
    __syncthreads();  // projection cache loaded
    for (; it < items; it += stride) {
      float acc[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
#pragma unroll
      for (int u = 0; u < kPoolUnroll; ++u) {
        const T* x = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] += Conv<T>::to_f(x[e]);
      }
      if (loader) {
#pragma unroll
        for (int e = 0; e < EPV; ++e) part[g * W + j * EPV + e] = acc[e];
      }
      // the next item's rows fly while this one is reduced and projected
      int b2 = 0, c2 = 0, n2 = 0, phys2 = -1;
      if (it + stride < items) {
        issue(phys1, n1);
        if (it + 2 * stride < items) pool_item(p, it + 2 * stride, b2, c2, n2, phys2);
      }
      __syncthreads();  // partials written
      float* out = p.out + ((int64_t)b * p.max_chunks + c) * out_w;
      if (phys < 0) {
        for (int i = tid; i < out_w; i += kPoolThreads) out[i] = 0.f;
      } else {
        const float inv = 1.f / (float)n;
        for (int d = tid; d < W; d += kPoolThreads) {
          float s = 0.f;
          for (int gg = 0; gg < groups; ++gg) s += part[gg * W + d];
          mean[d] = s * inv;
        }
        __syncthreads();  // mean complete
        if (!p.proj) {
          for (int d = tid; d < W; d += kPoolThreads) out[d] = mean[d];
        } else {
          project(out);
        }
      }
      __syncthreads();  // mean and partials consumed
      b = b1; c = c1; n = n1; phys = phys1;
      b1 = b2; c1 = c2; n1 = n2; phys1 = phys2;
    }
    return;
  }

  for (int64_t it = blockIdx.x; it < items; it += stride) {
    int b, c, n, phys;
    pool_item(p, it, b, c, n, phys);
    float* out = p.out + ((int64_t)b * p.max_chunks + c) * out_w;
    __syncthreads();  // previous item's mean/part reads are done (and the cache is loaded)
    if (phys < 0) {
      for (int i = tid; i < out_w; i += kPoolThreads) out[i] = 0.f;
      continue;
    }
    const T* rows = reinterpret_cast<const T*>(p.pool) + (int64_t)phys * p.block_size * p.row_width;
    const float inv = 1.f / (float)n;
    if (vec_ok) {
      const int j = tid % n_vec, g = tid / n_vec;
      float acc[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
      if (g < groups) {
        for (int r0 = g; r0 < n; r0 += groups * kPoolUnroll) {
          uint4 v[kPoolUnroll];
#pragma unroll
          for (int u = 0; u < kPoolUnroll; ++u) {
            const int r = r0 + u * groups;
            v[u] = r < n ? *reinterpret_cast<const uint4*>(rows + (int64_t)r * p.row_width + j * EPV)
                         : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < kPoolUnroll; ++u) {
            const T* x = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] += Conv<T>::to_f(x[e]);
          }
        }
#pragma unroll
        for (int e = 0; e < EPV; ++e) part[g * W + j * EPV + e] = acc[e];
      }
      __syncthreads();
      for (int d = tid; d < W; d += kPoolThreads) {
        float s = 0.f;
        for (int gg = 0; gg < groups; ++gg) s += part[gg * W + d];
        mean[d] = s * inv;
      }
    } else {
      for (int d = tid; d < W; d += kPoolThreads) {
        float s = 0.f;
        for (int r = 0; r < n; ++r) s += Conv<T>::to_f(rows[(int64_t)r * p.row_width + d]);
        mean[d] = s * inv;
      }
    }
    __syncthreads();
    if (!p.proj) {
      for (int d = tid; d < W; d += kPoolThreads) out[d] = mean[d];
      continue;
    }
    project(out);
  }
}

// ---------------------------------------------------------------------------
// chunk means then projection, as two kernels (many chunks at once)
// ---------------------------------------------------------------------------
constexpr int kMeanThreads = 256;

// One CTA per item: the mean of the chunk's rows (first W columns), fp32, into
// means[item][W].  Row groups of threads sum with 16-byte loads, kPoolUnroll
// rows in flight per thread; several CTAs per SM keep many chunks in flight.
template <typename T>
__global__ void __launch_bounds__(kMeanThreads) indexer_mean_kernel(PoolParams p, float* means, int vec_ok) {
  extern __shared__ __align__(16) float mpart[];  // [groups][W]
  const int W = p.width;
  const int64_t it = blockIdx.x;
  int b, c, n, phys;
  pool_item(p, it, b, c, n, phys);
  float* out = means + it * W;
  const int tid = threadIdx.x;
  if (phys < 0) {
    for (int d = tid; d < W; d += kMeanThreads) out[d] = 0.f;
    return;
  }
  const T* rows = reinterpret_cast<const T*>(p.pool) + (int64_t)phys * p.block_size * p.row_width;
  const float inv = 1.f / (float)n;
  if (!vec_ok) {
    for (int d = tid; d < W; d += kMeanThreads) {
      float acc = 0.f;
      for (int r = 0; r < n; ++r) acc += Conv<T>::to_f(rows[(int64_t)r * p.row_width + d]);
      out[d] = acc * inv;
    }
    return;
  }
  constexpr int EPV = 16 / (int)sizeof(T);
  const int n_vec = W / EPV;
  const int groups = kMeanThreads / n_vec;
  const int j = tid % n_vec, g = tid / n_vec;
  if (g < groups) {
    float acc[EPV];
#pragma unroll
    for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
    for (int r0 = g; r0 < n; r0 += groups * kPoolUnroll) {
      uint4 v[kPoolUnroll];
#pragma unroll
      for (int u = 0; u < kPoolUnroll; ++u) {
        const int r = r0 + u * groups;
        v[u] = r < n ? *reinterpret_cast<const uint4*>(rows + (int64_t)r * p.row_width + j * EPV)
                     : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kPoolUnroll; ++u) {
        const T* x = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] += Conv<T>::to_f(x[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < EPV; ++e) mpart[g * W + j * EPV + e] = acc[e];
  }
  __syncthreads();
  for (int d = tid; d < W; d += kMeanThreads) {
    float acc = 0.f;
    for (int gg = 0; gg < groups; ++gg) acc += mpart[gg * W + d];
    out[d] = acc * inv;
  }
}

constexpr int kProjTile = 64;   // items and outputs per CTA
constexpr int kProjK = 32;      // columns per step
constexpr int kProjPad = 68;    // smem row stride (floats): 16-byte aligned rows

// 8 consecutive elements as floats; 16-byte loads when `vec` (aligned rows).
__device__ __forceinline__ void load8(const float* src, bool valid, bool vec, int n_left, float* dst) {
  if (valid && vec) {
    const float4 x = *reinterpret_cast<const float4*>(src), y = *reinterpret_cast<const float4*>(src + 4);
    dst[0] = x.x; dst[1] = x.y; dst[2] = x.z; dst[3] = x.w;
    dst[4] = y.x; dst[5] = y.y; dst[6] = y.z; dst[7] = y.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[e] = (valid && e < n_left) ? src[e] : 0.f;
  }
}
template <typename TP>
__device__ __forceinline__ void load8(const TP* src, bool valid, bool vec, int n_left, float* dst) {
  if (valid && vec) {
    const uint4 x = *reinterpret_cast<const uint4*>(src);
    const TP* t = reinterpret_cast<const TP*>(&x);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[e] = Conv<TP>::to_f(t[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[e] = (valid && e < n_left) ? Conv<TP>::to_f(src[e]) : 0.f;
  }
}

// out[b][c][o] = sum_d means[item][d] * P[o][d] for 64 items x 64 outputs per
// CTA; each thread accumulates 4 items x 4 outputs in fp32, summing d in order.
// The next 32 columns of both operands are loaded into registers while the
// current ones are multiplied.
template <typename TP>
__global__ void __launch_bounds__(256) indexer_project_kernel(PoolParams p, const float* means, int64_t items) {
  __shared__ __align__(16) float As[kProjK][kProjPad];  // [d][item]
  __shared__ __align__(16) float Bs[kProjK][kProjPad];  // [d][output]
  const int tid = threadIdx.x;
  const int W = p.width, O = p.out_dim;
  const int64_t item0 = (int64_t)blockIdx.x * kProjTile;
  const int o0 = blockIdx.y * kProjTile;
  const TP* P = reinterpret_cast<const TP*>(p.proj);
  const int ti = tid >> 4, to = tid & 15;            // 4 items x 4 outputs
  const int l_row = tid & 63, l_k = (tid >> 6) * 8;  // loader: row, 8 columns
  const int64_t l_item = item0 + l_row;
  const int l_o = o0 + l_row;
  const bool a_ok = l_item < items, b_ok = l_o < O;
  const bool vec_a = (W % 4 == 0) && ((reinterpret_cast<uintptr_t>(means) & 15) == 0);
  const bool vec_b = (W % 8 == 0) && ((reinterpret_cast<uintptr_t>(P) & 15) == 0) && sizeof(TP) == 2;
  const float* a_src = means + (a_ok ? l_item : 0) * W + l_k;
  const TP* b_src = P + (int64_t)(b_ok ? l_o : 0) * W + l_k;
  float a_reg[8], b_reg[8];
  auto fetch = [&](int k0) {
    const int left = W - (k0 + l_k);
    load8(a_src + k0, a_ok && left > 0, vec_a && left >= 8, left, a_reg);
    load8(b_src + k0, b_ok && left > 0, vec_b && left >= 8, left, b_reg);
  };
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  fetch(0);
  for (int k0 = 0; k0 < W; k0 += kProjK) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      As[l_k + e][l_row] = a_reg[e];
      Bs[l_k + e][l_row] = b_reg[e];
    }
    __syncthreads();
    if (k0 + kProjK < W) fetch(k0 + kProjK);
#pragma unroll 8
    for (int kk = 0; kk < kProjK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ti * 4]);
      const float4 w = *reinterpret_cast<const float4*>(&Bs[kk][to * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t item = item0 + ti * 4 + i;
    if (item >= items) continue;
    const int b = (int)(item / p.chunk_count);
    const int c = p.chunk_begin + (int)(item - (int64_t)b * p.chunk_count);
    float* out = p.out + ((int64_t)b * p.max_chunks + c) * O;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int o = o0 + to * 4 + j;
      if (o < O) out[o] = acc[i][j];
    }
  }
}

// Tensor-core form of the projection for bf16 projection matrices: each fp32
// mean is split into two bf16 terms (hi = bf16(x), lo = bf16(x - hi): their sum
// is x to about 2^-18 relative), both multiplied by the bf16 matrix with
// mma.sync m16n8k16 and accumulated in fp32.  CTA = 64 chunks x 128 outputs,
// 4 warps of 16 chunks; 32 columns per step, staged in shared memory with
// 80-byte rows (ldmatrix of 8 consecutive rows hits 8 bank groups), the next
// step's operands loaded into registers while the current one is multiplied.
constexpr int kTcItems = 64, kTcOut = 128, kTcK = 32, kTcRow = kTcK + 8;

__device__ __forceinline__ uint32_t idx_smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void idx_ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void idx_mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(128) indexer_project_tc_kernel(PoolParams p, const float* means, int64_t items) {
  __shared__ __align__(16) __nv_bfloat16 Ah[kTcItems][kTcRow];
  __shared__ __align__(16) __nv_bfloat16 Al[kTcItems][kTcRow];
  __shared__ __align__(16) __nv_bfloat16 Bs[kTcOut][kTcRow];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int W = p.width, O = p.out_dim;
  const int64_t item0 = (int64_t)blockIdx.x * kTcItems;
  const int o0 = blockIdx.y * kTcOut;
  const __nv_bfloat16* P = reinterpret_cast<const __nv_bfloat16*>(p.proj);
  // loaders: A rows of 16 floats (two threads per chunk row), B rows of 32 bf16 (one thread per output)
  const int a_r = tid >> 1, a_c = (tid & 1) * 16;
  const int64_t a_item = item0 + a_r;
  const bool a_ok = a_item < items;
  const int b_o = o0 + tid;
  const bool b_ok = b_o < O;
  const float* a_src = means + (a_ok ? a_item : 0) * W + a_c;
  const __nv_bfloat16* b_src = P + (int64_t)(b_ok ? b_o : 0) * W;
  float4 a_reg[4];
  uint4 b_reg[4];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a_reg[j] = a_ok ? *reinterpret_cast<const float4*>(a_src + k0 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
      b_reg[j] = b_ok ? *reinterpret_cast<const uint4*>(b_src + k0 + 8 * j) : make_uint4(0, 0, 0, 0);
    }
  };
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_kof = (lane >> 4) * 8;
  const int b_row = (lane & 7) + ((lane >> 4) & 1) * 8, b_kof = ((lane >> 3) & 1) * 8;
  fetch(0);
  for (int k0 = 0; k0 < W; k0 += kTcK) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x[4] = {a_reg[j].x, a_reg[j].y, a_reg[j].z, a_reg[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(x[e]);
        Ah[a_r][a_c + 4 * j + e] = hi;
        Al[a_r][a_c + 4 * j + e] = __float2bfloat16_rn(x[e] - __bfloat162float(hi));
      }
      *reinterpret_cast<uint4*>(&Bs[tid][8 * j]) = b_reg[j];
    }
    __syncthreads();
    if (k0 + kTcK < W) fetch(k0 + kTcK);
#pragma unroll
    for (int ks = 0; ks < kTcK / 16; ++ks) {
      uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
      idx_ldsm4(idx_smem_u32(&Ah[16 * warp + a_row][ks * 16 + a_kof]), h0, h1, h2, h3);
      idx_ldsm4(idx_smem_u32(&Al[16 * warp + a_row][ks * 16 + a_kof]), l0, l1, l2, l3);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b0, b1, b2, b3;
        idx_ldsm4(idx_smem_u32(&Bs[16 * np + b_row][ks * 16 + b_kof]), b0, b1, b2, b3);
        idx_mma_bf16(acc[2 * np], h0, h1, h2, h3, b0, b1);
        idx_mma_bf16(acc[2 * np], l0, l1, l2, l3, b0, b1);
        idx_mma_bf16(acc[2 * np + 1], h0, h1, h2, h3, b2, b3);
        idx_mma_bf16(acc[2 * np + 1], l0, l1, l2, l3, b2, b3);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int64_t item = item0 + 16 * warp + g + 8 * hr;
    if (item >= items) continue;
    const int b = (int)(item / p.chunk_count);
    const int c = p.chunk_begin + (int)(item - (int64_t)b * p.chunk_count);
    float* out = p.out + ((int64_t)b * p.max_chunks + c) * O;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int o = o0 + nt * 8 + 2 * tig;
      if (o < O) out[o] = acc[nt][2 * hr];
      if (o + 1 < O) out[o + 1] = acc[nt][2 * hr + 1];
    }
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

// 4 consecutive elements as float4 (aligned: 16 bytes for fp32, 8 for 16-bit types)
__device__ __forceinline__ float4 load4f(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <typename T>
__device__ __forceinline__ float4 load4f(const T* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const T* t = reinterpret_cast<const T*>(&u);
  return make_float4(Conv<T>::to_f(t[0]), Conv<T>::to_f(t[1]), Conv<T>::to_f(t[2]), Conv<T>::to_f(t[3]));
}

constexpr int kDotChunks = 16;  // chunks per warp pass

// One warp: q . key[c] for the kDotChunks chunks c0 .. c0 + 15 (0 for c >= nc);
// lane u < kDotChunks returns chunk c0 + u.  With `vec` each lane reads 4
// consecutive dims of every chunk row at once, so a pass is one round trip.
template <typename T>
__device__ __forceinline__ float warp_chunk_dots(const T* qb, const T* kb, int dim, int c0, int nc, bool vec,
                                                 int lane) {
  float dot[kDotChunks];
#pragma unroll
  for (int u = 0; u < kDotChunks; ++u) dot[u] = 0.f;
  if (vec) {
    for (int d = lane * 4; d < dim; d += 128) {
      const float4 qv = load4f(qb + d);
      float4 kv[kDotChunks];
#pragma unroll
      for (int u = 0; u < kDotChunks; ++u)
        kv[u] = c0 + u < nc ? load4f(kb + (int64_t)(c0 + u) * dim + d) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < kDotChunks; ++u) {
        dot[u] = fmaf(qv.x, kv[u].x, dot[u]);
        dot[u] = fmaf(qv.y, kv[u].y, dot[u]);
        dot[u] = fmaf(qv.z, kv[u].z, dot[u]);
        dot[u] = fmaf(qv.w, kv[u].w, dot[u]);
      }
    }
  } else {
    for (int d = lane; d < dim; d += 32) {
      const float qd = Conv<T>::to_f(qb[d]);
#pragma unroll
      for (int u = 0; u < kDotChunks; ++u)
        if (c0 + u < nc) dot[u] = fmaf(qd, Conv<T>::to_f(kb[(int64_t)(c0 + u) * dim + d]), dot[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < kDotChunks; ++u) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], off);
  }
  float mine = dot[0];
#pragma unroll
  for (int u = 1; u < kDotChunks; ++u)
    if (lane == u) mine = dot[u];
  return mine;
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads) indexer_topk_kernel(
    const T* q, const T* keys, const int32_t* n_chunks_arr, int n_chunks0, int max_chunks, int dim, float scale,
    float bias, int k, int sort_n, int32_t* out_idx, float* out_score, float* all_scores, int vec) {
  extern __shared__ unsigned long long skeys[];  // [sort_n]
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // as in the sliced kernel
  const int b = blockIdx.x;
  int nc = n_chunks_arr ? n_chunks_arr[b] : n_chunks0;
  nc = max(0, min(nc, max_chunks));
  const T* qb = q + (int64_t)b * dim;
  const T* kb = keys + (int64_t)b * max_chunks * dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  constexpr int kU = kDotChunks;
  for (int c0 = warp * kU; c0 < sort_n; c0 += nw * kU) {
    const float mine = warp_chunk_dots(qb, kb, dim, c0, nc, vec != 0, lane);
    if (lane < kU) {
      const int c = c0 + lane;
      unsigned long long key = 0ull;  // below every real key
      if (c < nc) {
        const float s = 1.f / (1.f + expf(-(mine * scale + bias)));
        if (all_scores) all_scores[(int64_t)b * max_chunks + c] = s;
        key = ((unsigned long long)ordered_bits(s) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)c);
      }
      if (c < sort_n) skeys[c] = key;
    }
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


constexpr int kSliceChunks = 128;  // chunks scored and pre-selected by one CTA
constexpr int kSliceThreads = 256;
constexpr int kWarpMergeK = 64;        // k up to this: one warp merges the slices' sorted lists
constexpr int kMaxTopkChunks = 16384;  // chunks per sequence the top-k accepts
constexpr int kMaxMergeSlices = kMaxTopkChunks / kSliceChunks;
constexpr int kListsPerLane = (kMaxMergeSlices + 31) / 32;  // warp merge: lists owned by one lane

// Two-phase top-k over many CTAs.  CTA (slice, b) scores chunks
// [slice * 128, slice * 128 + 128) of sequence b and keeps the best
// `keep` = min(k, 128) of their (ordered score, inverted id) keys as
// candidates, in rank order.  Every member of the sequence's top-k is among the
// candidates of its slice, so the top-k of the union of candidates is the exact
// answer.  The CTA that takes the sequence's last ticket ranks the union and
// resets the ticket; no CTA waits for another.  Both selections rank keys
// instead of sorting them (no barrier stages).
template <typename T>
__global__ void __launch_bounds__(kSliceThreads) indexer_topk_sliced_kernel(
    const T* q, const T* keys, const int32_t* n_chunks_arr, int n_chunks0, int max_chunks, int dim, float scale,
    float bias, int k, int n_slices, int keep, int merge_n, unsigned long long* cand, int32_t* tickets,
    int32_t* out_idx, float* out_score, float* all_scores, int vec) {
  extern __shared__ unsigned long long sk[];  // [max(kSliceChunks, merge_n)]
  __shared__ int s_last;
  // a kernel launched as this one's programmatic dependent (the sparse attention) may be
  // scheduled once every CTA here has started; it still waits for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int slice = blockIdx.x, b = blockIdx.y;
  int nc = n_chunks_arr ? n_chunks_arr[b] : n_chunks0;
  nc = max(0, min(nc, max_chunks));
  const int c_begin = slice * kSliceChunks;
  const T* qb = q + (int64_t)b * dim;
  const T* kb = keys + (int64_t)b * max_chunks * dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  constexpr int kU = kDotChunks;
  for (int l0 = warp * kU; l0 < kSliceChunks; l0 += nw * kU) {
    const float mine = warp_chunk_dots(qb, kb, dim, c_begin + l0, nc, vec != 0, lane);
    if (lane < kU) {
      const int c = c_begin + l0 + lane;
      unsigned long long key = 0ull;  // below every real key
      if (c < nc) {
        const float s = 1.f / (1.f + expf(-(mine * scale + bias)));
        if (all_scores) all_scores[(int64_t)b * max_chunks + c] = s;
        key = ((unsigned long long)ordered_bits(s) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)c);
      }
      sk[l0 + lane] = key;
    }
  }
  __syncthreads();
  // selection by rank (no sort): rank = keys ahead of this one, ties to the lower index;
  // ranks are distinct, and the best `keep` land in rank order
  unsigned long long* mine = cand + ((int64_t)b * n_slices + slice) * keep;
  for (int i = threadIdx.x; i < kSliceChunks; i += blockDim.x) {
    const unsigned long long key = sk[i];
    int r = 0;
    for (int j = 0; j < kSliceChunks; ++j) {
      const unsigned long long kj = sk[j];
      r += (kj > key) || (kj == key && j < i);
    }
    if (r < keep) mine[r] = key;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&tickets[b], 1) == n_slices - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const unsigned long long* all = cand + (int64_t)b * n_slices * keep;
  const int n_cand = n_slices * keep;
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) sk[i] = __ldcg(all + i);
  __syncthreads();
  // the same rank selection over the union of candidates; output slots past the
  // valid chunks are -1 (real keys rank before the zero fillers)
  const int n_out = min(k, nc);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    if (i >= n_out) {
      out_idx[(int64_t)b * k + i] = -1;
      if (out_score) out_score[(int64_t)b * k + i] = -INFINITY;
    }
  }
  if (k <= kWarpMergeK) {
    // small k: one warp merges the slices' lists (each sorted, descending) by
    // repeatedly taking the largest list head.  Real keys are unique (score
    // bits, then the inverted chunk id) and above the zero fillers, so the
    // order is the same as ranking the union.
    if (warp == 0) {
      // lane owns lists lane + 32 j (j < kListsPerLane); their current heads and
      // the entries after them live in registers, so a step has no dependent
      // shared-memory load
      unsigned long long head[kListsPerLane], nxt[kListsPerLane];
      int pos[kListsPerLane];
#pragma unroll
      for (int j = 0; j < kListsPerLane; ++j) {
        const int L = lane + 32 * j;
        const bool has = L < n_slices;
        pos[j] = 0;
        head[j] = has ? sk[L * keep] : 0ull;
        nxt[j] = has && keep > 1 ? sk[L * keep + 1] : 0ull;
      }
      for (int i = 0; i < n_out; ++i) {
        unsigned long long best = head[0];
        int bj = 0;
#pragma unroll
        for (int j = 1; j < kListsPerLane; ++j)
          if (head[j] > best) {
            best = head[j];
            bj = j;
          }
        // 64-bit warp maximum as (high word, then low word among the high-word winners)
        const uint32_t hi = (uint32_t)(best >> 32), lo = (uint32_t)best;
        const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
        const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? lo : 0u);
        const unsigned long long m = ((unsigned long long)mhi << 32) | mlo;
        if (m == 0ull) break;  // only fillers left (cannot happen while i < n_out)
        if (best == m) {        // the one lane holding the largest head
          out_idx[(int64_t)b * k + i] = (int32_t)(0xFFFFFFFFu - lo);
          if (out_score) {
            const uint32_t u = (mhi & 0x80000000u) ? (mhi & 0x7FFFFFFFu) : ~mhi;
            out_score[(int64_t)b * k + i] = __uint_as_float(u);
          }
#pragma unroll
          for (int j = 0; j < kListsPerLane; ++j)
            if (j == bj) {
              head[j] = nxt[j];
              pos[j] += 1;
              nxt[j] = pos[j] + 1 < keep ? sk[(lane + 32 * j) * keep + pos[j] + 1] : 0ull;
            }
        }
        __syncwarp();
      }
    }
    if (threadIdx.x == 0) tickets[b] = 0;
    return;
  }
  // each slice's candidates are in rank order (descending): a candidate's global
  // rank is its place in its own list plus, per other list, the keys ahead of it
  // (binary search; equal keys count as ahead when their list comes first)
  for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
    const int L = i / keep;
    const unsigned long long key = sk[i];
    int r = i - L * keep;
    for (int M = 0; M < n_slices; ++M) {
      if (M == L) continue;
      const unsigned long long* lst = sk + M * keep;
      int lo = 0, hi = keep;
      if (M < L) {
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (lst[mid] >= key) lo = mid + 1; else hi = mid;
        }
      } else {
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (lst[mid] > key) lo = mid + 1; else hi = mid;
        }
      }
      r += lo;
    }
    if (r < n_out) {
      out_idx[(int64_t)b * k + r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
      if (out_score) {
        const uint32_t ob = (uint32_t)(key >> 32);
        const uint32_t u = (ob & 0x80000000u) ? (ob & 0x7FFFFFFFu) : ~ob;
        out_score[(int64_t)b * k + r] = __uint_as_float(u);
      }
    }
  }
  if (threadIdx.x == 0) tickets[b] = 0;
}

// ---------------------------------------------------------------------------
// query projection q[b] = W . h[b] (fp32 out): one read of W, HBM-bound
// ---------------------------------------------------------------------------
constexpr int kQueryRows = 1;    // output rows per CTA
constexpr int kQueryParts = 16;  // warps splitting d_model for one output row
constexpr int kQueryBatch = 8;   // sequences per CTA (grid.y covers the rest)

// CTA = (1 output row, up to 8 sequences), 16 warps: warp `part` sums part `part`
// of d_model for the row over the CTA's sequences with 16-byte loads, two vectors
// per lane in flight (W read once; the hidden rows are shared by every CTA through
// L2), then the 16 parts meet in shared memory.  At d_model 7168 a lane's loads are
// all in flight at once, and one CTA per output row spreads the 128 rows over the SMs.
template <typename T>
__global__ void __launch_bounds__(32 * kQueryRows * kQueryParts) indexer_query_kernel(
    const T* hidden, const T* w, float* out, int batch, int d_model, int out_dim, int vec) {
  __shared__ float part_sum[kQueryRows][kQueryParts][kQueryBatch];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_l = warp / kQueryParts, part = warp % kQueryParts;
  const int o = blockIdx.x * kQueryRows + row_l;
  const int b0 = blockIdx.y * kQueryBatch;
  const int nb = min(kQueryBatch, batch - b0);
  float acc[kQueryBatch];
#pragma unroll
  for (int j = 0; j < kQueryBatch; ++j) acc[j] = 0.f;
  if (o < out_dim) {
    const T* wr = w + (int64_t)o * d_model;
    if (vec) {
      constexpr int V = 16 / (int)sizeof(T);
      const int nv = d_model / V;
      const int v0 = part * nv / kQueryParts, v1 = (part + 1) * nv / kQueryParts;
      // two vectors per lane at a time: every load of the pair (W and the rows of the
      // CTA's sequences) is issued before any of them is used, so they are in flight together
      for (int v = v0 + lane; v < v1; v += 64) {
        const bool two = v + 32 < v1;
        uint4 wv[2], hv[2][kQueryBatch];
        wv[0] = __ldg(reinterpret_cast<const uint4*>(wr + (int64_t)v * V));
        wv[1] = two ? __ldg(reinterpret_cast<const uint4*>(wr + (int64_t)(v + 32) * V)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < kQueryBatch; ++j) {
          const T* hr = hidden + (int64_t)(b0 + (j < nb ? j : 0)) * d_model;
          hv[0][j] = *reinterpret_cast<const uint4*>(hr + (int64_t)v * V);
          hv[1][j] = two ? *reinterpret_cast<const uint4*>(hr + (int64_t)(v + 32) * V) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const T* wt = reinterpret_cast<const T*>(&wv[u]);
#pragma unroll
          for (int j = 0; j < kQueryBatch; ++j) {
            const T* ht = reinterpret_cast<const T*>(&hv[u][j]);
#pragma unroll
            for (int e = 0; e < V; ++e) acc[j] = fmaf(Conv<T>::to_f(wt[e]), Conv<T>::to_f(ht[e]), acc[j]);
          }
        }
      }
    } else {
      const int d0 = part * d_model / kQueryParts, d1 = (part + 1) * d_model / kQueryParts;
      for (int d = d0 + lane; d < d1; d += 32) {
        const float wd = Conv<T>::to_f(wr[d]);
#pragma unroll
        for (int j = 0; j < kQueryBatch; ++j)
          if (j < nb) acc[j] = fmaf(wd, Conv<T>::to_f(hidden[(int64_t)(b0 + j) * d_model + d]), acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kQueryBatch; ++j) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < kQueryBatch; ++j) part_sum[row_l][part][j] = acc[j];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kQueryRows * nb; e += blockDim.x) {
    const int r = e / nb, j = e - r * nb;
    const int oo = blockIdx.x * kQueryRows + r;
    if (oo < out_dim) {
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < kQueryParts; ++q) sum += part_sum[r][q][j];
      out[(int64_t)(b0 + j) * out_dim + oo] = sum;
    }
  }
}

struct TopkPlan {
  int n_slices, keep, merge_n;
  int64_t tickets_bytes, total;
};

TopkPlan topk_plan(int batch, int max_chunks, int k) {
  TopkPlan t;
  t.n_slices = (max_chunks + kSliceChunks - 1) / kSliceChunks;
  t.keep = k < kSliceChunks ? k : kSliceChunks;
  t.merge_n = t.n_slices * t.keep;  // candidates held in shared memory by the merging CTA
  if (t.merge_n < kSliceChunks) t.merge_n = kSliceChunks;
  t.tickets_bytes = ((int64_t)batch * 4 + 255) / 256 * 256;
  t.total = t.tickets_bytes + (int64_t)batch * t.n_slices * t.keep * 8;
  return t;
}
}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int64_t snapmind_indexer_pool_workspace_bytes(int32_t batch, int32_t chunk_count, int32_t width) {
  if (batch <= 0 || chunk_count <= 0 || width <= 0) return 0;
  return (int64_t)batch * chunk_count * width * (int64_t)sizeof(float);
}

int snapmind_indexer_pool_chunks(const void* pool, int dtype, int64_t row_width, int32_t width,
                                 const int32_t* block_tables, int64_t table_stride, int32_t table_width,
                                 const int32_t* seq_lens, int32_t batch, int32_t block_size, int32_t num_blocks,
                                 int32_t chunk_begin, int32_t chunk_count, int32_t max_chunks, const void* proj,
                                 int proj_dtype, int32_t out_dim, float* out, void* workspace,
                                 int64_t workspace_bytes, int32_t* err_word, void* stream) {
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
  const int esz = dtype_size(dtype);
  const int epv = 16 / esz;
  const int n_vec = width / epv;
  const int vec_ok = (width % epv == 0) && n_vec <= kPoolThreads && ((row_width * esz) % 16 == 0) &&
                     ((reinterpret_cast<uintptr_t>(pool) & 15) == 0);
  const int groups = vec_ok ? kPoolThreads / n_vec : 1;
  const int pd = proj ? proj_dtype : SNAPMIND_DTYPE_F32;
  const int64_t proj_bytes = proj ? (int64_t)out_dim * (width + 16 / dtype_size(pd)) * dtype_size(pd) : 0;
  const int cache_proj = proj && proj_bytes <= 160 * 1024;
  const size_t smem = (size_t)(cache_proj ? (proj_bytes + 15) / 16 * 16 : 0) + sizeof(float) * width * (1 + groups);
  SNAPMIND_CHECK_ARG(smem <= 220 * 1024, "indexer_pool_chunks: width too large for shared memory");
  const int64_t items = (int64_t)batch * chunk_count;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // many chunks with a projection and room for the means: two kernels
  const int64_t ws_need = snapmind_indexer_pool_workspace_bytes(batch, chunk_count, width);
  if (proj && workspace && workspace_bytes >= ws_need && items >= 4 * (int64_t)num_sms() &&
      items <= 0x7fffffff && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0) {
    float* means = static_cast<float*>(workspace);
    const int mean_vec = vec_ok && kMeanThreads % n_vec == 0 && n_vec <= kMeanThreads;
    const size_t msmem = mean_vec ? sizeof(float) * (size_t)width * (kMeanThreads / n_vec) : 0;
    SNAPMIND_CHECK_ARG(msmem <= 48 * 1024, "indexer_pool_chunks: width too large for the mean kernel");
    auto mean_go = [&](auto kernel) -> int {
      kernel<<<(unsigned)items, kMeanThreads, msmem, st>>>(p, means, mean_vec);
      return cuda_status(cudaGetLastError(), "indexer_mean launch");
    };
    int rc = dtype == SNAPMIND_DTYPE_F32    ? mean_go(indexer_mean_kernel<float>)
             : dtype == SNAPMIND_DTYPE_BF16 ? mean_go(indexer_mean_kernel<__nv_bfloat16>)
                                            : mean_go(indexer_mean_kernel<__half>);
    if (rc != SNAPMIND_OK) return rc;
    const bool tc = pd == SNAPMIND_DTYPE_BF16 && width % kTcK == 0 && (reinterpret_cast<uintptr_t>(proj) & 15) == 0;
    if (tc) {
      dim3 tgrid((unsigned)((items + kTcItems - 1) / kTcItems), (unsigned)((out_dim + kTcOut - 1) / kTcOut));
      SNAPMIND_CHECK_ARG(tgrid.y <= 65535, "indexer_pool_chunks: out_dim too large");
      indexer_project_tc_kernel<<<tgrid, 128, 0, st>>>(p, means, items);
      return cuda_status(cudaGetLastError(), "indexer_project_tc launch");
    }
    dim3 pgrid((unsigned)((items + kProjTile - 1) / kProjTile), (unsigned)((out_dim + kProjTile - 1) / kProjTile));
    SNAPMIND_CHECK_ARG(pgrid.y <= 65535, "indexer_pool_chunks: out_dim too large");
    auto proj_go = [&](auto kernel) -> int {
      kernel<<<pgrid, 256, 0, st>>>(p, means, items);
      return cuda_status(cudaGetLastError(), "indexer_project launch");
    };
    if (pd == SNAPMIND_DTYPE_F32) return proj_go(indexer_project_kernel<float>);
    if (pd == SNAPMIND_DTYPE_BF16) return proj_go(indexer_project_kernel<__nv_bfloat16>);
    return proj_go(indexer_project_kernel<__half>);
  }
  const int per_sm = smem > 110 * 1024 ? 1 : 2;
  const int grid = (int)(items < (int64_t)num_sms() * per_sm ? items : (int64_t)num_sms() * per_sm);
  auto go = [&](auto kernel) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "indexer_pool smem attribute");
    }
    kernel<<<grid, kPoolThreads, smem, st>>>(p, cache_proj, vec_ok);
    return cuda_status(cudaGetLastError(), "indexer_pool launch");
  };
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

int snapmind_indexer_query(const void* hidden, const void* w, int dtype, float* out, int32_t batch, int32_t d_model,
                           int32_t out_dim, void* stream) {
  const int esz = dtype_size(dtype);
  SNAPMIND_CHECK_ARG(esz > 0, "indexer_query: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && d_model > 0 && out_dim > 0, "indexer_query: bad sizes");
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(hidden && w && out, "indexer_query: null pointer");
  SNAPMIND_CHECK_ARG((batch + kQueryBatch - 1) / kQueryBatch <= 65535, "indexer_query: batch too large");
  const int vec = (d_model * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(hidden) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  dim3 grid((out_dim + kQueryRows - 1) / kQueryRows, (batch + kQueryBatch - 1) / kQueryBatch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int threads = 32 * kQueryRows * kQueryParts;
  switch (dtype) {
    case SNAPMIND_DTYPE_F32:
      indexer_query_kernel<float><<<grid, threads, 0, st>>>(static_cast<const float*>(hidden),
                                                           static_cast<const float*>(w), out, batch, d_model,
                                                           out_dim, vec);
      break;
    case SNAPMIND_DTYPE_BF16:
      indexer_query_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(hidden), static_cast<const __nv_bfloat16*>(w), out, batch, d_model,
          out_dim, vec);
      break;
    default:
      indexer_query_kernel<__half><<<grid, threads, 0, st>>>(static_cast<const __half*>(hidden),
                                                            static_cast<const __half*>(w), out, batch, d_model,
                                                            out_dim, vec);
  }
  SNAPMIND_LAUNCH_CHECK("indexer_query launch");
}

int64_t snapmind_indexer_topk_workspace_bytes(int32_t batch, int32_t max_chunks, int32_t k) {
  if (batch <= 0 || max_chunks <= 0 || k <= 0 || k > max_chunks) return 0;
  return topk_plan(batch, max_chunks, k).total;
}

int snapmind_indexer_topk(const void* q, const void* keys, int dtype, const int32_t* n_chunks, int32_t n_chunks0,
                          int32_t batch, int32_t max_chunks, int32_t dim, float scale, float bias, int32_t k,
                          int32_t* out_idx, float* out_score, float* all_scores, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  SNAPMIND_CHECK_ARG(dtype_size(dtype) > 0, "indexer_topk: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && max_chunks > 0 && max_chunks <= kMaxTopkChunks && dim > 0 && k > 0 &&
                         k <= max_chunks,
                     "indexer_topk: bad sizes (max_chunks <= 16384, 0 < k <= max_chunks)");
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(q && keys && out_idx, "indexer_topk: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int esz = dtype_size(dtype);
  const int vec = dim % 4 == 0 && (reinterpret_cast<uintptr_t>(q) % (4 * esz)) == 0 &&
                  (reinterpret_cast<uintptr_t>(keys) % (4 * esz)) == 0;
  if (workspace) {
    const TopkPlan t = topk_plan(batch, max_chunks, k);
    SNAPMIND_CHECK_ARG(workspace_bytes >= t.total, "indexer_topk: workspace needs %lld bytes, got %lld",
                       (long long)t.total, (long long)workspace_bytes);
    SNAPMIND_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 7) == 0, "indexer_topk: workspace not 8-byte aligned");
    SNAPMIND_CHECK_ARG(batch <= 65535, "indexer_topk: batch > 65535");
    int32_t* tickets = static_cast<int32_t*>(workspace);
    auto* cand = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + t.tickets_bytes);
    const size_t smem = sizeof(unsigned long long) * (size_t)t.merge_n;
    auto go2 = [&](auto kernel, const auto* qq, const auto* kk) -> int {
      if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_status(e, "indexer_topk smem attribute");
      }
      kernel<<<dim3(t.n_slices, batch), kSliceThreads, smem, st>>>(
          qq, kk, n_chunks, n_chunks0, max_chunks, dim, scale, bias, k, t.n_slices, t.keep, t.merge_n, cand, tickets,
          out_idx, out_score, all_scores, vec);
      return cuda_status(cudaGetLastError(), "indexer_topk launch");
    };
    switch (dtype) {
      case SNAPMIND_DTYPE_F32:
        return go2(indexer_topk_sliced_kernel<float>, static_cast<const float*>(q), static_cast<const float*>(keys));
      case SNAPMIND_DTYPE_BF16:
        return go2(indexer_topk_sliced_kernel<__nv_bfloat16>, static_cast<const __nv_bfloat16*>(q),
                   static_cast<const __nv_bfloat16*>(keys));
      default:
        return go2(indexer_topk_sliced_kernel<__half>, static_cast<const __half*>(q), static_cast<const __half*>(keys));
    }
  }
  int sort_n = 1;
  while (sort_n < max_chunks) sort_n <<= 1;
  const size_t smem = sizeof(unsigned long long) * sort_n;
  auto go = [&](auto kernel, const auto* qq, const auto* kk) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "indexer_topk smem attribute");
    }
    kernel<<<batch, kTopkThreads, smem, st>>>(qq, kk, n_chunks, n_chunks0, max_chunks, dim, scale, bias, k, sort_n,
                                              out_idx, out_score, all_scores, vec);
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
