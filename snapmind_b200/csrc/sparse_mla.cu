// Sparse MLA decode attention over selected chunks (sm_100a).
//
// For each sequence the attended positions are the union of an attention
// sink (positions < sink), a recent window (positions >= len - window) and
// the chunks chosen by the indexer's top-k (chunk = one block of the paged
// latent pool).  With the query absorbed into the latent space, the score of
// position t for head h is scale * (q_lat[h] . c_t + q_pe[h] . k_pe_t) and the
// output is the latent average sum_t p_t c_t (the value up-projection follows
// outside) — the MLA attention of snapmind/layers/attention/mla.py:217-245 in
// absorbed form, restricted to the selected positions.
//
// CTA = (split, group of 16 heads, sequence).  The CTA marks the included
// chunks in a shared bitmap, compacts them in ascending order, takes its
// share, and for each chunk stages the latent (block_size x R) and rope
// (block_size x P) rows in shared memory, computes the 16 x block_size scores
// (rotated 16-byte reads keep the row-per-thread access conflict-free), runs
// an online softmax per head and accumulates the latent output.  Splits merge
// through the same last-ticket combine as the paged GQA decode.
#include <cfloat>

#include "common.cuh"
#include "paged_decode.cuh"
#include "sparse_mla.cuh"

namespace snapmind {
namespace {

constexpr int kHeadsPerCta = 16;
constexpr int kThreads = 256;
constexpr int kMaxChunkBits = 8192;  // chunks per sequence covered by the bitmaps

template <typename T>
__global__ void __launch_bounds__(kThreads) sparse_mla_kernel(SparseParams p) {
  extern __shared__ float smem[];
  const int s = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int R = p.R, P = p.P, bs = p.bs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // shared layout
  float* q_lat = smem;                                  // [16][R]
  float* q_pe = q_lat + kHeadsPerCta * R;               // [16][P]
  float* S = q_pe + kHeadsPerCta * P;                   // [16][bs]
  float* m_sh = S + kHeadsPerCta * bs;                  // [16]
  float* l_sh = m_sh + kHeadsPerCta;                    // [16]
  float* al_sh = l_sh + kHeadsPerCta;                   // [16]
  uint32_t* sel_bits = reinterpret_cast<uint32_t*>(al_sh + kHeadsPerCta);  // [kMaxChunkBits/32]
  uint32_t* inc_bits = sel_bits + kMaxChunkBits / 32;                      // [kMaxChunkBits/32]
  int32_t* list = reinterpret_cast<int32_t*>(inc_bits + kMaxChunkBits / 32);  // compacted chunk ids
  __shared__ int s_count;
  T* tile_c = reinterpret_cast<T*>(list + kMaxChunkBits);  // [bs][R]
  T* tile_p = tile_c + (size_t)bs * R;                       // [bs][P]

  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  const int n_chunks = min((len + bs - 1) / bs, kMaxChunkBits);
  const int words = (n_chunks + 31) / 32;
  for (int i = tid; i < words; i += kThreads) {
    sel_bits[i] = 0u;
    inc_bits[i] = 0u;
  }
  __syncthreads();
  // selected chunks, then the chunks touched by the sink and the window
  for (int i = tid; i < p.k; i += kThreads) {
    const int c = p.selected[(int64_t)b * p.k + i];
    if (c >= 0 && c < n_chunks) {
      atomicOr(&sel_bits[c >> 5], 1u << (c & 31));
      atomicOr(&inc_bits[c >> 5], 1u << (c & 31));
    }
  }
  const int sink = min(p.sink, len);
  const int wstart = max(0, len - p.window);
  for (int c = tid; c < min((sink + bs - 1) / bs, n_chunks); c += kThreads)  // every chunk the sink touches
    atomicOr(&inc_bits[c >> 5], 1u << (c & 31));
  for (int c = wstart / bs + tid; c < n_chunks; c += kThreads) {
    if (len > wstart) atomicOr(&inc_bits[c >> 5], 1u << (c & 31));
  }
  __syncthreads();
  // compact (ascending) with warp 0
  if (warp == 0) {
    int base = 0;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const uint32_t word = (w0 + lane < words) ? inc_bits[w0 + lane] : 0u;
      const int cnt = __popc(word);
      int pre = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, off);
        if (lane >= off) pre += y;
      }
      int pos = base + pre - cnt;
      uint32_t wv = word;
      while (wv) {
        const int bit = __ffs(wv) - 1;
        list[pos++] = (w0 + lane) * 32 + bit;
        wv &= wv - 1;
      }
      base += __shfl_sync(0xffffffffu, pre, 31);
    }
    if (lane == 0) s_count = base;
  }
  // queries of this head group
  const int h0 = hg * kHeadsPerCta;
  const int nh = min(kHeadsPerCta, p.n_heads - h0);
  const T* qlb = reinterpret_cast<const T*>(p.q_lat) + ((int64_t)b * p.n_heads + h0) * R;
  const T* qpb = reinterpret_cast<const T*>(p.q_pe) + ((int64_t)b * p.n_heads + h0) * P;
  for (int i = tid; i < kHeadsPerCta * R; i += kThreads) q_lat[i] = (i / R < nh) ? Conv<T>::to_f(qlb[i]) : 0.f;
  for (int i = tid; i < kHeadsPerCta * P; i += kThreads) q_pe[i] = (i / P < nh) ? Conv<T>::to_f(qpb[i]) : 0.f;
  if (tid < kHeadsPerCta) {
    m_sh[tid] = -INFINITY;
    l_sh[tid] = 0.f;
  }
  __syncthreads();
  const int count = s_count;
  if (count == 0) {
    // nothing to attend (empty sequence, no sink/window/selection): zeros, like a softmax over no keys
    if (s == 0) {
      const DecodeParams& dz = p.dp;
      for (int i = tid; i < nh * R; i += kThreads) {
        T* o = reinterpret_cast<T*>(dz.out) + (int64_t)b * dz.out_stride_seq + (int64_t)(h0 + i / R) * dz.out_stride_head;
        o[i % R] = Conv<T>::from_f(0.f);
      }
    }
    return;
  }
  const int per = (count + p.n_splits - 1) / p.n_splits;
  const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);

  // output accumulators: thread -> head (tid / 16), dims [dslice, dslice + R/16)
  const int oh = tid / 16;
  const int dsl = (tid % 16) * (R / 16);
  float acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  const int nd = R / 16;  // <= 32

  for (int li = c_lo; li < c_hi; ++li) {
    const int c = list[li];
    const int32_t phys = (c < p.table_width) ? p.tables[(int64_t)b * p.table_stride + c] : -1;
    if ((phys < 0 || phys >= p.num_blocks) && tid == 0) flag_error(p.dp.err, SNAPMIND_DEVERR_BLOCK_ID);
    __syncthreads();
    const bool ok = phys >= 0 && phys < p.num_blocks;
    if (ok) {
      const uint4* srcc = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.latent) + (int64_t)phys * bs * R);
      const uint4* srcp = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.rope) + (int64_t)phys * bs * P);
      uint4* dc = reinterpret_cast<uint4*>(tile_c);
      uint4* dp = reinterpret_cast<uint4*>(tile_p);
      const int nc = bs * R * (int)sizeof(T) / 16, np_ = bs * P * (int)sizeof(T) / 16;
      for (int i = tid; i < nc; i += kThreads) dc[i] = srcc[i];
      for (int i = tid; i < np_; i += kThreads) dp[i] = srcp[i];
    }
    __syncthreads();
    const bool selected = (sel_bits[c >> 5] >> (c & 31)) & 1u;
    // scores: thread -> row r, heads hq*4 .. +3 (bs * 4 groups of 4 heads = 4 * bs threads)
    for (int task = tid; task < bs * 4; task += kThreads) {
      const int r = task % bs, hq = task / bs;
      const int pos = c * bs + r;
      const bool valid = ok && pos < len && (selected || pos < sink || pos >= wstart);
      float d4[4] = {0.f, 0.f, 0.f, 0.f};
      if (valid) {
        const T* crow = tile_c + (size_t)r * R;
        const T* prow = tile_p + (size_t)r * P;
        for (int j = 0; j < R; ++j) {
          const int col = (j + r) % R;
          const float x = Conv<T>::to_f(crow[col]);
#pragma unroll
          for (int u = 0; u < 4; ++u) d4[u] = fmaf(q_lat[(hq * 4 + u) * R + col], x, d4[u]);
        }
        for (int j = 0; j < P; ++j) {
          const int col = (j + r) % P;
          const float x = Conv<T>::to_f(prow[col]);
#pragma unroll
          for (int u = 0; u < 4; ++u) d4[u] = fmaf(q_pe[(hq * 4 + u) * P + col], x, d4[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) S[(hq * 4 + u) * bs + r] = valid ? d4[u] * p.scale : -INFINITY;
    }
    __syncthreads();
    // online softmax: warp w handles heads 2w, 2w+1
    for (int hh = warp * 2; hh < warp * 2 + 2; ++hh) {
      float mt = -INFINITY;
      for (int r = lane; r < bs; r += 32) mt = fmaxf(mt, S[hh * bs + r]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_old = m_sh[hh];
      const float m_new = fmaxf(m_old, mt);
      float sum = 0.f;
      for (int r = lane; r < bs; r += 32) {
        const float e = (m_new == -INFINITY) ? 0.f : expf(S[hh * bs + r] - m_new);
        S[hh * bs + r] = e;
        sum += e;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float al = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        al_sh[hh] = al;
        l_sh[hh] = l_sh[hh] * al + sum;
        m_sh[hh] = m_new;
      }
    }
    __syncthreads();
    // latent accumulation
    const float al = al_sh[oh];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] *= al;
    for (int r = 0; r < bs; ++r) {
      const float pr = S[oh * bs + r];
      if (pr == 0.f) continue;
      const T* crow = tile_c + (size_t)r * R + dsl;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nd) acc[i] = fmaf(pr, Conv<T>::to_f(crow[i]), acc[i]);
    }
    __syncthreads();
  }

  // partial of this split -> output or workspace, then the last-ticket merge
  const DecodeParams& dp = p.dp;
  const bool direct = (p.n_splits == 1);
  const float M = m_sh[oh], L = l_sh[oh];
  if (oh < nh) {
    if (direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)(h0 + oh) * dp.out_stride_head;
      for (int i = 0; i < nd; ++i) o[dsl + i] = Conv<T>::from_f(L > 0.f ? acc[i] / L : 0.f);
    } else {
      float* part = dp.partials + (((int64_t)b * dp.n_q_heads + h0 + oh) * dp.max_splits + s) * (R + 2);
      for (int i = 0; i < nd; ++i) part[2 + dsl + i] = acc[i];
      if (tid % 16 == 0) {
        part[0] = M;
        part[1] = L;
      }
    }
  }
  if (direct) return;
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(&dp.counters[b * dp.n_kv_heads + hg], 1);
    s_last = (ticket == p.n_splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  combine_splits<T>(dp, b, hg, p.n_splits, smem);
  if (tid == 0) dp.counters[b * dp.n_kv_heads + hg] = 0;
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int32_t snapmind_sparse_mla_default_splits(int32_t batch, int32_t n_heads, int32_t kv_lora_rank, int32_t rope_dim,
                                           int32_t block_size, int32_t dtype) {
  if (batch <= 0 || n_heads <= 0) return 1;
  if ((dtype == SNAPMIND_DTYPE_BF16 || dtype == SNAPMIND_DTYPE_F16) && n_heads == 128 && kv_lora_rank == 512 &&
      rope_dim == 64 && block_size == 64)
    return sparse_mla_umma_splits(batch);  // (split, output half) CTAs fill the SMs once
  const int groups = (n_heads + 31) / 32;
  const int per_seq = num_sms() / (groups * batch);
  return per_seq < 1 ? 1 : (per_seq > 64 ? 64 : per_seq);
}

int64_t snapmind_sparse_mla_workspace_bytes(int32_t batch, int32_t n_heads, int32_t kv_lora_rank, int32_t n_splits) {
  if (batch <= 0 || n_heads <= 0 || kv_lora_rank <= 0 || n_splits <= 0) return 0;
  const int groups = (n_heads + kHeadsPerCta - 1) / kHeadsPerCta;
  return workspace_layout(batch, n_heads, groups, kv_lora_rank, n_splits).total;
}

int snapmind_sparse_mla_decode(const void* q_lat, const void* q_pe, int dtype, const void* latent_pool,
                               const void* rope_pool, const int32_t* block_tables, int64_t table_stride,
                               int32_t table_width, const int32_t* seq_lens, const int32_t* selected, int32_t k,
                               int32_t sink, int32_t window, float scale, int32_t batch, int32_t n_heads,
                               int32_t kv_lora_rank, int32_t rope_dim, int32_t block_size, int32_t num_blocks,
                               int32_t n_splits, void* out, void* workspace, int64_t workspace_bytes,
                               int32_t* err_word, void* stream) {
  const int esz = dtype_size(dtype);
  SNAPMIND_CHECK_ARG(esz > 0, "sparse_mla_decode: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && batch <= 65535 && n_heads > 0 && k >= 0 && sink >= 0 && window >= 0 &&
                         n_splits >= 1 && n_splits <= 64 && block_size > 0 && block_size <= 128,
                     "sparse_mla_decode: bad sizes");
  SNAPMIND_CHECK_ARG(kv_lora_rank % 16 == 0 && kv_lora_rank <= 512 && rope_dim > 0 && rope_dim <= 256,
                     "sparse_mla_decode: kv_lora_rank must be a multiple of 16 up to 512, rope_dim <= 256");
  SNAPMIND_CHECK_ARG(((int64_t)block_size * kv_lora_rank * esz) % 16 == 0 &&
                         ((int64_t)block_size * rope_dim * esz) % 16 == 0,
                     "sparse_mla_decode: block rows must fill 16-byte vectors");
  SNAPMIND_CHECK_ARG(table_width <= kMaxChunkBits, "sparse_mla_decode: at most %d chunks per sequence",
                     kMaxChunkBits);
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(q_lat && q_pe && latent_pool && rope_pool && block_tables && seq_lens && out &&
                         (k == 0 || selected),
                     "sparse_mla_decode: null pointer");
  SNAPMIND_CHECK_ARG((reinterpret_cast<uintptr_t>(latent_pool) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(rope_pool) & 15) == 0,
                     "sparse_mla_decode: pools must be 16-byte aligned");
  const int groups = (n_heads + kHeadsPerCta - 1) / kHeadsPerCta;
  const WorkspaceLayout ws = workspace_layout(batch, n_heads, groups, kv_lora_rank, n_splits);
  SNAPMIND_CHECK_ARG(n_splits == 1 || (workspace && workspace_bytes >= ws.total),
                     "sparse_mla_decode: workspace needs %lld bytes", (long long)ws.total);
  SparseParams p;
  p.q_lat = q_lat;
  p.q_pe = q_pe;
  p.latent = latent_pool;
  p.rope = rope_pool;
  p.tables = block_tables;
  p.table_stride = table_stride;
  p.table_width = table_width;
  p.seq_lens = seq_lens;
  p.selected = selected;
  p.k = k;
  p.sink = sink;
  p.window = window;
  p.scale = scale;
  p.batch = batch;
  p.n_heads = n_heads;
  p.R = kv_lora_rank;
  p.P = rope_dim;
  p.bs = block_size;
  p.num_blocks = num_blocks;
  p.n_splits = n_splits;
  DecodeParams& dp = p.dp;
  dp = DecodeParams{};
  dp.out = out;
  dp.out_stride_seq = (int64_t)n_heads * kv_lora_rank;
  dp.out_stride_head = kv_lora_rank;
  dp.batch = batch;
  dp.n_q_heads = n_heads;
  dp.n_kv_heads = groups;
  dp.group = kHeadsPerCta;
  dp.head_dim = kv_lora_rank;
  dp.max_splits = n_splits;
  dp.counters = workspace ? reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + ws.counters_off) : nullptr;
  dp.partials = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + ws.partials_off) : nullptr;
  dp.err = err_word;
  SNAPMIND_CHECK_ARG(n_heads % kHeadsPerCta == 0, "sparse_mla_decode: n_heads must be a multiple of %d",
                     kHeadsPerCta);
  const size_t smem = sizeof(float) * (kHeadsPerCta * (kv_lora_rank + rope_dim + block_size) + 3 * kHeadsPerCta) +
                      sizeof(uint32_t) * 2 * (kMaxChunkBits / 32) + sizeof(int32_t) * kMaxChunkBits +
                      (size_t)block_size * (kv_lora_rank + rope_dim) * esz + 16;
  SNAPMIND_CHECK_ARG(smem <= 227 * 1024, "sparse_mla_decode: shared memory %zu exceeds the limit", smem);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (sparse_mla_umma_supported(p, dtype)) return launch_sparse_mla_umma(p, dtype, st);
  if (sparse_mla_tc_supported(p, dtype)) return launch_sparse_mla_tc(p, dtype, st);
  dim3 grid(n_splits, groups, batch);
  auto go = [&](auto kernel) -> int {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "sparse_mla smem attribute");
    kernel<<<grid, kThreads, smem, st>>>(p);
    return cuda_status(cudaGetLastError(), "sparse_mla launch");
  };
  switch (dtype) {
    case SNAPMIND_DTYPE_F32: return go(sparse_mla_kernel<float>);
    case SNAPMIND_DTYPE_BF16: return go(sparse_mla_kernel<__nv_bfloat16>);
    default: return go(sparse_mla_kernel<__half>);
  }
}

}  // extern "C"
