// Shared declarations of the paged GQA decode kernels.
#pragma once

#include "common.cuh"

namespace snapmind {

struct DecodeParams {
  const void* q;
  int64_t q_stride_seq, q_stride_head;  // elements
  const void* k_pool;
  const void* v_pool;
  const int32_t* tables;
  int64_t table_stride;
  int32_t table_width;
  const int32_t* seq_lens;
  const int32_t* seq_start = nullptr;  // per sequence: first attended token (NULL: 0)
  void* out;
  int64_t out_stride_seq, out_stride_head;  // elements
  float scale;
  int32_t batch, n_q_heads, n_kv_heads, group, head_dim, block_size, num_blocks;
  int32_t split_tokens, max_splits;
  int32_t* counters;  // [batch][n_kv_heads] tickets, zero between calls
  float* partials;    // [batch][n_q_heads][max_splits][head_dim + 2]: m, l, acc[head_dim]
  int32_t* err;
  // outputs written straight into the output buffers of several GPUs (peer stores);
  // n_peers = 0: the local `out` only
  void* const* peer_out = nullptr;       // [n_peers] output bases, rank order (own buffer included)
  int32_t n_peers = 0, head_offset = 0;  // q heads of this launch start at head_offset globally
  // the token at position seq_lens[b] - 1 of every sequence, [batch][n_kv_heads][head_dim] in
  // the pool's dtype, stored into the pool by the decode itself before it attends (NULL: none)
  const void* new_k = nullptr;
  const void* new_v = nullptr;
  int64_t new_stride_seq = 0, new_stride_head = 0;  // elements
};

// Destinations of a decode whose outputs go straight to several GPUs.
struct PeerArgs {
  void* const* out;  // device array [n]: output base on each rank (16-byte aligned)
  int32_t n, head_offset;
};

// One output element of (sequence b, q head `head` of this launch) to `out`.
template <typename T>
__device__ __forceinline__ void store_out(const DecodeParams& p, int b, int head, int d, float v) {
  reinterpret_cast<T*>(p.out)[(int64_t)b * p.out_stride_seq + (int64_t)head * p.out_stride_head + d] =
      Conv<T>::from_f(v);
}

__device__ __forceinline__ uint32_t bits16(__nv_bfloat16 x) { return __bfloat16_as_ushort(x); }
__device__ __forceinline__ uint32_t bits16(__half x) { return __half_as_ushort(x); }

// The output rows of heads [head0, head0 + G) of sequence b, value(g, d) each,
// stored into every GPU's output buffer at the global head: 16-byte stores
// (whole vectors cross NVLink), every peer in turn.  head_dim and the output
// strides are multiples of 16 bytes (checked by the host).
template <typename T, typename F>
__device__ __forceinline__ void emit_peer_rows(const DecodeParams& p, int b, int head0, int G, int D, F value) {
  constexpr int V = 16 / sizeof(T);
  const int per_row = D / V;
  for (int e = threadIdx.x; e < G * per_row; e += blockDim.x) {
    const int g = e / per_row, d0 = (e - g * per_row) * V;
    uint32_t w[4];
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = __float_as_uint(value(g, d0 + j));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = bits16(Conv<T>::from_f(value(g, d0 + 2 * j))) | (bits16(Conv<T>::from_f(value(g, d0 + 2 * j + 1))) << 16);
    }
    const uint4 v = make_uint4(w[0], w[1], w[2], w[3]);
    const int64_t off = (int64_t)b * p.out_stride_seq + (int64_t)(head0 + g + p.head_offset) * p.out_stride_head + d0;
    for (int r = 0; r < p.n_peers; ++r) *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.peer_out[r]) + off) = v;
  }
}

struct WorkspaceLayout {
  int64_t counters_off, partials_off, total;
};

inline WorkspaceLayout workspace_layout(int batch, int n_q_heads, int n_kv_heads, int head_dim,
                                        int max_splits) {
  WorkspaceLayout w;
  w.counters_off = 0;
  const int64_t counters = (int64_t)batch * n_kv_heads * sizeof(int32_t);
  w.partials_off = (counters + 255) / 256 * 256;
  w.total = w.partials_off +
            (int64_t)batch * n_q_heads * max_splits * (head_dim + 2) * (int64_t)sizeof(float);
  return w;
}

// Tokens per split: about 16 CTAs per SM over the batch at a mean length of
// max_seq_len / 2, at least 512 tokens (8 pipeline tiles, so the fill and the
// per-CTA merge stay small next to the streaming), rounded to whole 64-token
// tiles (and whole blocks).
inline int default_split_tokens(int batch, int n_kv_heads, int max_seq_len, int block_size) {
  if (block_size <= 0) return 0;
  const int64_t work = (int64_t)(batch > 0 ? batch : 1) * (n_kv_heads > 0 ? n_kv_heads : 1) *
                       (max_seq_len > 0 ? max_seq_len : 1) / 2;
  const int64_t target = (int64_t)num_sms() * 16;
  int64_t split = (work + target - 1) / target;
  int64_t unit = block_size;
  if (64 % block_size == 0) unit = 64;
  // splits of at least 512 tokens keep the TMA pipeline full; a small problem (fewer
  // than about two CTAs per SM at 512) takes shorter splits, down to one 64-token tile
  const int64_t rows = (int64_t)(batch > 0 ? batch : 1) * (n_kv_heads > 0 ? n_kv_heads : 1);
  const int64_t ctas_512 = rows * (((max_seq_len > 0 ? max_seq_len : 1) + 511) / 512);
  const int64_t min_split = ctas_512 < 2 * (int64_t)num_sms() ? unit : 512;
  if (split < min_split) split = min_split;
  if (split > 8192) split = 8192;
  split = (split + unit - 1) / unit * unit;
  return (int)split;
}

inline size_t combine_smem_bytes(const DecodeParams& p) { return sizeof(float) * 2 * p.group; }

// Merge the per-split (m, l, acc) partial states of (b, kv head) into the
// output: M = max m_s, L = sum l_s e^(m_s - M), out = sum acc_s e^(m_s - M) / L.
// Partials written by other CTAs are read with L1-bypassing loads.
template <typename T>
__device__ void combine_splits(const DecodeParams& p, int b, int kvh, int n_splits, float* sm) {
  const int G = p.group, D = p.head_dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float* s_M = sm;
  float* s_L = sm + G;
  const int64_t pstride = D + 2;
  const float* base = p.partials + ((int64_t)b * p.n_q_heads + kvh * G) * p.max_splits * pstride;
  __syncthreads();
  for (int g = warp; g < G; g += nw) {
    const float* pg = base + (int64_t)g * p.max_splits * pstride;
    float M = -INFINITY;
    for (int s = lane; s < n_splits; s += 32) M = fmaxf(M, __ldcg(pg + s * pstride));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    for (int s = lane; s < n_splits; s += 32)
      L += __ldcg(pg + s * pstride + 1) * expf(__ldcg(pg + s * pstride) - M);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) {
      s_M[g] = M;
      s_L[g] = L;
    }
  }
  __syncthreads();
  auto value = [&](int g, int d) {
    const float* pg = base + (int64_t)g * p.max_splits * pstride;
    const float M = s_M[g];
    float A = 0.f;
    for (int s = 0; s < n_splits; ++s)
      A += __ldcg(pg + s * pstride + 2 + d) * expf(__ldcg(pg + s * pstride) - M);
    return A / s_L[g];
  };
  if (p.n_peers > 0) {
    emit_peer_rows<T>(p, b, kvh * G, G, D, value);
    return;
  }
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    store_out<T>(p, b, kvh * G + g, d, value(g, d));
  }
}

// Tensor-core path (paged_decode_fast.cu).
bool decode_fast_supported(const DecodeParams& p, int dtype);
int launch_decode_fast(const DecodeParams& p, int dtype, cudaStream_t stream);

}  // namespace snapmind
