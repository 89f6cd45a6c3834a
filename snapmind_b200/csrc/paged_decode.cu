// Paged GQA decode attention (split-K flash decoding) for sm_100a.
//
// Math: for each sequence b and query head h (kv head h / G, G = Hq / H),
//     out[b, h] = softmax(q[b, h] . K[b, kv]^T * scale) V[b, kv]
// over the seq_lens[b] tokens reached through the block table — the
// repeat_interleave / matmul / softmax / matmul sequence of
// GroupedQueryAttention.forward (snapmind/layers/attention/gqa.py:69-82)
// applied to what PagedKVCache.fetch (snapmind/kv_cache/paged.py:56-78) would
// return, without materialising either.
//
// Work split: CTA (split s, kv head, sequence b) covers tokens
// [s*split_tokens, (s+1)*split_tokens).  Every CTA keeps an online-softmax
// state (m, l, acc) per query head of its group; a sequence with one split
// writes the output directly, otherwise each CTA stores its partial state in
// the workspace and the CTA that takes the last ticket of the (b, kv head)
// counter merges the partials and resets the counter (no CTA ever waits).
#include <cfloat>

#include "common.cuh"
#include "paged_decode.cuh"

namespace snapmind {

// ---------------------------------------------------------------------------
// generic CUDA-core kernel: any head_dim <= 256, group sizes up to 32 (16 for
// head_dim > 64, 8 for head_dim > 128); fp32, bf16 and f16 pools.
//
// Each warp takes 32-token tiles of its split (flash-decoding on CUDA cores):
//   * scores: lane = token; the lane reads its key row (16-byte loads when
//     aligned) against q in shared memory (broadcast reads), all query heads
//     of the group at once;
//   * online softmax: one warp max and one warp sum per head per tile;
//   * P V: lane = dims; P is broadcast from shared memory and each valid
//     token's value row is read coalesced.
// Warps merge in shared memory; splits merge through the last-ticket combine.
// ---------------------------------------------------------------------------
constexpr int kGenericWarps = 8;
constexpr int kTileTok = 32;

__device__ __forceinline__ float4 load4_as_f(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <typename T>
__device__ __forceinline__ float4 load4_as_f(const T* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const T* t = reinterpret_cast<const T*>(&u);
  return make_float4(Conv<T>::to_f(t[0]), Conv<T>::to_f(t[1]), Conv<T>::to_f(t[2]), Conv<T>::to_f(t[3]));
}

template <int GMAX, int NI>
constexpr int generic_smem_floats(int head_dim) {
  return GMAX * 32 * NI + kGenericWarps * kTileTok * GMAX + 2 * kGenericWarps * GMAX +
         kGenericWarps * GMAX * head_dim;
}

template <typename T, int NI, int GMAX>
__global__ void __launch_bounds__(kGenericWarps * 32, (GMAX <= 8 && NI <= 2) ? 2 : 1)
    paged_decode_generic_kernel(DecodeParams p) {
  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.group;
  const int D = p.head_dim;
  constexpr int DP = 32 * NI;  // padded head_dim of the q copy

  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  const int skip = p.seq_start ? max(0, p.seq_start[b]) : 0;  // tokens before the window start
  int n_splits = (len + p.split_tokens - 1) / p.split_tokens;
  if (n_splits > p.max_splits) {
    if (s == 0 && threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_SPLIT);
    n_splits = p.max_splits;
    len = p.max_splits * p.split_tokens;
  }
  if (len <= skip) {
    // softmax over zero keys: the reference's matmul over an empty dim gives 0
    if (s == 0) {
      if (p.n_peers > 0) {
        emit_peer_rows<T>(p, b, kvh * G, G, D, [](int, int) { return 0.f; });
      } else {
        for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
          const int g = e / D, d = e - g * D;
          store_out<T>(p, b, kvh * G + g, d, 0.f);
        }
      }
    }
    return;
  }
  if (s >= n_splits) return;
  const int t0 = s * p.split_tokens;
  const int t1 = min(len, t0 + p.split_tokens);

  // smem: [q: GMAX x DP][P: warps x 32 tokens x GMAX][merge: m, l, acc]
  extern __shared__ __align__(16) float sm[];
  float* q_s = sm;
  float* p_s = q_s + GMAX * DP;
  float* mrg = p_s + kGenericWarps * kTileTok * GMAX;

  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_stride_seq;
  for (int e = threadIdx.x; e < GMAX * DP; e += blockDim.x) {
    const int g = e / DP, d = e - g * DP;
    q_s[e] = (g < G && d < D) ? Conv<T>::to_f(qb[(int64_t)(kvh * G + g) * p.q_stride_head + d]) : 0.f;
  }
  __syncthreads();

  float m[GMAX], l[GMAX], acc[GMAX][NI];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < NI; ++i) acc[g][i] = 0.f;
  }

  const T* kpool = reinterpret_cast<const T*>(p.k_pool);
  const T* vpool = reinterpret_cast<const T*>(p.v_pool);
  const int32_t* table = p.tables + (int64_t)b * p.table_stride;
  const bool vec = (D % 4 == 0) && (reinterpret_cast<uintptr_t>(kpool) % (4 * sizeof(T)) == 0);
  float* pw = p_s + warp * kTileTok * GMAX;  // this warp's P tile [token][GMAX]

  for (int tile = t0 + warp * kTileTok; tile < t1; tile += kGenericWarps * kTileTok) {
    // ---- scores: lane = token
    const int t = tile + lane;
    bool valid = t < t1 && t >= skip;
    int64_t row = 0;
    if (valid) {
      const int j = t / p.block_size;
      const int off = t - j * p.block_size;
      const int32_t phys = j < p.table_width ? table[j] : -1;
      if (phys < 0 || phys >= p.num_blocks) {
        flag_error(p.err, j < p.table_width ? SNAPMIND_DEVERR_BLOCK_ID : SNAPMIND_DEVERR_TABLE);
        valid = false;
      } else {
        row = (((int64_t)phys * p.n_kv_heads + kvh) * p.block_size + off) * D;
      }
    }
    float sc[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g) sc[g] = 0.f;
    if (valid) {
      const T* kr = kpool + row;
      if (vec) {
        // kKv vector loads per round are issued before any of them is used
        constexpr int kKv = GMAX >= 32 ? 4 : 8;
        for (int d0 = 0; d0 < D; d0 += 4 * kKv) {
          float4 kv[kKv];
#pragma unroll
          for (int j = 0; j < kKv; ++j)
            kv[j] = d0 + 4 * j < D ? load4_as_f(kr + d0 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int j = 0; j < kKv; ++j) {
            if (d0 + 4 * j >= D) break;
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
              const float4 qv = *reinterpret_cast<const float4*>(q_s + g * DP + d0 + 4 * j);
              sc[g] = fmaf(qv.x, kv[j].x, sc[g]);
              sc[g] = fmaf(qv.y, kv[j].y, sc[g]);
              sc[g] = fmaf(qv.z, kv[j].z, sc[g]);
              sc[g] = fmaf(qv.w, kv[j].w, sc[g]);
            }
          }
        }
      } else {
        for (int d = 0; d < D; ++d) {
          const float kv = Conv<T>::to_f(kr[d]);
#pragma unroll
          for (int g = 0; g < GMAX; ++g) sc[g] = fmaf(q_s[g * DP + d], kv, sc[g]);
        }
      }
    }
    // ---- online softmax over the tile, per head
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      const float x = valid ? sc[g] * p.scale : -INFINITY;
      float tm = x;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
      const float m_new = fmaxf(m[g], tm);
      float corr = 1.f, pe = 0.f;
      if (m_new != -INFINITY) {
        corr = (m[g] == -INFINITY) ? 0.f : expf(m[g] - m_new);
        pe = valid ? expf(x - m_new) : 0.f;
      }
      float ps = pe;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[g] = l[g] * corr + ps;
#pragma unroll
      for (int i = 0; i < NI; ++i) acc[g][i] *= corr;
      m[g] = m_new;
      pw[lane * GMAX + g] = pe;
    }
    __syncwarp();
    // ---- P V: lane = dims
    const unsigned vmask = __ballot_sync(0xffffffffu, valid);
    constexpr int kPvUnroll = (NI <= 2 && GMAX < 32) ? 8 : 4;  // value rows in flight
#pragma unroll kPvUnroll
    for (int jt = 0; jt < kTileTok; ++jt) {
      const int64_t rj = __shfl_sync(0xffffffffu, row, jt);
      if (!((vmask >> jt) & 1u)) continue;
      const T* vr = vpool + rj;
      float vf[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int d = lane + 32 * i;
        vf[i] = d < D ? Conv<T>::to_f(vr[d]) : 0.f;
      }
      const float* pj = pw + jt * GMAX;
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        const float pg = pj[g];
#pragma unroll
        for (int i = 0; i < NI; ++i) acc[g][i] = fmaf(pg, vf[i], acc[g][i]);
      }
    }
    __syncwarp();  // the P tile is rewritten next iteration
  }

  // ---- merge the warps of this CTA ------------------------------------------
  float* sm_m = mrg;                                  // [warps][GMAX]
  float* sm_l = mrg + kGenericWarps * GMAX;           // [warps][GMAX]
  float* sm_acc = mrg + 2 * kGenericWarps * GMAX;     // [warps][GMAX][D]
  __shared__ int s_last;
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      sm_m[warp * GMAX + g] = m[g];
      sm_l[warp * GMAX + g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int d = lane + 32 * i;
      if (g < G && d < D) sm_acc[(warp * GMAX + g) * D + d] = acc[g][i];
    }
  }
  __syncthreads();

  const bool direct = (n_splits == 1);
  if (direct && p.n_peers > 0) {
    emit_peer_rows<T>(p, b, kvh * G, G, D, [&](int g, int d) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kGenericWarps; ++w) M = fmaxf(M, sm_m[w * GMAX + g]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < kGenericWarps; ++w) {
        const float mw = sm_m[w * GMAX + g];
        const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
        L += sm_l[w * GMAX + g] * f;
        A += sm_acc[(w * GMAX + g) * D + d] * f;
      }
      return A / L;
    });
    return;
  }
  float* part_base = p.partials + ((int64_t)b * p.n_q_heads + kvh * G) * p.max_splits * (D + 2);
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kGenericWarps; ++w) M = fmaxf(M, sm_m[w * GMAX + g]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kGenericWarps; ++w) {
      const float mw = sm_m[w * GMAX + g];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      L += sm_l[w * GMAX + g] * f;
      A += sm_acc[(w * GMAX + g) * D + d] * f;
    }
    if (direct) {
      store_out<T>(p, b, kvh * G + g, d, A / L);
    } else {
      float* part = part_base + ((int64_t)g * p.max_splits + s) * (D + 2);
      part[2 + d] = A;
      if (d == 0) {
        part[0] = M;
        part[1] = L;
      }
    }
  }
  if (direct) return;

  // ---- last-ticket merge of the split partials --------------------------------
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&p.counters[b * p.n_kv_heads + kvh], 1);
    s_last = (ticket == n_splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  combine_splits<T>(p, b, kvh, n_splits, sm);
  if (threadIdx.x == 0) p.counters[b * p.n_kv_heads + kvh] = 0;
}

template <typename T, int NI>
static int launch_generic_g(const DecodeParams& p, dim3 grid, cudaStream_t st) {
  auto go = [&](auto kernel, int gmax) -> int {
    size_t smem = sizeof(float) * ((size_t)gmax * 32 * NI + (size_t)kGenericWarps * kTileTok * gmax +
                                   2 * (size_t)kGenericWarps * gmax + (size_t)kGenericWarps * gmax * p.head_dim);
    const size_t comb = combine_smem_bytes(p);
    if (comb > smem) smem = comb;
    if (smem > 48 * 1024) {
      cudaError_t e =
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "paged_decode smem attribute");
    }
    kernel<<<grid, kGenericWarps * 32, smem, st>>>(p);
    return cuda_status(cudaGetLastError(), "paged_decode_generic launch");
  };
  if (p.group <= 1) return go(paged_decode_generic_kernel<T, NI, 1>, 1);
  if (p.group <= 2) return go(paged_decode_generic_kernel<T, NI, 2>, 2);
  if (p.group <= 4) return go(paged_decode_generic_kernel<T, NI, 4>, 4);
  if (p.group <= 8) return go(paged_decode_generic_kernel<T, NI, 8>, 8);
  if constexpr (NI <= 4) {
    if (p.group <= 16) return go(paged_decode_generic_kernel<T, NI, 16>, 16);
  }
  if constexpr (NI <= 2) {
    if (p.group <= 32) return go(paged_decode_generic_kernel<T, NI, 32>, 32);
  }
  set_last_error("paged_decode: group size %d with head_dim %d unsupported", p.group, p.head_dim);
  return SNAPMIND_ERR_UNSUPPORTED;
}

template <typename T>
static int launch_generic(const DecodeParams& p, dim3 grid, cudaStream_t st) {
  if (p.head_dim <= 32) return launch_generic_g<T, 1>(p, grid, st);
  if (p.head_dim <= 64) return launch_generic_g<T, 2>(p, grid, st);
  if (p.head_dim <= 128) return launch_generic_g<T, 4>(p, grid, st);
  return launch_generic_g<T, 8>(p, grid, st);
}

}  // namespace snapmind

using namespace snapmind;

extern "C" {

int32_t snapmind_paged_gqa_decode_split_tokens(int32_t batch, int32_t n_kv_heads,
                                               int32_t max_seq_len, int32_t block_size) {
  return default_split_tokens(batch, n_kv_heads, max_seq_len, block_size);
}

int64_t snapmind_paged_gqa_decode_workspace_bytes(int32_t batch, int32_t n_q_heads,
                                                  int32_t n_kv_heads, int32_t head_dim,
                                                  int32_t max_seq_len, int32_t split_tokens) {
  if (batch <= 0 || n_q_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || split_tokens <= 0)
    return 0;
  const int64_t max_splits = ((int64_t)(max_seq_len > 0 ? max_seq_len : 1) + split_tokens - 1) / split_tokens;
  return workspace_layout(batch, n_q_heads, n_kv_heads, head_dim, (int)max_splits).total;
}

}  // extern "C"

static int decode_entry(const void* q, int64_t q_stride_seq, int64_t q_stride_head, const void* k_pool,
                        const void* v_pool, int dtype, const int32_t* block_tables, int64_t table_stride_seq,
                        int32_t table_width, const int32_t* seq_lens, const int32_t* seq_starts, void* out,
                        int64_t out_stride_seq, int64_t out_stride_head, float scale, int32_t batch,
                        int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                        int32_t num_blocks, int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                        void* workspace, int64_t workspace_bytes, int32_t* err_word, void* stream,
                        const PeerArgs* peers = nullptr, const void* new_k = nullptr,
                        const void* new_v = nullptr, int64_t new_stride_seq = 0, int64_t new_stride_head = 0) {
  SNAPMIND_CHECK_ARG(dtype_size(dtype) > 0, "paged_decode: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && n_q_heads > 0 && n_kv_heads > 0 && head_dim > 0 &&
                         head_dim <= 256 && block_size > 0 && num_blocks > 0 && table_width >= 0,
                     "paged_decode: bad sizes");
  SNAPMIND_CHECK_ARG(n_q_heads % n_kv_heads == 0,
                     "paged_decode: n_q_heads (%d) must be a multiple of n_kv_heads (%d)",
                     n_q_heads, n_kv_heads);
  if (peers) {
    const int vec = 16 / dtype_size(dtype);  // elements per 16-byte peer store
    SNAPMIND_CHECK_ARG(peers->out && peers->n >= 1 && peers->head_offset >= 0,
                       "paged_decode_peers: bad peer arguments");
    SNAPMIND_CHECK_ARG(head_dim % vec == 0 && out_stride_seq % vec == 0 && out_stride_head % vec == 0,
                       "paged_decode_peers: head_dim and output strides must be multiples of 16 bytes");
  }
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(q && k_pool && v_pool && block_tables && seq_lens && (out || peers),
                     "paged_decode: null pointer");
  if (max_seq_len <= 0) max_seq_len = table_width * block_size;
  if (split_tokens <= 0)
    split_tokens = default_split_tokens(batch, n_kv_heads, max_seq_len, block_size);
  SNAPMIND_CHECK_ARG(split_tokens % block_size == 0,
                     "paged_decode: split_tokens (%d) must be a multiple of block_size (%d)",
                     split_tokens, block_size);
  const int max_splits = (max_seq_len + split_tokens - 1) / split_tokens;
  const WorkspaceLayout ws =
      workspace_layout(batch, n_q_heads, n_kv_heads, head_dim, max_splits > 0 ? max_splits : 1);
  SNAPMIND_CHECK_ARG(workspace != nullptr && workspace_bytes >= ws.total,
                     "paged_decode: workspace needs %lld bytes, got %lld", (long long)ws.total,
                     (long long)workspace_bytes);

  DecodeParams p;
  p.q = q;
  p.q_stride_seq = q_stride_seq;
  p.q_stride_head = q_stride_head;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.tables = block_tables;
  p.table_stride = table_stride_seq;
  p.table_width = table_width;
  p.seq_lens = seq_lens;
  p.seq_start = seq_starts;
  p.out = out;
  p.out_stride_seq = out_stride_seq;
  p.out_stride_head = out_stride_head;
  p.scale = scale;
  p.batch = batch;
  p.n_q_heads = n_q_heads;
  p.n_kv_heads = n_kv_heads;
  p.group = n_q_heads / n_kv_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.split_tokens = split_tokens;
  p.max_splits = max_splits > 0 ? max_splits : 1;
  p.counters = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + ws.counters_off);
  p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + ws.partials_off);
  p.err = err_word;
  if (peers) {
    p.peer_out = peers->out;
    p.n_peers = peers->n;
    p.head_offset = peers->head_offset;
  }
  p.new_k = new_k;
  p.new_v = new_v;
  p.new_stride_seq = new_stride_seq;
  p.new_stride_head = new_stride_head;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (!(flags & SNAPMIND_DECODE_FORCE_GENERIC)) {
    int rc = SNAPMIND_ERR_UNSUPPORTED;
    if (decode_fast_supported(p, dtype)) rc = launch_decode_fast(p, dtype, st);
    if (rc != SNAPMIND_ERR_UNSUPPORTED) return rc;
  }
  if (new_k != nullptr) {
    // the CUDA-core kernel attends only: store the token with the append kernel first
    const int rc = snapmind_kv_append(const_cast<void*>(k_pool), const_cast<void*>(v_pool), dtype, 0, new_k, new_v,
                                      dtype, 0, new_stride_seq, new_stride_head, 0, block_tables, table_stride_seq,
                                      0, table_width, seq_lens, -1, 1, batch, 1, n_kv_heads, head_dim, block_size,
                                      num_blocks, err_word, stream);
    if (rc != SNAPMIND_OK) return rc;
    p.new_k = p.new_v = nullptr;
  }
  dim3 grid(p.max_splits, n_kv_heads, batch);
  SNAPMIND_CHECK_ARG(grid.y <= 65535 && grid.z <= 65535, "paged_decode: grid too large");
  switch (dtype) {
    case SNAPMIND_DTYPE_F32: return launch_generic<float>(p, grid, st);
    case SNAPMIND_DTYPE_BF16: return launch_generic<__nv_bfloat16>(p, grid, st);
    default: return launch_generic<__half>(p, grid, st);
  }
}

extern "C" {

int snapmind_paged_gqa_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                              const void* k_pool, const void* v_pool, int dtype,
                              const int32_t* block_tables, int64_t table_stride_seq,
                              int32_t table_width, const int32_t* seq_lens, void* out,
                              int64_t out_stride_seq, int64_t out_stride_head, float scale,
                              int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t block_size, int32_t num_blocks,
                              int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                              void* workspace, int64_t workspace_bytes, int32_t* err_word,
                              void* stream) {
  return decode_entry(q, q_stride_seq, q_stride_head, k_pool, v_pool, dtype, block_tables, table_stride_seq,
                      table_width, seq_lens, nullptr, out, out_stride_seq, out_stride_head, scale, batch,
                      n_q_heads, n_kv_heads, head_dim, block_size, num_blocks, max_seq_len, split_tokens, flags,
                      workspace, workspace_bytes, err_word, stream);
}

int snapmind_paged_gqa_decode_append(const void* q, int64_t q_stride_seq, int64_t q_stride_head, void* k_pool,
                                     void* v_pool, int dtype, const int32_t* block_tables, int64_t table_stride_seq,
                                     int32_t table_width, const int32_t* seq_lens, const void* k_new,
                                     const void* v_new, int64_t new_stride_seq, int64_t new_stride_head, void* out,
                                     int64_t out_stride_seq, int64_t out_stride_head, float scale, int32_t batch,
                                     int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                     int32_t num_blocks, int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                                     void* workspace, int64_t workspace_bytes, int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(k_new != nullptr && v_new != nullptr, "paged_decode_append: k_new / v_new is NULL");
  SNAPMIND_CHECK_ARG(out != nullptr, "paged_decode_append: out is NULL");
  return decode_entry(q, q_stride_seq, q_stride_head, k_pool, v_pool, dtype, block_tables, table_stride_seq,
                      table_width, seq_lens, nullptr, out, out_stride_seq, out_stride_head, scale, batch,
                      n_q_heads, n_kv_heads, head_dim, block_size, num_blocks, max_seq_len, split_tokens, flags,
                      workspace, workspace_bytes, err_word, stream, nullptr, k_new, v_new, new_stride_seq,
                      new_stride_head);
}

int snapmind_paged_gqa_decode_window(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                     const void* k_pool, const void* v_pool, int dtype,
                                     const int32_t* block_tables, int64_t table_stride_seq,
                                     int32_t table_width, const int32_t* seq_lens, const int32_t* seq_starts,
                                     void* out, int64_t out_stride_seq, int64_t out_stride_head, float scale,
                                     int32_t batch, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                     int32_t block_size, int32_t num_blocks, int32_t max_seq_len,
                                     int32_t split_tokens, int32_t flags, void* workspace,
                                     int64_t workspace_bytes, int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(seq_starts != nullptr, "paged_decode_window: seq_starts is NULL");
  return decode_entry(q, q_stride_seq, q_stride_head, k_pool, v_pool, dtype, block_tables, table_stride_seq,
                      table_width, seq_lens, seq_starts, out, out_stride_seq, out_stride_head, scale, batch,
                      n_q_heads, n_kv_heads, head_dim, block_size, num_blocks, max_seq_len, split_tokens, flags,
                      workspace, workspace_bytes, err_word, stream);
}


int snapmind_paged_gqa_decode_peers(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                    const void* k_pool, const void* v_pool, int dtype,
                                    const int32_t* block_tables, int64_t table_stride_seq, int32_t table_width,
                                    const int32_t* seq_lens, const int32_t* seq_starts, void* const* peer_out,
                                    int32_t n_peers, int32_t head_offset, int64_t out_stride_seq,
                                    int64_t out_stride_head, float scale, int32_t batch, int32_t n_q_heads,
                                    int32_t n_kv_heads, int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                    int32_t max_seq_len, int32_t split_tokens, int32_t flags, void* workspace,
                                    int64_t workspace_bytes, int32_t* err_word, void* stream) {
  const PeerArgs peers{peer_out, n_peers, head_offset};
  return decode_entry(q, q_stride_seq, q_stride_head, k_pool, v_pool, dtype, block_tables, table_stride_seq,
                      table_width, seq_lens, seq_starts, nullptr, out_stride_seq, out_stride_head, scale, batch,
                      n_q_heads, n_kv_heads, head_dim, block_size, num_blocks, max_seq_len, split_tokens, flags,
                      workspace, workspace_bytes, err_word, stream, &peers);
}

}  // extern "C"
