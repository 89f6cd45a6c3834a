// Sparse MLA decode on the 5th-generation tensor cores (tcgen05, sm_100a):
// 128 heads, kv_lora_rank 512, rope 64, 64-token blocks, bf16/f16.
//
// A decode step of DeepSeek-style absorbed MLA is, per sequence, a 128-row
// attention: Q [128 heads x 576] against the attended latent rows
// [n x 576] (latent 512 | rope 64), output [128 x 512] over the first 512
// columns of the same rows.  The 128 heads are exactly the M = 128 of one
// tcgen05.mma, so:
//   CTA = (split s, output half dh, sequence b), 4 warps (thread = head row).
//   Shared memory (1024-aligned, 128-byte swizzle, written by TMA):
//     Q: 9 k-blocks x [128 rows x 64] = 144 KB, resident;
//     2 stages of 32 attended rows: 9 k-blocks x [32 rows x 64] = 36 KB each;
//     P: [128 x 32] bf16, 64-byte swizzle, written by the softmax threads.
//   TMEM (512 columns): O [128 x 256] f32 at column 0 (this CTA's half of the
//     512 output dims), S [128 x 32] f32 at column 256.
//   Per tile of 32 tokens (half a block):
//     S = Q K^T: 36 MMAs (M 128, N 32, K 16), K-major operands;
//     softmax: each thread loads its row of S from TMEM, masks the tokens
//       outside the selection, keeps a reference maximum that is raised only
//       when a score exceeds it by 2^8 (then O's row is rescaled in TMEM), and
//       writes P = exp2(s - m) as bf16 into shared memory;
//     O += P V: 2 MMAs (M 128, N 256, K 16), V = the tile's latent columns
//       [256 dh, 256 dh + 256) read MN-major from the same staged rows.
//   One thread issues TMA loads and MMAs; completion is tracked by mbarriers
//   (tcgen05.commit), every wait is bounded (about a second), and TMEM is
//   released on every path.
// Splits write fp32 partials (max, sum, unnormalised output) in the layout of
// the paged GQA decode; a second kernel merges them over all (sequence, head)
// rows in parallel.
//
// The attended positions are those of the mma.sync kernel (sparse_mla.cu):
// the selected chunks of the lookahead indexer
// (snapmind/layers/indexer/lookahead.py:11-106), the first `sink` positions
// and the last `window` positions; the attention is that of
// snapmind/layers/attention/mla.py:217-245 with the query absorbed.
#include <cuda.h>

#include "common.cuh"
#include "paged_decode.cuh"
#include "sm100.cuh"
#include "sparse_mla.cuh"

namespace snapmind {
namespace {

using namespace tc;

constexpr int kH = 128;                                 // heads = MMA M
constexpr int kR = 512, kP = 64;
constexpr int kKB = (kR + kP) / 64;                     // 9 k-blocks of 64 elements
constexpr int kBs = 64;                                 // block (chunk) size
constexpr int kTok = 32;                                // tokens per tile
constexpr int kDH = kR / 2;                             // output dims per CTA
constexpr int kThreads = 128;
constexpr uint32_t kQBlock = kH * 128;                  // one k-block of Q: 16 KB
constexpr uint32_t kQBytes = kKB * kQBlock;             // 144 KB
constexpr uint32_t kTBlock = kTok * 128;                // one k-block of a tile: 4 KB
constexpr uint32_t kTileBytes = kKB * kTBlock;          // 36 KB
constexpr uint32_t kPBytes = kH * kTok * 2;             // 8 KB
constexpr int kStages = 2;
constexpr int kBits = 4096;                             // chunks per sequence (bitmaps)
constexpr uint32_t kTmemCols = 512, kColO = 0, kColS = 256;
constexpr float kRescale = 8.f;                         // log2 headroom of the reference maximum

struct Ctrl {
  uint64_t full[kStages];
  uint64_t q_full;
  uint64_t mma;
  uint32_t tmem_base;
  int32_t count;
  int32_t tile_phys[kStages];
  int32_t tile_chunk[kStages];
  uint32_t sel_bits[kBits / 32];
  uint32_t inc_bits[kBits / 32];
  int32_t word_pre[kBits / 32 + 1];
};

constexpr size_t kSmemBytes = 1024 + kQBytes + kStages * kTileBytes + kPBytes + sizeof(Ctrl);
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ int chunk_of_rank(const Ctrl& C, int words, int rank) {
  int lo = 0, hi = words;  // last word w with word_pre[w] <= rank
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (C.word_pre[mid] <= rank) lo = mid; else hi = mid;
  }
  uint32_t word = C.inc_bits[lo];
  int k = rank - C.word_pre[lo];
  while (k-- > 0) word &= word - 1;
  return lo * 32 + __ffs(word) - 1;
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_umma_kernel(const __grid_constant__ CUtensorMap qlat_map, const __grid_constant__ CUtensorMap qpe_map,
                           const __grid_constant__ CUtensorMap lat_map, const __grid_constant__ CUtensorMap rope_map,
                           SparseParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = base;
  uint8_t* kv_s = q_s + kQBytes;
  uint8_t* p_s = kv_s + kStages * kTileBytes;
  Ctrl& C = *reinterpret_cast<Ctrl*>(p_s + kPBytes);

  const int s = blockIdx.x, dh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBf16, kH, kTok, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBf16, kH, kDH, false, true);

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(smem_u32(&C.full[i]), 1);
    mbar_init(smem_u32(&C.q_full), 1);
    mbar_init(smem_u32(&C.mma), 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }

  // ---- attended chunks of sequence b: bitmaps and the prefix of their counts
  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  int n_chunks = (len + kBs - 1) / kBs;
  if (n_chunks > kBits) {
    if (tid == 0 && s == 0 && dh == 0) flag_error(p.dp.err, SNAPMIND_DEVERR_TABLE);
    n_chunks = kBits;
    len = kBits * kBs;
  }
  const int words = (n_chunks + 31) / 32;
  for (int i = tid; i < words; i += kThreads) {
    C.sel_bits[i] = 0u;
    C.inc_bits[i] = 0u;
  }
  __syncthreads();
  for (int i = tid; i < p.k; i += kThreads) {
    const int c = p.selected[(int64_t)b * p.k + i];
    if (c >= 0 && c < n_chunks) {
      atomicOr(&C.sel_bits[c >> 5], 1u << (c & 31));
      atomicOr(&C.inc_bits[c >> 5], 1u << (c & 31));
    }
  }
  const int sink = min(p.sink, len);
  const int wstart = max(0, len - p.window);
  if (tid == 0 && sink > 0) atomicOr(&C.inc_bits[0], 1u);
  if (len > wstart)
    for (int c = wstart / kBs + tid; c < n_chunks; c += kThreads) atomicOr(&C.inc_bits[c >> 5], 1u << (c & 31));
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const int cnt = (w0 + lane < words) ? __popc(C.inc_bits[w0 + lane]) : 0;
      int pre = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, off);
        if (lane >= off) pre += y;
      }
      if (w0 + lane < words) C.word_pre[w0 + lane] = carry + pre - cnt;
      carry += __shfl_sync(0xffffffffu, pre, 31);
    }
    if (lane == 0) {
      C.word_pre[words] = carry;
      C.count = carry;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = C.tmem_base;
  const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's TMEM lanes
  const int count = C.count;
  const DecodeParams& dp = p.dp;
  const int head = tid;

  // tiles of this split: tile u = half (u & 1) of the (u >> 1)-th attended chunk
  const int total = 2 * count;
  const int per = (total + p.n_splits - 1) / max(p.n_splits, 1);
  const int u_lo = min(total, s * per), u_hi = min(total, u_lo + per);
  const int n_tiles = u_hi - u_lo;

  auto issue_tile = [&](int t) {  // thread 0
    const int st = t % kStages;
    const int u = u_lo + t;
    const int c = chunk_of_rank(C, words, u >> 1);
    int32_t phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
    if (phys >= p.num_blocks) phys = -1;
    C.tile_phys[st] = phys;
    C.tile_chunk[st] = c;
    const uint32_t bar = smem_u32(&C.full[st]);
    if (phys < 0) {
      flag_error(dp.err, SNAPMIND_DEVERR_BLOCK_ID);
      mbar_arrive(bar);
      return;
    }
    mbar_arrive_expect_tx(bar, kTileBytes);
    uint8_t* stage = kv_s + st * kTileBytes;
    const int y = phys * kBs + (u & 1) * kTok;
#pragma unroll
    for (int kb = 0; kb < kKB - 1; ++kb) tma_load_2d(smem_u32(stage + kb * kTBlock), &lat_map, kb * 64, y, bar);
    tma_load_2d(smem_u32(stage + (kKB - 1) * kTBlock), &rope_map, 0, y, bar);
  };

  bool aborted = false;
  int issued = 0, consumed = 0;
  bool mma_pending = false, q_pending = false;
  uint32_t mma_phase = 0;
  float m_ref = -INFINITY, l_run = 0.f;  // this thread's head row, log2 units of score * scale
  const float c2 = p.scale * 1.4426950408889634f;

  if (count > 0 && n_tiles > 0) {
    if (tid == 0) {
      const uint32_t qb = smem_u32(&C.q_full);
      mbar_arrive_expect_tx(qb, kQBytes);
#pragma unroll
      for (int kb = 0; kb < kKB - 1; ++kb) tma_load_2d(smem_u32(q_s + kb * kQBlock), &qlat_map, kb * 64, b * kH, qb);
      tma_load_2d(smem_u32(q_s + (kKB - 1) * kQBlock), &qpe_map, 0, b * kH, qb);
      for (int t = 0; t < min(kStages, n_tiles); ++t) issue_tile(t);
    }
    issued = min(kStages, n_tiles);
    q_pending = true;

    for (int t = 0; t < n_tiles; ++t) {
      const int st = t % kStages;
      uint8_t* stage = kv_s + st * kTileBytes;
      bool ok = true;
      if (t == 0) {
        ok = mbar_wait(smem_u32(&C.q_full), 0);
        if (ok) q_pending = false;
      }
      ok = ok && mbar_wait(smem_u32(&C.full[st]), (t / kStages) & 1);
      if (__syncthreads_or(!ok)) {
        aborted = true;
        break;
      }
      consumed = t + 1;
      const int phys = C.tile_phys[st], c = C.tile_chunk[st];
      const int pos0 = c * kBs + (t + u_lo) % 2 * kTok;
      // rows holding no token (past the end, or an unloaded tile): zero this CTA's V columns
      const int good = phys < 0 ? 0 : max(0, min(kTok, len - pos0));
      if (good < kTok) {
        const int rows = kTok - good;
        for (int e = tid; e < 4 * rows * 8; e += kThreads) {
          const int kb = dh * 4 + e / (rows * 8);
          const int r = good + (e / 8) % rows;
          *reinterpret_cast<uint4*>(stage + kb * kTBlock + r * 128 + (e & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      const bool selected = phys >= 0 && ((C.sel_bits[c >> 5] >> (c & 31)) & 1u);
      __syncthreads();

      // ---- S = Q K^T
      if (tid == 0) {
        tc_fence_after();
#pragma unroll 1
        for (int kb = 0; kb < kKB; ++kb) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(q_s + kb * kQBlock + kk * 32), 16, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(smem_u32(stage + kb * kTBlock + kk * 32), 16, 1024, kSwizzle128B);
            umma_f16(tmem + kColS, ad, bd, kIdescS, (kb | kk) != 0);
          }
        }
        umma_commit(smem_u32(&C.mma));
      }
      mma_pending = true;
      ok = mbar_wait(smem_u32(&C.mma), mma_phase);
      if (__syncthreads_or(!ok)) {
        aborted = true;
        break;
      }
      mma_phase ^= 1;
      mma_pending = false;
      tc_fence_after();
      // S(t) done, and with it O += P V of tile t - 1: its stage and P are free
      if (tid == 0 && t + 1 < n_tiles && t + 1 >= kStages) {
        issue_tile(t + 1);
      }
      if (t + 1 < n_tiles && t + 1 >= kStages) issued = t + 2;

      // ---- softmax of this thread's row
      float sv[kTok];
      tmem_ld32(t_row + kColS, sv);
      tmem_wait_ld();
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < kTok; ++j) {
        const int pos = pos0 + j;
        const bool valid = j < good && (selected || pos < sink || pos >= wstart);
        sv[j] = valid ? sv[j] * c2 : -INFINITY;
        mt = fmaxf(mt, sv[j]);
      }
      const bool raise = mt > m_ref + kRescale;
      const float m_new = raise ? mt : m_ref;
      if (__any_sync(0xffffffffu, raise && m_ref != -INFINITY)) {
        // O rows of this warp at the old reference maximum: rescale in TMEM
        const float alpha = (raise && m_ref != -INFINITY) ? exp2f(m_ref - m_new) : 1.f;
#pragma unroll 1
        for (int cc = 0; cc < kDH; cc += 32) {
          float o[32];
          tmem_ld32(t_row + kColO + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= alpha;
          tmem_st32(t_row + kColO + cc, o);
        }
        tmem_wait_st();
        l_run *= alpha;
      }
      m_ref = m_new;
      uint32_t pk[kTok / 2];
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < kTok / 2; ++j) {
        const float p0 = m_ref == -INFINITY ? 0.f : exp2f(sv[2 * j] - m_ref);
        const float p1 = m_ref == -INFINITY ? 0.f : exp2f(sv[2 * j + 1] - m_ref);
        psum += p0 + p1;
        pk[j] = pack2<T>(p0, p1);
      }
      l_run += psum;
      // row `head` of P: 64 bytes, 64-byte swizzle (16-byte chunk c of row r at chunk c ^ ((r >> 1) & 3))
      {
        uint8_t* prow = p_s + (head >> 3) * 512 + (head & 7) * 64;
        const int sw = (head >> 1) & 3;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
          *reinterpret_cast<uint4*>(prow + ((c4 ^ sw) << 4)) =
              make_uint4(pk[4 * c4], pk[4 * c4 + 1], pk[4 * c4 + 2], pk[4 * c4 + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();

      // ---- O += P V
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kTok / 16; ++ks) {
          const uint64_t ad = smem_desc(smem_u32(p_s + ks * 32), 16, 512, kSwizzle64B);
          const uint64_t bd =
              smem_desc(smem_u32(stage + dh * 4 * kTBlock + ks * 16 * 128), kTBlock, 1024, kSwizzle128B);
          umma_f16(tmem + kColO, ad, bd, kIdescPV, (t > 0 || ks > 0) ? 1u : 0u);
        }
        if (t + 1 == n_tiles) umma_commit(smem_u32(&C.mma));
      }
    }
    if (!aborted) {
      mma_pending = true;
      const bool ok = mbar_wait(smem_u32(&C.mma), mma_phase);
      if (__syncthreads_or(!ok)) aborted = true;
      else mma_pending = false;
      tc_fence_after();
    }
  }

  if (aborted) {
    if (tid == 0) {
      flag_error(dp.err, SNAPMIND_DEVERR_TIMEOUT);
      // wait (bounded) for what is still in flight before the memory is released
      if (q_pending) mbar_wait(smem_u32(&C.q_full), 0);
      for (int i = consumed; i < issued; ++i) mbar_wait(smem_u32(&C.full[i % kStages]), (i / kStages) & 1);
      if (mma_pending) mbar_wait(smem_u32(&C.mma), mma_phase);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    return;
  }

  const bool direct = (p.n_splits == 1);
  if (count == 0) {
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    if (s == 0 && direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)head * dp.out_stride_head +
             dh * kDH;
      for (int d = 0; d < kDH; d += 8) *reinterpret_cast<uint4*>(o + d) = make_uint4(0, 0, 0, 0);
    }
    if (!direct) {  // empty partials: the merge reads every split
      float* part = dp.partials + (((int64_t)b * dp.n_q_heads + head) * dp.max_splits + s) * (kR + 2);
      if (dh == 0) {
        part[0] = -INFINITY;
        part[1] = 0.f;
      }
      for (int d = 0; d < kDH; ++d) part[2 + dh * kDH + d] = 0.f;
    }
    return;
  }

  // ---- epilogue: this thread's row of O (256 columns)
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
  float* part = dp.partials + (((int64_t)b * dp.n_q_heads + head) * dp.max_splits + s) * (kR + 2);
  T* orow = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)head * dp.out_stride_head +
            dh * kDH;
#pragma unroll 1
  for (int cc = 0; cc < kDH; cc += 32) {
    float o[32];
    if (n_tiles > 0) {
      tmem_ld32(t_row + kColO + cc, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = 0.f;
    }
    if (direct) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        const uint4 v = make_uint4(pack2<T>(o[j] * inv, o[j + 1] * inv), pack2<T>(o[j + 2] * inv, o[j + 3] * inv),
                                   pack2<T>(o[j + 4] * inv, o[j + 5] * inv), pack2<T>(o[j + 6] * inv, o[j + 7] * inv));
        *reinterpret_cast<uint4*>(orow + cc + j) = v;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *reinterpret_cast<float2*>(part + 2 + dh * kDH + cc + j) = make_float2(o[j], o[j + 1]);
    }
  }
  if (!direct && dh == 0) {
    part[0] = m_ref == -INFINITY ? -INFINITY : m_ref * 0.6931471805599453f;  // natural-log units
    part[1] = l_run;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge of the split partials: one CTA per (sequence, 8 heads), 16-byte output stores.
template <typename T>
__global__ void __launch_bounds__(256) sparse_mla_merge_kernel(DecodeParams dp, int n_splits) {
  const int b = blockIdx.y;
  const int hl = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * 8 + hl;
  const int64_t pstride = kR + 2;
  const float* pg = dp.partials + ((int64_t)b * dp.n_q_heads + h) * dp.max_splits * pstride;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, __ldcg(pg + s * pstride));
  float L = 0.f;
  for (int s = 0; s < n_splits; ++s) {
    const float m = __ldcg(pg + s * pstride);
    if (m != -INFINITY) L += __ldcg(pg + s * pstride + 1) * expf(m - M);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  // lane covers dims [16 lane, 16 lane + 16)
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
  for (int s = 0; s < n_splits; ++s) {
    const float m = __ldcg(pg + s * pstride);
    if (m == -INFINITY) continue;
    const float f = expf(m - M);
    const float* a = pg + s * pstride + 2 + 16 * lane;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(a + j));
      acc[j] += v.x * f;
      acc[j + 1] += v.y * f;
    }
  }
  T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head + 16 * lane;
#pragma unroll
  for (int j = 0; j < 16; j += 8) {
    *reinterpret_cast<uint4*>(o + j) =
        make_uint4(pack2<T>(acc[j] * inv, acc[j + 1] * inv), pack2<T>(acc[j + 2] * inv, acc[j + 3] * inv),
                   pack2<T>(acc[j + 4] * inv, acc[j + 5] * inv), pack2<T>(acc[j + 6] * inv, acc[j + 7] * inv));
  }
}

}  // namespace

int sparse_mla_umma_splits(int batch) {
  const int per_seq = num_sms() / (2 * (batch > 0 ? batch : 1));
  return per_seq < 1 ? 1 : (per_seq > 64 ? 64 : per_seq);
}

bool sparse_mla_umma_supported(const SparseParams& p, int dtype) {
  const auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  return (dtype == SNAPMIND_DTYPE_BF16 || dtype == SNAPMIND_DTYPE_F16) && p.n_heads == kH && p.R == kR &&
         p.P == kP && p.bs == kBs && p.table_width <= kBits && p.batch <= 65535 && a16(p.q_lat) && a16(p.q_pe) &&
         a16(p.latent) && a16(p.rope) && a16(p.dp.out) && encode_tiled() != nullptr;
}

int launch_sparse_mla_umma(const SparseParams& p, int dtype, cudaStream_t st) {
  const bool bf16 = dtype == SNAPMIND_DTYPE_BF16;
  CUtensorMap qlat, qpe, lat, rope;
  const uint64_t rows = (uint64_t)p.num_blocks * kBs;
  if (!tensor_map_2d(&qlat, bf16, p.q_lat, kR, (uint64_t)p.batch * kH, kR * 2, 64, kH) ||
      !tensor_map_2d(&qpe, bf16, p.q_pe, kP, (uint64_t)p.batch * kH, kP * 2, 64, kH) ||
      !tensor_map_2d(&lat, bf16, p.latent, kR, rows, kR * 2, 64, kTok) ||
      !tensor_map_2d(&rope, bf16, p.rope, kP, rows, kP * 2, 64, kTok)) {
    set_last_error("sparse_mla_umma: tensor map encoding failed");
    return SNAPMIND_ERR_CUDA;
  }
  auto go = [&](auto kernel, auto merge) -> int {
    static bool attr = false;
    if (!attr) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e != cudaSuccess) return cuda_status(e, "sparse_mla_umma smem attribute");
      attr = true;
    }
    kernel<<<dim3(p.n_splits, 2, p.batch), kThreads, kSmemBytes, st>>>(qlat, qpe, lat, rope, p);
    int rc = cuda_status(cudaGetLastError(), "sparse_mla_umma launch");
    if (rc != SNAPMIND_OK || p.n_splits == 1) return rc;
    merge<<<dim3(kH / 8, p.batch), 256, 0, st>>>(p.dp, p.n_splits);
    return cuda_status(cudaGetLastError(), "sparse_mla_merge launch");
  };
  return bf16 ? go(sparse_mla_umma_kernel<__nv_bfloat16>, sparse_mla_merge_kernel<__nv_bfloat16>)
              : go(sparse_mla_umma_kernel<__half>, sparse_mla_merge_kernel<__half>);
}

}  // namespace snapmind
