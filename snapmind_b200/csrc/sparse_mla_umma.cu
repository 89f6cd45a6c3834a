// Sparse MLA decode on the 5th-generation tensor cores (tcgen05, sm_100a):
// 128 heads, kv_lora_rank 512, rope 64, 64-token blocks, bf16/f16.
//
// A decode step of DeepSeek-style absorbed MLA is, per sequence, a 128-row
// attention: Q [128 heads x 576] against the attended latent rows
// [n x 576] (latent 512 | rope 64), output [128 x 512] over the first 512
// columns of the same rows.  The 128 heads are exactly the M = 128 of one
// tcgen05.mma, so:
//   CTA = (split s, output half dh, sequence b), 6 warps: warps 0-3 softmax
//   (thread = head row = TMEM lane), warp 4 TMA producer, warp 5 MMA issuer.
//   Shared memory (1024-aligned, 128-byte swizzle, written by TMA):
//     Q: 9 k-blocks x [128 rows x 64] = 144 KB, resident;
//     one attended chunk (block) of 64 rows as two 32-row stages,
//       9 k-blocks x [64 rows x 64] (72 KB: one 3-D TMA box for the 8 latent
//       k-blocks, one 2-D box for the rope k-block);
//     P: [128 x 32] bf16, 64-byte swizzle, written by the softmax threads.
//   TMEM (512 columns): O [128 x 256] f32 at column 0 (this CTA's half of the
//     512 output dims); the scores of a chunk [128 x 64] f32 as two
//     accumulator chains (even and odd k-blocks) at columns 256 and 320.
//   Per chunk of 64 tokens (two tiles of 32):
//     S = Q K^T: 36 MMAs (M 128, N 64, K 16), K-major operands, alternating
//       between the two chains so consecutive MMAs do not wait on one
//       accumulator;
//     softmax, per tile: each thread loads and adds its row of both chains
//       from TMEM, masks the tokens outside the selection, keeps a reference
//       maximum that is raised only when a score exceeds it by 2^8 (then O's
//       row is rescaled in TMEM), and writes P = exp2(s - m) as bf16 into
//       shared memory;
//     O += P V per tile: 2 MMAs (M 128, N 256, K 16), V = the tile's latent
//       columns [256 dh, 256 dh + 256) read MN-major from the staged rows.
//   Pipeline: the producer loads the next chunk once O += P V of the current
//   chunk's second tile has completed, resolving its block id beforehand; the
//   MMA warp polls (non-blocking) and issues whichever is ready first: O += P V
//   of the oldest tile whose P is written, or S of the next staged chunk.
//   Handshakes are mbarriers (tcgen05.commit for the tensor core), every wait
//   is bounded (about a second) and ends early once another role gave up, and
//   TMEM is released on every path.
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
constexpr int kSoftmaxThreads = 128;                    // warps 0-3: one head row per thread
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr int kThreads = 192;
constexpr uint32_t kQBlock = kH * 128;                  // one k-block of Q: 16 KB
constexpr uint32_t kQBytes = kKB * kQBlock;             // 144 KB
constexpr uint32_t kTBlock = kTok * 128;                // one k-block of a tile: 4 KB
constexpr uint32_t kTileBytes = kKB * kTBlock;          // 36 KB
constexpr uint32_t kPBytes = kH * kTok * 2;             // 8 KB
constexpr int kStages = 2;
constexpr int kBits = 4096;                             // chunks per sequence (bitmaps)
// TMEM columns: O (f32) at 0; the scores of a chunk as two accumulator chains of 64 columns
constexpr uint32_t kTmemCols = 512, kColO = 0, kColS = 256, kSChain = 64;
constexpr float kRescale = 8.f;                         // log2 headroom of the reference maximum
// The two stages interleave per k-block: k-block kb of stage st at
// kb * kKBStride + st * kTBlock, so the 64 rows of a stage pair are contiguous
// in every k-block and one N = 64 MMA scores two tiles.
constexpr uint32_t kKBStride = kStages * kTBlock;
static_assert(kStages == 2, "tiles are scored in pairs of stages");

struct Ctrl {
  uint64_t full;             // producer -> MMA, softmax: the chunk (both tiles) staged
  uint64_t empty;            // MMA commit after O += P V of the chunk's second tile
  uint64_t s_full[2];        // MMA commit after S = Q K^T: S buffer ready
  uint64_t s_empty[2];       // softmax threads: S buffer read
  uint64_t q_full;
  uint64_t p_full;           // softmax threads: P written (and O rescaled)
  uint64_t o_done;           // MMA commit after O += P V
  uint32_t tmem_base;
  int32_t abort;
  int32_t count;
  int32_t chunk_phys;        // block and chunk id of the staged chunk
  int32_t chunk_id;
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

// 2^x by the hardware approximation (MUFU.EX2); -inf -> 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// Waits of the pipeline roles: bounded, and cut short once another role gave up.
__device__ __forceinline__ bool role_wait(const Ctrl& C, uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<const volatile int32_t*>(&C.abort)) return false;
    if (clock64() - t0 > kWaitTicks) return false;
  }
  return true;
}

__device__ __forceinline__ void give_up(Ctrl& C, int32_t* err) {
  atomicExch(&C.abort, 1);
  flag_error(err, SNAPMIND_DEVERR_TIMEOUT);
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
  constexpr uint32_t kIdescS2 = idesc_f16(kBf16, kH, 2 * kTok, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBf16, kH, kDH, false, true);
  const DecodeParams& dp = p.dp;

  if (tid == 0) {
    mbar_init(smem_u32(&C.full), 1);
    mbar_init(smem_u32(&C.empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&C.s_full[i]), 1);
      mbar_init(smem_u32(&C.s_empty[i]), kSoftmaxThreads);
    }
    mbar_init(smem_u32(&C.q_full), 1);
    mbar_init(smem_u32(&C.p_full), kSoftmaxThreads);
    mbar_init(smem_u32(&C.o_done), 1);
    C.abort = 0;
    mbar_init_fence();
    // Q depends only on the sequence: its copy overlaps the selection set-up below
    const uint32_t qb = smem_u32(&C.q_full);
    mbar_arrive_expect_tx(qb, kQBytes);
#pragma unroll
    for (int kb = 0; kb < kKB - 1; ++kb) tma_load_2d(smem_u32(q_s + kb * kQBlock), &qlat_map, kb * 64, b * kH, qb);
    tma_load_2d(smem_u32(q_s + (kKB - 1) * kQBlock), &qpe_map, 0, b * kH, qb);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }

  // ---- attended chunks of sequence b: bitmaps and the prefix of their counts
  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  int n_chunks = (len + kBs - 1) / kBs;
  if (n_chunks > kBits) {
    if (tid == 0 && s == 0 && dh == 0) flag_error(dp.err, SNAPMIND_DEVERR_TABLE);
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
  const int count = C.count;

  // chunks of this split; tile t = half (t & 1) of chunk c_lo + (t >> 1)
  const int per = (count + p.n_splits - 1) / max(p.n_splits, 1);
  const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);
  const int n_tiles = 2 * (c_hi - c_lo);
  const bool direct = (p.n_splits == 1);

  if (n_tiles > 0) {
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0) {
        // block of the i-th chunk of the split, resolved before the stages free up
        auto locate = [&](int i, int& c, int32_t& phys) {
          c = chunk_of_rank(C, words, c_lo + i);
          phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
          if (phys >= p.num_blocks) phys = -1;
        };
        const int n_ck = n_tiles / 2;
        int c_next;
        int32_t phys_next;
        locate(0, c_next, phys_next);
        int issued = 0;
        for (int i = 0; i < n_ck; ++i) {
          const int c = c_next;
          const int32_t phys = phys_next;
          if (i >= 1 && !role_wait(C, smem_u32(&C.empty), (i - 1) & 1)) {
            give_up(C, dp.err);
            break;
          }
          C.chunk_phys = phys;
          C.chunk_id = c;
          const uint32_t bar = smem_u32(&C.full);
          if (phys < 0) {
            flag_error(dp.err, SNAPMIND_DEVERR_BLOCK_ID);
            mbar_arrive(bar);
          } else {
            // the chunk's 64 rows, k-block by k-block: both stages in one copy
            mbar_arrive_expect_tx(bar, kStages * kTileBytes);
            const int y = phys * kBs;
            tma_load_3d(smem_u32(kv_s), &lat_map, 0, y, 0, bar);  // the 8 latent k-blocks
            tma_load_2d(smem_u32(kv_s + (kKB - 1) * kKBStride), &rope_map, 0, y, bar);
          }
          issued = i + 1;
          if (i + 1 < n_ck) locate(i + 1, c_next, phys_next);
        }
        // before the shared memory is released: every copy issued has landed (bounded)
        if (issued > 0) mbar_wait(smem_u32(&C.full), (issued - 1) & 1);
        mbar_wait(smem_u32(&C.q_full), 0);
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- MMA issuer
      if (lane == 0) {
        bool ok = role_wait(C, smem_u32(&C.q_full), 0);
        uint32_t last_bar = 0, last_parity = 0;  // the latest commit: covers every MMA issued
        auto issue_pv = [&](int t) {  // O += P V of tile t
          const uint8_t* stage = kv_s + (t % kStages) * kTBlock;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kTok / 16; ++ks) {
            const uint64_t ad = smem_desc(smem_u32(p_s + ks * 32), 16, 512, kSwizzle64B);
            const uint64_t bd =
                smem_desc(smem_u32(stage + dh * 4 * kKBStride + ks * 16 * 128), kKBStride, 1024, kSwizzle128B);
            umma_f16(tmem + kColO, ad, bd, kIdescPV, (t > 0 || ks > 0) ? 1u : 0u);
          }
          if (t & 1) umma_commit(smem_u32(&C.empty));
          umma_commit(smem_u32(&C.o_done));
          last_bar = smem_u32(&C.o_done);
          last_parity = t & 1;
        };
        // S = Q K^T of both tiles of a chunk (N = 64: tile t in columns 0-31,
        // t + 1 in 32-63), as two independent accumulator chains (even and odd
        // k-blocks) that the softmax threads add.
        auto issue_s = [&](int t) {
          tc_fence_after();
#pragma unroll 1
          for (int kb = 0; kb < kKB; ++kb) {
            const uint32_t d = tmem + kColS + (kb & 1) * kSChain;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc(smem_u32(q_s + kb * kQBlock + kk * 32), 16, 1024, kSwizzle128B);
              const uint64_t bd = smem_desc(smem_u32(kv_s + kb * kKBStride + kk * 32), 16, 1024, kSwizzle128B);
              umma_f16(d, ad, bd, kIdescS2, (kb > 1 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(smem_u32(&C.s_full[0]));
          umma_commit(smem_u32(&C.s_full[1]));
          last_bar = smem_u32(&C.s_full[1]);
          last_parity = (t >> 1) & 1;
        };
        // Issue whichever is ready: O += P V of the oldest tile whose P is written
        // (it frees a stage for the producer), else S of the next staged tile (at
        // most two S buffers ahead of O += P V).
        int ns = 0, np = 0;  // next tile to score (even), next tile for O += P V
        long long idle_since = clock64();
        while (ok && np < n_tiles) {
          bool progressed = false;
          if (np < ns && mbar_test_wait(smem_u32(&C.p_full), np & 1)) {
            issue_pv(np++);
            progressed = true;
          } else if (ns < n_tiles) {
            // the chunk of tiles ns, ns + 1 once staged and both S buffers were read
            const uint32_t par = (ns >> 1) & 1, prev = ((ns >> 1) - 1) & 1;
            if (mbar_test_wait(smem_u32(&C.full), par) &&
                (ns < 2 || (mbar_test_wait(smem_u32(&C.s_empty[0]), prev) &&
                            mbar_test_wait(smem_u32(&C.s_empty[1]), prev)))) {
              issue_s(ns);
              ns += 2;
              progressed = true;
            }
          }
          if (progressed) {
            idle_since = clock64();
          } else if (*reinterpret_cast<const volatile int32_t*>(&C.abort) || clock64() - idle_since > kWaitTicks) {
            ok = false;
          }
        }
        if (!ok) {
          give_up(C, dp.err);
          if (last_bar) mbar_wait(last_bar, last_parity);  // MMAs in flight finish (bounded) before TMEM goes
        }
      }
    } else {
      // ---------------------------------------------------------------- softmax warps 0-3
      const int head = tid;  // TMEM lane = head row
      const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);
      const float c2 = p.scale * 1.4426950408889634f;
      float m_ref = -INFINITY, l_run = 0.f;  // log2 units of score * scale
      bool ok = true;
      for (int t = 0; t < n_tiles; ++t) {
        const int st = t % kStages, sb = t & 1;
        ok = role_wait(C, smem_u32(&C.full), (t >> 1) & 1) && role_wait(C, smem_u32(&C.s_full[sb]), (t >> 1) & 1);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        const int phys = C.chunk_phys, c = C.chunk_id;
        const int pos0 = c * kBs + (t & 1) * kTok;
        const int good = phys < 0 ? 0 : max(0, min(kTok, len - pos0));  // rows holding a token
        // attended tokens of the tile as a bit mask: [0, good) for a selected chunk,
        // else [0, min(good, sink - pos0)) and [max(0, wstart - pos0), good)
        uint32_t vmask;
        {
          const uint32_t below_good = good >= 32 ? 0xffffffffu : ((1u << good) - 1u);
          const bool selected = phys >= 0 && ((C.sel_bits[c >> 5] >> (c & 31)) & 1u);
          if (selected) {
            vmask = below_good;
          } else {
            const int a = max(0, min(32, sink - pos0));
            const int w = max(0, min(32, wstart - pos0));
            const uint32_t sink_bits = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
            const uint32_t win_bits = w >= 32 ? 0u : ~((1u << w) - 1u);
            vmask = (sink_bits | win_bits) & below_good;
          }
        }
        tc_fence_after();
        float sv[kTok], sv2[kTok];
        tmem_ld32(t_row + kColS + sb * kTok, sv);
        tmem_ld32(t_row + kColS + kSChain + sb * kTok, sv2);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < kTok; ++j) sv[j] += sv2[j];
        tc_fence_before();
        mbar_arrive(smem_u32(&C.s_empty[sb]));
        // masked row maximum (raw scores; scale > 0), as a tree
        float mx[kTok / 2];
#pragma unroll
        for (int j = 0; j < kTok / 2; ++j)
          mx[j] = fmaxf((vmask >> (2 * j)) & 1u ? sv[2 * j] : -INFINITY,
                        (vmask >> (2 * j + 1)) & 1u ? sv[2 * j + 1] : -INFINITY);
#pragma unroll
        for (int w = kTok / 4; w >= 1; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) mx[j] = fmaxf(mx[j], mx[j + w]);
        const float mt = mx[0] * c2;
        const bool raise = mt > m_ref + kRescale;
        const float m_old = m_ref;
        m_ref = raise ? mt : m_ref;
        // P = 2^(s c2 - m) for attended tokens, 0 elsewhere
        uint32_t pk[kTok / 2];
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < kTok / 2; ++j) {
          const float e0 = ex2_approx(fmaf(sv[2 * j], c2, -m_ref));
          const float e1 = ex2_approx(fmaf(sv[2 * j + 1], c2, -m_ref));
          const float p0 = (vmask >> (2 * j)) & 1u ? e0 : 0.f;
          const float p1 = (vmask >> (2 * j + 1)) & 1u ? e1 : 0.f;
          ps[j & 3] += p0 + p1;
          pk[j] = pack2<T>(p0, p1);
        }
        // O += P V of tile t - 1 has finished: P is free and O holds it
        if (t >= 1) {
          ok = role_wait(C, smem_u32(&C.o_done), (t - 1) & 1);
          if (__any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, raise && m_old != -INFINITY)) {
          // O rows of this warp at the old reference maximum: rescale in TMEM
          const float alpha = (raise && m_old != -INFINITY) ? exp2f(m_old - m_ref) : 1.f;
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
        l_run += (ps[0] + ps[1]) + (ps[2] + ps[3]);
        {  // row `head` of P: 64 bytes, 64-byte swizzle (chunk c of row r at c ^ ((r >> 1) & 3))
          uint8_t* prow = p_s + (head >> 3) * 512 + (head & 7) * 64;
          const int sw = (head >> 1) & 3;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            *reinterpret_cast<uint4*>(prow + ((c4 ^ sw) << 4)) =
                make_uint4(pk[4 * c4], pk[4 * c4 + 1], pk[4 * c4 + 2], pk[4 * c4 + 3]);
        }
        if (good < kTok) {  // rows holding no token: zero this CTA's V columns (S of the tile is done)
          uint8_t* stage = kv_s + st * kTBlock;
          const int rows = kTok - good;
          for (int e = tid; e < 4 * rows * 8; e += kSoftmaxThreads) {
            const int kb = dh * 4 + e / (rows * 8);
            const int r = good + (e / 8) % rows;
            *reinterpret_cast<uint4*>(stage + kb * kKBStride + r * 128 + (e & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(smem_u32(&C.p_full));
      }
      if (ok) {
        ok = role_wait(C, smem_u32(&C.o_done), (n_tiles - 1) & 1);
        ok = !__any_sync(0xffffffffu, !ok);
      }
      if (!ok) {
        give_up(C, dp.err);
      } else {
        // ---- epilogue: this thread's row of O (256 columns)
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        float* part = dp.partials + (((int64_t)b * dp.n_q_heads + head) * dp.max_splits + s) * (kR + 2);
        T* orow = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq +
                  (int64_t)head * dp.out_stride_head + dh * kDH;
#pragma unroll 1
        for (int cc = 0; cc < kDH; cc += 32) {
          float o[32];
          tmem_ld32(t_row + kColO + cc, o);
          tmem_wait_ld();
          if (direct) {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              *reinterpret_cast<uint4*>(orow + cc + j) =
                  make_uint4(pack2<T>(o[j] * inv, o[j + 1] * inv), pack2<T>(o[j + 2] * inv, o[j + 3] * inv),
                             pack2<T>(o[j + 4] * inv, o[j + 5] * inv), pack2<T>(o[j + 6] * inv, o[j + 7] * inv));
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
      }
    }
  } else if (tid < kSoftmaxThreads) {
    // no tile in this split: an empty partial (or a zero output when nothing is attended)
    const int head = tid;
    if (tid == 0) mbar_wait(smem_u32(&C.q_full), 0);  // the Q copy lands before the CTA exits (bounded)
    if (direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)head * dp.out_stride_head +
             dh * kDH;
      for (int d = 0; d < kDH; d += 8) *reinterpret_cast<uint4*>(o + d) = make_uint4(0, 0, 0, 0);
    } else if (dh == 0) {
      float* part = dp.partials + (((int64_t)b * dp.n_q_heads + head) * dp.max_splits + s) * (kR + 2);
      part[0] = -INFINITY;
      part[1] = 0.f;
    }
  }

  // ---- every role is done with shared memory and TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge of the split partials: one warp per (sequence, head, 128 output dims);
// lanes read the splits' (max, sum) pairs in parallel, then every lane
// accumulates 4 dims over all splits with independent loads.
template <typename T>
__global__ void __launch_bounds__(256) sparse_mla_merge_kernel(DecodeParams dp, int n_splits) {
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int q4 = w & 3, h = (w >> 2) % kH, b = (w >> 2) / kH;
  if (b >= dp.batch) return;
  const int64_t pstride = kR + 2;
  const float* pg = dp.partials + ((int64_t)b * dp.n_q_heads + h) * dp.max_splits * pstride;
  float m_l[2], l_l[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int sp = lane + 32 * i;
    m_l[i] = sp < n_splits ? __ldcg(pg + sp * pstride) : -INFINITY;
    l_l[i] = sp < n_splits ? __ldcg(pg + sp * pstride + 1) : 0.f;
  }
  float M = fmaxf(m_l[0], m_l[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float f_l[2], L = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    f_l[i] = m_l[i] == -INFINITY ? 0.f : expf(m_l[i] - M);
    L += l_l[i] * f_l[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int d = q4 * 128 + lane * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // splits without attended tokens (factor 0) may hold stale values: select, never multiply
#pragma unroll 8
  for (int sp = 0; sp < n_splits; ++sp) {
    const float f = __shfl_sync(0xffffffffu, sp < 32 ? f_l[0] : f_l[1], sp & 31);
    const float2 a = __ldcg(reinterpret_cast<const float2*>(pg + sp * pstride + 2 + d));
    const float2 c = __ldcg(reinterpret_cast<const float2*>(pg + sp * pstride + 4 + d));
    if (f != 0.f) {
      acc[0] = fmaf(a.x, f, acc[0]);
      acc[1] = fmaf(a.y, f, acc[1]);
      acc[2] = fmaf(c.x, f, acc[2]);
      acc[3] = fmaf(c.y, f, acc[3]);
    }
  }
  T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head + d;
  *reinterpret_cast<uint2*>(o) = make_uint2(pack2<T>(acc[0] * inv, acc[1] * inv), pack2<T>(acc[2] * inv, acc[3] * inv));
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
      !tensor_map_col_blocks(&lat, bf16, p.latent, rows, kR * 2, kKB - 1, kBs) ||
      !tensor_map_2d(&rope, bf16, p.rope, kP, rows, kP * 2, 64, kBs)) {
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
    merge<<<dim3(p.batch * kH * 4 / 8), 256, 0, st>>>(p.dp, p.n_splits);
    return cuda_status(cudaGetLastError(), "sparse_mla_merge launch");
  };
  return bf16 ? go(sparse_mla_umma_kernel<__nv_bfloat16>, sparse_mla_merge_kernel<__nv_bfloat16>)
              : go(sparse_mla_umma_kernel<__half>, sparse_mla_merge_kernel<__half>);
}

}  // namespace snapmind
