// Sparse MLA decode on the 5th-generation tensor cores (tcgen05, sm_100a):
// 128 heads, kv_lora_rank 512, rope 64, 64-token blocks, bf16/f16.
//
// A decode step of DeepSeek-style absorbed MLA is, per sequence, a 128-row
// attention: Q [128 heads x 576] against the attended latent rows
// [n x 576] (latent 512 | rope 64), output [128 x 512] over the first 512
// columns of the same rows.  A full-width output accumulator (128 x 512 f32)
// would fill a whole SM's tensor memory and a full Q (144 KB) most of its
// shared memory, so four independent CTAs share each (split, sequence):
//   CTA q = 2 hh + dh owns heads [64 hh, 64 hh + 64) and output dims
//   [256 dh, 256 dh + 256).  Each scores its 64 heads over the full
//   576-wide contraction (tcgen05.mma with M = 64), so no partial result ever
//   crosses between CTAs; the two dh CTAs of a head half compute the same
//   scores (bit for bit: same inputs, same instruction sequence) and each
//   applies them to its own half of V.
// CTA = 6 warps: warps 0-3 softmax, warp 4 TMA producer, warp 5 MMA issuer.
//   Shared memory (1024-aligned, 128-byte swizzle, written by TMA):
//     Q: 9 k-blocks x [64 rows x 64] = 72 KB, resident;
//     2 stages of one attended chunk of 64 rows, 9 k-blocks x [64 x 64]
//       (72 KB: one 3-D TMA box for the 8 latent k-blocks, one 2-D box for
//       the rope k-block);
//     P: [64 heads x 64 tokens] bf16 = 8 KB, written by the softmax threads.
//   TMEM (M = 64 accumulators keep row m in lane 32 (m / 16) + m % 16):
//     O [64 x 256] f32 at column 0; two score buffers [64 x 64] at columns 256
//     and 320.
//   Per chunk of 64 tokens:
//     S = Q K^T: 36 MMAs (M 64, N 64, K 16), K-major operands;
//     softmax: warp w owns head rows 16 w .. 16 w + 15, four threads per row
//       (tcgen05.ld.16x256b: thread t holds rows t / 4 and t / 4 + 8, 16 of
//       the 64 tokens each; row maxima and sums take two shuffles); tokens
//       outside the selection are masked; a reference maximum is raised only
//       when a score exceeds it by 2^8 (then O's rows are rescaled in TMEM);
//       P = exp2(s - m) is written as bf16;
//     O += P V: 4 MMAs (M 64, N 256, K 16), V = this CTA's 4 latent k-blocks
//       of the staged rows, read MN-major.
//   The MMA warp issues whatever is ready (PV of the oldest chunk whose P is
//   written, else the scores of the next staged chunk), so the scores of the
//   next chunk overlap the softmax of the current one.  The producer keeps one
//   chunk loading and the next kPrefetch chunks prefetched into L2 (TMA
//   prefetch, no shared memory), so a stage that frees up is refilled from L2.
//   Handshakes are mbarriers (tcgen05.commit for the tensor core), every wait
//   is bounded (about a second) and ends early once another role gave up, and
//   TMEM is released on every path.
// Splits write fp32 partials (unnormalised output [sequence][split][dim][head],
// max and sum [sequence][split][2][head]) into the workspace region the paged
// GQA decode layout sizes for them; a second kernel merges them.
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

constexpr int kH = 128;                                 // heads of a sequence
constexpr int kHC = 64;                                 // heads per CTA = MMA M
constexpr int kR = 512, kP = 64;
constexpr int kKB = (kR + kP) / 64;                     // 9 k-blocks of 64 elements
constexpr int kBs = 64;                                 // block (chunk) size = tokens per score tile
constexpr int kDH = kR / 2;                             // output dims per CTA
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr int kThreads = 192;
constexpr uint32_t kQBlock = kHC * 128;                 // one k-block of Q: 8 KB
constexpr uint32_t kQBytes = kKB * kQBlock;             // 72 KB
constexpr uint32_t kStBlock = kBs * 128;                // one k-block of a chunk: 8 KB
constexpr uint32_t kStageBytes = kKB * kStBlock;        // 72 KB
constexpr int kStages = 2;
constexpr uint32_t kPBytes = kHC * kBs * 2;             // 8 KB
constexpr int kBits = 3072;                             // chunks per sequence (bitmaps; longer tables take the mma.sync kernel)
constexpr uint32_t kTmemCols = 512, kColO = 0, kColS = 256;
constexpr float kRescale = 8.f;                         // log2 headroom of the reference maximum
constexpr int kPrefetch = 4;                            // chunks prefetched into L2 ahead of the load
constexpr int kRing = 64;                               // resolved (chunk, block) pairs kept ahead

struct Ctrl {
  uint64_t full[kStages];    // producer -> MMA, softmax: chunk staged
  uint64_t empty[kStages];   // MMA commit after O += P V of the chunk: stage free
  uint64_t s_full[2];        // MMA commit after S = Q K^T: buffer ready
  uint64_t s_empty[2];       // softmax threads: buffer read
  uint64_t q_full;
  uint64_t p_full;           // softmax threads: P written (and O rescaled)
  uint64_t o_done;           // MMA commit after O += P V
  uint32_t tmem_base;
  int32_t abort;
  int32_t count;
  int32_t chunk_phys[kStages];  // block and chunk id of each staged chunk
  int32_t chunk_id[kStages];
  int32_t ring_c[kRing];        // chunk id and block of chunk j of the split at j % kRing
  int32_t ring_p[kRing];
  uint32_t sel_bits[kBits / 32];
  uint32_t inc_bits[kBits / 32];
  int32_t word_pre[kBits / 32 + 1];
};

constexpr size_t kSmemBytes = 1024 + kQBytes + kStages * kStageBytes + kPBytes + sizeof(Ctrl);
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

// Maximum over the four threads that share a row (lanes 4 r .. 4 r + 3).
__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
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
  uint8_t* st_s = q_s + kQBytes;
  uint8_t* p_s = st_s + kStages * kStageBytes;
  Ctrl& C = *reinterpret_cast<Ctrl*>(p_s + kPBytes);

  const int hh = blockIdx.x >> 1, dh = blockIdx.x & 1;  // head half, output-dim half
  const int s = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBf16, kHC, kBs, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBf16, kHC, kDH, false, true);
  const DecodeParams& dp = p.dp;
  const int q_row0 = b * kH + hh * kHC;  // first row of this CTA's heads in q_lat / q_pe

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&C.full[i]), 1);
      mbar_init(smem_u32(&C.empty[i]), 1);
    }
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
    tma_load_3d(smem_u32(q_s), &qlat_map, 0, q_row0, 0, qb);  // the 8 latent k-blocks
    tma_load_2d(smem_u32(q_s + (kKB - 1) * kQBlock), &qpe_map, 0, q_row0, qb);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }

  // ---- attended chunks of sequence b: bitmaps and the prefix of their counts
  // (the length and the first selected ids are loaded together)
  const int sel0 = tid < p.k ? p.selected[(int64_t)b * p.k + tid] : -1;
  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  int n_chunks = (len + kBs - 1) / kBs;
  if (n_chunks > kBits) {
    if (tid == 0 && s == 0 && blockIdx.x == 0) flag_error(dp.err, SNAPMIND_DEVERR_TABLE);
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
    const int c = i == tid ? sel0 : p.selected[(int64_t)b * p.k + i];
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

  // chunks of this split (the same for the four CTAs of a (split, sequence))
  const int per = (count + p.n_splits - 1) / max(p.n_splits, 1);
  const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);
  const int n_ck = c_hi - c_lo;
  const bool direct = (p.n_splits == 1);

  if (n_ck > 0) {
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------------- TMA producer
      // The warp resolves the blocks of 32 chunks at a time (one table read per lane)
      // into a ring; lane 0 loads chunk i into stage i % 2 once PV(i - 2) freed it,
      // and keeps chunks up to i + kPrefetch prefetched into L2, so a load that
      // waited for its stage finds its rows there.
      int located = 0, prefetched = min(n_ck, kStages), issued = 0;
      bool ok = true;
      for (int i = 0; i < n_ck && ok; ++i) {
        if (min(n_ck, i + kPrefetch + 1) > located) {  // warp-uniform
          const int j = located + lane;
          if (j < n_ck) {
            const int c = chunk_of_rank(C, words, c_lo + j);
            int32_t phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
            if (phys >= p.num_blocks) phys = -1;
            C.ring_c[j % kRing] = c;
            C.ring_p[j % kRing] = phys;
          }
          __syncwarp();
          located += 32;
        }
        if (lane == 0) {
          const int st = i % kStages;
          if (i >= kStages && !role_wait(C, smem_u32(&C.empty[st]), ((i / kStages) - 1) & 1)) {
            give_up(C, dp.err);
            ok = false;
          } else {
            const int32_t phys = C.ring_p[i % kRing];
            C.chunk_phys[st] = phys;
            C.chunk_id[st] = C.ring_c[i % kRing];
            const uint32_t bar = smem_u32(&C.full[st]);
            if (phys < 0) {
              flag_error(dp.err, SNAPMIND_DEVERR_BLOCK_ID);
              mbar_arrive(bar);
            } else {
              uint8_t* stage = st_s + st * kStageBytes;
              mbar_arrive_expect_tx(bar, kStageBytes);
              const int y = phys * kBs;
              tma_load_3d(smem_u32(stage), &lat_map, 0, y, 0, bar);  // the 8 latent k-blocks
              tma_load_2d(smem_u32(stage + (kKB - 1) * kStBlock), &rope_map, 0, y, bar);
            }
            issued = i + 1;
            for (; prefetched < min(n_ck, i + kPrefetch + 1); ++prefetched) {
              const int32_t pp = C.ring_p[prefetched % kRing];
              if (pp >= 0) {
                tma_prefetch_3d(&lat_map, 0, pp * kBs, 0);
                tma_prefetch_2d(&rope_map, 0, pp * kBs);
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (lane == 0) {
        // before the shared memory is released: every copy issued has landed (bounded)
        for (int j = max(0, issued - kStages); j < issued; ++j)
          mbar_wait(smem_u32(&C.full[j % kStages]), (j / kStages) & 1);
        mbar_wait(smem_u32(&C.q_full), 0);
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- MMA issuer
      if (lane == 0) {
        bool ok = role_wait(C, smem_u32(&C.q_full), 0);
        uint32_t last_bar = 0, last_parity = 0;  // the latest commit: covers every MMA issued
        auto issue_s = [&](int i) {  // S = Q K^T of chunk i over the full 576 columns
          const uint8_t* stage = st_s + (i % kStages) * kStageBytes;
          const uint32_t d = tmem + kColS + (i & 1) * kBs;
          tc_fence_after();
#pragma unroll 1
          for (int kb = 0; kb < kKB; ++kb) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc(smem_u32(q_s + kb * kQBlock + kk * 32), 16, 1024, kSwizzle128B);
              const uint64_t bd = smem_desc(smem_u32(stage + kb * kStBlock + kk * 32), 16, 1024, kSwizzle128B);
              umma_f16(d, ad, bd, kIdescS, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(smem_u32(&C.s_full[i & 1]));
          last_bar = smem_u32(&C.s_full[i & 1]);
          last_parity = (i >> 1) & 1;
        };
        auto issue_pv = [&](int i) {  // O += P V of chunk i (this CTA's 256 output dims)
          const uint8_t* v = st_s + (i % kStages) * kStageBytes + dh * 4 * kStBlock;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kBs / 16; ++ks) {
            const uint64_t ad = smem_desc(smem_u32(p_s + ks * 32), 16, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(smem_u32(v + ks * 16 * 128), kStBlock, 1024, kSwizzle128B);
            umma_f16(tmem + kColO, ad, bd, kIdescPV, (i > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&C.empty[i % kStages]));
          umma_commit(smem_u32(&C.o_done));
          last_bar = smem_u32(&C.o_done);
          last_parity = i & 1;
        };
        // Issue whichever is ready: O += P V of the oldest chunk whose P is written (it
        // frees a stage), else the scores of the next staged chunk (at most two score
        // buffers ahead).  Between polls the thread backs off briefly, leaving the
        // issue slots of its SM sub-partition to the softmax warp there.
        int ns = 0, np = 0;  // next chunk to score, next chunk for O += P V
        long long idle_since = clock64();
        while (ok && np < n_ck) {
          bool progressed = false;
          if (np < ns && mbar_test_wait(smem_u32(&C.p_full), np & 1)) {
            issue_pv(np++);
            progressed = true;
          } else if (ns < n_ck && mbar_test_wait(smem_u32(&C.full[ns % kStages]), (ns / kStages) & 1) &&
                     (ns < 2 || mbar_test_wait(smem_u32(&C.s_empty[ns & 1]), ((ns >> 1) - 1) & 1))) {
            issue_s(ns++);
            progressed = true;
          }
          if (progressed) {
            idle_since = clock64();
          } else if (*reinterpret_cast<const volatile int32_t*>(&C.abort) || clock64() - idle_since > kWaitTicks) {
            ok = false;
          } else {
            __nanosleep(32);
          }
        }
        if (!ok) {
          give_up(C, dp.err);
          if (last_bar) mbar_wait(last_bar, last_parity);  // MMAs in flight finish (bounded) before TMEM goes
        }
      }
    } else {
      // ---------------------------------------------------------------- softmax warps 0-3
      // thread: rows ra = 16 warp + lane / 4 and rb = ra + 8 of this CTA's 64 heads,
      // tokens 8 j + 2 cq + {0, 1} of every chunk (j = 0..7)
      const int cq = lane & 3;
      const int ra = warp * 16 + (lane >> 2), rb = ra + 8;
      const uint32_t t_w = tmem + ((uint32_t)(warp * 32) << 16);
      const float c2 = p.scale * 1.4426950408889634f;
      float ma_ref = -INFINITY, mb_ref = -INFINITY, la = 0.f, lb = 0.f;  // log2 units of score * scale
      uint8_t* prow_a = p_s + ra * 128;
      uint8_t* prow_b = p_s + rb * 128;
      const uint32_t psw = (uint32_t)(ra & 7);  // rb & 7 is the same
      bool ok = true;
      for (int i = 0; i < n_ck; ++i) {
        const int st = i % kStages, sb = i & 1;
        ok = role_wait(C, smem_u32(&C.full[st]), (i / kStages) & 1) &&
             role_wait(C, smem_u32(&C.s_full[sb]), (i >> 1) & 1);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
        const int phys = C.chunk_phys[st], c = C.chunk_id[st];
        const int pos0 = c * kBs;
        const int good = phys < 0 ? 0 : max(0, min(kBs, len - pos0));  // rows holding a token
        // attended tokens of the chunk as a bit mask: [0, good) for a selected chunk,
        // else [0, min(good, sink - pos0)) and [max(0, wstart - pos0), good)
        uint64_t vmask;
        {
          const uint64_t below_good = good >= 64 ? ~0ull : ((1ull << good) - 1ull);
          const bool selected = phys >= 0 && ((C.sel_bits[c >> 5] >> (c & 31)) & 1u);
          if (selected) {
            vmask = below_good;
          } else {
            const int a = max(0, min(64, sink - pos0));
            const int w = max(0, min(64, wstart - pos0));
            const uint64_t sink_bits = a >= 64 ? ~0ull : ((1ull << a) - 1ull);
            const uint64_t win_bits = w >= 64 ? 0ull : ~((1ull << w) - 1ull);
            vmask = (sink_bits | win_bits) & below_good;
          }
        }
        const uint64_t tmask = vmask >> (2 * cq);  // bit 8 j + e: token 8 j + 2 cq + e
        tc_fence_after();
        float sv[32];
        tmem_ld16x256b_x8(t_w + kColS + sb * kBs, sv);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(smem_u32(&C.s_empty[sb]));
        // masked row maxima (raw scores; scale > 0)
        float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool on = (tmask >> (8 * j + e)) & 1ull;
            mxa = fmaxf(mxa, on ? sv[4 * j + e] : -INFINITY);
            mxb = fmaxf(mxb, on ? sv[4 * j + 2 + e] : -INFINITY);
          }
        }
        const float mta = quad_max(mxa) * c2, mtb = quad_max(mxb) * c2;
        const bool raise_a = mta > ma_ref + kRescale, raise_b = mtb > mb_ref + kRescale;
        const float ma_old = ma_ref, mb_old = mb_ref;
        ma_ref = raise_a ? mta : ma_ref;
        mb_ref = raise_b ? mtb : mb_ref;
        // P = 2^(s c2 - m) for attended tokens, 0 elsewhere
        uint32_t pa[8], pb[8];
        float sa = 0.f, sb_ = 0.f;  // this chunk's terms (added after any rescale of la, lb)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool on0 = (tmask >> (8 * j)) & 1ull, on1 = (tmask >> (8 * j + 1)) & 1ull;
          const float a0 = on0 ? ex2_approx(fmaf(sv[4 * j], c2, -ma_ref)) : 0.f;
          const float a1 = on1 ? ex2_approx(fmaf(sv[4 * j + 1], c2, -ma_ref)) : 0.f;
          const float b0 = on0 ? ex2_approx(fmaf(sv[4 * j + 2], c2, -mb_ref)) : 0.f;
          const float b1 = on1 ? ex2_approx(fmaf(sv[4 * j + 3], c2, -mb_ref)) : 0.f;
          sa += a0 + a1;
          sb_ += b0 + b1;
          pa[j] = pack2<T>(a0, a1);
          pb[j] = pack2<T>(b0, b1);
        }
        // O += P V of the previous chunk has finished: P is free and O holds it
        if (i >= 1) {
          ok = role_wait(C, smem_u32(&C.o_done), (i - 1) & 1);
          if (__any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        const bool resc_a = raise_a && ma_old != -INFINITY, resc_b = raise_b && mb_old != -INFINITY;
        if (__any_sync(0xffffffffu, resc_a || resc_b)) {
          // O rows of this warp at the old reference maxima: rescale in TMEM
          const float alpha_a = resc_a ? exp2f(ma_old - ma_ref) : 1.f;
          const float alpha_b = resc_b ? exp2f(mb_old - mb_ref) : 1.f;
#pragma unroll 1
          for (int cc = 0; cc < kDH; cc += 64) {
            float o[32];
            tmem_ld16x256b_x8(t_w + kColO + cc, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              o[4 * j] *= alpha_a;
              o[4 * j + 1] *= alpha_a;
              o[4 * j + 2] *= alpha_b;
              o[4 * j + 3] *= alpha_b;
            }
            tmem_st16x256b_x8(t_w + kColO + cc, o);
          }
          tmem_wait_st();
          la *= alpha_a;
          lb *= alpha_b;
        }
        la += sa;
        lb += sb_;
        // rows ra, rb of P: 128 bytes each, 128-byte swizzle (16-byte piece j at j ^ (row & 7))
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t off = (((uint32_t)j ^ psw) << 4) + 4 * cq;
          *reinterpret_cast<uint32_t*>(prow_a + off) = pa[j];
          *reinterpret_cast<uint32_t*>(prow_b + off) = pb[j];
        }
        if (good < kBs) {  // rows holding no token: zero this CTA's V columns (the scores are done)
          uint8_t* v = st_s + st * kStageBytes + dh * 4 * kStBlock;
          const int rows = kBs - good;
          for (int e = tid; e < 4 * rows * 8; e += kSoftmaxThreads) {
            const int kb = e / (rows * 8);
            const int row = good + (e / 8) % rows;
            *reinterpret_cast<uint4*>(v + kb * kStBlock + row * 128 + (e & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(smem_u32(&C.p_full));
      }
      if (ok) {
        ok = role_wait(C, smem_u32(&C.o_done), (n_ck - 1) & 1);
        ok = !__any_sync(0xffffffffu, !ok);
      }
      if (!ok) {
        give_up(C, dp.err);
      } else {
        // ---- epilogue: rows ra, rb of O (256 columns)
        tc_fence_after();
        const float lta = quad_sum(la), ltb = quad_sum(lb);
        const float inv_a = lta > 0.f ? 1.f / lta : 0.f, inv_b = ltb > 0.f ? 1.f / ltb : 0.f;
        const int ha = hh * kHC + ra, hb = hh * kHC + rb;
        // partials [sequence][split][dim][head], then max and sum [sequence][split][2][head]
        const int64_t bs_ = (int64_t)b * p.n_splits + s;
        float* part = dp.partials + (bs_ * kR + dh * kDH) * kH;
        float* ml = dp.partials + (int64_t)p.batch * p.n_splits * kR * kH + bs_ * 2 * kH;
        T* out_a = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)ha * dp.out_stride_head +
                   dh * kDH;
        T* out_b = out_a + 8 * dp.out_stride_head;
#pragma unroll 1
        for (int cc = 0; cc < kDH; cc += 64) {
          float o[32];
          tmem_ld16x256b_x8(t_w + kColO + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int d = cc + 8 * j + 2 * cq;
            if (direct) {
              *reinterpret_cast<uint32_t*>(out_a + d) = pack2<T>(o[4 * j] * inv_a, o[4 * j + 1] * inv_a);
              *reinterpret_cast<uint32_t*>(out_b + d) = pack2<T>(o[4 * j + 2] * inv_b, o[4 * j + 3] * inv_b);
            } else {
              part[(int64_t)d * kH + ha] = o[4 * j];
              part[(int64_t)(d + 1) * kH + ha] = o[4 * j + 1];
              part[(int64_t)d * kH + hb] = o[4 * j + 2];
              part[(int64_t)(d + 1) * kH + hb] = o[4 * j + 3];
            }
          }
        }
        if (!direct && dh == 0 && cq == 0) {
          ml[ha] = ma_ref == -INFINITY ? -INFINITY : ma_ref * 0.6931471805599453f;  // natural-log units
          ml[hb] = mb_ref == -INFINITY ? -INFINITY : mb_ref * 0.6931471805599453f;
          ml[kH + ha] = lta;
          ml[kH + hb] = ltb;
        }
      }
    }
  } else if (tid < kHC) {
    // no chunk in this split: an empty partial (or a zero output when nothing is attended)
    const int h = hh * kHC + tid;
    if (tid == 0) mbar_wait(smem_u32(&C.q_full), 0);  // the Q copy lands before the CTA exits (bounded)
    if (direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head +
             dh * kDH;
      for (int d = 0; d < kDH; d += 8) *reinterpret_cast<uint4*>(o + d) = make_uint4(0, 0, 0, 0);
    } else if (dh == 0) {
      float* ml = dp.partials + (int64_t)p.batch * p.n_splits * kR * kH + ((int64_t)b * p.n_splits + s) * 2 * kH;
      ml[h] = -INFINITY;
      ml[kH + h] = 0.f;
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

// Merge of the split partials: CTA = (sequence, 16 output dims), thread = head.
// Every load of a warp reads 32 heads of one (split, dim): one 128-byte line.
// Splits without attended tokens (weight 0) may hold stale values: their
// terms are skipped, never multiplied.
constexpr int kMergeDims = 16;

template <typename T>
__global__ void __launch_bounds__(kH) sparse_mla_merge_kernel(DecodeParams dp, int n_splits) {
  const int b = blockIdx.x / (kR / kMergeDims), d0 = (blockIdx.x % (kR / kMergeDims)) * kMergeDims;
  const int h = threadIdx.x;
  if (b >= dp.batch) return;
  const float* ml = dp.partials + (int64_t)dp.batch * n_splits * kR * kH + (int64_t)b * n_splits * 2 * kH + h;
  float M = -INFINITY;
  for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, __ldcg(ml + sp * 2 * kH));
  float L = 0.f, acc[kMergeDims];
#pragma unroll
  for (int j = 0; j < kMergeDims; ++j) acc[j] = 0.f;
  const float* part = dp.partials + ((int64_t)b * n_splits * kR + d0) * kH + h;
  for (int sp = 0; sp < n_splits; ++sp) {
    const float m = __ldcg(ml + sp * 2 * kH);
    if (m == -INFINITY) continue;
    const float f = expf(m - M);
    L = fmaf(__ldcg(ml + sp * 2 * kH + kH), f, L);
    const float* ps = part + (int64_t)sp * kR * kH;
    float v[kMergeDims];
#pragma unroll
    for (int j = 0; j < kMergeDims; ++j) v[j] = __ldcg(ps + j * kH);
#pragma unroll
    for (int j = 0; j < kMergeDims; ++j) acc[j] = fmaf(v[j], f, acc[j]);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head + d0;
#pragma unroll
  for (int j = 0; j < kMergeDims; j += 8)
    *reinterpret_cast<uint4*>(o + j) =
        make_uint4(pack2<T>(acc[j] * inv, acc[j + 1] * inv), pack2<T>(acc[j + 2] * inv, acc[j + 3] * inv),
                   pack2<T>(acc[j + 4] * inv, acc[j + 5] * inv), pack2<T>(acc[j + 6] * inv, acc[j + 7] * inv));
}

}  // namespace

int sparse_mla_umma_splits(int batch) {
  const int per_seq = num_sms() / (4 * (batch > 0 ? batch : 1));  // 4 CTAs per (split, sequence)
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
  // Q rows of 64 heads and chunk rows of 64 tokens: all 8 latent k-blocks in one 3-D box, rope in a 2-D box
  if (!tensor_map_col_blocks(&qlat, bf16, p.q_lat, (uint64_t)p.batch * kH, kR * 2, kR / 64, kHC) ||
      !tensor_map_2d(&qpe, bf16, p.q_pe, kP, (uint64_t)p.batch * kH, kP * 2, 64, kHC) ||
      !tensor_map_col_blocks(&lat, bf16, p.latent, rows, kR * 2, kR / 64, kBs) ||
      !tensor_map_2d(&rope, bf16, p.rope, kP, rows, kP * 2, 64, kBs)) {
    set_last_error("sparse_mla_umma: tensor map encoding failed");
    return SNAPMIND_ERR_CUDA;
  }
  // one flag per instantiation: both kernels have the same function type
  static bool attr_set[2] = {false, false};
  auto go = [&](auto kernel, auto merge) -> int {
    bool& attr = attr_set[bf16 ? 0 : 1];
    if (!attr) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e != cudaSuccess) return cuda_status(e, "sparse_mla_umma smem attribute");
      attr = true;
    }
    // x = 2 (head half) + (output-dim half)
    kernel<<<dim3(4, p.n_splits, p.batch), kThreads, kSmemBytes, st>>>(qlat, qpe, lat, rope, p);
    int rc = cuda_status(cudaGetLastError(), "sparse_mla_umma launch");
    if (rc != SNAPMIND_OK || p.n_splits == 1) return rc;
    merge<<<dim3(p.batch * (kR / kMergeDims)), kH, 0, st>>>(p.dp, p.n_splits);
    return cuda_status(cudaGetLastError(), "sparse_mla_merge launch");
  };
  return bf16 ? go(sparse_mla_umma_kernel<__nv_bfloat16>, sparse_mla_merge_kernel<__nv_bfloat16>)
              : go(sparse_mla_umma_kernel<__half>, sparse_mla_merge_kernel<__half>);
}

}  // namespace snapmind
