// Sparse MLA decode on the 5th-generation tensor cores (tcgen05, sm_100a):
// 128 heads, kv_lora_rank 512, rope 64, 64-token blocks, bf16/f16.
//
// A decode step of DeepSeek-style absorbed MLA is, per sequence, a 128-row
// attention: Q [128 heads x 576] against the attended latent rows
// [n x 576] (latent 512 | rope 64), output [128 x 512] over the first 512
// columns of the same rows.  The 128 heads are the M = 128 of one
// tcgen05.mma.  The output accumulator (128 x 512 f32) would fill a whole
// SM's tensor memory, so two CTAs of a cluster share each (split, sequence):
//   CTA r (cluster rank r = 0, 1) owns latent columns [256 r, 256 r + 256)
//   and rope columns [32 r, 32 r + 32), a split of the 576-wide contraction
//   whose latent part is also exactly the V columns of its output half.
//   Each attended row is therefore loaded once per pair (288 columns into
//   each CTA), and each CTA computes a partial score tile
//   S_r = Q[:, cols r] K[:, cols r]^T; the two partial tiles are exchanged
//   through distributed shared memory and added, in the same order-free way
//   (a + b == b + a in IEEE arithmetic) on both sides, so both CTAs hold
//   bit-identical scores, softmax state and P.
// CTA = 6 warps: warps 0-3 softmax (thread = head row = TMEM lane), warp 4
// TMA producer, warp 5 MMA issuer.  Shared memory (1024-aligned):
//   Q part: 4 latent k-blocks [128 rows x 64] (128-byte swizzle, 64 KB) and
//     the rope half [128 x 32] (64-byte swizzle, 8 KB), resident;
//   3 stages of one attended chunk of 64 rows: 4 latent k-blocks [64 x 64]
//     (32 KB, one 3-D TMA box) and the rope half [64 x 32] (4 KB);
//   X (32 KB): the peer's partial scores of the current chunk, row h's 64
//     fp32 in two 128-byte halves at h * 128 (tokens 0-31) and
//     16 KB + h * 128 (tokens 32-63), 16-byte pieces swizzled by (h & 7).
//     P [128 x 64] (bf16, 128-byte swizzle, the A operand of O += P V)
//     overwrites the first half after the thread read it: row h of P is
//     exactly the bytes of row h's first half, so only thread h touches them.
//   TMEM: O [128 x 256] f32 (this CTA's output half) at column 0; two
//     partial score buffers [128 x 64] at columns 256 and 320.
// Per chunk of 64 tokens:
//   MMA: S_r = 18 MMAs (M 128, N 64, K 16) into a score buffer; later
//     O += P V: 4 MMAs (M 128, N 256, K 16), V = the staged latent rows read
//     MN-major.  Commits free the stage and mark O current.
//   softmax thread h: loads its partial row from TMEM; once its own previous
//     O += P V has completed (P and O are free) it tells the peer that its X
//     may be overwritten; once the peer says the same, it stores its partial
//     row into the peer's X (st.shared::cluster) and arrives on the peer's
//     barrier; it waits for the peer's row in its own X, adds, masks the
//     tokens outside the selection, keeps a reference maximum that is raised
//     only when a score exceeds it by 2^8 (then O's row is rescaled in TMEM),
//     and writes P = exp2(s - m) as bf16.
// Every wait is bounded (about a second) and ends early once a role of
// either CTA gave up; a CTA that gives up also raises the peer's abort flag.
// All threads of both CTAs meet at a cluster barrier before exit, so neither
// leaves while the other may still write into its shared memory.  TMEM is
// released on every path.  Nothing here touches another GPU's memory; the
// TMA loads carry no multicast.
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
constexpr int kBs = 64;                                 // block (chunk) size = tokens per score tile
constexpr int kLatBlocks = 4;                           // latent k-blocks of 64 columns per CTA
constexpr int kRopeHalf = kP / 2;                       // rope columns per CTA
constexpr int kDH = kR / 2;                             // output dims per CTA
constexpr int kSoftmaxThreads = 128;                    // warps 0-3: one head row per thread
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr int kThreads = 192;
constexpr uint32_t kQBlock = kH * 128;                  // one latent k-block of Q: 16 KB
constexpr uint32_t kQLatBytes = kLatBlocks * kQBlock;   // 64 KB
constexpr uint32_t kQRopeBytes = kH * kRopeHalf * 2;    // 8 KB
constexpr uint32_t kStBlock = kBs * 128;                // one latent k-block of a chunk: 8 KB
constexpr uint32_t kStLatBytes = kLatBlocks * kStBlock; // 32 KB
constexpr uint32_t kStRopeBytes = kBs * kRopeHalf * 2;  // 4 KB
constexpr uint32_t kStageBytes = kStLatBytes + kStRopeBytes;
constexpr int kStages = 3;
constexpr uint32_t kXHalf = kH * 128;                   // 16 KB: 32 fp32 per row
constexpr uint32_t kXBytes = 2 * kXHalf;
constexpr int kBits = 4096;                             // chunks per sequence (bitmaps)
constexpr uint32_t kTmemCols = 512, kColO = 0, kColS = 256;
constexpr float kRescale = 8.f;                         // log2 headroom of the reference maximum
static_assert(kStageBytes % 1024 == 0 && kQLatBytes % 1024 == 0 && (kQLatBytes + kQRopeBytes) % 1024 == 0,
              "swizzled tiles stay 1024-byte aligned");

struct Ctrl {
  uint64_t full[kStages];    // producer -> MMA, softmax: chunk staged
  uint64_t empty[kStages];   // MMA commit after O += P V of the chunk: stage free
  uint64_t s_full[2];        // MMA commit after the partial scores: buffer ready
  uint64_t s_empty[2];       // softmax threads: buffer read
  uint64_t q_full;
  uint64_t p_full;           // softmax threads: P written (and O rescaled)
  uint64_t o_done;           // MMA commit after O += P V
  uint64_t x_full;           // the peer's 128 threads: their partial scores are in X
  uint64_t x_empty;          // the peer's 128 threads: the peer's X may take ours
  uint32_t tmem_base;
  int32_t abort;             // set by a role of this CTA or of the peer that gave up
  int32_t count;
  int32_t chunk_phys[kStages];  // block and chunk id of each staged chunk
  int32_t chunk_id[kStages];
  uint32_t sel_bits[kBits / 32];
  uint32_t inc_bits[kBits / 32];
  int32_t word_pre[kBits / 32 + 1];
};

constexpr size_t kSmemBytes = 1024 + kQLatBytes + kQRopeBytes + kStages * kStageBytes + kXBytes + sizeof(Ctrl);
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

__device__ __forceinline__ bool aborted(const Ctrl& C) {
  return *reinterpret_cast<const volatile int32_t*>(&C.abort) != 0;
}

// Waits of the pipeline roles: bounded, and cut short once a role of either CTA gave up.
__device__ __forceinline__ bool role_wait(const Ctrl& C, uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (aborted(C) || clock64() - t0 > kWaitTicks) return false;
  }
  return true;
}
// The same for a barrier the peer CTA arrives on (acquire at cluster scope).
__device__ __forceinline__ bool peer_wait(const Ctrl& C, uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (aborted(C) || clock64() - t0 > kWaitTicks) return false;
  }
  return true;
}

__device__ __forceinline__ void give_up(Ctrl& C, uint32_t peer_abort, int32_t* err) {
  atomicExch(&C.abort, 1);
  st_cluster_u32(peer_abort, 1u);
  flag_error(err, SNAPMIND_DEVERR_TIMEOUT);
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    sparse_mla_umma_kernel(const __grid_constant__ CUtensorMap qlat_map, const __grid_constant__ CUtensorMap qpe_map,
                           const __grid_constant__ CUtensorMap lat_map, const __grid_constant__ CUtensorMap rope_map,
                           SparseParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = base;
  uint8_t* q_rope = q_s + kQLatBytes;
  uint8_t* st_s = q_rope + kQRopeBytes;
  uint8_t* x_s = st_s + kStages * kStageBytes;
  Ctrl& C = *reinterpret_cast<Ctrl*>(x_s + kXBytes);

  const uint32_t r = cluster_ctarank();  // contraction half and output half of this CTA
  const uint32_t peer = r ^ 1u;
  const int s = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBf16, kH, kBs, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBf16, kH, kDH, false, true);
  const DecodeParams& dp = p.dp;
  const uint32_t peer_abort = mapa_shared(smem_u32(&C.abort), peer);

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
    mbar_init(smem_u32(&C.x_full), kSoftmaxThreads);
    mbar_init(smem_u32(&C.x_empty), kSoftmaxThreads);
    C.abort = 0;
    mbar_init_fence();
    // Q depends only on the sequence: its copy overlaps the selection set-up below
    const uint32_t qb = smem_u32(&C.q_full);
    mbar_arrive_expect_tx(qb, kQLatBytes + kQRopeBytes);
    tma_load_3d(smem_u32(q_s), &qlat_map, 0, b * kH, kLatBlocks * (int)r, qb);
    tma_load_2d(smem_u32(q_rope), &qpe_map, kRopeHalf * (int)r, b * kH, qb);
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
    if (tid == 0 && s == 0 && r == 0) flag_error(dp.err, SNAPMIND_DEVERR_TABLE);
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
  // both CTAs' barriers are initialised before either arrives on the other's
  cluster_sync_all();
  const uint32_t tmem = C.tmem_base;
  const int count = C.count;

  // chunks of this split (the same for both CTAs of the pair)
  const int per = (count + p.n_splits - 1) / max(p.n_splits, 1);
  const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);
  const int n_ck = c_hi - c_lo;
  const bool direct = (p.n_splits == 1);

  if (n_ck > 0) {
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------------- TMA producer
      if (lane == 0) {
        // block of the i-th chunk of the split, resolved before its stage frees up
        auto locate = [&](int i, int& c, int32_t& phys) {
          c = chunk_of_rank(C, words, c_lo + i);
          phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
          if (phys >= p.num_blocks) phys = -1;
        };
        int c_next;
        int32_t phys_next;
        locate(0, c_next, phys_next);
        int issued = 0;
        for (int i = 0; i < n_ck; ++i) {
          const int st = i % kStages;
          const int c = c_next;
          const int32_t phys = phys_next;
          if (i >= kStages && !role_wait(C, smem_u32(&C.empty[st]), ((i / kStages) - 1) & 1)) {
            give_up(C, peer_abort, dp.err);
            break;
          }
          C.chunk_phys[st] = phys;
          C.chunk_id[st] = c;
          const uint32_t bar = smem_u32(&C.full[st]);
          if (phys < 0) {
            flag_error(dp.err, SNAPMIND_DEVERR_BLOCK_ID);
            mbar_arrive(bar);
          } else {
            uint8_t* stage = st_s + st * kStageBytes;
            mbar_arrive_expect_tx(bar, kStageBytes);
            const int y = phys * kBs;
            tma_load_3d(smem_u32(stage), &lat_map, 0, y, kLatBlocks * (int)r, bar);  // 4 latent k-blocks
            tma_load_2d(smem_u32(stage + kStLatBytes), &rope_map, kRopeHalf * (int)r, y, bar);
          }
          issued = i + 1;
          if (i + 1 < n_ck) locate(i + 1, c_next, phys_next);
        }
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
        auto issue_pv = [&](int i) {  // O += P V of chunk i
          const uint8_t* stage = st_s + (i % kStages) * kStageBytes;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kBs / 16; ++ks) {
            const uint64_t ad = smem_desc(smem_u32(x_s + ks * 32), 16, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(smem_u32(stage + ks * 16 * 128), kStBlock, 1024, kSwizzle128B);
            umma_f16(tmem + kColO, ad, bd, kIdescPV, (i > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&C.empty[i % kStages]));
          umma_commit(smem_u32(&C.o_done));
          last_bar = smem_u32(&C.o_done);
          last_parity = i & 1;
        };
        auto issue_s = [&](int i) {  // partial scores of chunk i over this CTA's 288 columns
          const uint8_t* stage = st_s + (i % kStages) * kStageBytes;
          const uint32_t d = tmem + kColS + (i & 1) * kBs;
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < kLatBlocks; ++j) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc(smem_u32(q_s + j * kQBlock + kk * 32), 16, 1024, kSwizzle128B);
              const uint64_t bd = smem_desc(smem_u32(stage + j * kStBlock + kk * 32), 16, 1024, kSwizzle128B);
              umma_f16(d, ad, bd, kIdescS, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(q_rope + kk * 32), 16, 512, kSwizzle64B);
            const uint64_t bd = smem_desc(smem_u32(stage + kStLatBytes + kk * 32), 16, 512, kSwizzle64B);
            umma_f16(d, ad, bd, kIdescS, 1u);
          }
          umma_commit(smem_u32(&C.s_full[i & 1]));
          last_bar = smem_u32(&C.s_full[i & 1]);
          last_parity = (i >> 1) & 1;
        };
        // Issue whichever is ready: O += P V of the oldest chunk whose P is written
        // (it frees a stage for the producer), else the scores of the next staged
        // chunk (at most two score buffers ahead of the softmax).
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
          } else if (aborted(C) || clock64() - idle_since > kWaitTicks) {
            ok = false;
          }
        }
        if (!ok) {
          give_up(C, peer_abort, dp.err);
          if (last_bar) mbar_wait(last_bar, last_parity);  // MMAs in flight finish (bounded) before TMEM goes
        }
      }
    } else {
      // ---------------------------------------------------------------- softmax warps 0-3
      const int h = tid;  // TMEM lane = head row
      const uint32_t t_row = tmem + ((uint32_t)(warp * 32) << 16);
      const float c2 = p.scale * 1.4426950408889634f;
      const uint32_t sw = (uint32_t)(h & 7) << 4;
      const uint32_t x_lo = smem_u32(x_s) + h * 128, x_hi = x_lo + kXHalf;  // row h, tokens 0-31 / 32-63
      const uint32_t px_lo = mapa_shared(x_lo, peer), px_hi = mapa_shared(x_hi, peer);
      const uint32_t peer_xfull = mapa_shared(smem_u32(&C.x_full), peer);
      const uint32_t peer_xempty = mapa_shared(smem_u32(&C.x_empty), peer);
      float m_ref = -INFINITY, l_run = 0.f;  // log2 units of score * scale
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
        tc_fence_after();
        float sv[kBs];
        tmem_ld32(t_row + kColS + sb * kBs, sv);
        tmem_ld32(t_row + kColS + sb * kBs + 32, sv + 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(smem_u32(&C.s_empty[sb]));
        if (i >= 1) {
          // O += P V of the previous chunk has finished: our P (in X) and O are free,
          // so the peer may write this chunk's partial scores into our X
          ok = role_wait(C, smem_u32(&C.o_done), (i - 1) & 1);
          if (__any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mbar_arrive_cluster(peer_xempty);
          ok = peer_wait(C, smem_u32(&C.x_empty), (i - 1) & 1);  // the peer's X is free for ours
          if (__any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
          }
        }
        // our partial row into the peer's X, then the peer's partial row from ours
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t off = ((uint32_t)j << 4) ^ sw;
          st_cluster_v4(px_lo + off, sv[4 * j], sv[4 * j + 1], sv[4 * j + 2], sv[4 * j + 3]);
          st_cluster_v4(px_hi + off, sv[32 + 4 * j], sv[32 + 4 * j + 1], sv[32 + 4 * j + 2], sv[32 + 4 * j + 3]);
        }
        mbar_arrive_cluster(peer_xfull);
        ok = peer_wait(C, smem_u32(&C.x_full), i & 1);
        if (__any_sync(0xffffffffu, !ok)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t off = ((uint32_t)j << 4) ^ sw;
          float4 a, bb;
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(a.x), "=f"(a.y), "=f"(a.z), "=f"(a.w)
                       : "r"(x_lo + off));
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(bb.x), "=f"(bb.y), "=f"(bb.z), "=f"(bb.w)
                       : "r"(x_hi + off));
          sv[4 * j] += a.x;
          sv[4 * j + 1] += a.y;
          sv[4 * j + 2] += a.z;
          sv[4 * j + 3] += a.w;
          sv[32 + 4 * j] += bb.x;
          sv[32 + 4 * j + 1] += bb.y;
          sv[32 + 4 * j + 2] += bb.z;
          sv[32 + 4 * j + 3] += bb.w;
        }
        // masked row maximum (raw scores; scale > 0), as a tree
        float mx[kBs / 2];
#pragma unroll
        for (int j = 0; j < kBs / 2; ++j)
          mx[j] = fmaxf((vmask >> (2 * j)) & 1ull ? sv[2 * j] : -INFINITY,
                        (vmask >> (2 * j + 1)) & 1ull ? sv[2 * j + 1] : -INFINITY);
#pragma unroll
        for (int w = kBs / 4; w >= 1; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) mx[j] = fmaxf(mx[j], mx[j + w]);
        const float mt = mx[0] * c2;
        const bool raise = mt > m_ref + kRescale;
        const float m_old = m_ref;
        m_ref = raise ? mt : m_ref;
        // P = 2^(s c2 - m) for attended tokens, 0 elsewhere: row h over the first
        // half of X (bytes this thread alone has read), 128-byte swizzle
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = 8 * j + 2 * e;
            const float e0 = ex2_approx(fmaf(sv[t], c2, -m_ref));
            const float e1 = ex2_approx(fmaf(sv[t + 1], c2, -m_ref));
            const float p0 = (vmask >> t) & 1ull ? e0 : 0.f;
            const float p1 = (vmask >> (t + 1)) & 1ull ? e1 : 0.f;
            ps[e] += p0 + p1;
            pk[e] = pack2<T>(p0, p1);
          }
          const uint32_t off = ((uint32_t)j << 4) ^ sw;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(x_lo + off), "r"(pk[0]), "r"(pk[1]),
                       "r"(pk[2]), "r"(pk[3])
                       : "memory");
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
        if (good < kBs) {  // rows holding no token: zero this CTA's V columns (the scores are done)
          uint8_t* stage = st_s + st * kStageBytes;
          const int rows = kBs - good;
          for (int e = tid; e < kLatBlocks * rows * 8; e += kSoftmaxThreads) {
            const int kb = e / (rows * 8);
            const int row = good + (e / 8) % rows;
            *reinterpret_cast<uint4*>(stage + kb * kStBlock + row * 128 + (e & 7) * 16) = make_uint4(0, 0, 0, 0);
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
        give_up(C, peer_abort, dp.err);
      } else {
        // ---- epilogue: this thread's row of O (256 columns)
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        float* part = dp.partials + (((int64_t)b * dp.n_q_heads + h) * dp.max_splits + s) * (kR + 2);
        T* orow = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq +
                  (int64_t)h * dp.out_stride_head + r * kDH;
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
              *reinterpret_cast<float2*>(part + 2 + r * kDH + cc + j) = make_float2(o[j], o[j + 1]);
          }
        }
        if (!direct && r == 0) {
          part[0] = m_ref == -INFINITY ? -INFINITY : m_ref * 0.6931471805599453f;  // natural-log units
          part[1] = l_run;
        }
      }
    }
  } else if (tid < kSoftmaxThreads) {
    // no chunk in this split: an empty partial (or a zero output when nothing is attended)
    const int h = tid;
    if (tid == 0) mbar_wait(smem_u32(&C.q_full), 0);  // the Q copy lands before the CTA exits (bounded)
    if (direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head +
             r * kDH;
      for (int d = 0; d < kDH; d += 8) *reinterpret_cast<uint4*>(o + d) = make_uint4(0, 0, 0, 0);
    } else if (r == 0) {
      float* part = dp.partials + (((int64_t)b * dp.n_q_heads + h) * dp.max_splits + s) * (kR + 2);
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
  // no CTA leaves while its peer may still write into its shared memory
  cluster_sync_all();
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
  // each CTA loads its 4 of the 8 latent k-blocks and its 32 of the 64 rope columns
  if (!tensor_map_col_blocks(&qlat, bf16, p.q_lat, (uint64_t)p.batch * kH, kR * 2, kR / 64, kH, kLatBlocks) ||
      !tensor_map_2d_sw64(&qpe, bf16, p.q_pe, kP, (uint64_t)p.batch * kH, kP * 2, kH) ||
      !tensor_map_col_blocks(&lat, bf16, p.latent, rows, kR * 2, kR / 64, kBs, kLatBlocks) ||
      !tensor_map_2d_sw64(&rope, bf16, p.rope, kP, rows, kP * 2, kBs)) {
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
    // clusters of the two CTAs (x = 0, 1) of each (split, sequence)
    kernel<<<dim3(2, p.n_splits, p.batch), kThreads, kSmemBytes, st>>>(qlat, qpe, lat, rope, p);
    int rc = cuda_status(cudaGetLastError(), "sparse_mla_umma launch");
    if (rc != SNAPMIND_OK || p.n_splits == 1) return rc;
    merge<<<dim3(p.batch * kH * 4 / 8), 256, 0, st>>>(p.dp, p.n_splits);
    return cuda_status(cudaGetLastError(), "sparse_mla_merge launch");
  };
  return bf16 ? go(sparse_mla_umma_kernel<__nv_bfloat16>, sparse_mla_merge_kernel<__nv_bfloat16>)
              : go(sparse_mla_umma_kernel<__half>, sparse_mla_merge_kernel<__half>);
}

}  // namespace snapmind
