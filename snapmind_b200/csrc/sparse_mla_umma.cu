// Sparse MLA decode on the 5th-generation tensor cores (tcgen05, sm_100a):
// 128 heads, kv_lora_rank 512, rope 64, 64-token blocks, bf16/f16.
//
// A decode step of DeepSeek-style absorbed MLA is, per sequence, a 128-row
// attention: Q [128 heads x 576] against the attended latent rows
// [n x 576] (latent 512 | rope 64), output [128 x 512] over the first 512
// columns of the same rows.
//
// Orientation.  A tcgen05.mma of M = 64 rows takes as long as one of M = 128
// (its time follows N), so the M side of every product here is 128 attended
// tokens (two 64-token chunks), and the heads are the N side:
//   S^T [128 tokens x 64 heads] = K [128 x 576] . Q^T: 36 MMAs (M 128, N 64, K 16);
//   O^T [512 dims x 64 heads] += V^T [512 x 128] . P^T [128 x 64]: 32 MMAs
//     (4 blocks of 128 dims x 8 steps of 16 tokens).
// CTA = (head half hh, split, sequence): heads [64 hh, 64 hh + 64), every
// output dim, the split's attended chunks two at a time ("pairs").  No
// product is computed twice and nothing crosses between CTAs.
// CTA = 10 warps: warps 0-7 softmax in two groups of 32 heads (warp w reads TMEM
// lanes 32 (w % 4) ..: thread = token of the pair, both groups on the same lanes),
// warp 8 TMA producer, warp 9 MMA issuer.  The producer and MMA warps run their
// loops with every lane and one elected lane issues each copy, MMA and commit.
//   Shared memory (1024-aligned, 128-byte swizzle):
//     Q^T: 9 k-blocks x [64 heads x 64] = 72 KB, resident;
//     one pair stage: 9 k-blocks x [128 tokens x 64] = 144 KB (chunk 2q in
//       rows 0-63 of every k-block, chunk 2q + 1 in rows 64-127; one 2-D TMA
//       box per (chunk, k-block)).  Once the scores are done the rope k-block
//       is free and holds P^T [128 tokens x 64 heads] for P V.
//   TMEM (M = 128: row m in lane m): O^T as 4 blocks [128 dims x 64 heads] at
//     columns 0-255, S^T [128 tokens x 64 heads] at column 256.
//   Per pair: S^T over the 9 k-blocks (K-major operands); softmax: each group
//     loads its token's 32 scores (tcgen05.ld 32x32b) and masks the token if
//     it is not attended; the scores are checked against a per-head reference
//     maximum that is raised only when a score exceeds it by 2^8 (then the
//     exact per-head maximum of the pair is reduced across the group and O's
//     columns are rescaled in TMEM); P = exp2(s - m) is written as the group's
//     half of a bf16 row of P^T; a row that holds no token is zeroed in the
//     latent k-blocks (0 x garbage must not reach O); O^T += V^T P^T (V^T read
//     MN-major from the staged rows, P^T MN-major); meanwhile the per-head
//     sums of P are reduced across each warp by a transposing butterfly.
//   The producer refills the stage in five groups (latent k-blocks 2 g, 2 g + 1
//   for g < 4, then rope): group g of the next pair loads as soon as O^T block
//   g += V^T P^T of this pair is done, so the refill runs under the rest of
//   P V and the next scores start on the groups already landed.  It keeps the
//   next kPrefetch chunks prefetched into L2 (TMA prefetch, no shared memory),
//   so the refill is served from L2.  The epilogue stores O^T block j as soon
//   as the last pair's block j is done.
//   Handshakes are mbarriers (tcgen05.commit for the tensor core), every wait
//   is bounded (about a second) and ends early once another role gave up, and
//   TMEM is released on every path.
// Splits write fp32 partials (unnormalised output [sequence][split][head][dim],
// then max and sum [sequence][split][2][head]) into the workspace region the
// paged GQA decode layout sizes for them; a second kernel merges them.
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
constexpr int kHC = 64;                                 // heads per CTA = MMA N
constexpr int kR = 512, kP = 64;
constexpr int kKB = (kR + kP) / 64;                     // 9 k-blocks of 64 elements
constexpr int kBs = 64;                                 // block (chunk) size
constexpr int kPair = 2 * kBs;                          // tokens per pair = MMA M
constexpr int kGroupHeads = 32;                         // heads of one softmax group
constexpr int kSoftmaxThreads = 256;                    // two groups of 4 warps (128 token lanes each)
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kQBlock = kHC * 128;                 // one k-block of Q^T: 8 KB
constexpr uint32_t kQBytes = kKB * kQBlock;             // 72 KB
constexpr uint32_t kHalfBlock = kBs * 128;              // one chunk's rows of a k-block: 8 KB
constexpr uint32_t kStBlock = kPair * 128;              // one k-block of the pair: 16 KB
constexpr uint32_t kStageBytes = kKB * kStBlock;        // 144 KB
constexpr uint32_t kPOff = (kKB - 1) * kStBlock;        // P^T in the rope k-block
constexpr int kMaxSelected = 256;                       // selected chunk ids per sequence (more take the mma.sync kernel)
constexpr uint32_t kTmemCols = 512, kColO = 0, kColS = 256;
constexpr float kRescale = 8.f;                         // log2 headroom of the reference maximum
constexpr int kPrefetch = 4;                            // chunks prefetched into L2 ahead of the load
constexpr int kRing = 64;                               // resolved (chunk, block) pairs kept ahead
// The stage is refilled in groups: group g < 4 = latent k-blocks 2 g, 2 g + 1 (the V rows
// of output block g), group 4 = the rope k-block (P^T during P V).  Group g of the next pair
// loads as soon as O^T block g += V^T P^T is done, so the refill overlaps the rest of P V.
constexpr int kGroups = 5;
__host__ __device__ constexpr uint32_t group_bytes(int g) { return g < kGroups - 1 ? 2 * kHalfBlock : kHalfBlock; }

struct Ctrl {
  uint64_t full[kGroups];       // producer -> MMA: group g of the pair staged
  uint64_t empty[kGroups - 1];  // MMA commit after O^T block g += V^T P^T: latent group g free
  uint64_t s_full;  // MMA commit after S^T: scores ready
  uint64_t p_full;  // softmax threads: P^T written, empty rows zeroed (and O rescaled)
  uint64_t o_done;  // MMA commit after O^T += V^T P^T
  uint64_t q_full;
  uint32_t tmem_base;
  int32_t abort;
  int32_t rescale[2];           // per softmax group: a raise step must rescale some head's O columns
  int32_t n_extra;               // selected chunks outside the window and the sink chunks
  int32_t sel_wfirst, sel_slast; // the first window chunk / the last sink chunk is among the selected
  int32_t ring_c[kRing];        // chunk id, block and "selected" flag of chunk j of the split at j % kRing
  int32_t ring_p[kRing];
  int32_t ring_s[kRing];
  int32_t extra[kMaxSelected];  // those chunks, in selected order
  float m_ref[kHC];             // per-head reference maximum (log2 units of score * scale)
  float alpha[kHC];             // per-head rescale factor of a raise step; 1 / sum in the epilogue
  float red[8][kGroupHeads];    // per softmax warp: partial maxima / sums of its group's heads
};

constexpr size_t kSmemBytes = 1024 + kQBytes + kStageBytes + sizeof(Ctrl);
static_assert(kSmemBytes <= 232448, "shared memory budget");

// The attended chunks of a sequence, in the order the splits share them out:
// the window chunks [wfirst, n_chunks) ascending, then the chunks the sink touches
// [0, sink_chunks) that the window does not hold, then the selected chunks outside
// both (first occurrence, in selected order).  Chunk of list position r and whether
// that chunk is among the selected (which decides its positions outside the sink and
// the window: only the first window chunk and the last sink chunk can have such).
struct ChunkList {
  int wfirst, n_win, sink_chunks, n_sink;
};
__device__ __forceinline__ void chunk_at(const Ctrl& C, const ChunkList& L, int r, int& c, int& sel) {
  if (r < L.n_win) {
    c = L.wfirst + r;
    sel = r == 0 ? C.sel_wfirst : 1;  // later window chunks lie wholly inside the window
    return;
  }
  r -= L.n_win;
  if (r < L.n_sink) {
    c = r;
    sel = c == L.sink_chunks - 1 ? C.sel_slast : 1;  // earlier sink chunks lie wholly inside the sink
    return;
  }
  c = C.extra[r - L.n_sink];
  sel = 1;
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
template <typename T> __device__ __forceinline__ T to_elem(float x);
template <> __device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half to_elem<__half>(float x) { return __float2half_rn(x); }

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

// Named barriers of the softmax threads (the producer and MMA warps do not take part):
// 1 + g over the 128 threads of group g, 3 over both groups.
__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
// The group barrier, returning whether `v` holds in any of its 128 threads.
__device__ __forceinline__ bool group_any(int g, bool v) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.or.pred q, %2, 128, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(1 + g)
      : "memory");
  return r != 0;
}
// Barrier 3 over all 256 softmax threads, returning whether `v` holds in any of them.
__device__ __forceinline__ bool softmax_any(bool v) {
  uint32_t r;
  asm volatile(
      "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.or.pred q, 3, 256, p; selp.u32 %0, 1, 0, q; }"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// Reduces N (32 or 64) values per lane over the warp's 32 lanes by a transposing
// butterfly (N - 2 or N - 1 shuffles): afterwards lane l holds the sum (or maximum)
// over the warp of value l in v[0] (N = 32), or of values 2 l and 2 l + 1 in v[0] and
// v[1] (N = 64).
template <int N, bool kMax>
__device__ __forceinline__ void warp_transpose_reduce(float (&v)[N], int lane) {
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int mask = 16 >> step;        // partner distance
    const int n = (N / 2) >> step;      // this lane keeps n of its current 2 n values
    const bool upper = (lane & mask) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = upper ? v[i] : v[i + n];
      const float keep = upper ? v[i + n] : v[i];
      const float got = __shfl_xor_sync(0xffffffffu, send, mask);
      v[i] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_mla_umma_kernel(const __grid_constant__ CUtensorMap qlat_map, const __grid_constant__ CUtensorMap qpe_map,
                           const __grid_constant__ CUtensorMap lat_map, const __grid_constant__ CUtensorMap lat3_map,
                           const __grid_constant__ CUtensorMap rope_map, SparseParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = base;
  uint8_t* st_s = q_s + kQBytes;
  Ctrl& C = *reinterpret_cast<Ctrl*>(st_s + kStageBytes);

  const int hh = blockIdx.x;  // head half
  const int s = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = idesc_f16(kBf16, kPair, kHC, false, false);
  constexpr uint32_t kIdescPV = idesc_f16(kBf16, kPair, kHC, true, true);
  const DecodeParams& dp = p.dp;
  const int q_row0 = b * kH + hh * kHC;  // first row of this CTA's heads in q_lat / q_pe

  if (tid == 0) {
    for (int g = 0; g < kGroups; ++g) mbar_init(smem_u32(&C.full[g]), 1);
    for (int g = 0; g < kGroups - 1; ++g) mbar_init(smem_u32(&C.empty[g]), 1);
    mbar_init(smem_u32(&C.s_full), 1);
    mbar_init(smem_u32(&C.p_full), kSoftmaxThreads);
    mbar_init(smem_u32(&C.o_done), 1);
    mbar_init(smem_u32(&C.q_full), 1);
    C.abort = 0;
    C.rescale[0] = C.rescale[1] = 0;
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&C.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (tid < kHC) C.m_ref[tid] = -INFINITY;
  // The kernel is launched as a programmatic dependent of the previous kernel on the
  // stream (the top-k selection that writes `selected`): everything above is on-chip,
  // and no input is read before this wait for that grid to complete.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) {
    // Q depends only on the sequence: its copy overlaps the selection set-up below
    const uint32_t qb = smem_u32(&C.q_full);
    mbar_arrive_expect_tx(qb, kQBytes);
    tma_load_3d(smem_u32(q_s), &qlat_map, 0, q_row0, 0, qb);  // the 8 latent k-blocks
    tma_load_2d(smem_u32(q_s + (kKB - 1) * kQBlock), &qpe_map, 0, q_row0, qb);
  }

  // ---- the attended chunks of sequence b (the same list in every CTA of the sequence)
  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  const int n_chunks = (len + kBs - 1) / kBs;
  const int sink = min(p.sink, len);
  const int wstart = max(0, len - p.window);
  ChunkList L;
  L.wfirst = len > wstart ? wstart / kBs : n_chunks;
  L.n_win = n_chunks - L.wfirst;
  L.sink_chunks = (sink + kBs - 1) / kBs;
  L.n_sink = min(L.sink_chunks, L.wfirst);
  if (warp == kProducerWarp) {
    // The selected ids outside the window and the sink chunks (first occurrences, in
    // order), then this split's first list entries with their block-table entries, so
    // the first copies can go out as soon as the CTA-wide barrier below opens.
    int n_extra = 0;
    bool sw = false, sz = false;
    for (int i0 = 0; i0 < p.k; i0 += 32) {  // warp-uniform
      const int i = i0 + lane;
      int c = i < p.k ? p.selected[(int64_t)b * p.k + i] : -1;
      if (c >= n_chunks) c = -1;
      sw |= __any_sync(0xffffffffu, c >= 0 && c == L.wfirst);
      sz |= __any_sync(0xffffffffu, c >= 0 && c == L.sink_chunks - 1);
      bool keep = c >= L.sink_chunks && c < L.wfirst;
#pragma unroll 1
      for (int d = 1; d < 32; ++d) {  // a repeat of an id in an earlier lane
        const int o = __shfl_up_sync(0xffffffffu, c, d);
        if (lane >= d && o == c) keep = false;
      }
      if (keep)
        for (int e = 0; e < n_extra; ++e)  // or of an id kept from an earlier batch
          if (C.extra[e] == c) {
            keep = false;
            break;
          }
      const uint32_t m = __ballot_sync(0xffffffffu, keep);
      if (keep) C.extra[n_extra + __popc(m & ((1u << lane) - 1u))] = c;
      n_extra += __popc(m);
      __syncwarp();
    }
    if (lane == 0) {
      C.n_extra = n_extra;
      C.sel_wfirst = sw;
      C.sel_slast = sz;
    }
    __syncwarp();
    const int count = L.n_win + L.n_sink + n_extra;
    int per = (count + p.n_splits - 1) / max(p.n_splits, 1);
    per += per & 1;
    const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);
    if (lane < c_hi - c_lo) {  // list entries c_lo .. c_lo + 31 of this split
      int c, sel;
      chunk_at(C, L, c_lo + lane, c, sel);
      int32_t phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
      if (phys >= p.num_blocks) phys = -1;
      C.ring_c[lane] = c;
      C.ring_p[lane] = phys;
      C.ring_s[lane] = sel;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = C.tmem_base;
  const int count = L.n_win + L.n_sink + C.n_extra;

  // chunks of this split (the same for both head halves): an even count per split, so
  // only the last split can end in a half-empty pair
  int per = (count + p.n_splits - 1) / max(p.n_splits, 1);
  per += per & 1;
  const int c_lo = min(count, s * per), c_hi = min(count, c_lo + per);
  const int n_ck = c_hi - c_lo;
  const int n_pairs = (n_ck + 1) / 2;
  const bool direct = (p.n_splits == 1);

  if (n_ck > 0) {
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------------- TMA producer
      // The warp resolves the list entries 32 at a time (one table read per lane) into a
      // ring (the first 32 before the set-up barrier).  Then, with every lane running the
      // loop and one elected lane
      // issuing, it loads group g of pair q into the stage once O^T block g += V^T P^T
      // of pair q - 1 is done (the rope group once all of P V is done), and keeps the
      // chunks up to 2 q + 2 + kPrefetch prefetched into L2, so the refill finds its
      // rows there.
      const uint32_t leader = elect_one_sync();
      int located = 32, prefetched = min(n_ck, 2);
      int armed[kGroups];  // the last pair whose copies group g's full barrier counts (-1: none)
#pragma unroll
      for (int g = 0; g < kGroups; ++g) armed[g] = -1;
      bool ok = true;
      for (int q = 0; q < n_pairs && ok; ++q) {
        while (min(n_ck, 2 * q + 2 + kPrefetch) > located) {  // warp-uniform
          const int j = located + lane;
          if (j < n_ck) {
            int c, sel;
            chunk_at(C, L, c_lo + j, c, sel);
            int32_t phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
            if (phys >= p.num_blocks) phys = -1;
            C.ring_c[j % kRing] = c;
            C.ring_p[j % kRing] = phys;
            C.ring_s[j % kRing] = sel;
          }
          __syncwarp();
          located += 32;
        }
        int32_t phys[2];
        int n_valid = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * q + h;
          phys[h] = i < n_ck ? C.ring_p[i % kRing] : -1;
          if (phys[h] >= 0) ++n_valid;
          else if (i < n_ck && lane == 0) flag_error(dp.err, SNAPMIND_DEVERR_BLOCK_ID);
        }
#pragma unroll 1
        for (int g = 0; g < kGroups; ++g) {
          if (q > 0) {
            const uint32_t freed = g < kGroups - 1 ? smem_u32(&C.empty[g]) : smem_u32(&C.o_done);
            ok = __all_sync(0xffffffffu, role_wait(C, freed, (q - 1) & 1));
            if (!ok) {
              if (lane == 0) give_up(C, dp.err);
              break;
            }
          }
          const uint32_t bar = smem_u32(&C.full[g]);
          if (n_valid == 0) {
            mbar_arrive_p(leader, bar);
          } else {
            mbar_arrive_expect_tx_p(leader, bar, n_valid * group_bytes(g));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (phys[h] < 0) continue;
              const int y = phys[h] * kBs;
              if (g < kGroups - 1) {
                tma_load_2d_p(leader, smem_u32(st_s + 2 * g * kStBlock + h * kHalfBlock), &lat_map, 2 * g * 64, y,
                              bar);
                tma_load_2d_p(leader, smem_u32(st_s + (2 * g + 1) * kStBlock + h * kHalfBlock), &lat_map,
                              (2 * g + 1) * 64, y, bar);
              } else {
                tma_load_2d_p(leader, smem_u32(st_s + (kKB - 1) * kStBlock + h * kHalfBlock), &rope_map, 0, y, bar);
              }
            }
          }
          armed[g] = q;
        }
        // L2 prefetch of the chunks after this pair, queued behind the pair's own copies
        for (; ok && prefetched < min(n_ck, 2 * q + 2 + kPrefetch); ++prefetched) {
          const int32_t pb = C.ring_p[prefetched % kRing];
          if (pb >= 0) {
            tma_prefetch_3d_p(leader, &lat3_map, 0, pb * kBs, 0);
            tma_prefetch_2d_p(leader, &rope_map, 0, pb * kBs);
          }
        }
      }
      // before the shared memory is released: every copy issued has landed (bounded)
#pragma unroll 1
      for (int g = 0; g < kGroups; ++g)
        if (armed[g] >= 0) mbar_wait(smem_u32(&C.full[g]), armed[g] & 1);
      mbar_wait(smem_u32(&C.q_full), 0);
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- MMA issuer
      // Every lane runs the loop and its waits; one elected lane issues the MMAs and
      // commits.
      const uint32_t leader = elect_one_sync();
      bool ok = __all_sync(0xffffffffu, role_wait(C, smem_u32(&C.q_full), 0));
      uint32_t last_bar = 0, last_parity = 0;  // the latest commit: covers every MMA issued
      for (int q = 0; q < n_pairs && ok; ++q) {
        // S^T = K Q^T over the 576 columns: the stage's token rows (A) against Q^T (B),
        // each group as soon as it has landed
        bool kb_issued = false;
#pragma unroll 1
        for (int kb = 0; kb < kKB; ++kb) {
          if (kb % 2 == 0) {  // first k-block of group kb / 2 (the rope k-block is group 4)
            ok = __all_sync(0xffffffffu, role_wait(C, smem_u32(&C.full[kb / 2]), q & 1));
            if (!ok) break;
            tc_fence_after();
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(st_s + kb * kStBlock + kk * 32), 16, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(smem_u32(q_s + kb * kQBlock + kk * 32), 16, 1024, kSwizzle128B);
            umma_f16_p(leader, tmem + kColS, ad, bd, kIdescS, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          kb_issued = true;
        }
        if (!ok) {
          if (kb_issued) {  // cover the score MMAs already issued for this pair
            umma_commit_p(leader, smem_u32(&C.s_full));
            last_bar = smem_u32(&C.s_full);
            last_parity = q & 1;
          }
          break;
        }
        umma_commit_p(leader, smem_u32(&C.s_full));
        last_bar = smem_u32(&C.s_full);
        last_parity = q & 1;
        ok = __all_sync(0xffffffffu, role_wait(C, smem_u32(&C.p_full), q & 1));
        if (!ok) break;
        tc_fence_after();
        // O^T += V^T P^T: dim block j = latent k-blocks 2 j, 2 j + 1 (MN-major), P^T
        // (MN-major), 16 tokens a step
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int ks = 0; ks < kPair / 16; ++ks) {
            const uint64_t ad =
                smem_desc(smem_u32(st_s + 2 * j * kStBlock + ks * 16 * 128), kStBlock, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(smem_u32(st_s + kPOff + ks * 16 * 128), kStBlock, 1024, kSwizzle128B);
            umma_f16_p(leader, tmem + kColO + j * kHC, ad, bd, kIdescPV, (q > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit_p(leader, smem_u32(&C.empty[j]));  // latent group j may refill for the next pair
        }
        umma_commit_p(leader, smem_u32(&C.o_done));
        last_bar = smem_u32(&C.o_done);
        last_parity = q & 1;
      }
      if (!ok) {
        if (lane == 0) give_up(C, dp.err);
        if (last_bar) mbar_wait(last_bar, last_parity);  // MMAs in flight finish (bounded) before TMEM goes
      }
    } else {
      // ---------------------------------------------------------------- softmax warps 0-7
      // thread = token t of the pair (TMEM lane t, warp w reads lanes 32 (w % 4) ..) and
      // head group hg: heads [32 hg, 32 hg + 32) of the CTA's 64; token t is row t % 64 of
      // chunk 2 q + t / 64
      const int t = tid & (kPair - 1);
      const int hg = tid >> 7;
      const int h0 = hg * kGroupHeads;
      const uint32_t t_w = tmem + ((uint32_t)((warp & 3) * 32) << 16);
      const float c2 = p.scale * 1.4426950408889634f;
      uint8_t* prow = st_s + kPOff + t * 128;
      const uint32_t psw = (uint32_t)(t & 7);
      float lsum = 0.f;  // sum of P over this warp's tokens for head h0 + lane
      bool ok = true;
      for (int q = 0; q < n_pairs; ++q) {
        // S^T done: every group of the pair landed (both groups take this check every pair)
        ok = ok && role_wait(C, smem_u32(&C.s_full), q & 1);
        if (softmax_any(!ok)) {
          ok = false;
          break;
        }
        const int i = 2 * q + (t >> 6);
        int c = 0, phys = -1, sel = 0;
        if (i < n_ck) {
          c = C.ring_c[i % kRing];  // kept until chunk i + 64 is resolved
          phys = C.ring_p[i % kRing];
          sel = C.ring_s[i % kRing];
        }
        const int pos = c * kBs + (t & 63);
        const bool real = phys >= 0 && pos < len;  // the row holds a token
        const bool att = real && (sel != 0 || pos < sink || pos >= wstart);
        tc_fence_after();
        float v[kGroupHeads];
        tmem_ld32(t_w + kColS + h0, v);
        tmem_wait_ld();
        // raise step: an attended score exceeds its head's reference maximum by 2^8
        bool need = false;
        if (att) {
#pragma unroll
          for (int h = 0; h < kGroupHeads; ++h) need |= v[h] * c2 > C.m_ref[h0 + h] + kRescale;
        }
        if (group_any(hg, need)) {
          // the scores are reduced in place (fewer live registers) and reloaded from TMEM below
#pragma unroll
          for (int h = 0; h < kGroupHeads; ++h) v[h] = att ? v[h] * c2 : -INFINITY;
          warp_transpose_reduce<kGroupHeads, true>(v, lane);
          C.red[warp][lane] = v[0];
          group_sync(hg);
          if (t < kGroupHeads) {
            const int w0 = hg * 4;
            const float m = fmaxf(fmaxf(C.red[w0][t], C.red[w0 + 1][t]), fmaxf(C.red[w0 + 2][t], C.red[w0 + 3][t]));
            const float old = C.m_ref[h0 + t];
            float a = 1.f;
            if (m > old + kRescale) {
              C.m_ref[h0 + t] = m;
              if (old != -INFINITY) {
                a = exp2f(old - m);
                C.rescale[hg] = 1;
              }
            }
            C.alpha[h0 + t] = a;
          }
          group_sync(hg);
          if (C.rescale[hg]) {  // O^T columns of the raised heads (O^T += V^T P^T of pair q - 1 is done)
            // A failed wait does not leave the loop here: the other group is not in this
            // branch, and both groups must meet at every barrier over all softmax threads.
            // The abort flag makes the next shared check end the loop for both.
            ok = role_wait(C, smem_u32(&C.o_done), (q - 1) & 1);
            if (group_any(hg, !ok)) {
              if (t == 0) give_up(C, dp.err);
              ok = false;
            } else {
              tc_fence_after();
#pragma unroll 1
              for (int j = 0; j < 4; ++j) {
                float o[kGroupHeads];
                tmem_ld32(t_w + kColO + j * kHC + h0, o);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < kGroupHeads; ++e) o[e] *= C.alpha[h0 + e];
                tmem_st32(t_w + kColO + j * kHC + h0, o);
              }
              tmem_wait_st();
            }
            lsum *= C.alpha[h0 + lane];
            group_sync(hg);  // every thread has read the factors before the flag is cleared
            if (t == 0) C.rescale[hg] = 0;
          }
          tmem_ld32(t_w + kColS + h0, v);  // the scores again (S^T stays until the next pair's scores)
          tmem_wait_ld();
        }
        // P = 2^(s c2 - m) for an attended token, 0 otherwise; this group's half of row t
        // of P^T (128-byte swizzle: 16-byte piece j of the row at j ^ (t & 7))
#pragma unroll
        for (int h = 0; h < kGroupHeads; ++h) v[h] = att ? ex2_approx(fmaf(v[h], c2, -C.m_ref[h0 + h])) : 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w4 = make_uint4(pack2<T>(v[8 * j], v[8 * j + 1]), pack2<T>(v[8 * j + 2], v[8 * j + 3]),
                                      pack2<T>(v[8 * j + 4], v[8 * j + 5]), pack2<T>(v[8 * j + 6], v[8 * j + 7]));
          *reinterpret_cast<uint4*>(prow + (((uint32_t)(4 * hg + j) ^ psw) << 4)) = w4;
        }
        if (!real) {  // a row without a token: zero it in the latent k-blocks (V^T of P V), half per group
#pragma unroll
          for (int kb = 4 * hg; kb < 4 * hg + 4; ++kb) {
            uint4* row = reinterpret_cast<uint4*>(st_s + kb * kStBlock + t * 128);
#pragma unroll
            for (int e = 0; e < 8; ++e) row[e] = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(smem_u32(&C.p_full));
        // the per-head sums of P over this warp's tokens, while O^T += V^T P^T runs
        warp_transpose_reduce<kGroupHeads, false>(v, lane);
        lsum += v[0];
      }
      {  // every softmax thread takes this shared check, whichever way its loop ended:
         // block 0 of the last pair's P V is done (blocks 1-3 are waited for one by one
         // below, so the first stores overlap the rest of P V)
        const bool fine = ok && role_wait(C, smem_u32(&C.empty[0]), (n_pairs - 1) & 1);
        ok = !softmax_any(!fine);
      }
      if (!ok) {
        give_up(C, dp.err);
      } else {
        // ---- epilogue: per-head totals, then O^T rows d = 128 j + t of this group's heads
        tc_fence_after();
        C.red[warp][lane] = lsum;
        group_sync(hg);
        const int64_t bs_ = (int64_t)b * p.n_splits + s;
        if (t < kGroupHeads) {
          const int w0 = hg * 4;
          const float l = C.red[w0][t] + C.red[w0 + 1][t] + C.red[w0 + 2][t] + C.red[w0 + 3][t];
          C.alpha[h0 + t] = l > 0.f ? 1.f / l : 0.f;
          if (!direct) {
            // max and sum [sequence][split][2][head]
            float* ml = dp.partials + (int64_t)p.batch * p.n_splits * kR * kH + bs_ * 2 * kH + hh * kHC + h0;
            const float m = C.m_ref[h0 + t];
            ml[t] = m == -INFINITY ? -INFINITY : m * 0.6931471805599453f;  // natural-log units
            ml[kH + t] = l;
          }
        }
        group_sync(hg);
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          if (j > 0) {  // O^T block j is final once the last pair's block j has completed
            if (!role_wait(C, smem_u32(&C.empty[j]), (n_pairs - 1) & 1)) {
              give_up(C, dp.err);
              break;
            }
            tc_fence_after();
          }
          const int d = j * kPair + t;
          float o[kGroupHeads];
          tmem_ld32(t_w + kColO + j * kHC + h0, o);
          tmem_wait_ld();
          if (direct) {
            T* out = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq +
                     (int64_t)(hh * kHC + h0) * dp.out_stride_head + d;
#pragma unroll
            for (int h = 0; h < kGroupHeads; ++h)
              out[(int64_t)h * dp.out_stride_head] = to_elem<T>(o[h] * C.alpha[h0 + h]);
          } else {
            // partials [sequence][split][head][dim]: the warp's 32 dims of each head are one
            // 128-byte line
            float* part = dp.partials + (bs_ * kH + hh * kHC + h0) * kR + d;
#pragma unroll
            for (int h = 0; h < kGroupHeads; ++h) part[(int64_t)h * kR] = o[h];
          }
        }
      }
    }
  } else if (tid < kHC) {
    // no chunk in this split: an empty partial (or a zero output when nothing is attended)
    const int h = hh * kHC + tid;
    if (tid == 0) mbar_wait(smem_u32(&C.q_full), 0);  // the Q copy lands before the CTA exits (bounded)
    if (direct) {
      T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head;
      for (int d = 0; d < kR; d += 8) *reinterpret_cast<uint4*>(o + d) = make_uint4(0, 0, 0, 0);
    } else {
      float* ml = dp.partials + (int64_t)p.batch * p.n_splits * kR * kH + ((int64_t)b * p.n_splits + s) * 2 * kH;
      ml[h] = -INFINITY;
      ml[kH + h] = 0.f;
    }
  }

  // ---- every role is done with shared memory and TMEM
  tc_fence_before();
  __syncthreads();
  // the merge kernel may launch now; it still waits for this whole grid before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge of the split partials: CTA = (sequence, head), thread = 4 output dims, so
// every load of a warp is 512 contiguous bytes of one (split, head).  The splits are
// taken kMergeBatch at a time: each thread first issues the loads of its four dims of
// every split of the batch, all independent, then the first threads stage the splits'
// max and sum in shared memory, and the rows are folded in with a running maximum.
// At most 64 registers a thread, so a batch of 128 sequences x heads fits in one wave.
// Splits without attended tokens (max -inf, weight 0) may hold stale rows: their
// terms are selected away, never multiplied.
constexpr int kMergeBatch = 10;

template <typename T>
__global__ void __launch_bounds__(kR / 4, 8) sparse_mla_merge_kernel(DecodeParams dp, int n_splits) {
  __shared__ float s_m[kMergeBatch], s_l[kMergeBatch];
  const int b = blockIdx.x / kH, h = blockIdx.x % kH;
  const int d = threadIdx.x * 4;
  // launched as a programmatic dependent of the attention kernel: its partials are
  // complete and visible once this returns
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (b >= dp.batch) return;
  const float* ml = dp.partials + (int64_t)dp.batch * n_splits * kR * kH + (int64_t)b * n_splits * 2 * kH + h;
  const float* part = dp.partials + ((int64_t)b * n_splits * kH + h) * kR + d;
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < n_splits; s0 += kMergeBatch) {  // uniform over the CTA
    float4 v[kMergeBatch];
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i)
      if (s0 + i < n_splits) v[i] = __ldcg(reinterpret_cast<const float4*>(part + (int64_t)(s0 + i) * kH * kR));
    if (threadIdx.x < kMergeBatch) {
      const int sp = s0 + threadIdx.x;
      s_m[threadIdx.x] = sp < n_splits ? __ldcg(ml + sp * 2 * kH) : -INFINITY;
      s_l[threadIdx.x] = sp < n_splits ? __ldcg(ml + sp * 2 * kH + kH) : 0.f;
    }
    __syncthreads();
    float mb = M;
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) mb = fmaxf(mb, s_m[i]);
    if (mb != -INFINITY) {  // something attended so far
      const float r = M == -INFINITY ? 0.f : expf(M - mb);
      L *= r;
      acc.x *= r;
      acc.y *= r;
      acc.z *= r;
      acc.w *= r;
      M = mb;
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        const float m = s_m[i];
        if (m != -INFINITY) {
          const float f = expf(m - M);
          L = fmaf(s_l[i], f, L);
          acc.x = fmaf(v[i].x, f, acc.x);
          acc.y = fmaf(v[i].y, f, acc.y);
          acc.z = fmaf(v[i].z, f, acc.z);
          acc.w = fmaf(v[i].w, f, acc.w);
        }
      }
    }
    __syncthreads();  // the next batch overwrites s_m / s_l
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* o = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)h * dp.out_stride_head + d;
  *reinterpret_cast<uint2*>(o) = make_uint2(pack2<T>(acc.x * inv, acc.y * inv), pack2<T>(acc.z * inv, acc.w * inv));
}

}  // namespace

int sparse_mla_umma_splits(int batch) {
  const int per_seq = num_sms() / (2 * (batch > 0 ? batch : 1));  // 2 CTAs (head halves) per (split, sequence)
  return per_seq < 1 ? 1 : (per_seq > 64 ? 64 : per_seq);
}

bool sparse_mla_umma_supported(const SparseParams& p, int dtype) {
  const auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  return (dtype == SNAPMIND_DTYPE_BF16 || dtype == SNAPMIND_DTYPE_F16) && p.n_heads == kH && p.R == kR &&
         p.P == kP && p.bs == kBs && p.k <= kMaxSelected && p.batch <= 65535 && a16(p.q_lat) && a16(p.q_pe) &&
         a16(p.latent) && a16(p.rope) && a16(p.dp.out) && encode_tiled() != nullptr;
}

int launch_sparse_mla_umma(const SparseParams& p, int dtype, cudaStream_t st) {
  const bool bf16 = dtype == SNAPMIND_DTYPE_BF16;
  CUtensorMap qlat, qpe, lat, lat3, rope;
  const uint64_t rows = (uint64_t)p.num_blocks * kBs;
  // Q^T rows of 64 heads: all 8 latent k-blocks in one 3-D box, rope in a 2-D box.  Chunk
  // rows of 64 tokens: one 2-D box per latent k-block (the pair stage interleaves two
  // chunks in every k-block) and one for rope; the 3-D map prefetches a chunk's latent rows.
  if (!tensor_map_col_blocks(&qlat, bf16, p.q_lat, (uint64_t)p.batch * kH, kR * 2, kR / 64, kHC) ||
      !tensor_map_2d(&qpe, bf16, p.q_pe, kP, (uint64_t)p.batch * kH, kP * 2, 64, kHC) ||
      !tensor_map_2d(&lat, bf16, p.latent, kR, rows, kR * 2, 64, kBs) ||
      !tensor_map_col_blocks(&lat3, bf16, p.latent, rows, kR * 2, kR / 64, kBs) ||
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
    // Both kernels are programmatic dependent launches: each one's launch and on-chip
    // set-up overlap the tail of the kernel before it, and each waits (griddepcontrol.wait)
    // for that kernel to complete before it reads any input.
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, p.n_splits, p.batch);  // x = head half
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    int rc = cuda_status(cudaLaunchKernelEx(&cfg, kernel, qlat, qpe, lat, lat3, rope, p), "sparse_mla_umma launch");
    if (rc != SNAPMIND_OK || p.n_splits == 1) return rc;
    cfg.gridDim = dim3(p.batch * kH);
    cfg.blockDim = dim3(kR / 4);
    cfg.dynamicSmemBytes = 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, merge, p.dp, p.n_splits), "sparse_mla_merge launch");
  };
  return bf16 ? go(sparse_mla_umma_kernel<__nv_bfloat16>, sparse_mla_merge_kernel<__nv_bfloat16>)
              : go(sparse_mla_umma_kernel<__half>, sparse_mla_merge_kernel<__half>);
}

}  // namespace snapmind
