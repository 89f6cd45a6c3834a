// Tensor-core paged GQA decode for sm_100a: TMA-staged K/V tiles, mma.sync
// m16n8k16 (bf16/f16 in, fp32 accumulate), split-K with last-ticket merge.
//
// Why mma.sync and not tcgen05: a decode step has one query token per
// sequence, so the query group of a kv head is G <= 8 rows.  tcgen05.mma tiles
// start at M = 64; here the M dimension is the 16 keys of a tile
// (S^T = K . Q^T, N = 8 query heads) and the kernel is HBM bound at about
// 4 flop per byte — the tensor cores only need to keep the issue rate low,
// which the 16x8x16 legacy MMA already does (about 4 instructions per key).
//
// CTA = (split s, kv head, sequence b): 1 producer warp + 4 consumer warps.
//   producer: copies the split's block-table slice into shared memory, then
//     for each 64-token tile issues TMA loads (cp.async.bulk.tensor, 128-byte
//     swizzle) of the tile's (block, kv head) K and V rows into a ring of
//     NSTAGE stages, each guarded by full/empty mbarriers;
//   consumer warp w: keys [16w, 16w+16) of every tile —
//     S^T = K Q^T (8 MMAs over head_dim 128), online softmax in base 2
//     (scale * log2 e folded in), P^T moved from accumulator to operand
//     layout with 4 shuffles, O^T += V^T P^T (8 MMAs, V^T via ldmatrix.trans).
// Every mbarrier wait is bounded (about a second of clock64 ticks); on
// timeout the CTA flags SNAPMIND_DEVERR_TIMEOUT, stops issuing, waits (again
// bounded) for its copies in flight and returns.
#include <cuda.h>

#include "paged_decode.cuh"

namespace snapmind {

namespace {

constexpr int kD = 128;          // head_dim handled by this kernel
constexpr int kTile = 64;        // keys per pipeline stage
constexpr int kConsumers = 4;    // consumer warps, 16 keys each
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kStages = 3;
constexpr int kHalfBytes = kTile * 128;          // 64 keys x 64 dims x 2 bytes
constexpr int kStageBytes = 4 * kHalfBytes;      // K lo/hi + V lo/hi
constexpr int kMaxTableEntries = 512;            // per split
constexpr long long kWaitTicks = 2000000000LL;   // ~1 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false when the barrier did not complete within kWaitTicks.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitTicks) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Issue from a convergent warp: the producer warp runs its loop with every lane and
// one elected lane (`leader` non-zero) issues each copy and barrier arrive.
__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred;
  asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}" : "=r"(pred));
  return pred;
}
__device__ __forceinline__ void tma_load_2d_p(uint32_t leader, uint32_t dst, const CUtensorMap* map, int x, int y,
                                              uint32_t bar) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %0, 0; @p cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%1], [%2, {%3, %4}], [%5]; }" ::"r"(leader),
      "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_p(uint32_t leader, uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 st; setp.ne.b32 p, %0, 0; @p mbarrier.arrive.expect_tx.shared::cta.b64 st, [%1], "
      "%2; }" ::"r"(leader),
      "r"(bar), "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__half>(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                                 uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128-byte-swizzled half tile (rows of 128 bytes, pattern period 8 rows).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return row * 128 + ((chunk ^ (row & 7)) << 4);
}

struct FastSmem {
  // placed right after the stage ring (which starts 1024-byte aligned)
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int32_t table[kMaxTableEntries];
  int issued;
  int abort;
};

constexpr size_t kSmemBytes = kStages * kStageBytes + sizeof(FastSmem) + 1024;

__device__ __forceinline__ int read_abort(const FastSmem& S) {
  return *reinterpret_cast<const volatile int*>(&S.abort);
}

template <typename T, int BS>
__global__ void __launch_bounds__(kThreads, 2)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FastSmem& S = *reinterpret_cast<FastSmem*>(ring + kStages * kStageBytes);
  __shared__ int s_last;

  const int s = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group;

  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  const int skip = p.seq_start ? max(0, p.seq_start[b]) : 0;  // tokens before the window start
  int n_splits = (len + p.split_tokens - 1) / p.split_tokens;
  const int new_pos = len - 1;  // the position of this step's token, when the launch stores it
  if (n_splits > p.max_splits) {
    if (s == 0 && threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_SPLIT);
    n_splits = p.max_splits;
    len = p.max_splits * p.split_tokens;
  }
  if (len <= skip) {
    if (s == 0) {
      if (p.n_peers > 0) {
        emit_peer_rows<T>(p, b, kvh * G, G, kD, [](int, int) { return 0.f; });
      } else {
        for (int e = threadIdx.x; e < G * kD; e += blockDim.x) {
          const int g = e / kD, d = e - g * kD;
          store_out<T>(p, b, kvh * G + g, d, 0.f);
        }
      }
    }
    return;
  }
  if (s >= n_splits) return;
  const int t0 = s * p.split_tokens;
  const int t1 = min(len, t0 + p.split_tokens);
  const int n_tiles = (t1 - t0 + kTile - 1) / kTile;
  const int blk0 = t0 / BS;
  const int n_blk = (t1 - t0 + BS - 1) / BS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&S.full[i]), 1);
      mbar_init(smem_u32(&S.empty[i]), kConsumers);
    }
    S.abort = 0;
    S.issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // block-table slice of this split, validated once
  const int32_t* trow_ptr = p.tables + (int64_t)b * p.table_stride;
  for (int j = threadIdx.x; j < n_blk; j += blockDim.x) {
    const int jj = blk0 + j;
    int32_t phys = -1;
    if (jj < p.table_width) {
      phys = trow_ptr[jj];
      if (phys < 0 || phys >= p.num_blocks) {
        flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
        phys = -1;
      }
    } else {
      flag_error(p.err, SNAPMIND_DEVERR_TABLE);
    }
    S.table[j] = phys;
  }
  if (p.new_k != nullptr && warp == 0 && new_pos >= t0 && new_pos < t1) {
    // this split holds the step's token: store its K and V rows of head kvh into the pool
    // (lanes 0-15 K, 16-31 V, 16 bytes each), then make them visible to the TMA loads below
    const int jj = new_pos / BS;
    const int32_t phys = jj < p.table_width ? trow_ptr[jj] : -1;
    if (phys >= 0 && phys < p.num_blocks) {
      const bool is_v = lane >= 16;
      const T* src = reinterpret_cast<const T*>(is_v ? p.new_v : p.new_k) + (int64_t)b * p.new_stride_seq +
                     (int64_t)kvh * p.new_stride_head + (lane & 15) * 8;
      T* dst = reinterpret_cast<T*>(const_cast<void*>(is_v ? p.v_pool : p.k_pool)) +
               (((int64_t)phys * p.n_kv_heads + kvh) * BS + new_pos % BS) * kD + (lane & 15) * 8;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
  }
  __syncthreads();

  const float c = p.scale * 1.4426950408889634f;  // scale * log2(e)
  const int g = lane >> 2, tig = lane & 3;
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;  // running max (raw score) of heads 2tig, 2tig+1
  float l0 = 0.f, l1 = 0.f;              // this lane's share of the softmax sums

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer
    // every lane runs the loop and its waits; one elected lane issues the copies
    const uint32_t leader = elect_one();
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i % kStages;
      const uint32_t parity = ((i / kStages) & 1) ^ 1;
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&S.empty[st]), parity))) {
        if (lane == 0) {
          flag_error(p.err, SNAPMIND_DEVERR_TIMEOUT);
          atomicExch(&S.abort, 1);
        }
        break;
      }
      if (__any_sync(0xffffffffu, read_abort(S) != 0)) break;
      const int tile_t0 = t0 + i * kTile;
      const int tile_n = min(kTile, t1 - tile_t0);
      const int jb = (tile_t0 - t0) / BS;     // first block of the tile (split-relative)
      const int nb = (tile_n + BS - 1) / BS;  // blocks holding valid keys
      uint32_t bytes = 0;
      for (int j = 0; j < nb; ++j)
        if (S.table[jb + j] >= 0) bytes += 4u * BS * 128u;
      const uint32_t fb = smem_u32(&S.full[st]);
      mbar_arrive_expect_tx_p(leader, fb, bytes);
      uint8_t* stage = ring + st * kStageBytes;
      for (int j = 0; j < nb; ++j) {
        const int32_t phys = S.table[jb + j];
        if (phys < 0) continue;
        const int y = (phys * p.n_kv_heads + kvh) * BS;
        const uint32_t row_off = j * BS * 128;
        tma_load_2d_p(leader, smem_u32(stage + 0 * kHalfBytes + row_off), &kmap, 0, y, fb);
        tma_load_2d_p(leader, smem_u32(stage + 1 * kHalfBytes + row_off), &kmap, 64, y, fb);
        tma_load_2d_p(leader, smem_u32(stage + 2 * kHalfBytes + row_off), &vmap, 0, y, fb);
        tma_load_2d_p(leader, smem_u32(stage + 3 * kHalfBytes + row_off), &vmap, 64, y, fb);
      }
      if (lane == 0) S.issued = i + 1;
    }
  } else {
    // ------------------------------------------------------------ consumers
    // Q^T fragments (B operand, 16 dims x 8 heads): head g, dims 16k + 2tig (+8)
    uint32_t qf[8][2];
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_stride_seq +
                      (int64_t)(kvh * G + (g < G ? g : 0)) * p.q_stride_head;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        qf[k][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + 16 * k + 2 * tig) : 0u;
        qf[k][1] = g < G ? *reinterpret_cast<const uint32_t*>(qrow + 16 * k + 8 + 2 * tig) : 0u;
      }
    }
    // ldmatrix row/chunk of this lane
    const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8;  // K (A operand): key rows 0-15
    const int lchk = lane >> 4;                           // chunk 0/1 of a 16-dim step
    const int vrow = (lane & 7) + ((lane >> 4) & 1) * 8;  // V^T (trans): key rows 0-15
    const int vchk = (lane >> 3) & 1;

    for (int i = 0; i < n_tiles; ++i) {
      const int st = i % kStages;
      const uint32_t parity = (i / kStages) & 1;
      if (read_abort(S)) break;
      if (!mbar_wait(smem_u32(&S.full[st]), parity)) {
        flag_error(p.err, SNAPMIND_DEVERR_TIMEOUT);
        atomicExch(&S.abort, 1);
        break;
      }
      const int tile_t0 = t0 + i * kTile;
      const int valid = min(16, t1 - (tile_t0 + 16 * warp));  // keys of this warp in the tile
      const int lead = skip - (tile_t0 + 16 * warp);          // leading keys before the window start
      uint8_t* stage = ring + st * kStageBytes;
      const uint32_t kbase = smem_u32(stage);
      const uint32_t vbase = smem_u32(stage + 2 * kHalfBytes);
      // a warp computes only if one of its keys is attended (keeps every score row finite)
      const bool loaded = valid > 0 && lead < valid && S.table[(tile_t0 - t0 + 16 * warp) / BS] >= 0;
      if (loaded) {
        if (valid < 16) {
          // zero V rows past the sequence end so that zero weights never meet NaN garbage
          for (int e = lane; e < (16 - valid) * 16; e += 32) {
            const int r = 16 * warp + valid + e / 16;
            const int ch = e & 15;
            *reinterpret_cast<uint4*>(stage + 2 * kHalfBytes + (ch >> 3) * kHalfBytes + swz(r, ch & 7)) =
                make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
        }
        // ---- S^T = K Q^T : 16 keys x 8 heads
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kbase + (k >> 2) * kHalfBytes + swz(16 * warp + lrow, (k & 3) * 2 + lchk), a0, a1, a2, a3);
          mma16816<T>(sc, a0, a1, a2, a3, qf[k][0], qf[k][1]);
        }
        // keys g and g+8 of this warp's 16; heads 2tig, 2tig+1
        if (g >= valid || g < lead) sc[0] = sc[1] = -INFINITY;
        if (g + 8 >= valid || g + 8 < lead) sc[2] = sc[3] = -INFINITY;
        float mt0 = fmaxf(sc[0], sc[2]), mt1 = fmaxf(sc[1], sc[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
          mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
        }
        const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
        const float al0 = exp2f((m0 - mn0) * c), al1 = exp2f((m1 - mn1) * c);
        m0 = mn0;
        m1 = mn1;
        const float p0 = exp2f((sc[0] - mn0) * c), p1 = exp2f((sc[1] - mn1) * c);
        const float p2 = exp2f((sc[2] - mn0) * c), p3 = exp2f((sc[3] - mn1) * c);
        l0 = l0 * al0 + p0 + p2;
        l1 = l1 * al1 + p1 + p3;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt][0] *= al0;
          o[mt][1] *= al1;
          o[mt][2] *= al0;
          o[mt][3] *= al1;
        }
        // ---- P^T operand (16 keys x 8 heads): lane (g, tig) needs keys 2tig(+1)(+8) of head g
        const uint32_t pr01 = pack2<T>(p0, p1), pr23 = pack2<T>(p2, p3);
        const int src = 8 * tig + (g >> 1);
        const uint32_t x = __shfl_sync(0xffffffffu, pr01, src);
        const uint32_t y = __shfl_sync(0xffffffffu, pr01, src + 4);
        const uint32_t z = __shfl_sync(0xffffffffu, pr23, src);
        const uint32_t w = __shfl_sync(0xffffffffu, pr23, src + 4);
        const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
        const uint32_t pb0 = __byte_perm(x, y, sel);
        const uint32_t pb1 = __byte_perm(z, w, sel);
        // ---- O^T += V^T P^T : 128 dims x 8 heads
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vbase + (mt >> 2) * kHalfBytes + swz(16 * warp + vrow, (mt & 3) * 2 + vchk), a0, a1, a2,
                    a3);
          mma16816<T>(o[mt], a0, a1, a2, a3, pb0, pb1);
        }
        if (valid < 16) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&S.empty[st]));
    }
    // sums over the 8 lanes that share tig
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
  }
  __syncthreads();  // the ring is idle: every issued copy was consumed (or the CTA aborts)

  if (S.abort) {
    // wait (bounded) for the latest copy of each stage before leaving
    if (threadIdx.x == 0) {
      const int issued = S.issued;
      for (int i = max(0, issued - kStages); i < issued; ++i) {
        const uint32_t bar = smem_u32(&S.full[i % kStages]);
        const long long tstart = clock64();
        while (!mbar_try_wait(bar, (i / kStages) & 1)) {
          if (clock64() - tstart > kWaitTicks) break;
        }
      }
    }
    __syncthreads();
    return;
  }

  float* mo = reinterpret_cast<float*>(ring);  // [warp][8 heads][128 dims]
  float* mm = mo + kConsumers * 8 * kD;        // [warp][8]
  float* ml = mm + kConsumers * 8;             // [warp][8]
  if (warp < kConsumers) {
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d0 = 16 * mt + g;
      mo[(warp * 8 + 2 * tig) * kD + d0] = o[mt][0];
      mo[(warp * 8 + 2 * tig + 1) * kD + d0] = o[mt][1];
      mo[(warp * 8 + 2 * tig) * kD + d0 + 8] = o[mt][2];
      mo[(warp * 8 + 2 * tig + 1) * kD + d0 + 8] = o[mt][3];
    }
    if (g == 0) {
      mm[warp * 8 + 2 * tig] = m0 * p.scale;  // natural-log units, like the partials
      mm[warp * 8 + 2 * tig + 1] = m1 * p.scale;
      ml[warp * 8 + 2 * tig] = l0;
      ml[warp * 8 + 2 * tig + 1] = l1;
    }
  }
  __syncthreads();

  // ---- merge the 4 consumer warps
  const bool direct = (n_splits == 1);
  if (direct && p.n_peers > 0) {
    emit_peer_rows<T>(p, b, kvh * G, G, kD, [&](int h, int d) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, mm[w * 8 + h]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float mw = mm[w * 8 + h];
        const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
        L += ml[w * 8 + h] * f;
        A += mo[(w * 8 + h) * kD + d] * f;
      }
      return A / L;
    });
    return;
  }
  float* part_base = p.partials + ((int64_t)b * p.n_q_heads + kvh * G) * p.max_splits * (kD + 2);
  for (int e = threadIdx.x; e < G * kD; e += blockDim.x) {
    const int h = e / kD, d = e - h * kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, mm[w * 8 + h]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) {
      const float mw = mm[w * 8 + h];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      L += ml[w * 8 + h] * f;
      A += mo[(w * 8 + h) * kD + d] * f;
    }
    if (direct) {
      store_out<T>(p, b, kvh * G + h, d, A / L);
    } else {
      float* part = part_base + ((int64_t)h * p.max_splits + s) * (kD + 2);
      part[2 + d] = A;
      if (d == 0) {
        part[0] = M;
        part[1] = L;
      }
    }
  }
  if (direct) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&p.counters[b * p.n_kv_heads + kvh], 1);
    s_last = (ticket == n_splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  combine_splits<T>(p, b, kvh, n_splits, mo);
  if (threadIdx.x == 0) p.counters[b * p.n_kv_heads + kvh] = 0;
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D view of one layer's pool: rows of head_dim elements, (block, head, slot) major.
bool make_pool_map(CUtensorMap* map, const void* base, int64_t rows, int dtype, int bs) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kD * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)bs};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == SNAPMIND_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int BS>
int launch_tc(const DecodeParams& p, int dtype, cudaStream_t st) {
  CUtensorMap kmap, vmap;
  const int64_t rows = (int64_t)p.num_blocks * p.n_kv_heads * BS;
  if (!make_pool_map(&kmap, p.k_pool, rows, dtype, BS) || !make_pool_map(&vmap, p.v_pool, rows, dtype, BS)) {
    return SNAPMIND_ERR_UNSUPPORTED;  // the caller falls back to the CUDA-core kernel
  }
  auto kernel = paged_decode_tc_kernel<T, BS>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "paged_decode_tc smem attribute");
    attr_set = true;
  }
  dim3 grid(p.max_splits, p.n_kv_heads, p.batch);
  kernel<<<grid, kThreads, kSmemBytes, st>>>(kmap, vmap, p);
  return cuda_status(cudaGetLastError(), "paged_decode_tc launch");
}

}  // namespace

bool decode_fast_supported(const DecodeParams& p, int dtype) {
  if (dtype != SNAPMIND_DTYPE_BF16 && dtype != SNAPMIND_DTYPE_F16) return false;
  if (p.head_dim != kD || p.group < 1 || p.group > 8) return false;
  if (p.block_size != 16 && p.block_size != 32 && p.block_size != 64) return false;
  if (p.split_tokens % kTile != 0 || p.split_tokens / p.block_size > kMaxTableEntries) return false;
  if (p.q_stride_head % 2 != 0 || p.q_stride_seq % 2 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(p.q) & 3) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(p.k_pool) & 15) != 0 || (reinterpret_cast<uintptr_t>(p.v_pool) & 15) != 0)
    return false;
  if (p.new_k != nullptr &&  // the stored rows move as 16-byte vectors
      (((reinterpret_cast<uintptr_t>(p.new_k) | reinterpret_cast<uintptr_t>(p.new_v)) & 15) != 0 ||
       p.new_stride_seq % 8 != 0 || p.new_stride_head % 8 != 0 || p.seq_start != nullptr || p.n_peers > 0))
    return false;
  if ((int64_t)p.num_blocks * p.n_kv_heads * p.block_size >= (int64_t)1 << 31) return false;
  if (p.batch > 65535 || p.n_kv_heads > 65535) return false;
  return true;
}

int launch_decode_fast(const DecodeParams& p, int dtype, cudaStream_t stream) {
  const bool bf = dtype == SNAPMIND_DTYPE_BF16;
  switch (p.block_size) {
    case 16: return bf ? launch_tc<__nv_bfloat16, 16>(p, dtype, stream) : launch_tc<__half, 16>(p, dtype, stream);
    case 32: return bf ? launch_tc<__nv_bfloat16, 32>(p, dtype, stream) : launch_tc<__half, 32>(p, dtype, stream);
    default: return bf ? launch_tc<__nv_bfloat16, 64>(p, dtype, stream) : launch_tc<__half, 64>(p, dtype, stream);
  }
}

}  // namespace snapmind
