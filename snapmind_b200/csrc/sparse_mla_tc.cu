// Tensor-core sparse MLA decode (bf16/f16, kv_lora_rank 512, rope 64,
// 64-token chunks) for sm_100a.
//
// CTA = (split, group of 16 MT heads, sequence), 8 MT warps (MT = 2 when the
// heads divide by 32).  Each m-tile of 16 heads is the M dimension of
// mma.sync m16n8k16 — a dense tile, which is why this kernel uses tensor cores
// while the paged GQA decode (query group <= 8) is byte-bound anyway.  Per
// 64-token tile of attended positions:
//   * latent + rope rows (1152 bytes) are staged by cp.async into rows padded
//     to 1168 bytes (ldmatrix of 8 consecutive rows hits 8 distinct bank
//     groups), double-buffered; rows outside the selection are zero-filled;
//     the staged tile serves every m-tile of the CTA;
//   * S = Q K^T: warp (mt, wm) owns tokens [8 wm, 8 wm + 8) of m-tile mt:
//     36 k-steps x 1 MMA on four accumulator chains (k mod 4);
//   * the tile's row maxima / sums are merged across the 8 warps of an m-tile
//     in shared memory (online softmax in base 2, scale folded in), P is
//     staged as bf16;
//   * O += P V: warp (mt, wm) owns output dims [64 wm, 64 wm + 64):
//     4 k-steps x 8 MMAs, V^T fragments via ldmatrix.trans.
// Splits merge through the last-ticket combine of the paged GQA decode.
#include "common.cuh"
#include "paged_decode.cuh"
#include "sparse_mla.cuh"

namespace snapmind {
namespace {

constexpr int kR = 512, kP = 64, kRow = kR + kP;  // 576 elements
constexpr int kRowBytes = kRow * 2 + 16;          // padded smem row: 1168 bytes
constexpr int kTileRows = 64;
constexpr int kPRowBytes = kTileRows * 2 + 16;    // P row: 144 bytes
constexpr int kBits = 8192;                       // chunks per sequence (bitmaps)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}

template <typename T>
__device__ __forceinline__ void mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                    uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  T a = Conv<T>::from_f(lo), b = Conv<T>::from_f(hi);
  return (uint32_t)(*reinterpret_cast<uint16_t*>(&a)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&b)) << 16);
}

constexpr int kWPM = 8;       // warps per 16-head m-tile
constexpr int kMaxWarps = 16;

struct TcSmem {
  uint32_t sel_bits[kBits / 32];
  uint32_t inc_bits[kBits / 32];
  int32_t word_pre[kBits / 32 + 1];  // included chunks before each bitmap word
  float red_max[kMaxWarps][16];
  float red_sum[kMaxWarps][16];
  int32_t tile_chunk[2];
};

// smem: [Q: 16 MT rows][KV: 2 x 64 rows][P: 16 MT rows x 144 B][TcSmem]
constexpr size_t kKvBytes = (size_t)kTileRows * kRowBytes;
constexpr size_t tc_smem_bytes(int mt) {
  return (size_t)16 * mt * kRowBytes + 2 * kKvBytes + (size_t)16 * mt * kPRowBytes + sizeof(TcSmem) + 128;
}

// chunk id of the rank-th included chunk (rank < count)
__device__ __forceinline__ int chunk_of_rank(const TcSmem& S, int words, int rank) {
  int lo = 0, hi = words;  // find last word w with word_pre[w] <= rank
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (S.word_pre[mid] <= rank) lo = mid; else hi = mid;
  }
  uint32_t word = S.inc_bits[lo];
  int k = rank - S.word_pre[lo];
  while (k-- > 0) word &= word - 1;
  return lo * 32 + __ffs(word) - 1;
}

// MT m-tiles of 16 heads per CTA, kWPM = 8 warps per m-tile: warp = 8 mt + wm.
// S = Q K^T: warp (mt, wm) scores heads [16 mt, 16 mt + 16) against tokens
// [8 wm, 8 wm + 8) of the tile; O += P V: warp (mt, wm) owns those heads x
// latent dims [64 wm, 64 wm + 64).  The K/V tile in shared memory serves
// all m-tiles; small per-warp accumulators keep 16 warps resident.
template <typename T, int MT>
__global__ void __launch_bounds__(32 * kWPM * MT, 1) sparse_mla_tc_kernel(SparseParams p) {
  constexpr int kWarps = kWPM * MT;
  constexpr int kThreads = 32 * kWarps;
  constexpr size_t kQBytes = (size_t)16 * MT * kRowBytes;
  constexpr size_t kPBytes = (size_t)16 * MT * kPRowBytes;
  extern __shared__ __align__(128) unsigned char sm_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
  unsigned char* q_s = base;
  unsigned char* kv_s = q_s + kQBytes;
  unsigned char* p_s = kv_s + 2 * kKvBytes;
  TcSmem& S = *reinterpret_cast<TcSmem*>(p_s + kPBytes);
  __shared__ int s_count;

  const int s = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = warp / kWPM, wm = warp % kWPM;
  const int g = lane >> 2, tig = lane & 3;
  const int bs = kTileRows;

  int len = p.seq_lens[b];
  if (len < 0) len = 0;
  int n_chunks = (len + bs - 1) / bs;
  if (n_chunks > kBits) {
    if (tid == 0 && s == 0 && hg == 0) flag_error(p.dp.err, SNAPMIND_DEVERR_TABLE);
    n_chunks = kBits;
    len = kBits * bs;
  }
  const int words = (n_chunks + 31) / 32;
  for (int i = tid; i < words; i += kThreads) {
    S.sel_bits[i] = 0u;
    S.inc_bits[i] = 0u;
  }
  __syncthreads();
  for (int i = tid; i < p.k; i += kThreads) {
    const int c = p.selected[(int64_t)b * p.k + i];
    if (c >= 0 && c < n_chunks) {
      atomicOr(&S.sel_bits[c >> 5], 1u << (c & 31));
      atomicOr(&S.inc_bits[c >> 5], 1u << (c & 31));
    }
  }
  const int sink = min(p.sink, len);
  const int wstart = max(0, len - p.window);
  for (int c = tid; c < min((sink + bs - 1) / bs, n_chunks); c += kThreads)  // every chunk the sink touches
    atomicOr(&S.inc_bits[c >> 5], 1u << (c & 31));
  if (len > wstart)
    for (int c = wstart / bs + tid; c < n_chunks; c += kThreads) atomicOr(&S.inc_bits[c >> 5], 1u << (c & 31));
  __syncthreads();
  if (warp == 0) {  // exclusive prefix of popcounts per word
    int carry = 0;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const int cnt = (w0 + lane < words) ? __popc(S.inc_bits[w0 + lane]) : 0;
      int pre = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, off);
        if (lane >= off) pre += y;
      }
      if (w0 + lane < words) S.word_pre[w0 + lane] = carry + pre - cnt;
      carry += __shfl_sync(0xffffffffu, pre, 31);
    }
    if (lane == 0) {
      S.word_pre[words] = carry;
      s_count = carry;
    }
  }
  // Q rows of the CTA's heads (q_lat | q_pe), bf16/f16, padded
  const int h0 = hg * 16 * MT;
  for (int i = tid; i < 16 * MT * (kRow / 8); i += kThreads) {
    const int h = i / (kRow / 8), v = i - h * (kRow / 8);
    const T* src = v < kR / 8 ? reinterpret_cast<const T*>(p.q_lat) + ((int64_t)b * p.n_heads + h0 + h) * kR + v * 8
                              : reinterpret_cast<const T*>(p.q_pe) + ((int64_t)b * p.n_heads + h0 + h) * kP + (v - kR / 8) * 8;
    *reinterpret_cast<uint4*>(q_s + h * kRowBytes + v * 16) = *reinterpret_cast<const uint4*>(src);
  }
  __syncthreads();
  const int count = s_count;
  if (count == 0) {
    if (s == 0) {
      for (int i = tid; i < 16 * MT * kR; i += kThreads) {
        T* o = reinterpret_cast<T*>(p.dp.out) + (int64_t)b * p.dp.out_stride_seq +
               (int64_t)(h0 + i / kR) * p.dp.out_stride_head;
        o[i % kR] = Conv<T>::from_f(0.f);
      }
    }
    return;
  }
  const int per = (count + p.n_splits - 1) / p.n_splits;
  const int r_lo = min(count, s * per), r_hi = min(count, r_lo + per);
  const int n_tiles = r_hi - r_lo;

  // stage one chunk's rows into buffer `buf`: warp w copies rows w, w + kWarps, ...;
  // lanes copy the 72 16-byte vectors of a row (latent 64, rope 8)
  auto stage = [&](int tile, int buf) {
    const int c = chunk_of_rank(S, words, r_lo + tile);
    int32_t phys = c < p.table_width ? p.tables[(int64_t)b * p.table_stride + c] : -1;
    if (phys >= p.num_blocks) phys = -1;
    if (phys < 0 && tid == 0) flag_error(p.dp.err, SNAPMIND_DEVERR_BLOCK_ID);
    if (tid == 0) S.tile_chunk[buf] = phys < 0 ? -1 : c;
    const bool selected = (S.sel_bits[c >> 5] >> (c & 31)) & 1u;
    const T* lat = reinterpret_cast<const T*>(p.latent) + (int64_t)max(phys, 0) * bs * kR;
    const T* rp = reinterpret_cast<const T*>(p.rope) + (int64_t)max(phys, 0) * bs * kP;
    unsigned char* dst = kv_s + buf * kKvBytes;
    for (int r = warp; r < bs; r += kWarps) {
      const int pos = c * bs + r;
      const bool valid = phys >= 0 && pos < len && (selected || pos < sink || pos >= wstart);
      const uint32_t drow = smem_u32(dst + r * kRowBytes);
      cp_async16(drow + lane * 16, lat + (int64_t)r * kR + lane * 8, valid);
      cp_async16(drow + (lane + 32) * 16, lat + (int64_t)r * kR + (lane + 32) * 8, valid);
      if (lane < kRow / 8 - 64) cp_async16(drow + (lane + 64) * 16, rp + (int64_t)r * kP + lane * 8, valid);
    }
  };

  const float c2 = p.scale * 1.4426950408889634f;
  float m_run[2] = {-INFINITY, -INFINITY};  // heads g, g+8 of this warp's m-tile
  float l_run[2] = {0.f, 0.f};
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  // ldmatrix lane addressing
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8;  // Q / P rows 0-15 of the m-tile
  const int a_kof = (lane >> 4) * 8;                      // +8 elements for matrices 2,3
  const int b_tok = lane & 7;                             // K rows (8 tokens) for B non-trans
  const int b_kof = (lane >> 3) * 8;                      // matrices 0-3: k offsets 0, 8, 16, 24
  const int v_tok = (lane & 7) + ((lane >> 3) & 1) * 8;   // V^T: tokens 0-15 (matrices 0,1 / 2,3)
  const int v_dof = (lane >> 4) * 8;
  const unsigned char* q_rows = q_s + (16 * mt + a_row) * kRowBytes;
  unsigned char* p_rows = p_s + 16 * mt * kPRowBytes;

  if (n_tiles > 0) {
    stage(0, 0);
    cp_async_commit();
  }
  for (int t = 0; t < n_tiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < n_tiles) stage(t + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    const int c = S.tile_chunk[buf];
    const unsigned char* kv = kv_s + buf * kKvBytes;
    // ---- S = Q K^T for tokens [8 wm, 8 wm + 8): one B load covers two k-steps;
    //      four accumulator chains (k mod 4)
    float acc4[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) acc4[c][0] = acc4[c][1] = acc4[c][2] = acc4[c][3] = 0.f;
    const unsigned char* k_rows = kv + (8 * wm + b_tok) * kRowBytes;
    for (int k = 0; k < kRow / 16; k += 4) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t b0, b1, b2, b3;
        ldsm4(smem_u32(k_rows + ((k + 2 * h2) * 16 + b_kof) * 2), b0, b1, b2, b3);
        uint32_t a0, a1, a2, a3;
        ldsm4(smem_u32(q_rows + ((k + 2 * h2) * 16 + a_kof) * 2), a0, a1, a2, a3);
        mma<T>(acc4[2 * h2], a0, a1, a2, a3, b0, b1);
        ldsm4(smem_u32(q_rows + ((k + 2 * h2 + 1) * 16 + a_kof) * 2), a0, a1, a2, a3);
        mma<T>(acc4[2 * h2 + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    float sc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) sc[e] = (acc4[0][e] + acc4[1][e]) + (acc4[2][e] + acc4[3][e]);
    // validity of this thread's 2 token columns (rows g and g + 8)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = 8 * wm + 2 * tig + e;
      const int pos = c * bs + r;
      const bool selected = c >= 0 && ((S.sel_bits[c >> 5] >> (c & 31)) & 1u);
      const bool valid = c >= 0 && pos < len && (selected || pos < sink || pos >= wstart);
      if (!valid) {
        sc[e] = -INFINITY;
        sc[2 + e] = -INFINITY;
      }
      mx[0] = fmaxf(mx[0], sc[e]);
      mx[1] = fmaxf(mx[1], sc[2 + e]);
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], off));
      mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], off));
    }
    if (tig == 0) {
      S.red_max[warp][g] = mx[0];
      S.red_max[warp][g + 8] = mx[1];
    }
    __syncthreads();
    float m_new[2], alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float tm = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWPM; ++w) tm = fmaxf(tm, S.red_max[kWPM * mt + w][g + 8 * hh]);
      m_new[hh] = fmaxf(m_run[hh], tm);
      alpha[hh] = (m_run[hh] == -INFINITY) ? 0.f : exp2f((m_run[hh] - m_new[hh]) * c2);
    }
    float ps[2] = {0.f, 0.f};
    {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hh = e >> 1;
        pv[e] = (m_new[hh] == -INFINITY) ? 0.f : exp2f((sc[e] - m_new[hh]) * c2);
        ps[hh] += pv[e];
      }
      const int col = 8 * wm + 2 * tig;
      *reinterpret_cast<uint32_t*>(p_rows + g * kPRowBytes + col * 2) = pack_pair<T>(pv[0], pv[1]);
      *reinterpret_cast<uint32_t*>(p_rows + (g + 8) * kPRowBytes + col * 2) = pack_pair<T>(pv[2], pv[3]);
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      ps[0] += __shfl_xor_sync(0xffffffffu, ps[0], off);
      ps[1] += __shfl_xor_sync(0xffffffffu, ps[1], off);
    }
    if (tig == 0) {
      S.red_sum[warp][g] = ps[0];
      S.red_sum[warp][g + 8] = ps[1];
    }
    __syncthreads();
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float tsum = 0.f;
#pragma unroll
      for (int w = 0; w < kWPM; ++w) tsum += S.red_sum[kWPM * mt + w][g + 8 * hh];
      l_run[hh] = l_run[hh] * alpha[hh] + tsum;
      m_run[hh] = m_new[hh];
    }
    // ---- O (16 heads x dims [64 wm, 64 wm + 64)) += P V
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }
#pragma unroll
    for (int ks = 0; ks < kTileRows / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm4(smem_u32(p_rows + a_row * kPRowBytes + (ks * 16 + a_kof) * 2), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int d0 = 64 * wm + np * 16;
        uint32_t b0, b1, b2, b3;
        ldsm4t(smem_u32(kv + (ks * 16 + v_tok) * kRowBytes + (d0 + v_dof) * 2), b0, b1, b2, b3);
        mma<T>(o[2 * np], a0, a1, a2, a3, b0, b1);
        mma<T>(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // P and this KV buffer are reused
  }
  cp_async_wait0();

  // ---- partial of this split -> output or workspace, then the last-ticket merge
  const DecodeParams& dp = p.dp;
  const bool direct = (p.n_splits == 1);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int hh = e >> 1;
      const int head = 16 * mt + g + 8 * hh;
      const int d = 64 * wm + nt * 8 + 2 * tig + (e & 1);
      if (direct) {
        T* out = reinterpret_cast<T*>(dp.out) + (int64_t)b * dp.out_stride_seq + (int64_t)(h0 + head) * dp.out_stride_head;
        out[d] = Conv<T>::from_f(l_run[hh] > 0.f ? o[nt][e] / l_run[hh] : 0.f);
      } else {
        float* part = dp.partials + (((int64_t)b * dp.n_q_heads + h0 + head) * dp.max_splits + s) * (kR + 2);
        part[2 + d] = o[nt][e];
        if (d == 0) {
          part[0] = m_run[hh] == -INFINITY ? -INFINITY : m_run[hh] * p.scale;  // natural-log units
          part[1] = l_run[hh];
        }
      }
    }
  }
  if (direct) return;
  // one ticket per CTA, on the counter of its first 16-head group
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  const int grp0 = hg * MT;
  if (tid == 0) {
    const int ticket = atomicAdd(&dp.counters[b * dp.n_kv_heads + grp0], 1);
    s_last = (ticket == p.n_splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int m = 0; m < MT; ++m) combine_splits<T>(dp, b, grp0 + m, p.n_splits, reinterpret_cast<float*>(base));
  if (tid == 0) dp.counters[b * dp.n_kv_heads + grp0] = 0;
}

}  // namespace

bool sparse_mla_tc_supported(const SparseParams& p, int dtype) {
  return (dtype == SNAPMIND_DTYPE_BF16 || dtype == SNAPMIND_DTYPE_F16) && p.R == kR && p.P == kP &&
         p.bs == kTileRows && p.n_heads % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(p.q_lat) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.q_pe) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(p.latent) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.rope) & 15) == 0;
}

int launch_sparse_mla_tc(const SparseParams& p, int dtype, cudaStream_t st) {
  // 32 heads (two m-tiles, 8 warps) per CTA when they divide evenly
  const int mt = p.n_heads % 32 == 0 ? 2 : 1;
  dim3 grid(p.n_splits, p.n_heads / (16 * mt), p.batch);
  auto go = [&](auto kernel, size_t smem) -> int {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "sparse_mla_tc smem attribute");
    kernel<<<grid, 32 * kWPM * mt, smem, st>>>(p);
    return cuda_status(cudaGetLastError(), "sparse_mla_tc launch");
  };
  if (dtype == SNAPMIND_DTYPE_BF16) {
    return mt == 2 ? go(sparse_mla_tc_kernel<__nv_bfloat16, 2>, tc_smem_bytes(2))
                   : go(sparse_mla_tc_kernel<__nv_bfloat16, 1>, tc_smem_bytes(1));
  }
  return mt == 2 ? go(sparse_mla_tc_kernel<__half, 2>, tc_smem_bytes(2)) : go(sparse_mla_tc_kernel<__half, 1>, tc_smem_bytes(1));
}

}  // namespace snapmind
