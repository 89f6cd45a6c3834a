// Paged KV append / gather / compaction / block reservation for sm_100a.
//
// These kernels are HBM-bound byte movers.  The pool layout
// pool[layer][block][head][slot][dim] makes every (block, head) tile of
// block_size x head_dim elements contiguous, so:
//   * append writes one head_dim row per (token, head), 16-byte vectors;
//   * gather copies whole contiguous tiles into the (H, T, D) layout that
//     PagedKVCache.fetch returns (snapmind/kv_cache/paged.py:56-78) — reads and
//     writes are both fully coalesced, every pool byte is read once.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace snapmind {

static thread_local char g_last_error[512] = "";

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

// ---------------------------------------------------------------------------
// append
// ---------------------------------------------------------------------------
struct AppendParams {
  char* pool[2];            // K, V layer-0 base
  const char* in[2];        // K, V input base
  int64_t pool_layer_stride;  // bytes
  int64_t in_stride_layer, in_stride_seq, in_stride_head, in_stride_tok;  // bytes
  const int32_t* tables;
  int64_t table_stride_seq, table_stride_layer;
  int32_t table_width;
  const int32_t* slot_starts;
  int32_t slot_start0;
  int32_t n_layers, batch, n_tokens, n_heads, block_size, num_blocks;
  int32_t row_bytes_in, row_bytes_out;  // head_dim * element size
  int32_t head_dim;
  int32_t nkv;  // 2 for K and V pools, 1 for a single pool (v pointers NULL)
  int32_t* err;
};

// Resolve the destination row of (layer, b, t); returns nullptr (and flags)
// when the table entry is missing or out of range.
__device__ __forceinline__ int64_t append_dst_row(const AppendParams& p, int layer, int b, int t,
                                                  int h) {
  const int slot = (p.slot_starts ? p.slot_starts[b] : 0) + p.slot_start0 + t;
  const int j = slot / p.block_size;
  const int off = slot - j * p.block_size;
  if (slot < 0 || j >= p.table_width) {
    flag_error(p.err, SNAPMIND_DEVERR_TABLE);
    return -1;
  }
  const int32_t phys =
      p.tables[(int64_t)layer * p.table_stride_layer + (int64_t)b * p.table_stride_seq + j];
  if (phys < 0 || phys >= p.num_blocks) {
    flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
    return -1;
  }
  return (((int64_t)phys * p.n_heads + h) * p.block_size + off);
}

// Same dtype on both sides: a byte copy in W-byte vectors.  A team of lanes copies one
// row (one token of one head of one layer): vpr lanes when a row's vpr vectors divide
// the warp (two 256-byte rows per warp at head_dim 128 in 16-bit), else the whole warp.
// The row's coordinates and destination are resolved once per row, not per vector.
template <int W>
__global__ void __launch_bounds__(256) kv_append_copy_kernel(AppendParams p) {
  using V = typename VecT<W>::type;
  const int vpr = p.row_bytes_out / W;  // vectors per row
  const int team = (vpr < 32 && 32 % vpr == 0) ? vpr : 32;
  const int per_warp = 32 / team;
  const int lane = threadIdx.x & 31;
  const int sub = lane / team, sl = lane - sub * team;
  const int64_t rows = (int64_t)p.n_layers * p.batch * p.n_tokens * p.nkv * p.n_heads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * per_warp + sub; r < rows;
       r += warps * per_warp) {
    int64_t q = r;
    const int h = (int)(q % p.n_heads); q /= p.n_heads;
    const int kv = (int)(q % p.nkv); q /= p.nkv;
    const int t = (int)(q % p.n_tokens); q /= p.n_tokens;
    const int b = (int)(q % p.batch);
    const int layer = (int)(q / p.batch);
    const int64_t row = append_dst_row(p, layer, b, t, h);
    if (row < 0) continue;
    const V* src = reinterpret_cast<const V*>(p.in[kv] + layer * p.in_stride_layer + b * p.in_stride_seq +
                                              h * p.in_stride_head + t * p.in_stride_tok);
    V* dst = reinterpret_cast<V*>(p.pool[kv] + layer * p.pool_layer_stride + row * p.row_bytes_out);
    for (int v = sl; v < vpr; v += team) dst[v] = src[v];
  }
}

// Different dtypes: element-wise conversion (round to nearest even).
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) kv_append_convert_kernel(AppendParams p) {
  const int D = p.head_dim;
  const int64_t rows = (int64_t)p.n_layers * p.batch * p.n_tokens * p.nkv * p.n_heads;
  const int64_t total = rows * D;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / D;
    const int d = (int)(idx - r * D);
    int64_t q = r;
    const int h = (int)(q % p.n_heads); q /= p.n_heads;
    const int kv = (int)(q % p.nkv); q /= p.nkv;
    const int t = (int)(q % p.n_tokens); q /= p.n_tokens;
    const int b = (int)(q % p.batch);
    const int layer = (int)(q / p.batch);
    const int64_t row = append_dst_row(p, layer, b, t, h);
    if (row < 0) continue;
    const Tin* src = reinterpret_cast<const Tin*>(p.in[kv] + layer * p.in_stride_layer +
                                                  b * p.in_stride_seq + h * p.in_stride_head +
                                                  t * p.in_stride_tok);
    Tout* dst = reinterpret_cast<Tout*>(p.pool[kv] + layer * p.pool_layer_stride +
                                        row * p.row_bytes_out);
    dst[d] = Conv<Tout>::from_f(Conv<Tin>::to_f(src[d]));
  }
}

template <typename Tin>
static void launch_convert_from(int pool_dtype, const AppendParams& p, int grid, cudaStream_t s) {
  switch (pool_dtype) {
    case SNAPMIND_DTYPE_F32: kv_append_convert_kernel<Tin, float><<<grid, 256, 0, s>>>(p); break;
    case SNAPMIND_DTYPE_BF16:
      kv_append_convert_kernel<Tin, __nv_bfloat16><<<grid, 256, 0, s>>>(p);
      break;
    default: kv_append_convert_kernel<Tin, __half><<<grid, 256, 0, s>>>(p); break;
  }
}

// ---------------------------------------------------------------------------
// gather
// ---------------------------------------------------------------------------
struct GatherParams {
  const char* pool[2];
  char* out[2];
  int64_t pool_layer_stride, out_layer_stride;  // bytes
  int64_t out_capacity_rows;                    // token rows (x heads) one layer's output holds
  const int32_t* tables;
  int64_t table_stride_seq, table_stride_layer;
  int32_t table_width;
  const int32_t* seq_lens;
  int32_t seq_len0;
  int32_t n_layers, batch, n_heads, block_size, num_blocks;
  int32_t row_bytes;
  int32_t nkv;  // 2 for K and V pools, 1 for a single pool
  int32_t* err;
};

// Block-wide exclusive scan of ceil(len/bs) and len over the batch, written to
// shared memory (cu_blocks[0..B], cu_tokens[0..B]).  Runs once per CTA.
__device__ void scan_lengths(const GatherParams& p, int32_t* cu_blocks, int32_t* cu_tok) {
  __shared__ int32_t s_wb[32], s_wt[32];
  __shared__ int32_t s_carry_b, s_carry_t;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  if (tid == 0) { s_carry_b = 0; s_carry_t = 0; }
  __syncthreads();
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int b = base + tid;
    int len = 0;
    if (b < p.batch) len = p.seq_lens ? p.seq_lens[b] : p.seq_len0;
    if (len < 0) len = 0;
    int nb = (len + p.block_size - 1) / p.block_size;
    int xb = nb, xt = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int yb = __shfl_up_sync(0xffffffffu, xb, o);
      int yt = __shfl_up_sync(0xffffffffu, xt, o);
      if (lane >= o) { xb += yb; xt += yt; }
    }
    if (lane == 31) { s_wb[warp] = xb; s_wt[warp] = xt; }
    __syncthreads();
    if (warp == 0) {
      int wb = lane < nwarps ? s_wb[lane] : 0;
      int wt = lane < nwarps ? s_wt[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int yb = __shfl_up_sync(0xffffffffu, wb, o);
        int yt = __shfl_up_sync(0xffffffffu, wt, o);
        if (lane >= o) { wb += yb; wt += yt; }
      }
      if (lane < nwarps) { s_wb[lane] = wb; s_wt[lane] = wt; }
    }
    __syncthreads();
    const int pre_b = (warp > 0 ? s_wb[warp - 1] : 0) + s_carry_b;
    const int pre_t = (warp > 0 ? s_wt[warp - 1] : 0) + s_carry_t;
    if (b < p.batch) {
      cu_blocks[b] = pre_b + xb - nb;
      cu_tok[b] = pre_t + xt - len;
    }
    __syncthreads();
    if (tid == blockDim.x - 1) {
      s_carry_b = pre_b + xb;
      s_carry_t = pre_t + xt;
    }
    __syncthreads();
  }
  if (tid == 0) {
    cu_blocks[p.batch] = s_carry_b;
    cu_tok[p.batch] = s_carry_t;
  }
  __syncthreads();
}

constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 4;

template <int W>
__global__ void __launch_bounds__(kGatherThreads) kv_gather_kernel(GatherParams p) {
  using V = typename VecT<W>::type;
  extern __shared__ int32_t smem_i32[];
  int32_t* cu_blocks = smem_i32;
  int32_t* cu_tok = smem_i32 + p.batch + 1;
  scan_lengths(p, cu_blocks, cu_tok);
  const int total_blocks = cu_blocks[p.batch];
  if (total_blocks == 0) return;
  if ((int64_t)cu_tok[p.batch] * p.n_heads > p.out_capacity_rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_TABLE);
    return;
  }
  const int64_t items = (int64_t)p.n_layers * p.nkv * total_blocks;
  const int vrow = p.row_bytes / W;  // vectors per token row
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int gb = (int)(it % total_blocks);
    const int rest = (int)(it / total_blocks);
    const int kv = rest % p.nkv;
    const int layer = rest / p.nkv;
    const int b = upper_bound_i32(cu_blocks, p.batch + 1, gb) - 1;
    const int j = gb - cu_blocks[b];
    const int len = cu_tok[b + 1] - cu_tok[b];
    const int rows = min(p.block_size, len - j * p.block_size);
    if (j >= p.table_width) {
      if (threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_TABLE);
      continue;
    }
    const int32_t phys =
        p.tables[(int64_t)layer * p.table_stride_layer + (int64_t)b * p.table_stride_seq + j];
    if (phys < 0 || phys >= p.num_blocks) {
      if (threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
      continue;
    }
    const char* src = p.pool[kv] + layer * p.pool_layer_stride +
                      (int64_t)phys * p.n_heads * p.block_size * p.row_bytes;
    char* dst = p.out[kv] + layer * p.out_layer_stride +
                ((int64_t)cu_tok[b] * p.n_heads + (int64_t)j * p.block_size) * p.row_bytes;
    const int vhead = rows * vrow;        // vectors per head in this tile
    const int total = vhead * p.n_heads;  // vectors in this work item
    const int64_t src_hstride = (int64_t)p.block_size * p.row_bytes;
    const int64_t dst_hstride = (int64_t)len * p.row_bytes;
    for (int v0 = threadIdx.x; v0 < total; v0 += kGatherThreads * kGatherUnroll) {
      V buf[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int v = v0 + u * kGatherThreads;
        if (v < total) {
          const int h = v / vhead, w = v - h * vhead;
          buf[u] = reinterpret_cast<const V*>(src + h * src_hstride)[w];
        }
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int v = v0 + u * kGatherThreads;
        if (v < total) {
          const int h = v / vhead, w = v - h * vhead;
          reinterpret_cast<V*>(dst + h * dst_hstride)[w] = buf[u];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// compaction copy (evict)
// ---------------------------------------------------------------------------
constexpr int kMaxCopySlots = 64;
struct CopySlotsParams {
  char* pool[2];
  int32_t src_block[kMaxCopySlots], src_row[kMaxCopySlots];
  int32_t dst_block[kMaxCopySlots], dst_row[kMaxCopySlots];
  int32_t n, n_heads, block_size, num_blocks, row_bytes;
  int32_t* err;
};

// One CTA per (K|V, head): stage all n source rows in shared memory, then
// write them, so overlapping source/destination rows behave like the
// reference's clone-before-assign.
__global__ void __launch_bounds__(256) kv_copy_slots_kernel(CopySlotsParams p) {
  extern __shared__ uint32_t stage[];
  const int kv = blockIdx.x & 1;
  const int h = blockIdx.x >> 1;
  const int words = p.row_bytes / 4;
  for (int i = 0; i < p.n; ++i) {
    if (p.src_block[i] < 0 || p.src_block[i] >= p.num_blocks || p.dst_block[i] < 0 ||
        p.dst_block[i] >= p.num_blocks) {
      if (threadIdx.x == 0) flag_error(p.err, SNAPMIND_DEVERR_BLOCK_ID);
      return;
    }
  }
  for (int e = threadIdx.x; e < p.n * words; e += blockDim.x) {
    const int i = e / words, w = e - i * words;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(
        p.pool[kv] +
        (((int64_t)p.src_block[i] * p.n_heads + h) * p.block_size + p.src_row[i]) * p.row_bytes);
    stage[e] = src[w];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.n * words; e += blockDim.x) {
    const int i = e / words, w = e - i * words;
    uint32_t* dst = reinterpret_cast<uint32_t*>(
        p.pool[kv] +
        (((int64_t)p.dst_block[i] * p.n_heads + h) * p.block_size + p.dst_row[i]) * p.row_bytes);
    dst[w] = stage[e];
  }
}

// ---------------------------------------------------------------------------
// batched block reservation / release (device free stack)
// ---------------------------------------------------------------------------
struct ReserveParams {
  int32_t* tables;
  int64_t table_stride;
  int32_t table_width;
  int32_t* seq_lens;
  const int32_t* seq_ids;  // release only
  int32_t batch, n_new, block_size;
  int32_t* free_stack;
  int32_t* free_top;
  int32_t num_blocks;
  int32_t* err;
};

// Exclusive block-wide scan of one int per thread; returns the prefix and
// writes the block total to *total.
__device__ int block_exclusive_scan(int x, int* total) {
  __shared__ int s_w[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_w[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? s_w[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nwarps) s_w[lane] = w;
  }
  __syncthreads();
  const int pre = (warp > 0 ? s_w[warp - 1] : 0) + incl - x;
  *total = s_w[nwarps - 1];
  __syncthreads();
  return pre;
}

__global__ void __launch_bounds__(1024) kv_reserve_kernel(ReserveParams p) {
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  // pass 1: total demand and table-width check
  int need_total = 0;
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int need = 0;
    if (b < p.batch) {
      const int old_len = p.seq_lens[b];
      const int new_len = old_len + p.n_new;
      const int have = (old_len + p.block_size - 1) / p.block_size;
      const int want = (new_len + p.block_size - 1) / p.block_size;
      need = want - have;
      if (want > p.table_width || old_len < 0) atomicOr(&s_bad, SNAPMIND_DEVERR_TABLE);
    }
    int tot;
    block_exclusive_scan(need, &tot);
    need_total += tot;
  }
  __syncthreads();
  const int top = *p.free_top;
  if (threadIdx.x == 0 && need_total > top) s_bad |= SNAPMIND_DEVERR_OUT_OF_BLOCKS;
  __syncthreads();
  if (s_bad) {
    if (threadIdx.x == 0) flag_error(p.err, s_bad);
    return;
  }
  // pass 2: deterministic assignment, ascending sequence order
  int carry = 0;
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int need = 0, have = 0, old_len = 0;
    if (b < p.batch) {
      old_len = p.seq_lens[b];
      have = (old_len + p.block_size - 1) / p.block_size;
      need = (old_len + p.n_new + p.block_size - 1) / p.block_size - have;
    }
    int tot;
    const int pre = block_exclusive_scan(need, &tot) + carry;
    if (b < p.batch) {
      for (int k = 0; k < need; ++k) {
        p.tables[(int64_t)b * p.table_stride + have + k] = p.free_stack[top - 1 - (pre + k)];
      }
      p.seq_lens[b] = old_len + p.n_new;
    }
    carry += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *p.free_top = top - need_total;
}

__global__ void __launch_bounds__(1024) kv_release_kernel(ReserveParams p) {
  // p.batch = number of listed sequences
  int carry = 0;
  const int top = *p.free_top;
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  int total = 0;
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int nb = 0;
    if (i < p.batch) {
      const int s = p.seq_ids[i];
      const int len = p.seq_lens[s];
      nb = (len + p.block_size - 1) / p.block_size;
      if (nb > p.table_width) atomicOr(&s_bad, SNAPMIND_DEVERR_TABLE);
    }
    int tot;
    block_exclusive_scan(nb, &tot);
    total += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0 && top + total > p.num_blocks) s_bad |= SNAPMIND_DEVERR_BLOCK_ID;
  __syncthreads();
  if (s_bad) {
    if (threadIdx.x == 0) flag_error(p.err, s_bad);
    return;
  }
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int nb = 0, s = 0;
    if (i < p.batch) {
      s = p.seq_ids[i];
      nb = (p.seq_lens[s] + p.block_size - 1) / p.block_size;
    }
    int tot;
    const int pre = block_exclusive_scan(nb, &tot) + carry;
    if (i < p.batch) {
      for (int k = 0; k < nb; ++k) {
        p.free_stack[top + pre + k] = p.tables[(int64_t)s * p.table_stride + k];
      }
    }
    __syncthreads();  // every read of seq_lens[s] above precedes the reset below
    if (i < p.batch) p.seq_lens[s] = 0;
    carry += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *p.free_top = top + total;
}

}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_abi_version(void) { return 1; }

const char* snapmind_last_error(void) { return g_last_error; }

int snapmind_kv_append(void* k_pool, void* v_pool, int pool_dtype, int64_t pool_layer_stride,
                       const void* k_new, const void* v_new, int in_dtype,
                       int64_t in_stride_layer, int64_t in_stride_seq, int64_t in_stride_head,
                       int64_t in_stride_tok, const int32_t* block_tables,
                       int64_t table_stride_seq, int64_t table_stride_layer, int32_t table_width,
                       const int32_t* slot_starts, int32_t slot_start0, int32_t n_layers,
                       int32_t batch, int32_t n_tokens, int32_t n_heads, int32_t head_dim,
                       int32_t block_size, int32_t num_blocks, int32_t* err_word, void* stream) {
  const int esz_out = dtype_size(pool_dtype), esz_in = dtype_size(in_dtype);
  SNAPMIND_CHECK_ARG(esz_out > 0 && esz_in > 0, "kv_append: unknown dtype");
  SNAPMIND_CHECK_ARG(n_layers >= 0 && batch >= 0 && n_tokens >= 0 && n_heads > 0 && head_dim > 0 &&
                         block_size > 0 && num_blocks > 0 && table_width >= 0,
                     "kv_append: bad sizes");
  const int nkv = v_pool ? 2 : 1;
  const int64_t rows = (int64_t)n_layers * batch * n_tokens * nkv * n_heads;
  if (rows == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(k_pool && k_new && block_tables && ((v_pool == nullptr) == (v_new == nullptr)),
                     "kv_append: null pointer (v_pool and v_new are both set or both NULL)");
  AppendParams p;
  p.pool[0] = static_cast<char*>(k_pool);
  p.pool[1] = static_cast<char*>(v_pool);
  p.in[0] = static_cast<const char*>(k_new);
  p.in[1] = static_cast<const char*>(v_new);
  p.pool_layer_stride = pool_layer_stride * esz_out;
  p.in_stride_layer = in_stride_layer * esz_in;
  p.in_stride_seq = in_stride_seq * esz_in;
  p.in_stride_head = in_stride_head * esz_in;
  p.in_stride_tok = in_stride_tok * esz_in;
  p.tables = block_tables;
  p.table_stride_seq = table_stride_seq;
  p.table_stride_layer = table_stride_layer;
  p.table_width = table_width;
  p.slot_starts = slot_starts;
  p.slot_start0 = slot_start0;
  p.n_layers = n_layers;
  p.batch = batch;
  p.n_tokens = n_tokens;
  p.n_heads = n_heads;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.row_bytes_in = head_dim * esz_in;
  p.row_bytes_out = head_dim * esz_out;
  p.head_dim = head_dim;
  p.nkv = nkv;
  p.err = err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int max_grid = num_sms() * 8;
  if (pool_dtype == in_dtype) {
    const int w = vec_width(p.row_bytes_out, p.in_stride_layer, p.in_stride_seq, p.in_stride_head,
                            p.in_stride_tok);
    const int w2 = vec_width(reinterpret_cast<uintptr_t>(k_new), reinterpret_cast<uintptr_t>(v_new),
                             reinterpret_cast<uintptr_t>(k_pool), reinterpret_cast<uintptr_t>(v_pool),
                             p.pool_layer_stride);
    const int vw = w < w2 ? w : w2;
    const int vpr = p.row_bytes_out / (vw > 1 ? vw : 1);
    const int per_warp = (vpr < 32 && 32 % vpr == 0) ? 32 / vpr : 1;
    const int64_t blocks = (rows + 8 * per_warp - 1) / (8 * per_warp);  // 8 warps per block
    const int grid = (int)(blocks < max_grid ? blocks : max_grid);
    switch (vw) {
      case 16: kv_append_copy_kernel<16><<<grid, 256, 0, s>>>(p); break;
      case 8: kv_append_copy_kernel<8><<<grid, 256, 0, s>>>(p); break;
      case 4: kv_append_copy_kernel<4><<<grid, 256, 0, s>>>(p); break;
      case 2: kv_append_copy_kernel<2><<<grid, 256, 0, s>>>(p); break;
      default:
        set_last_error("kv_append: misaligned rows");
        return SNAPMIND_ERR_BAD_ARGUMENT;
    }
  } else {
    const int64_t total = rows * head_dim;
    const int grid = (int)((total + 255) / 256 < max_grid ? (total + 255) / 256 : max_grid);
    switch (in_dtype) {
      case SNAPMIND_DTYPE_F32: launch_convert_from<float>(pool_dtype, p, grid, s); break;
      case SNAPMIND_DTYPE_BF16: launch_convert_from<__nv_bfloat16>(pool_dtype, p, grid, s); break;
      default: launch_convert_from<__half>(pool_dtype, p, grid, s); break;
    }
  }
  SNAPMIND_LAUNCH_CHECK("kv_append launch");
}

int snapmind_kv_gather(const void* k_pool, const void* v_pool, int dtype, int64_t pool_layer_stride,
                       void* k_out, void* v_out, int64_t out_layer_stride,
                       int64_t out_layer_capacity, const int32_t* block_tables, int64_t table_stride_seq,
                       int64_t table_stride_layer, int32_t table_width, const int32_t* seq_lens,
                       int32_t seq_len0, int32_t n_layers, int32_t batch, int32_t n_heads,
                       int32_t head_dim, int32_t block_size, int32_t num_blocks,
                       int32_t* err_word, void* stream) {
  const int esz = dtype_size(dtype);
  SNAPMIND_CHECK_ARG(esz > 0, "kv_gather: unknown dtype");
  SNAPMIND_CHECK_ARG(n_layers >= 0 && batch >= 0 && batch <= 8192 && n_heads > 0 && head_dim > 0 &&
                         block_size > 0 && num_blocks > 0,
                     "kv_gather: bad sizes");
  if (n_layers == 0 || batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(k_pool && k_out && block_tables && ((v_pool == nullptr) == (v_out == nullptr)),
                     "kv_gather: null pointer (v_pool and v_out are both set or both NULL)");
  GatherParams p;
  p.pool[0] = static_cast<const char*>(k_pool);
  p.pool[1] = static_cast<const char*>(v_pool);
  p.out[0] = static_cast<char*>(k_out);
  p.out[1] = static_cast<char*>(v_out);
  p.pool_layer_stride = pool_layer_stride * esz;
  p.out_layer_stride = out_layer_stride * esz;
  p.out_capacity_rows = out_layer_capacity / head_dim;
  p.tables = block_tables;
  p.table_stride_seq = table_stride_seq;
  p.table_stride_layer = table_stride_layer;
  p.table_width = table_width;
  p.seq_lens = seq_lens;
  p.seq_len0 = seq_len0;
  p.n_layers = n_layers;
  p.batch = batch;
  p.n_heads = n_heads;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.row_bytes = head_dim * esz;
  p.nkv = v_pool ? 2 : 1;
  p.err = err_word;
  const int vw = vec_width(p.row_bytes, reinterpret_cast<uintptr_t>(k_pool),
                           reinterpret_cast<uintptr_t>(v_pool), reinterpret_cast<uintptr_t>(k_out),
                           reinterpret_cast<uintptr_t>(v_out));
  const int vw2 = vec_width(p.pool_layer_stride, p.out_layer_stride);
  const int w = vw < vw2 ? vw : vw2;
  const size_t smem = 2 * sizeof(int32_t) * (size_t)(batch + 1);
  const int grid = num_sms() * 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kernel) -> int {
    if (smem > 48 * 1024) {
      cudaError_t e =
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_status(e, "kv_gather smem attribute");
    }
    kernel<<<grid, kGatherThreads, smem, s>>>(p);
    return cuda_status(cudaGetLastError(), "kv_gather launch");
  };
  switch (w) {
    case 16: return launch(kv_gather_kernel<16>);
    case 8: return launch(kv_gather_kernel<8>);
    case 4: return launch(kv_gather_kernel<4>);
    case 2: return launch(kv_gather_kernel<2>);
    default: set_last_error("kv_gather: misaligned rows"); return SNAPMIND_ERR_BAD_ARGUMENT;
  }
}

int snapmind_kv_copy_slots(void* k_pool, void* v_pool, int dtype, const int32_t* src_blocks,
                           const int32_t* src_rows, const int32_t* dst_blocks,
                           const int32_t* dst_rows, int32_t n, int32_t n_heads, int32_t head_dim,
                           int32_t block_size, int32_t num_blocks, int32_t* err_word,
                           void* stream) {
  const int esz = dtype_size(dtype);
  SNAPMIND_CHECK_ARG(esz > 0, "kv_copy_slots: unknown dtype");
  SNAPMIND_CHECK_ARG(n >= 0 && n <= kMaxCopySlots, "kv_copy_slots: n must be in [0, %d]",
                     kMaxCopySlots);
  SNAPMIND_CHECK_ARG((head_dim * esz) % 4 == 0, "kv_copy_slots: row bytes must be a multiple of 4");
  if (n == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(k_pool && v_pool && src_blocks && src_rows && dst_blocks && dst_rows,
                     "kv_copy_slots: null pointer");
  CopySlotsParams p;
  p.pool[0] = static_cast<char*>(k_pool);
  p.pool[1] = static_cast<char*>(v_pool);
  for (int i = 0; i < n; ++i) {
    SNAPMIND_CHECK_ARG(src_rows[i] >= 0 && src_rows[i] < block_size && dst_rows[i] >= 0 &&
                           dst_rows[i] < block_size,
                       "kv_copy_slots: row outside the block");
    p.src_block[i] = src_blocks[i];
    p.src_row[i] = src_rows[i];
    p.dst_block[i] = dst_blocks[i];
    p.dst_row[i] = dst_rows[i];
  }
  p.n = n;
  p.n_heads = n_heads;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.row_bytes = head_dim * esz;
  p.err = err_word;
  const size_t smem = (size_t)n * p.row_bytes;
  SNAPMIND_CHECK_ARG(smem <= 200 * 1024, "kv_copy_slots: rows too large");
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kv_copy_slots_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "kv_copy_slots smem attribute");
  }
  kv_copy_slots_kernel<<<2 * n_heads, 256, smem, static_cast<cudaStream_t>(stream)>>>(p);
  SNAPMIND_LAUNCH_CHECK("kv_copy_slots launch");
}

int snapmind_kv_reserve(int32_t* block_tables, int64_t table_stride_seq, int32_t table_width,
                        int32_t* seq_lens, int32_t batch, int32_t n_new, int32_t block_size,
                        int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                        int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(batch >= 0 && n_new >= 0 && block_size > 0 && table_width >= 0,
                     "kv_reserve: bad sizes");
  if (batch == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(block_tables && seq_lens && free_stack && free_top,
                     "kv_reserve: null pointer");
  ReserveParams p{block_tables, table_stride_seq, table_width, seq_lens, nullptr, batch, n_new,
                  block_size, free_stack, free_top, num_blocks, err_word};
  kv_reserve_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(p);
  SNAPMIND_LAUNCH_CHECK("kv_reserve launch");
}

int snapmind_kv_release(int32_t* block_tables, int64_t table_stride_seq, int32_t table_width,
                        int32_t* seq_lens, const int32_t* seq_ids, int32_t n_release,
                        int32_t block_size, int32_t* free_stack, int32_t* free_top,
                        int32_t num_blocks, int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(n_release >= 0 && block_size > 0, "kv_release: bad sizes");
  if (n_release == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(block_tables && seq_lens && seq_ids && free_stack && free_top,
                     "kv_release: null pointer");
  ReserveParams p{block_tables, table_stride_seq, table_width, seq_lens, seq_ids, n_release, 0,
                  block_size, free_stack, free_top, num_blocks, err_word};
  kv_release_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(p);
  SNAPMIND_LAUNCH_CHECK("kv_release launch");
}

}  // extern "C"
