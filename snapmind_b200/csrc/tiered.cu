// Tiered-cache support kernels for sm_100a.
//
// kv_concat: the live view of the tiered cache is the token-dimension
// concatenation of its hot chunks (in chunk order) and the active chunk
// (snapmind/kv_cache/tiered.py:156-182).  Every (segment, row) pair is one
// contiguous run of n_tokens x head_dim elements on both sides, so one CTA per
// pair copies it with W-byte vectors; K and V go to separate CTAs.
#include "common.cuh"

namespace snapmind {
namespace {

constexpr int kMaxSegs = 256;

struct ConcatParams {
  const char* src[2][kMaxSegs];
  int64_t row_stride[kMaxSegs];  // bytes
  int32_t n_bytes[kMaxSegs];     // bytes per row of the segment
  int64_t out_off[kMaxSegs];     // byte offset of the segment inside an output row
  char* out[2];
  int64_t out_row_stride;        // bytes
  int32_t n_segs;
};

template <int W>
__global__ void __launch_bounds__(256) kv_concat_kernel(ConcatParams p) {
  using V = typename VecT<W>::type;
  const int seg = blockIdx.x, row = blockIdx.y, kv = blockIdx.z;
  const int nvec = p.n_bytes[seg] / W;
  const V* src = reinterpret_cast<const V*>(p.src[kv][seg] + row * p.row_stride[seg]);
  V* dst = reinterpret_cast<V*>(p.out[kv] + row * p.out_row_stride + p.out_off[seg]);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[i] = src[i];
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" int snapmind_kv_concat(const snapmind_segment* segs, int32_t n_segs, int32_t rows,
                                  int32_t head_dim, int dtype, void* k_out, void* v_out,
                                  int64_t out_row_stride, void* stream) {
  const int esz = dtype_size(dtype);
  SNAPMIND_CHECK_ARG(esz > 0, "kv_concat: unknown dtype");
  SNAPMIND_CHECK_ARG(n_segs >= 0 && rows >= 0 && rows <= 65535 && head_dim > 0, "kv_concat: bad sizes");
  if (n_segs == 0 || rows == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG(segs && k_out && v_out, "kv_concat: null pointer");
  const int64_t row_bytes = (int64_t)head_dim * esz;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t tok_off = 0;
  for (int base = 0; base < n_segs; base += kMaxSegs) {
    const int n = n_segs - base < kMaxSegs ? n_segs - base : kMaxSegs;
    ConcatParams p;
    p.out[0] = static_cast<char*>(k_out);
    p.out[1] = static_cast<char*>(v_out);
    p.out_row_stride = out_row_stride * row_bytes;
    p.n_segs = n;
    int64_t align = p.out_row_stride | reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out);
    for (int i = 0; i < n; ++i) {
      const snapmind_segment& s = segs[base + i];
      SNAPMIND_CHECK_ARG(s.n_tokens >= 0 && s.row_stride >= s.n_tokens,
                         "kv_concat: segment %d has bad sizes", base + i);
      SNAPMIND_CHECK_ARG(s.n_tokens == 0 || (s.k && s.v), "kv_concat: segment %d has a null pointer",
                         base + i);
      p.src[0][i] = static_cast<const char*>(s.k);
      p.src[1][i] = static_cast<const char*>(s.v);
      p.row_stride[i] = s.row_stride * row_bytes;
      p.n_bytes[i] = (int32_t)(s.n_tokens * row_bytes);
      p.out_off[i] = tok_off * row_bytes;
      tok_off += s.n_tokens;
      align |= p.row_stride[i] | p.n_bytes[i] | p.out_off[i] | reinterpret_cast<uintptr_t>(s.k) |
               reinterpret_cast<uintptr_t>(s.v);
    }
    SNAPMIND_CHECK_ARG(tok_off <= out_row_stride, "kv_concat: output row holds %lld tokens, segments need %lld",
                       (long long)out_row_stride, (long long)tok_off);
    dim3 grid(n, rows, 2);
    if (align % 16 == 0) kv_concat_kernel<16><<<grid, 256, 0, st>>>(p);
    else if (align % 8 == 0) kv_concat_kernel<8><<<grid, 256, 0, st>>>(p);
    else if (align % 4 == 0) kv_concat_kernel<4><<<grid, 256, 0, st>>>(p);
    else kv_concat_kernel<2><<<grid, 256, 0, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "kv_concat launch");
  }
  return SNAPMIND_OK;
}
