// Rotary position encoding of q and k in place, one launch for both, for the
// paged attention plugin.
//
// Rotate-half convention of snapmind's RotaryPositionalEncoding
// (snapmind/layers/positional/rope.py:47-61):
//   x_rot[d] = x[d] * cos[p][d] + rotate_half(x)[d] * sin[p][d],
//   rotate_half(x)[d] = -x[d + D/2] for d < D/2, x[d - D/2] otherwise,
// with cos/sin rows of the module's tables (fp32, [n_pos][D]) cast to the
// tensor's dtype first and each product and the sum rounded to that dtype, as
// the three separate torch ops do — so the result is bit-identical to
// apply_to_qk on the same device.  Position of token t of sequence b:
// positions[b * pos_stride_b + t], or t when positions is NULL (apply_to_qk
// without position_ids).
#include "common.cuh"

namespace snapmind {
namespace {

struct RopeTensor {
  char* base;
  int64_t stride_b, stride_h, stride_t;  // elements
  int32_t n_heads;
};

template <typename T>
__device__ __forceinline__ T rope_round(float x) {
  return Conv<T>::from_f(x);
}

// one thread per (tensor row, pair of dims d and d + D/2)
template <typename T>
__global__ void rope_qk_kernel(RopeTensor q, RopeTensor k, int batch, int n_tok, int head_dim,
                               const float* cos_t, const float* sin_t, int64_t n_pos, const int64_t* positions,
                               int64_t pos_stride_b, int32_t* err) {
  const int half = head_dim / 2;
  const int64_t rows_q = (int64_t)batch * q.n_heads * n_tok;
  const int64_t rows = rows_q + (int64_t)batch * k.n_heads * n_tok;
  const int64_t total = rows * half;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / half;
    const int d = (int)(e - r * half);
    const bool is_q = r < rows_q;
    const RopeTensor& ten = is_q ? q : k;
    const int64_t rr = is_q ? r : r - rows_q;
    const int t = (int)(rr % n_tok);
    const int64_t bh = rr / n_tok;
    const int h = (int)(bh % ten.n_heads);
    const int b = (int)(bh / ten.n_heads);
    const int64_t pos = positions ? positions[(int64_t)b * pos_stride_b + t] : t;
    if (pos < 0 || pos >= n_pos) {
      flag_error(err, SNAPMIND_DEVERR_POSITION);
      continue;
    }
    T* x = reinterpret_cast<T*>(ten.base) + b * ten.stride_b + h * ten.stride_h + t * ten.stride_t;
    const float* c = cos_t + pos * head_dim;
    const float* s = sin_t + pos * head_dim;
    const float x0 = Conv<T>::to_f(x[d]), x1 = Conv<T>::to_f(x[d + half]);
    // cos/sin in the tensor's dtype (apply_to_qk casts the tables with .to(q.dtype))
    const float c0 = Conv<T>::to_f(rope_round<T>(c[d])), c1 = Conv<T>::to_f(rope_round<T>(c[d + half]));
    const float s0 = Conv<T>::to_f(rope_round<T>(s[d])), s1 = Conv<T>::to_f(rope_round<T>(s[d + half]));
    // x * cos, rotate_half(x) * sin, their sum: each rounded to T
    const float a0 = Conv<T>::to_f(rope_round<T>(__fmul_rn(x0, c0)));
    const float b0 = Conv<T>::to_f(rope_round<T>(__fmul_rn(-x1, s0)));
    const float a1 = Conv<T>::to_f(rope_round<T>(__fmul_rn(x1, c1)));
    const float b1 = Conv<T>::to_f(rope_round<T>(__fmul_rn(x0, s1)));
    x[d] = rope_round<T>(__fadd_rn(a0, b0));
    x[d + half] = rope_round<T>(__fadd_rn(a1, b1));
  }
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_rope_qk(void* q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_t, int32_t n_q_heads,
                     void* k, int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_t, int32_t n_kv_heads,
                     int dtype, int32_t batch, int32_t n_tok, int32_t head_dim, const float* cos_table,
                     const float* sin_table, int64_t n_pos, const int64_t* positions, int64_t pos_stride_b,
                     int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(dtype_size(dtype) > 0, "rope_qk: unknown dtype");
  SNAPMIND_CHECK_ARG(batch >= 0 && n_tok >= 0 && n_q_heads >= 0 && n_kv_heads >= 0 && head_dim > 0 &&
                         head_dim % 2 == 0 && n_pos > 0,
                     "rope_qk: bad sizes (head_dim must be even)");
  const int64_t total = ((int64_t)batch * (n_q_heads + n_kv_heads) * n_tok) * (head_dim / 2);
  if (total == 0) return SNAPMIND_OK;
  SNAPMIND_CHECK_ARG((q || n_q_heads == 0) && (k || n_kv_heads == 0) && cos_table && sin_table,
                     "rope_qk: null pointer");
  RopeTensor tq{static_cast<char*>(q), q_stride_b, q_stride_h, q_stride_t, n_q_heads};
  RopeTensor tk{static_cast<char*>(k), k_stride_b, k_stride_h, k_stride_t, n_kv_heads};
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int grid = (int)(want < (int64_t)num_sms() * 8 ? want : (int64_t)num_sms() * 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SNAPMIND_DTYPE_F32:
      rope_qk_kernel<float><<<grid, threads, 0, st>>>(tq, tk, batch, n_tok, head_dim, cos_table, sin_table, n_pos,
                                                      positions, pos_stride_b, err_word);
      break;
    case SNAPMIND_DTYPE_BF16:
      rope_qk_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(tq, tk, batch, n_tok, head_dim, cos_table, sin_table,
                                                              n_pos, positions, pos_stride_b, err_word);
      break;
    default:
      rope_qk_kernel<__half><<<grid, threads, 0, st>>>(tq, tk, batch, n_tok, head_dim, cos_table, sin_table, n_pos,
                                                       positions, pos_stride_b, err_word);
  }
  return cuda_status(cudaGetLastError(), "rope_qk launch");
}

}  // extern "C"
