// Shared definitions for the snapmind_b200 KV-cache kernels (sm_100a).
//
// Every exported entry point is `extern "C"`, takes plain device pointers,
// element strides and sizes, a cudaStream_t passed as `void*`, and returns an
// int status (SNAPMIND_OK ... SNAPMIND_ERR_*).  The message of the most recent
// failure on the calling host thread is available from snapmind_last_error().
//
// Device-side checks never trap: a kernel that meets an out-of-range block id,
// slot or split index skips the access and ORs a bit into the caller-supplied
// device error word (may be NULL), which the host reads at its own sync point.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/snapmind_b200.h"

namespace snapmind {

// ---- host-side error reporting -------------------------------------------
void set_last_error(const char* fmt, ...);

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SNAPMIND_OK;
  set_last_error("%s: %s", what, cudaGetErrorString(e));
  return SNAPMIND_ERR_CUDA;
}

#define SNAPMIND_CHECK_ARG(cond, ...)            \
  do {                                           \
    if (!(cond)) {                               \
      ::snapmind::set_last_error(__VA_ARGS__);   \
      return SNAPMIND_ERR_BAD_ARGUMENT;          \
    }                                            \
  } while (0)

#define SNAPMIND_LAUNCH_CHECK(what) \
  return ::snapmind::cuda_status(cudaGetLastError(), what)

inline int dtype_size(int dtype) {
  switch (dtype) {
    case SNAPMIND_DTYPE_F32: return 4;
    case SNAPMIND_DTYPE_BF16: return 2;
    case SNAPMIND_DTYPE_F16: return 2;
    default: return 0;
  }
}

inline int num_sms() {
  static int cached = 0;
  if (cached == 0) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached = n > 0 ? n : 148;
  }
  return cached;
}

// ---- device helpers ---------------------------------------------------------
__device__ __forceinline__ void flag_error(int32_t* err, int32_t bit) {
  if (err != nullptr) atomicOr(err, bit);
}

template <typename T> struct Conv;
template <> struct Conv<float> {
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct Conv<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Conv<__half> {
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

// 16-byte vector type used by the copy kernels.
struct __align__(16) Vec16 { uint32_t x, y, z, w; };
struct __align__(8) Vec8 { uint32_t x, y; };

template <int BYTES> struct VecT;
template <> struct VecT<16> { using type = Vec16; };
template <> struct VecT<8> { using type = Vec8; };
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<2> { using type = uint16_t; };

// Largest power-of-two vector width (<= 16 bytes) dividing every given value.
inline int vec_width(int64_t a, int64_t b = 0, int64_t c = 0, int64_t d = 0, int64_t e = 0) {
  for (int w = 16; w >= 2; w >>= 1) {
    if (a % w == 0 && b % w == 0 && c % w == 0 && d % w == 0 && e % w == 0) return w;
  }
  return 1;
}

__device__ __forceinline__ int upper_bound_i32(const int32_t* a, int n, int32_t x) {
  // first index i in [0, n) with a[i] > x, or n
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] <= x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

}  // namespace snapmind
