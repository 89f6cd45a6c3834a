// Peer memory for the KV-head-sharded decode: the decode kernel of every rank
// stores its finished output rows straight into every rank's output buffer
// (NVLink peer stores through CUDA IPC mappings).  After it, on the same
// stream, one warp publishes the call's epoch into every rank's flag array and
// waits, bounded, until every rank's epoch has arrived.  No reference
// counterpart: snapmind runs on one device.  This replaces an all-gather of the
// per-rank head slices.
//
// Only plain loads and stores reach peer memory; no TMA touches it.
#include <cuda.h>
#include <string.h>

#include "common.cuh"

namespace snapmind {
namespace {

// A wait gives up after this long (ns of %globaltimer) and reports
// SNAPMIND_DEVERR_TIMEOUT; the ranks' decodes take microseconds, so only a
// rank that never launched its step (or a host stall of that length) reaches it.
constexpr unsigned long long kPeerWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* ptr) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int32_t* ptr, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// SIGNAL: lane r writes `epoch` into element `rank` of rank r's flag array.
// The decode before this kernel on the stream has completed; the system-scope
// fence orders its peer stores before the flags.  WAIT: lane r waits for
// flags[r] to reach `epoch` (epochs only grow; the signed difference tolerates
// wrap-around).
__global__ void peer_sync_kernel(int32_t* const* peer_flags, const int32_t* flags, int n, int rank, int32_t epoch,
                                 int what, int32_t* err) {
  if (what & SNAPMIND_PEER_SIGNAL) {
    __threadfence_system();
    for (int r = threadIdx.x; r < n; r += blockDim.x) st_release_sys(peer_flags[r] + rank, epoch);
  }
  if (!(what & SNAPMIND_PEER_WAIT)) return;
  const unsigned long long t0 = global_ns();
  for (int r = threadIdx.x; r < n; r += blockDim.x) {
    while ((int32_t)(ld_acquire_sys(flags + r) - epoch) < 0) {
      if (global_ns() - t0 > kPeerWaitNs) {
        flag_error(err, SNAPMIND_DEVERR_TIMEOUT);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncwarp();
  __threadfence_system();
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  }
  return fn;
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_peer_sync(int32_t* const* peer_flags, const int32_t* flags, int32_t n_peers, int32_t rank,
                       int32_t epoch, int32_t what, int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(n_peers >= 1 && n_peers <= 1024 && rank >= 0 && rank < n_peers && epoch > 0 &&
                         (what & ~(SNAPMIND_PEER_SIGNAL | SNAPMIND_PEER_WAIT)) == 0,
                     "peer_sync: bad arguments");
  SNAPMIND_CHECK_ARG(!(what & SNAPMIND_PEER_SIGNAL) || peer_flags != nullptr, "peer_sync: peer_flags is NULL");
  SNAPMIND_CHECK_ARG(!(what & SNAPMIND_PEER_WAIT) || flags != nullptr, "peer_sync: flags is NULL");
  if (what == 0) return SNAPMIND_OK;
  peer_sync_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(peer_flags, flags, n_peers, rank, epoch, what,
                                                                    err_word);
  return cuda_status(cudaGetLastError(), "peer_sync launch");
}

int snapmind_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  SNAPMIND_CHECK_ARG(ptr && handle_out && offset_out, "ipc_export: null pointer");
  AddressRangeFn fn = address_range_fn();
  if (!fn) {
    set_last_error("ipc_export: cuMemGetAddressRange is unavailable");
    return SNAPMIND_ERR_UNSUPPORTED;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_last_error("ipc_export: %p is not device memory of this context", ptr);
    return SNAPMIND_ERR_BAD_ARGUMENT;
  }
  cudaIpcMemHandle_t h;
  const int rc = cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  if (rc != SNAPMIND_OK) return rc;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return SNAPMIND_OK;
}

int snapmind_ipc_open(const void* handle, int64_t offset, void** ptr_out) {
  SNAPMIND_CHECK_ARG(handle && ptr_out && offset >= 0, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const int rc = cuda_status(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess),
                             "cudaIpcOpenMemHandle");
  if (rc != SNAPMIND_OK) return rc;
  *ptr_out = static_cast<char*>(base) + offset;
  return SNAPMIND_OK;
}

int snapmind_ipc_close(void* ptr, int64_t offset) {
  SNAPMIND_CHECK_ARG(ptr && offset >= 0, "ipc_close: bad arguments");
  return cuda_status(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset), "cudaIpcCloseMemHandle");
}

}  // extern "C"
