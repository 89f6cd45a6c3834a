// Paged GQA decode for callers that cannot allocate device memory.
//
// snapmind_paged_gqa_decode needs a scratch workspace (split tickets and
// partial softmax states) that its caller allocates.  Some callers of this
// library cannot do that on the decode path: a host bound through the C ABI
// (a cgo / JNI / ctypes binding) that has no CUDA allocator of its own and
// whose device memory is owned by another allocator (for example PyTorch's
// caching allocator, which a foreign caller cannot reach), or a serving loop
// that must not call cudaMalloc between steps because cudaMalloc can
// synchronise the device.  For them this file keeps the scratch in a fixed
// file-scope device array, so the entry point below allocates nothing.
//
// Limits and behaviour:
//   * the array holds SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES (16 MiB); a call
//     whose workspace would need more is rejected with a clear error;
//   * every GPU that loads this library holds one such array until the
//     process exits;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current); make
//     that first call before any stream capture;
//   * all calls on a device share the one array and it keeps the last call's
//     contents: each call clears the ticket counters it needs (an async
//     memset on the caller's stream), and calls that overlap on the GPU — on
//     different streams, or from several host threads without ordering —
//     race on the shared scratch and must not be issued.
#include <mutex>

#include "common.cuh"
#include "paged_decode.cuh"

namespace snapmind {
namespace {

static __device__ __align__(256) uint8_t g_decode_scratch[SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "paged_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_last_error("paged_decode_noalloc: device ordinal %d out of range", dev);
    return SNAPMIND_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess) return cuda_status(e, "paged_decode_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return SNAPMIND_OK;
}

}  // namespace
}  // namespace snapmind

using namespace snapmind;

extern "C" {

int snapmind_paged_gqa_decode_noalloc(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                      const void* k_pool, const void* v_pool, int dtype,
                                      const int32_t* block_tables, int64_t table_stride_seq,
                                      int32_t table_width, const int32_t* seq_lens, void* out,
                                      int64_t out_stride_seq, int64_t out_stride_head, float scale,
                                      int32_t batch, int32_t n_q_heads, int32_t n_kv_heads,
                                      int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                      int32_t max_seq_len, int32_t split_tokens, int32_t flags,
                                      int32_t* err_word, void* stream) {
  SNAPMIND_CHECK_ARG(batch >= 0 && n_q_heads > 0 && n_kv_heads > 0 && head_dim > 0 && block_size > 0 &&
                         table_width >= 0,
                     "paged_decode_noalloc: bad sizes");
  if (batch == 0) return SNAPMIND_OK;
  // the same split plan snapmind_paged_gqa_decode would use
  if (max_seq_len <= 0) max_seq_len = table_width * block_size;
  if (split_tokens <= 0) split_tokens = default_split_tokens(batch, n_kv_heads, max_seq_len, block_size);
  const int64_t need = snapmind_paged_gqa_decode_workspace_bytes(batch, n_q_heads, n_kv_heads, head_dim,
                                                                 max_seq_len, split_tokens);
  SNAPMIND_CHECK_ARG(need > 0, "paged_decode_noalloc: bad split plan");
  SNAPMIND_CHECK_ARG(need <= (int64_t)SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES,
                     "paged_decode_noalloc: this call needs %lld bytes of scratch but the static scratch "
                     "holds %lld; use a larger split_tokens, a smaller batch or max_seq_len, or "
                     "snapmind_paged_gqa_decode with a caller-owned workspace",
                     (long long)need, (long long)SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != SNAPMIND_OK) return rc;
  // the split tickets must start at zero; the partials need no clearing
  const WorkspaceLayout ws = workspace_layout(batch, n_q_heads, n_kv_heads, head_dim,
                                              (max_seq_len + split_tokens - 1) / split_tokens);
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(scratch) + ws.counters_off, 0,
                                  (size_t)batch * n_kv_heads * sizeof(int32_t),
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "paged_decode_noalloc: clearing tickets");
  return snapmind_paged_gqa_decode(q, q_stride_seq, q_stride_head, k_pool, v_pool, dtype, block_tables,
                                   table_stride_seq, table_width, seq_lens, out, out_stride_seq,
                                   out_stride_head, scale, batch, n_q_heads, n_kv_heads, head_dim,
                                   block_size, num_blocks, max_seq_len, split_tokens, flags, scratch,
                                   (int64_t)SNAPMIND_NOALLOC_DECODE_SCRATCH_BYTES, err_word, stream);
}

}  // extern "C"
