// Tensor-core paged GQA decode (bf16, sm_100a).  Not yet enabled: every
// shape takes the CUDA-core kernel in paged_decode.cu.
#include "paged_decode.cuh"

namespace snapmind {

bool decode_fast_supported(const DecodeParams&, int) { return false; }

int launch_decode_fast(const DecodeParams&, int, cudaStream_t) {
  return SNAPMIND_ERR_UNSUPPORTED;
}

}  // namespace snapmind
