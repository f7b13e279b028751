// Tensor-core paged decode kernels (placeholder until the mma path lands).
#include "decode_common.cuh"

namespace qkv {

bool decode_mma_supported(const DecodeParams&, bool) { return false; }

int launch_decode_mma(const DecodeParams&, bool, cudaStream_t) {
  return QKV_ERR_UNSUPPORTED;
}

}  // namespace qkv
