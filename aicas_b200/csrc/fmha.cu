#include <cstdio>
#include "fmha.cuh"

namespace aicas {
uint32_t fmha_capabilities() { return 0u; }
int run_fmha(const aicas_fmha_params*, bool, cudaStream_t, unsigned int*, char* err, size_t errlen) {
  snprintf(err, errlen, "tensor-core attention is not built yet");
  return AICAS_ERR_UNSUPPORTED;
}
}  // namespace aicas
