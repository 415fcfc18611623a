// Tensor-core (tcgen05) flash attention: causal GQA prefill and packed varlen.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "../../include/aicas_b200.h"

namespace aicas {

// AICAS_CAP_* bits for the attention kernels compiled into this library.
uint32_t fmha_capabilities();

// Launches the forward kernel for validated parameters.  Returns an AICAS_*
// status and writes a message into err on failure.
int run_fmha(const aicas_fmha_params* p, bool varlen, cudaStream_t stream, unsigned int* dev_err, char* err,
             size_t errlen);

}  // namespace aicas
