// Vision QKV projection with the RoPE in its epilogue (tcgen05): host entry point.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "../../include/aicas_b200.h"

namespace aicas {

// Launches the kernel for validated parameters on a device with `sms` SMs.
// Returns an AICAS_* status and writes a message into err on failure.
int run_vision_qkv(const aicas_vision_qkv_params* p, int sms, cudaStream_t stream, unsigned int* dev_err, char* err,
                   size_t errlen);

}  // namespace aicas
