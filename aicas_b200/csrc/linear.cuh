// Decode-side weight-streaming products (tcgen05): host entry points.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "../../include/aicas_b200.h"

namespace aicas {

// Bytes of workspace run_linear needs for validated parameters on a device
// with `sms` SMs.  Returns an AICAS_* status.
int plan_linear_workspace(const aicas_linear_params* p, int sms, size_t* bytes, char* err, size_t errlen);

// Launches the kernel for validated parameters.  Returns an AICAS_* status and
// writes a message into err on failure.
int run_linear(const aicas_linear_params* p, int sms, void* workspace, size_t workspace_bytes, cudaStream_t stream,
               unsigned int* dev_err, char* err, size_t errlen);

}  // namespace aicas
