// Launch entry points of every kernel, for the host engine and the C ABI.
#pragma once
#include <cuda_runtime.h>

#include "attention.cuh"
#include "conv.cuh"
#include "decode_types.cuh"
#include "norm.cuh"
#include "q8_gemv.cuh"
#include "q8_prefill.cuh"

namespace lfm3 {

cudaError_t launch_q8_gemv(const GemvParams& p, int grid, cudaStream_t stream,
                           bool pdl);

// Reads and clears the device error word (bounded waits that gave up).
unsigned take_device_error();

// Records the message lfm3_last_error() returns on this thread; returns code.
int set_last_error(int code, const char* message);

// Process-wide count of kernels this library has launched.
void note_launch(int kernels = 1);
unsigned long long launch_count();

}  // namespace lfm3
