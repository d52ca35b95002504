// Launch entry points of every kernel, for the host engine and the C ABI.
#pragma once
#include <cuda_runtime.h>

#include "attention.cuh"
#include "conv.cuh"
#include "decode_types.cuh"
#include "norm.cuh"
#include "q8_gemv.cuh"
#include "q8_prefill.cuh"
#include "sampling.cuh"

namespace lfm3 {

cudaError_t launch_q8_gemv(const GemvParams& p, int grid, cudaStream_t stream,
                           bool pdl);

// Reads and clears the device error word (bounded waits that gave up).
unsigned take_device_error();
// One bounded wait that nothing ends, given up after limit_ns (the device
// error word then holds kErrWaitProbe): exercises the failure path.
cudaError_t launch_wait_probe(uint64_t limit_ns, cudaStream_t stream);

// Records the message lfm3_last_error() returns on this thread; returns code.
int set_last_error(int code, const char* message);

// Raises a kernel's dynamic shared memory limit to `bytes` on the current
// device, once per (kernel, device, bytes): function attributes belong to
// each device's context. Thread-safe.
cudaError_t ensure_dynamic_smem(const void* kernel, int bytes);

// Process-wide count of kernels this library has launched.
void note_launch(int kernels = 1);
unsigned long long launch_count();

// kernel<<<grid, block, smem, stream>>>(args...), counted. With pdl the
// kernel may start while the previous kernel in the stream finishes
// (programmatic stream serialization): it must reach grid_dependency_wait()
// before it touches anything an earlier kernel writes or reads.
template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block,
                          size_t smem, cudaStream_t stream, bool pdl,
                          Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  config.attrs = attr;
  config.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&config, kernel, Params(args)...);
}

}  // namespace lfm3
