// The stream type of the reference's operator header (hip/ops.hpp) mapped to
// CUDA, as an extension build on the B200 library supplies it. TEST
// INFRASTRUCTURE: used by tests/test_ops_shim.py to compile the reference's
// own header against include/lfm3_gpu_ops.inl.
#pragma once
#include <cuda_runtime.h>
using hipStream_t = cudaStream_t;
