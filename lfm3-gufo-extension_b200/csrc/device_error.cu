// The device error word and its host accessor.
#include "common.cuh"
#include "kernels.cuh"

#include <atomic>

namespace lfm3 {

__device__ unsigned g_device_error = 0;

namespace {
std::atomic<unsigned long long> g_launches{0};
}
void note_launch(int kernels) { g_launches += kernels; }
unsigned long long launch_count() { return g_launches.load(); }

unsigned take_device_error() {
  unsigned value = 0;
  if (cudaMemcpyFromSymbol(&value, g_device_error, sizeof(value)) !=
      cudaSuccess)
    return ~0u;
  if (value) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  }
  return value;
}

}  // namespace lfm3
