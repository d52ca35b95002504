// The device error word and its host accessor.
#include "common.cuh"
#include "kernels.cuh"

#include <atomic>
#include <mutex>
#include <set>
#include <tuple>

namespace lfm3 {

__device__ unsigned g_device_error = 0;

namespace {
std::atomic<unsigned long long> g_launches{0};
}
void note_launch(int kernels) { g_launches += kernels; }
unsigned long long launch_count() { return g_launches.load(); }

cudaError_t ensure_dynamic_smem(const void* kernel, int bytes) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return e;
  static std::mutex mutex;
  static std::set<std::tuple<const void*, int, int>> done;
  const std::lock_guard<std::mutex> lock(mutex);
  if (done.count({kernel, device, bytes}))
    return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           bytes);
  if (e == cudaSuccess)
    done.insert({kernel, device, bytes});
  return e;
}

namespace {
// One thread waits on an mbarrier that nothing arrives at: the bounded wait
// gives up after limit_ns and records kErrWaitProbe.
__global__ void wait_probe_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  mbar_wait(&bar, 0, kErrWaitProbe, limit_ns);
}
}  // namespace

cudaError_t launch_wait_probe(uint64_t limit_ns, cudaStream_t stream) {
  note_launch();
  wait_probe_kernel<<<1, 1, 0, stream>>>(limit_ns);
  return cudaGetLastError();
}

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
