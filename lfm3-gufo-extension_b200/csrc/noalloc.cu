// Decode attention for callers that cannot allocate device memory.
//
// lfm3_cuda_attention (the reference's Attention operator) needs a scratch
// buffer from the caller for the per-span partial results and merge tickets
// of a long key history. Some callers cannot provide one: a serving loop
// that owns every byte of device memory through a fixed arena sized at
// start-up, or a latency-critical thread that must not call cudaMalloc
// (which can synchronise the device and stall every stream) between decode
// steps. lfm3_cuda_attention_decode_noalloc runs the same kernel with its
// scratch in a file-scope device array instead, so it allocates nothing.
//
// The array is sized for at most kNoAllocMaxHeads query heads (about 1 MiB)
// and lives on every GPU that loads this library until the process exits.
// Every call shares it and it keeps the last call's contents: the merge
// tickets are cleared on each call, and calls that overlap on the GPU (two
// streams, or two host threads) race on it and must be serialised by the
// caller.
#include <cuda.h>

#include <mutex>

#include "../../include/lfm3_cuda.h"
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kNoAllocMaxHeads = 32;
constexpr size_t kNoAllocPartialFloats =
    size_t(kNoAllocMaxHeads) * kMaxDecodeSplits * (kHeadDim + 2);
constexpr size_t kNoAllocTicketWords = 256;

// Partials of one decode row (heads x spans x (max, sum, 128 values)), then
// the tickets of its KV groups.
static __device__ __align__(256) float
    g_noalloc_scratch[kNoAllocPartialFloats + kNoAllocTicketWords];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
// Per device: the array's device address and the context it was looked up
// in. cudaDeviceReset ends that context and a later call runs in a new one
// where the module (and the array) is loaded again, possibly elsewhere, so
// a cached address is only reused in the context it came from.
float* g_scratch[kMaxDevices] = {};
CUcontext g_context[kMaxDevices] = {};

// The calling thread's current context (driver API, reached through the
// runtime so the library needs no link against libcuda).
cudaError_t current_context(CUcontext* ctx) {
  using GetCurrent = CUresult (*)(CUcontext*);
  static GetCurrent get = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault,
                                &status) != cudaSuccess ||
        status != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<GetCurrent>(fn);
  }();
  if (!get)
    return cudaErrorNotSupported;
  return get(ctx) == CUDA_SUCCESS ? cudaSuccess : cudaErrorDeviceUninitialized;
}

// The device address of g_noalloc_scratch on the current device. In host
// code the array's name is only a host-side stand-in, so the address is
// looked up with that device current: once per device and context (the
// first call on a device, or the first after a cudaDeviceReset), and reused
// while that context lives.
cudaError_t scratch_address(float** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return e;
  if (device < 0 || device >= kMaxDevices)
    return cudaErrorInvalidDevice;
  // (before the runtime's first call on this device there is no current
  // context yet: the lookup below creates it, and the next call, seeing a
  // different context, looks the address up once more)
  CUcontext ctx = nullptr;
  if ((e = current_context(&ctx)) != cudaSuccess)
    return e;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch[device] || g_context[device] != ctx) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess)
      return e;
    g_scratch[device] = static_cast<float*>(ptr);
    g_context[device] = ctx;
  }
  *out = g_scratch[device];
  return cudaSuccess;
}

}  // namespace
}  // namespace lfm3

extern "C" int lfm3_cuda_attention_decode_noalloc(
    const float* q, const uint16_t* k, const uint16_t* v, const float* gate,
    const uint16_t* cache_k, const uint16_t* cache_v, float* out, int heads,
    int kv_heads, int dim, int position, int capacity, int window,
    void* stream) {
  using namespace lfm3;
  if (dim != kHeadDim || kv_heads <= 0 || heads % kv_heads ||
      (heads / kv_heads != 2 && heads / kv_heads != 4 &&
       heads / kv_heads != 8))
    return set_last_error(LFM3_ERR_UNSUPPORTED,
                          "unsupported LFM3 attention shape");
  if (heads > kNoAllocMaxHeads)
    return set_last_error(
        LFM3_ERR_UNSUPPORTED,
        "lfm3_cuda_attention_decode_noalloc: more than 32 query heads exceeds "
        "its static scratch; use lfm3_cuda_attention with a scratch buffer");
  if (!q || !k || !v || !gate || !cache_k || !cache_v || !out ||
      capacity <= 0 || position < 0)
    return set_last_error(LFM3_ERR_INVALID, "invalid attention arguments");
  float* scratch = nullptr;
  if (const cudaError_t e = scratch_address(&scratch); e != cudaSuccess)
    return set_last_error(LFM3_ERR_CUDA, cudaGetErrorString(e));
  const auto s = static_cast<cudaStream_t>(stream);
  unsigned* tickets = reinterpret_cast<unsigned*>(scratch + kNoAllocPartialFloats);
  if (const cudaError_t e = cudaMemsetAsync(
          tickets, 0, kNoAllocTicketWords * sizeof(unsigned), s);
      e != cudaSuccess)
    return set_last_error(LFM3_ERR_CUDA, cudaGetErrorString(e));
  DecodeAttentionParams p{};
  p.q = q;
  p.gate = gate;
  p.ldq = heads * kHeadDim;
  p.ldg = heads;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.window = window;
  p.max_splits = kMaxDecodeSplits;
  p.out_f32 = out;
  p.partials = scratch;
  p.tickets = tickets;
  p.position = position;
  p.ring_k = reinterpret_cast<const __half*>(cache_k);
  p.ring_v = reinterpret_cast<const __half*>(cache_v);
  p.chunk_k = reinterpret_cast<const __half*>(k);
  p.chunk_v = reinterpret_cast<const __half*>(v);
  p.capacity = capacity;
  if (const cudaError_t e = launch_decode_attention(p, 1, s, false);
      e != cudaSuccess)
    return set_last_error(LFM3_ERR_CUDA, cudaGetErrorString(e));
  return LFM3_OK;
}
