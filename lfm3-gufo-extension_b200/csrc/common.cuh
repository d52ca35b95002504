// Shared device helpers for the sm_100a kernels: PTX wrappers (mbarrier,
// bulk copies, mma.sync, programmatic dependent launch), fp16 packing, the
// split-activation record format and the device error word.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lfm3 {

// ---- device error word ------------------------------------------------------
// Bounded waits that give up record a code here and return; the host reads
// it after the stream synchronises (lfm3_cuda_take_device_error).
enum DeviceError : unsigned {
  kErrNone = 0,
  kErrGemvFullWait = 1,
  kErrGemvEmptyWait = 2,
  kErrPrefillWait = 3,
  kErrTmemAlloc = 4,
  kErrWaitProbe = 5,  // lfm3_cuda_wait_probe's deliberate wait
};
// Defined once in device_error.cu (the library is built with relocatable
// device code).
extern __device__ unsigned g_device_error;

__device__ __forceinline__ void report_error(unsigned code) {
  atomicCAS(&g_device_error, 0u, code);
}

// Every mbarrier wait gives up after this much time on the global timer:
// far beyond any legitimate wait (microseconds), so only a broken pipeline
// reaches it, and the kernel then returns instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier / bulk copy -----------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Waits for the phase with this parity; false (and an error report) once
// limit_ns (kWaitLimitNs by default) have passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned error_code,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity))
    return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity))
      return true;
    if (global_timer_ns() - start > limit_ns) {
      report_error(error_code);
      return false;
    }
  }
}
// One contiguous global -> shared copy completing on bar. Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src,
                                          uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// An L2 policy for data read once per round (streamed weights): its lines
// are the first to go, so code, activations and the cache stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}
// bulk_load with an L2 cache policy.
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src,
                                               uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Asks L2 to fetch [src, src + bytes) (16-byte aligned, bytes % 16 == 0);
// completes on its own, nothing waits for it.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src),
               "r"(bytes)
               : "memory");
}

// One tiled TMA copy of a 3-D box at coordinates (x0, x1, x2) of `map` (a
// __grid_constant__ kernel parameter) completing on bar. x0 * element size
// must be a multiple of 16 bytes; the weight maps always start x0 at 0.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* map, int x0,
                                            int x1, int x2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(x1), "r"(x2),
      "r"(smem_addr(bar))
      : "memory");
}

// One tiled TMA copy of a 2-D box at (x0, x1) of `map`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int x0,
                                            int x1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x0), "r"(x1),
      "r"(smem_addr(bar))
      : "memory");
}

// ---- programmatic dependent launch ------------------------------------------
// Work before grid_dependency_wait() may only touch data that no earlier
// kernel in the stream writes (weights); everything else comes after it.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// ---- named barrier among a subset of warps ---------------------------------
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- mma.sync m16n8k16 f16 x f16 -> f32 -------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4],
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- Q8 codes -> f16 ----------------------------------------------------------
// Four signed codes (one little-endian word) become two half2 values, exactly:
// flipping the sign bit makes each code an unsigned byte u = q + 128, the
// byte is placed under the fp16 exponent of 1024 (0x64uu = 1024 + u), and
// subtracting 1152 leaves q.
__device__ __forceinline__ void codes_to_half2(uint32_t word, uint32_t& lo,
                                               uint32_t& hi) {
  const uint32_t u = word ^ 0x80808080u;
  lo = __byte_perm(u, 0x64646464u, 0x5150);
  hi = __byte_perm(u, 0x64646464u, 0x5352);
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152
  __half2 l = *reinterpret_cast<__half2*>(&lo);
  __half2 h = *reinterpret_cast<__half2*>(&hi);
  l = __hsub2(l, bias);
  h = __hsub2(h, bias);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}

// ---- split activations --------------------------------------------------------
// Decode projections read FP32 activations as two fp16 terms, x = hi + lo
// with hi = rn(x) and lo = rn(x - hi) (22 significant bits). Element k of a
// row lives in 32-byte record k / 8: hi[8] then lo[8], so one thread of the
// projection fetches both terms of 8 consecutive elements with two 16-byte
// loads.
struct SplitPair {
  __half hi, lo;
};
__device__ __forceinline__ SplitPair split_value(float v) {
  const __half hi = __float2half_rn(v);
  const __half lo = __float2half_rn(v - __half2float(hi));
  return {hi, lo};
}
// Writes element k of row `row` (row length K) into the split buffer.
__device__ __forceinline__ void store_split(void* split, int row, int K, int k,
                                            float v) {
  const SplitPair p = split_value(v);
  __half* rec =
      reinterpret_cast<__half*>(split) + (size_t(row) * (K / 8) + k / 8) * 16;
  rec[k % 8] = p.hi;
  rec[8 + k % 8] = p.lo;
}
// Writes 8 consecutive elements (k0 % 8 == 0) as one record.
__device__ __forceinline__ void store_split8(void* split, int row, int K,
                                             int k0, const float (&v)[8]) {
  union {
    __half h[16];
    uint4 u[2];
  } rec;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const SplitPair p = split_value(v[i]);
    rec.h[i] = p.hi;
    rec.h[8 + i] = p.lo;
  }
  uint4* dst =
      reinterpret_cast<uint4*>(split) + (size_t(row) * (K / 8) + k0 / 8) * 2;
  dst[0] = rec.u[0];
  dst[1] = rec.u[1];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace lfm3
