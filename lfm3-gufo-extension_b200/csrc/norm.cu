// Row kernels: embedding gather, fused residual + sandwich RMSNorm, FP16
// row scaling, split records. One CTA of 256 threads per row; each thread
// owns 8 consecutive elements (H <= 2048 x ... in 8-element groups).
#include <cuda_bf16.h>

#include "common.cuh"
#include "norm.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxGroups = 4;  // 8-element groups per thread: H <= 8192

__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0)
    scratch[warp] = v;
  __syncthreads();
  float total = 0;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w)
    total += scratch[w];
  return total;
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
  v = warp_max(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0)
    scratch[warp] = v;
  __syncthreads();
  float total = 0;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w)
    total = fmaxf(total, scratch[w]);
  return total;
}

__device__ __forceinline__ int row_exponent(float maximum) {
  return maximum > 0 ? 14 - ilogbf(maximum) : 0;
}

// This thread's groups of a weight vector (8 consecutive values each).
template <int G>
__device__ __forceinline__ void load_groups(const float* w, int H,
                                            float (&dst)[G][8]) {
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (w && k0 < H) {
      const float4 a = *reinterpret_cast<const float4*>(w + k0);
      const float4 b = *reinterpret_cast<const float4*>(w + k0 + 4);
      dst[j][0] = a.x, dst[j][1] = a.y, dst[j][2] = a.z, dst[j][3] = a.w;
      dst[j][4] = b.x, dst[j][5] = b.y, dst[j][6] = b.z, dst[j][7] = b.w;
    }
  }
}

// Normalises v (this thread's groups of row `row`) with the norm weights nw
// (this thread's groups) and writes every requested output.
template <int G>
__device__ void finish_norm(float (&v)[G][8], int groups,
                            const float (&nw)[G][8], NormOut out, int row,
                            int H, float eps, float* scratch) {
  float squares = 0;
  for (int j = 0; j < groups; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i)
      squares = fmaf(v[j][i], v[j][i], squares);
  const float inv = 1.0F / sqrtf(block_sum(squares, scratch) / float(H) + eps);
  float maximum = 0;
  for (int j = 0; j < groups; ++j) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[j][i] = (v[j][i] * inv) * nw[j][i];
      maximum = fmaxf(maximum, fabsf(v[j][i]));
    }
  }
  for (int j = 0; j < groups; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (out.f32) {
      float* dst = out.f32 + size_t(row) * H + k0;
      *reinterpret_cast<float4*>(dst) =
          make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      *reinterpret_cast<float4*>(dst + 4) =
          make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
    }
    if (out.split)
      store_split8(out.split, row, H, k0, v[j]);
  }
  if (out.half) {
    const int e = row_exponent(block_max(maximum, scratch));
    if (threadIdx.x == 0)
      out.scale[row] = ldexpf(1.0F, -e);
    for (int j = 0; j < groups; ++j) {
      const int k0 = (threadIdx.x + j * kNormThreads) * 8;
      union {
        __half h[8];
        uint4 u;
      } pack;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        pack.h[i] = __float2half_rn(ldexpf(v[j][i], e));
      *reinterpret_cast<uint4*>(out.half + size_t(row) * H + k0) = pack.u;
    }
  }
}

// G: 8-element groups per thread (H <= 2048 G)
template <int G>
__global__ void __launch_bounds__(kNormThreads)
    residual_norm_kernel(const float* __restrict__ branch,
                         const float* __restrict__ post_w, float* x,
                         const float* __restrict__ norm_w, NormOut out, int H,
                         float eps, SplitBranch split) {
  __shared__ float scratch[kNormThreads / 32];
  // the norm weights do not depend on the previous kernel: load them while
  // it finishes
  float pw[G][8], nw[G][8];
  load_groups<G>(post_w, H, pw);
  load_groups<G>(norm_w, H, nw);
  grid_dependency_wait();
  allow_dependents();
  const int row = blockIdx.x, groups = H / 8 / kNormThreads + 1;
  const bool has_branch = branch || split.partial;
  float v[G][8];
  float b[G][8];
  float* xr = x + size_t(row) * H;
  int live = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (j >= groups || k0 >= H)
      break;
    live = j + 1;
    const float4 a0 = *reinterpret_cast<const float4*>(xr + k0);
    const float4 a1 = *reinterpret_cast<const float4*>(xr + k0 + 4);
    v[j][0] = a0.x, v[j][1] = a0.y, v[j][2] = a0.z, v[j][3] = a0.w;
    v[j][4] = a1.x, v[j][5] = a1.y, v[j][6] = a1.z, v[j][7] = a1.w;
    if (branch) {
      const float* br = branch + size_t(row) * H + k0;
      const float4 c0 = *reinterpret_cast<const float4*>(br);
      const float4 c1 = *reinterpret_cast<const float4*>(br + 4);
      b[j][0] = c0.x, b[j][1] = c0.y, b[j][2] = c0.z, b[j][3] = c0.w;
      b[j][4] = c1.x, b[j][5] = c1.y, b[j][6] = c1.z, b[j][7] = c1.w;
      if (split.second) {  // the other half of a K split, added second
        const float* br2 = split.second + size_t(row) * H + k0;
        const float4 e0 = *reinterpret_cast<const float4*>(br2);
        const float4 e1 = *reinterpret_cast<const float4*>(br2 + 4);
        b[j][0] += e0.x, b[j][1] += e0.y, b[j][2] += e0.z, b[j][3] += e0.w;
        b[j][4] += e1.x, b[j][5] += e1.y, b[j][6] += e1.z, b[j][7] += e1.w;
      }
    } else if (split.partial) {
      // the branch is scale[row] * (sum over K splits, in split order)
      const int tile = (k0 >> 8) * split.token_tiles + (row >> 8);
      const float* src = split.partial +
                         size_t(tile) * split.splits * kSplitTileFloats +
                         (row & 255) * 256 + (k0 & 255);
      float4 s0 = __ldcg(reinterpret_cast<const float4*>(src));
      float4 s1 = __ldcg(reinterpret_cast<const float4*>(src + 4));
      for (int q = 1; q < split.splits; ++q) {
        const float* sq = src + size_t(q) * kSplitTileFloats;
        const float4 d0 = __ldcg(reinterpret_cast<const float4*>(sq));
        const float4 d1 = __ldcg(reinterpret_cast<const float4*>(sq + 4));
        s0.x += d0.x, s0.y += d0.y, s0.z += d0.z, s0.w += d0.w;
        s1.x += d1.x, s1.y += d1.y, s1.z += d1.z, s1.w += d1.w;
      }
      const float sc = split.scale ? split.scale[row] : 1.0F;
      b[j][0] = s0.x * sc, b[j][1] = s0.y * sc, b[j][2] = s0.z * sc,
      b[j][3] = s0.w * sc;
      b[j][4] = s1.x * sc, b[j][5] = s1.y * sc, b[j][6] = s1.z * sc,
      b[j][7] = s1.w * sc;
    }
  }
  if (has_branch) {
    if (post_w) {
      float squares = 0;
      for (int j = 0; j < live; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          squares = fmaf(b[j][i], b[j][i], squares);
      const float inv =
          1.0F / sqrtf(block_sum(squares, scratch) / float(H) + eps);
      for (int j = 0; j < live; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          b[j][i] = (b[j][i] * inv) * pw[j][i];
    }
    for (int j = 0; j < live; ++j) {
      const int k0 = (threadIdx.x + j * kNormThreads) * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = v[j][i] + b[j][i];
      *reinterpret_cast<float4*>(xr + k0) =
          make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      *reinterpret_cast<float4*>(xr + k0 + 4) =
          make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
    }
  }
  if (norm_w)
    finish_norm(v, live, nw, out, row, H, eps, scratch);
}

// Eight values of one row per thread as three exact bf16 planes.
__global__ void split_bf16_rows_kernel(const float* __restrict__ x,
                                       __nv_bfloat16* planes, int rows, int K,
                                       int plane_rows) {
  grid_dependency_wait();
  allow_dependents();
  const size_t e = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (e >= size_t(rows) * K)
    return;
  const int r = int(e / K), k = int(e % K);
  const float4 a = *reinterpret_cast<const float4*>(x + e);
  const float4 b = *reinterpret_cast<const float4*>(x + e + 4);
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  union {
    __nv_bfloat16 h[8];
    uint4 u;
  } t[3];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float rest = v[i];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      t[q].h[i] = __float2bfloat16_rn(rest);
      rest -= __bfloat162float(t[q].h[i]);
    }
  }
#pragma unroll
  for (int q = 0; q < 3; ++q)
    *reinterpret_cast<uint4*>(planes + (size_t(q) * plane_rows + r) * K + k) =
        t[q].u;
}

__device__ __forceinline__ float half_bits(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

template <int G>
__global__ void __launch_bounds__(kNormThreads)
    embed_norm_kernel(const uint8_t* __restrict__ table, uint32_t type,
                      const uint32_t* __restrict__ ids,
                      const uint32_t* __restrict__ tokens, float* x,
                      const float* __restrict__ norm_w, NormOut out, int H,
                      float eps) {
  __shared__ float scratch[kNormThreads / 32];
  float nw[G][8];
  load_groups<G>(norm_w, H, nw);
  grid_dependency_wait();
  allow_dependents();
  const int row = blockIdx.x, groups = H / 8 / kNormThreads + 1;
  const uint32_t token = ids ? ids[row] : tokens[row];
  float v[G][8];
  int live = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (j >= groups || k0 >= H)
      break;
    live = j + 1;
    if (type == 8) {  // Q8_0: 8 codes of one block
      const uint8_t* blk = table + size_t(token) * (H / 32) * 34 +
                           size_t(k0 / 32) * 34;
      const float d = half_bits(*reinterpret_cast<const uint16_t*>(blk));
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = float(int8_t(blk[2 + k0 % 32 + i])) * d;
    } else if (type == 30 || type == 1) {  // BF16 / F16
      const uint16_t* r =
          reinterpret_cast<const uint16_t*>(table) + size_t(token) * H + k0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = type == 30 ? __uint_as_float(uint32_t(r[i]) << 16)
                             : half_bits(r[i]);
    } else {  // F32
      const float* r = reinterpret_cast<const float*>(table) +
                       size_t(token) * H + k0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = r[i];
    }
    float* xr = x + size_t(row) * H + k0;
    *reinterpret_cast<float4*>(xr) =
        make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
    *reinterpret_cast<float4*>(xr + 4) =
        make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
  }
  if (norm_w)
    finish_norm(v, live, nw, out, row, H, eps, scratch);
}

// One row per CTA held in registers, G 8-element groups per thread
// (K <= 2048 G, K % 8 == 0): maximum, exponent, then 16-byte stores.
template <int G>
__global__ void __launch_bounds__(kNormThreads)
    half_rows_kernel(const float* __restrict__ x,
                     const unsigned* __restrict__ row_max, __half* values,
                     float* scale, int K) {
  __shared__ float scratch[kNormThreads / 32];
  grid_dependency_wait();
  allow_dependents();
  const int row = blockIdx.x;
  const float* src = x + size_t(row) * K;
  float v[G][8];
  float m = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (k0 >= K)
      break;
    const float4 a = *reinterpret_cast<const float4*>(src + k0);
    const float4 b = *reinterpret_cast<const float4*>(src + k0 + 4);
    v[j][0] = a.x, v[j][1] = a.y, v[j][2] = a.z, v[j][3] = a.w;
    v[j][4] = b.x, v[j][5] = b.y, v[j][6] = b.z, v[j][7] = b.w;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m = fmaxf(m, fabsf(v[j][i]));
  }
  const float maximum =
      row_max ? __uint_as_float(row_max[row]) : block_max(m, scratch);
  const int e = row_exponent(maximum);
  if (threadIdx.x == 0)
    scale[row] = ldexpf(1.0F, -e);
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int k0 = (threadIdx.x + j * kNormThreads) * 8;
    if (k0 >= K)
      break;
    union {
      __half h[8];
      uint4 u;
    } pack;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pack.h[i] = __float2half_rn(ldexpf(v[j][i], e));
    *reinterpret_cast<uint4*>(values + size_t(row) * K + k0) = pack.u;
  }
}

// Any K: two passes over the row.
__global__ void __launch_bounds__(kNormThreads)
    half_rows_any_kernel(const float* __restrict__ x,
                         const unsigned* __restrict__ row_max, __half* values,
                         float* scale, int K) {
  __shared__ float scratch[kNormThreads / 32];
  grid_dependency_wait();
  allow_dependents();
  const int row = blockIdx.x;
  const float* src = x + size_t(row) * K;
  float maximum;
  if (row_max) {
    maximum = __uint_as_float(row_max[row]);
  } else {
    float m = 0;
    for (int k = threadIdx.x; k < K; k += kNormThreads)
      m = fmaxf(m, fabsf(src[k]));
    maximum = block_max(m, scratch);
  }
  const int e = row_exponent(maximum);
  if (threadIdx.x == 0)
    scale[row] = ldexpf(1.0F, -e);
  for (int k = threadIdx.x; k < K; k += kNormThreads)
    values[size_t(row) * K + k] = __float2half_rn(ldexpf(src[k], e));
}

__global__ void __launch_bounds__(256)
    row_copies_kernel(const __grid_constant__ RowCopies c) {
  grid_dependency_wait();
  allow_dependents();
  const int i = blockIdx.y, e = blockIdx.x * blockDim.x + threadIdx.x;
  if (c.error_out && i == 0 && e == 0)
    *c.error_out = *const_cast<volatile unsigned*>(&g_device_error);
  if (c.vector[i]) {
    if (e < c.floats[i] / 4)
      reinterpret_cast<float4*>(c.dst[i])[e] =
          reinterpret_cast<const float4*>(c.src[i])[e];
  } else if (e < c.floats[i]) {
    c.dst[i][e] = c.src[i][e];
  }
}

__global__ void split_rows_kernel(const float* __restrict__ x, void* split,
                                  int rows, int K) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // record index
  const int per_row = K / 8;
  if (i >= rows * per_row)
    return;
  const int row = i / per_row, k0 = (i % per_row) * 8;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    v[j] = x[size_t(row) * K + k0 + j];
  store_split8(split, row, K, k0, v);
}

cudaError_t launch_pdl(const void* func, dim3 grid, dim3 block,
                       cudaStream_t stream, bool pdl, void** args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  config.attrs = attr;
  config.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelExC(&config, func, args);
}

}  // namespace

cudaError_t launch_residual_norm(const float* branch, const float* post_w,
                                 float* x, const float* norm_w, NormOut out,
                                 int rows, int H, float eps,
                                 cudaStream_t stream, bool pdl,
                                 const SplitBranch* split,
                                 const float* branch2) {
  if (H % 8 || H > kNormThreads * 8 * kNormMaxGroups)
    return cudaErrorInvalidValue;
  SplitBranch sb{};
  if (split) {
    sb = *split;
    if (branch || !sb.partial || sb.splits < 1 ||
        sb.token_tiles < (rows + 255) / 256 || H % 256 || sb.second)
      return cudaErrorInvalidValue;
  }
  if (branch2) {
    if (!branch || split)
      return cudaErrorInvalidValue;
    sb.second = branch2;
  }
  if (!rows)
    return cudaSuccess;
  void* args[] = {&branch, &post_w, &x, &norm_w, &out, &H, &eps, &sb};
  const void* kernel =
      H <= 2048   ? reinterpret_cast<const void*>(residual_norm_kernel<1>)
      : H <= 4096 ? reinterpret_cast<const void*>(residual_norm_kernel<2>)
                  : reinterpret_cast<const void*>(residual_norm_kernel<4>);
  return launch_pdl(kernel, dim3(rows), dim3(kNormThreads), stream, pdl, args);
}

cudaError_t launch_embed_norm(const void* table, uint32_t type,
                              const uint32_t* ids, const uint32_t* tokens,
                              float* x, const float* norm_w, NormOut out,
                              int rows, int H, float eps, cudaStream_t stream,
                              bool pdl) {
  if (H % 32 || H > kNormThreads * 8 * kNormMaxGroups)
    return cudaErrorInvalidValue;
  if (!rows)
    return cudaSuccess;
  const uint8_t* t = static_cast<const uint8_t*>(table);
  void* args[] = {&t, &type, &ids, &tokens, &x, &norm_w, &out, &H, &eps};
  const void* kernel =
      H <= 2048   ? reinterpret_cast<const void*>(embed_norm_kernel<1>)
      : H <= 4096 ? reinterpret_cast<const void*>(embed_norm_kernel<2>)
                  : reinterpret_cast<const void*>(embed_norm_kernel<4>);
  return launch_pdl(kernel, dim3(rows), dim3(kNormThreads), stream, pdl, args);
}

cudaError_t launch_half_rows(const float* x, const unsigned* row_max,
                             __half* values, float* scale, int rows, int K,
                             cudaStream_t stream, bool pdl) {
  if (!rows)
    return cudaSuccess;
  const int groups = (K / 8 + kNormThreads - 1) / kNormThreads;
  const bool vector = K % 8 == 0 && groups <= 8 &&
                      reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(values) % 16 == 0;
  const auto kernel = !vector      ? half_rows_any_kernel
                      : groups <= 1 ? half_rows_kernel<1>
                      : groups <= 2 ? half_rows_kernel<2>
                      : groups <= 4 ? half_rows_kernel<4>
                                    : half_rows_kernel<8>;
  return launch_kernel(kernel, dim3(rows), dim3(kNormThreads), 0, stream, pdl,
                       x, row_max, values, scale, K);
}

cudaError_t launch_split_bf16_rows(const float* x, void* planes, int rows,
                                   int K, int plane_rows, cudaStream_t stream,
                                   bool pdl) {
  if (rows <= 0)
    return cudaSuccess;
  if (K % 8 || rows > plane_rows || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(planes) % 16)
    return cudaErrorInvalidValue;
  const size_t groups = size_t(rows) * K / 8;
  return launch_kernel(split_bf16_rows_kernel,
                       dim3(unsigned((groups + 255) / 256)), dim3(256), 0,
                       stream, pdl, x, static_cast<__nv_bfloat16*>(planes),
                       rows, K, plane_rows);
}

cudaError_t launch_row_copies(const RowCopies& copies, cudaStream_t stream,
                              bool pdl) {
  if (copies.count < 0 || copies.count > kMaxRowCopies)
    return cudaErrorInvalidValue;
  RowCopies c = copies;
  int most = 0;  // pieces of the longest copy
  for (int i = 0; i < c.count; ++i) {
    if (c.floats[i] < 0 || (c.floats[i] && (!c.src[i] || !c.dst[i])))
      return cudaErrorInvalidValue;
    c.vector[i] = c.floats[i] % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(c.src[i]) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(c.dst[i]) % 16 == 0;
    const int pieces = c.vector[i] ? c.floats[i] / 4 : c.floats[i];
    most = pieces > most ? pieces : most;
  }
  if (!c.count || !most) {
    if (!c.error_out)
      return cudaSuccess;
    c.count = 1;  // one (empty) copy still reports the error word
    c.floats[0] = 0;
    most = 1;
  }
  return launch_kernel(row_copies_kernel, dim3((most + 255) / 256, c.count),
                       dim3(256), 0, stream, pdl, c);
}

cudaError_t launch_split_rows(const float* x, void* split, int rows, int K,
                              cudaStream_t stream) {
  if (K % 8)
    return cudaErrorInvalidValue;
  const int records = rows * (K / 8);
  if (!records)
    return cudaSuccess;
  note_launch();
  split_rows_kernel<<<(records + 255) / 256, 256, 0, stream>>>(x, split, rows,
                                                               K);
  return cudaGetLastError();
}

}  // namespace lfm3
