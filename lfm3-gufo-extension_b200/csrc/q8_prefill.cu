// Prompt-pass Q8_0 projections (mma.sync path).
//
// CTA tile: 128 weight rows x 64 tokens, K streamed in 256-column chunks
// (8 Q8 blocks). A producer warp moves each chunk's weight rows (272 bytes
// each) and token rows (512 bytes of fp16) into a 3-stage shared-memory ring
// with bulk copies; 8 consumer warps (2 x 4, 64 rows x 16 tokens each)
// decode the codes exactly to fp16 and run two m16n8k16 MMAs per block and
// tile, then apply the block scale: acc += d * C, the reference's order
// (hip/q8_prefill.hpp:563-569). Row scales of the activations apply after
// the K loop.
#include "common.cuh"
#include "q8_prefill.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kPM = 128, kPN = 64, kPStages = 3, kPWarps = 8;
constexpr int kPThreads = (kPWarps + 1) * 32;
constexpr int kWChunk = 272;    // bytes per weight row per chunk
constexpr int kXChunk = 512;    // bytes per token row per chunk
constexpr int kXPitch = 576;    // padded: 8 tokens of a warp hit 32 banks

struct PrefillSmem {
  uint8_t w[kPStages][kPM * kWChunk];
  uint8_t x[kPStages][kPN * kXPitch];
  uint64_t full[kPStages];
  uint64_t empty[kPStages];
};

__device__ __forceinline__ const uint8_t* prefill_source(
    const PrefillParams& p, int t, int i, size_t row_bytes) {
  if (p.kind == kPrefillPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    const int row = (t - p.first_tile[j]) * kPM + i;
    return row < p.o[j].rows ? p.o[j].w + size_t(row) * row_bytes : nullptr;
  }
  // SwiGLU: rows 0-63 of the tile belong to consumer row-half 0, 64-127 to
  // half 1; within a half, 32 gate rows then the same 32 up rows.
  const int half = i / 64, within = i % 64;
  const int row = t * 64 + half * 32 + (within & 31);
  if (row >= p.o[0].rows)
    return nullptr;
  return p.o[within < 32 ? 0 : 1].w + size_t(row) * row_bytes;
}

__global__ void __launch_bounds__(kPThreads, 1)
    q8_prefill_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  PrefillSmem& s = *reinterpret_cast<PrefillSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int t = blockIdx.x, token0 = blockIdx.y * kPN;
  const int chunks = p.K / 256;
  const size_t row_bytes = size_t(p.K / 32) * 34;
  if (tid == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kPWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kPWarps) {
    int stage = 0;
    uint32_t phase = 0;
    const uint8_t* src[4];
    unsigned rows = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      src[j] = prefill_source(p, t, lane + 32 * j, row_bytes);
      rows += __popc(__ballot_sync(0xffffffffu, src[j] != nullptr));
    }
    const int tokens = min(kPN, p.tokens - token0);
    for (int c = 0; c < chunks; ++c) {
      if (!mbar_wait(&s.empty[stage], phase ^ 1, kErrPrefillWait))
        return;
      if (lane == 0)
        mbar_arrive_expect_tx(&s.full[stage],
                              rows * kWChunk + tokens * kXChunk);
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (src[j])
          bulk_load(s.w[stage] + (lane + 32 * j) * kWChunk,
                    src[j] + size_t(c) * kWChunk, kWChunk, &s.full[stage]);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int tok = lane + 32 * j;
        if (tok < tokens)
          bulk_load(s.x[stage] + tok * kXPitch,
                    p.x + size_t(token0 + tok) * p.K + size_t(c) * 256,
                    kXChunk, &s.full[stage]);
      }
      if (++stage == kPStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    return;
  }

  const int g = lane / 4, cq = lane % 4;
  const int wm = warp / 4, wn = warp % 4;
  float acc[4][2][4];
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[m][n][j] = 0;
  int stage = 0;
  uint32_t phase = 0;
  for (int c = 0; c < chunks; ++c) {
    if (!mbar_wait(&s.full[stage], phase, kErrPrefillWait))
      return;
    const uint8_t* wst = s.w[stage] + wm * 64 * kWChunk;
    const uint8_t* xst = s.x[stage] + (wn * 16) * kXPitch;
#pragma unroll 2
    for (int blk = 0; blk < 8; ++blk) {
      uint4 xb[2];
#pragma unroll
      for (int n = 0; n < 2; ++n)
        xb[n] = *reinterpret_cast<const uint4*>(
            xst + (n * 8 + g) * kXPitch + (blk * 32 + 8 * cq) * 2);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t w[2][2];
        float d[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint8_t* row = wst + (m * 16 + g + h * 8) * kWChunk + blk * 34;
          d[h] = __half2float(*reinterpret_cast<const __half*>(row));
          const uint8_t* q = row + 2 + 8 * cq;
          if (blk & 1) {
            const uint32_t* pw = reinterpret_cast<const uint32_t*>(q);
            w[h][0] = pw[0];
            w[h][1] = pw[1];
          } else {
            const uint32_t* pw = reinterpret_cast<const uint32_t*>(q - 2);
            const uint32_t v0 = pw[0], v1 = pw[1], v2 = pw[2];
            w[h][0] = __funnelshift_r(v0, v1, 16);
            w[h][1] = __funnelshift_r(v1, v2, 16);
          }
        }
        uint32_t a1[4], a2[4];
        codes_to_half2(w[0][0], a1[0], a1[2]);
        codes_to_half2(w[1][0], a1[1], a1[3]);
        codes_to_half2(w[0][1], a2[0], a2[2]);
        codes_to_half2(w[1][1], a2[1], a2[3]);
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          float cc[4] = {0, 0, 0, 0};
          mma_f16(cc, a1, xb[n].x, xb[n].y);
          mma_f16(cc, a2, xb[n].z, xb[n].w);
          acc[m][n][0] = fmaf(d[0], cc[0], acc[m][n][0]);
          acc[m][n][1] = fmaf(d[0], cc[1], acc[m][n][1]);
          acc[m][n][2] = fmaf(d[1], cc[2], acc[m][n][2]);
          acc[m][n][3] = fmaf(d[1], cc[3], acc[m][n][3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0)
      mbar_arrive(&s.empty[stage]);
    if (++stage == kPStages) {
      stage = 0;
      phase ^= 1;
    }
  }

  // ---- epilogue
  if (p.kind == kPrefillPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    const int row0 = (t - p.first_tile[j]) * kPM + wm * 64;
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = row0 + m * 16 + g + (e >= 2 ? 8 : 0);
          const int tok = token0 + wn * 16 + n * 8 + 2 * cq + (e & 1);
          if (row < p.o[j].rows && tok < p.tokens)
            p.o[j].out[size_t(tok) * p.o[j].ld + row] =
                acc[m][n][e] * p.scale[tok];
        }
    return;
  }
  // SwiGLU: m-tiles 0,1 gate and 2,3 up of the same rows
  const int row0 = t * 64 + wm * 32;
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    float top[2] = {0, 0};
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row0 + m * 16 + g + (e >= 2 ? 8 : 0);
        const int tok = token0 + wn * 16 + n * 8 + 2 * cq + (e & 1);
        if (tok < p.tokens && row < p.o[0].rows) {
          const float scale = p.scale[tok];
          const float gv = acc[m][n][e] * scale, uv = acc[m + 2][n][e] * scale;
          const float sig = 1.0F / (1.0F + expf(-gv));
          const float value = (gv * sig) * uv;
          p.o[0].out[size_t(tok) * p.o[0].ld + row] = value;
          top[e & 1] = fmaxf(top[e & 1], fabsf(value));
        }
      }
    // lanes with the same cq share tokens: reduce over g
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float m = top[e];
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
      const int tok = token0 + wn * 16 + n * 8 + 2 * cq + e;
      if (g == 0 && tok < p.tokens && p.row_max)
        atomicMax(p.row_max + tok, __float_as_uint(m));
    }
  }
}

}  // namespace

cudaError_t launch_q8_prefill(PrefillParams p, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(
        q8_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        int(sizeof(PrefillSmem)));
    if (e != cudaSuccess)
      return e;
    configured = true;
  }
  if (p.K % 256 || p.tokens <= 0)
    return cudaErrorInvalidValue;
  const dim3 grid(p.row_tiles, (p.tokens + kPN - 1) / kPN);
  note_launch();
  q8_prefill_kernel<<<grid, kPThreads, sizeof(PrefillSmem), stream>>>(p);
  return cudaGetLastError();
}

}  // namespace lfm3
