// Prompt-pass Q8_0 projections on the fifth-generation tensor cores
// (tcgen05, accumulators in tensor memory).
//
// A work unit is 128 weight rows x 128 tokens over all K; CTAs (one per SM)
// take units round-robin, token tile fastest, so the CTAs sharing a weight
// tile run together and read it once from HBM. Warp roles:
//   warp 0     TMA producer: raw Q8 rows (272-byte chunks = 8 blocks) and
//              the fp16 activation tile of every block (128 tokens x 32,
//              64-byte swizzle)
//   warps 1-4  converters: each thread owns one weight row, decodes its
//              codes exactly to fp16 into the 64-byte-swizzled K-major A
//              tile of one block and records the block scale d
//   warp 5     one thread issues tcgen05.mma (M128 N128 K16, twice per
//              block) into one of four TMEM buffers and commits
//   warps 6-13 epilogue: each thread owns one weight row (TMEM lane) and
//              one half of the 128 token columns, loads the block's 64 sums
//              and accumulates acc += d * C in FP32
// so every K32 block is scaled as in the reference (acc = fma(d, c, acc),
// hip/q8_prefill.hpp:563-569), with the row scale of the FP16 activations
// applied after K. Stages hand over through mbarriers; every wait is
// bounded. SwiGLU units hold 64 gate rows and the same 64 up rows and
// write silu(g) * u with per-token maxima (atomicMax) for the down
// projection's FP16 conversion.
#include "common.cuh"
#include "kernels.cuh"
#include "q8_prefill.cuh"
#include "tensor_map.hpp"

namespace lfm3 {
namespace {

constexpr int kTM = 128, kTN = 128;
constexpr int kWStages = 2, kASlots = 4, kBSlots = 6, kTBufs = 4;
constexpr int kWRowBytes = 272;                    // 8 blocks
constexpr int kWStageBytes = kTM * kWRowBytes;     // 34,816
constexpr int kABytes = kTM * 64, kBBytes = kTN * 64;
constexpr int kThreads = 448;  // 14 warps: <= 128 registers each
constexpr int kXchPitch = kTN + 1;

struct __align__(1024) PrefillSmem {
  uint8_t a[kASlots][kABytes];
  uint8_t b[kBSlots][kBBytes];
  uint8_t w[kWStages][kWStageBytes];
  float d[kASlots][kTM];
  float xch[64 * kXchPitch];
  uint64_t w_full[kWStages], w_empty[kWStages];
  uint64_t b_full[kBSlots], b_empty[kBSlots];
  uint64_t a_full[kASlots], a_empty[kASlots];
  uint64_t d_full[kASlots], d_empty[kASlots];
  uint64_t t_full[kTBufs], t_empty[kTBufs];
  uint32_t tmem_base;
};

// tcgen05 instruction descriptor: kind::f16, A and B fp16 K-major, D fp32,
// M = 128, N = 128.
constexpr uint32_t kInstrDesc =
    (1u << 4) | (uint32_t(kTN >> 3) << 17) | (uint32_t(kTM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand with 64-byte rows and
// the 64-byte swizzle: 8-row groups 512 bytes apart.
__device__ __forceinline__ uint64_t sw64_desc(const void* p) {
  const uint32_t addr = smem_addr(p);
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) |
         (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(4) << 61);
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
        "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
        "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
        "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
        "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// acc (two lanes) += d * v (two lanes), FP32, one packed instruction.
__device__ __forceinline__ void fma2(float2& acc, float d, uint32_t v0,
                                     uint32_t v1) {
  unsigned long long a = (unsigned long long)__float_as_uint(acc.x) |
                         ((unsigned long long)__float_as_uint(acc.y) << 32);
  const unsigned long long dd = (unsigned long long)__float_as_uint(d) |
                                ((unsigned long long)__float_as_uint(d) << 32);
  const unsigned long long vv =
      (unsigned long long)v0 | ((unsigned long long)v1 << 32);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(dd), "l"(vv));
  acc.x = __uint_as_float(uint32_t(a));
  acc.y = __uint_as_float(uint32_t(a >> 32));
}

struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int slots) {
    if (++slot == slots) {
      slot = 0;
      phase ^= 1;
    }
  }
};

__device__ __forceinline__ int output_of(const PrefillParams& p, int t) {
  int j = 0;
#pragma unroll
  for (int q = 1; q < 4; ++q)
    if (q < p.n_out && t >= p.first_tile[q])
      j = q;
  return j;
}

__global__ void __launch_bounds__(kThreads, 1)
    q8_prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PrefillSmem& s = *reinterpret_cast<PrefillSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int token_tiles = (p.tokens + kTN - 1) / kTN;
  const int units = p.row_tiles * token_tiles;
  const int blocks = p.K / 32, stages = blocks / 8;

  if (tid == 0) {
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(&s.w_full[i], 1);
      mbar_init(&s.w_empty[i], 4);
    }
    for (int i = 0; i < kBSlots; ++i) {
      mbar_init(&s.b_full[i], 1);
      mbar_init(&s.b_empty[i], 1);
    }
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(&s.a_full[i], 4);
      mbar_init(&s.a_empty[i], 1);
      mbar_init(&s.d_full[i], 4);
      mbar_init(&s.d_empty[i], 8);
    }
    for (int i = 0; i < kTBufs; ++i) {
      mbar_init(&s.t_full[i], 1);
      mbar_init(&s.t_empty[i], 8);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile(
        "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::
            "r"(smem_addr(&s.tmem_base)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---- producer
    if (lane == 0) {
      Ring w, b;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int rt = u / token_tiles, tok0 = (u % token_tiles) * kTN;
        for (int st = 0; st < stages; ++st) {
          if (!mbar_wait(&s.w_empty[w.slot], w.phase ^ 1, kErrPrefillWait))
            goto done;
          mbar_arrive_expect_tx(&s.w_full[w.slot], kWStageBytes);
          if (p.kind == kPrefillPlain) {
            const int j = output_of(p, rt);
            tma_load_3d(s.w[w.slot], &p.w_maps[j], 0, st * 17,
                        (rt - p.first_tile[j]) * kTM, &s.w_full[w.slot]);
          } else {
            tma_load_3d(s.w[w.slot], &p.w_maps[0], 0, st * 17, rt * 64,
                        &s.w_full[w.slot]);
            tma_load_3d(s.w[w.slot] + 64 * kWRowBytes, &p.w_maps[1], 0,
                        st * 17, rt * 64, &s.w_full[w.slot]);
          }
          w.next(kWStages);
          for (int kb = st * 8; kb < st * 8 + 8; ++kb) {
            if (!mbar_wait(&s.b_empty[b.slot], b.phase ^ 1, kErrPrefillWait))
              goto done;
            mbar_arrive_expect_tx(&s.b_full[b.slot], kBBytes);
            tma_load_2d(s.b[b.slot], &p.x_map, kb * 32, p.x_row0 + tok0,
                        &s.b_full[b.slot]);
            b.next(kBSlots);
          }
        }
      }
    }
  } else if (warp <= 4) {
    // ---- converters: thread owns weight row r of the unit
    const int r = (warp - 1) * 32 + lane;
    Ring w, a;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      for (int st = 0; st < stages; ++st) {
        if (!mbar_wait(&s.w_full[w.slot], w.phase, kErrPrefillWait))
          goto done;
        uint32_t raw[68];
        {
          const uint4* row =
              reinterpret_cast<const uint4*>(s.w[w.slot] + r * kWRowBytes);
#pragma unroll
          for (int i = 0; i < 17; ++i) {
            const uint4 v = row[i];
            raw[4 * i] = v.x;
            raw[4 * i + 1] = v.y;
            raw[4 * i + 2] = v.z;
            raw[4 * i + 3] = v.w;
          }
        }
        __syncwarp();
        if (lane == 0)
          mbar_arrive(&s.w_empty[w.slot]);
        w.next(kWStages);
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
          // block blk: d at byte 34 blk, codes at 34 blk + 2
          const int o = 34 * blk;
          const uint32_t dw = raw[o / 4];
          const uint16_t dbits = (o % 4) ? uint16_t(dw >> 16) : uint16_t(dw);
          uint32_t codes[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c = o + 2 + 4 * i;
            codes[i] = (c % 4) ? __funnelshift_r(raw[c / 4], raw[c / 4 + 1], 16)
                               : raw[c / 4];
          }
          uint32_t h[16];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            codes_to_half2(codes[i], h[2 * i], h[2 * i + 1]);
          if (!mbar_wait(&s.a_empty[a.slot], a.phase ^ 1, kErrPrefillWait) ||
              !mbar_wait(&s.d_empty[a.slot], a.phase ^ 1, kErrPrefillWait))
            goto done;
          uint8_t* dst = s.a[a.slot] + r * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(dst + ((c ^ ((r >> 1) & 3)) * 16)) =
                make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
          s.d[a.slot][r] = __half2float(__ushort_as_half(dbits));
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&s.a_full[a.slot]);
            mbar_arrive(&s.d_full[a.slot]);
          }
          a.next(kASlots);
        }
      }
    }
  } else if (warp == 5) {
    // ---- MMA issue
    if (lane == 0) {
      Ring a, b, t;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        for (int kb = 0; kb < blocks; ++kb) {
          if (!mbar_wait(&s.a_full[a.slot], a.phase, kErrPrefillWait) ||
              !mbar_wait(&s.b_full[b.slot], b.phase, kErrPrefillWait) ||
              !mbar_wait(&s.t_empty[t.slot], t.phase ^ 1, kErrPrefillWait))
            goto done;
          tc_fence_after();
          const uint32_t d_tmem = tmem + uint32_t(t.slot * kTN);
          const uint64_t da = sw64_desc(s.a[a.slot]);
          const uint64_t db = sw64_desc(s.b[b.slot]);
          tc_mma(d_tmem, da, db, 0);
          tc_mma(d_tmem, da + 2, db + 2, 1);  // second K16: +32 bytes
          tc_commit(&s.a_empty[a.slot]);
          tc_commit(&s.b_empty[b.slot]);
          tc_commit(&s.t_full[t.slot]);
          a.next(kASlots);
          b.next(kBSlots);
          t.next(kTBufs);
        }
      }
    }
  } else {
    // ---- epilogue: thread owns weight row r = TMEM lane and token columns
    // col0 .. col0 + 63
    const int quarter = warp % 4, col0 = ((warp - 6) / 4) * 64;
    const int r = quarter * 32 + lane;
    Ring a, t;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int rt = u / token_tiles, tok0 = (u % token_tiles) * kTN;
      float2 acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        acc[j] = make_float2(0.f, 0.f);
      for (int kb = 0; kb < blocks; ++kb) {
        if (!mbar_wait(&s.t_full[t.slot], t.phase, kErrPrefillWait) ||
            !mbar_wait(&s.d_full[a.slot], a.phase, kErrPrefillWait))
          goto done;
        tc_fence_after();
        const float d = s.d[a.slot][r];
        const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) +
                              uint32_t(t.slot * kTN + col0);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t v[32];
          tc_ld32(base + q * 32, v);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            fma2(acc[q * 16 + j], d, v[2 * j], v[2 * j + 1]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.t_empty[t.slot]);
          mbar_arrive(&s.d_empty[a.slot]);
        }
        a.next(kASlots);
        t.next(kTBufs);
      }
      // ---- unit complete: row scales of the tokens, then the outputs
      const int ntok = min(kTN, p.tokens - tok0);
      if (p.kind == kPrefillPlain) {
        const int j = output_of(p, rt);
        const int row = (rt - p.first_tile[j]) * kTM + r;
        if (row < p.o[j].rows) {
          float* out = p.o[j].out + row;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int t0 = col0 + 2 * c;
            if (t0 < ntok)
              out[size_t(tok0 + t0) * p.o[j].ld] = acc[c].x * p.scale[tok0 + t0];
            if (t0 + 1 < ntok)
              out[size_t(tok0 + t0 + 1) * p.o[j].ld] =
                  acc[c].y * p.scale[tok0 + t0 + 1];
          }
        }
      } else {
        // rows 0-63 gate, 64-127 up of the same 64 indices
        float* x = s.xch;
        if (r >= 64)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            x[(r - 64) * kXchPitch + col0 + 2 * c] = acc[c].x;
            x[(r - 64) * kXchPitch + col0 + 2 * c + 1] = acc[c].y;
          }
        named_barrier(2, 256);
        const int row = rt * 64 + r;
        if (r < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int c = col0 + i;
            const float scale = c < ntok ? p.scale[tok0 + c] : 0.f;
            const float gv = (i & 1 ? acc[i / 2].y : acc[i / 2].x) * scale;
            const float uv = x[r * kXchPitch + c] * scale;
            // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
            const float sig = 1.0F / (1.0F + expf(-gv));
            const float h = (gv * sig) * uv;
            if (c < ntok && row < p.o[0].rows)
              p.o[0].out[size_t(tok0 + c) * p.o[0].ld + row] = h;
            x[r * kXchPitch + c] = row < p.o[0].rows ? fabsf(h) : 0.f;
          }
        }
        named_barrier(2, 256);
        if (p.row_max) {
          // two threads per token column, 32 rows each
          const int e = (warp - 6) * 32 + lane, c = e & 127, r0 = (e >> 7) * 32;
          if (c < ntok) {
            float m = 0.f;
            for (int i = r0; i < r0 + 32; ++i)
              m = fmaxf(m, x[i * kXchPitch + c]);
            atomicMax(p.row_max + tok0 + c, __float_as_uint(m));
          }
        }
        named_barrier(2, 256);
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(
        tmem));
  }
}

}  // namespace

cudaError_t launch_q8_prefill(PrefillParams p, const __half* x, int x_rows,
                              cudaStream_t stream) {
  static bool configured = false;
  const int smem = int(sizeof(PrefillSmem)) + 1024;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(
        q8_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        smem);
    if (e != cudaSuccess)
      return e;
    configured = true;
  }
  if (p.K % 256 || p.tokens <= 0)
    return cudaErrorInvalidValue;
  const size_t row_bytes = size_t(p.K / 32) * 34;
  const int outputs = p.kind == kPrefillPlain ? p.n_out : 2;
  for (int j = 0; j < outputs; ++j) {
    const cudaError_t e =
        encode_row_map(&p.w_maps[j], p.o[j].w, row_bytes, p.o[j].rows,
                       kWRowBytes, p.kind == kPrefillPlain ? kTM : 64);
    if (e != cudaSuccess)
      return e;
  }
  cudaError_t e = encode_activation_map(&p.x_map, x, x_rows, p.K, kTN, 32);
  if (e != cudaSuccess)
    return e;
  int device = 0, sms = 148;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int units = p.row_tiles * ((p.tokens + kTN - 1) / kTN);
  note_launch();
  q8_prefill_tc_kernel<<<units < sms ? units : sms, kThreads, smem, stream>>>(
      p);
  return cudaGetLastError();
}

}  // namespace lfm3
