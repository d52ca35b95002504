// Prompt-pass Q8_0 projections on the fifth-generation tensor cores
// (tcgen05 MMA, accumulators in tensor memory).
//
// Exact split of the block scales. The reference sums each K32 block in FP32
// and scales it (acc = fma(d, c, acc), hip/q8_prefill.hpp:563-569). Here each
// weight w = q * d (q the integer code, d the block's fp16 scale) is written
// as w = hi + lo with hi = fp16(q * d) and lo = fp16(q * d - hi) (one rounded
// multiply and one fused multiply-add in fp16). q * d has at most 18
// significant bits and its last bit is a multiple of 2^-24, so the rounding
// residual is itself an fp16 number and hi + lo == q * d exactly (true for
// every code and every fp16 scale below 516; larger scales, weights beyond
// 65504, would overflow hi). The tensor cores multiply hi and lo by the FP16
// activations exactly (11 x 11 significant bits) and accumulate in FP32, so
// each output is the reference's real-valued sum up to FP32 rounding order,
// with twice the MMA work and no per-block epilogue: the K loop stays in the
// tensor pipe.
//
// A tile is 256 weight rows x 256 prompt rows over a K range (split-K for
// matrices with few tiles: FP32 partial sums per split, then a bandwidth-
// bound pass adds them in split order, hip/ops.hip:2039-2119). Persistent
// CTAs (one per SM) take units round-robin, split and prompt tile fastest,
// so the CTAs sharing a weight tile run together and read it once from HBM.
// Warp roles:
//   warp 0      TMA producer: the fp16 activation tile of every K32 block
//               (256 rows x 32, 64-byte swizzle)
//   warp 1      one thread issues tcgen05.mma: per block, two accumulators
//               (rows 0-127, 128-255) x {hi, lo} x two K16 steps, M128 N256,
//               into the accumulator pair (all 512 TMEM columns; the next
//               tile's MMAs wait for the epilogue to read it); commits every
//               stage and every finished tile
//   warps 2-9   converters: thread r owns weight row r of the tile. Raw Q8
//               rows arrive by TMA 8 blocks (272 bytes per row) at a time,
//               issued by warp 2's lane 0 as soon as the previous chunk is in
//               registers; per block each thread writes its row of the hi and
//               lo A tiles (fp16, K-major, 64-byte swizzle)
//   warps 10-13 epilogue: thread owns one TMEM lane (weight row) of both
//               accumulators; applies the prompt-row scales and writes the
//               outputs (SwiGLU: silu(g) * u, optionally per-row maxima;
//               split tiles: the FP32 partial sums)
// BF16 weights (p.bf16, the numerical-reference models) skip the converters:
// warp 0 also loads the weight tiles (two 128-row boxes of the [rows][K]
// bf16 matrix, 64-byte swizzle) and the activations are three bf16 planes
// whose sum is the FP32 input exactly, so each K32 block is 2 accumulators
// x 3 planes x 2 K16 steps of bf16 MMAs: exact products, FP32
// accumulation, the precision of the reference's exact BF16 x FP32 GEMM
// (hip/ops.hip:1917-2005). Planes 1 and 2 of a stage sit where the Q8 mode
// keeps its lo tile and raw weight rows.
// Stages hand over through mbarriers and every wait is bounded: a pipeline
// that stops making progress reports kErrPrefillWait and the CTA returns.
// When that happens every copy and MMA it issued is seconds old and complete.
#include "common.cuh"
#include "kernels.cuh"
#include "q8_prefill.cuh"
#include "tensor_map.hpp"

namespace lfm3 {
namespace {

constexpr int kTM = 128;                      // rows per accumulator
constexpr int kRows = kPrefillTileRows;       // 256
constexpr int kTN = kPrefillTileTokens;       // 256
// accumulator pairs that fit the 512 TMEM columns (each pair 2 x kTN)
constexpr int kAccBufs = 512 / (2 * kTN);
constexpr int kStages = 3;
constexpr int kWRowBytes = 272;               // 8 blocks of 34 bytes
constexpr int kWBytes = kRows * kWRowBytes;   // 69,632
constexpr int kAPartBytes = kRows * 64;       // 256 rows x 32 fp16
constexpr int kBBytes = kTN * 64;             // kTN rows x 32 fp16
constexpr int kThreads = 14 * 32;

struct __align__(1024) PrefillSmem {
  uint8_t a_hi[kStages][kAPartBytes];  // bf16: the weight tile
  uint8_t a_lo[kStages][kAPartBytes];  // bf16: activation plane 1
  uint8_t b[kStages][kBBytes];         // activation tile (bf16: plane 0)
  uint8_t w[kWBytes];                  // bf16: plane 2 of stage s at s * kBBytes
  uint64_t w_full, w_empty;
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[kAccBufs], acc_empty[kAccBufs];
  uint32_t tmem_base;
};

// tcgen05 instruction descriptor: kind::f16, A and B fp16 K-major, D fp32,
// M = 128, N = kTN; the same with A and B bf16.
constexpr uint32_t kInstrDesc =
    (1u << 4) | (uint32_t(kTN >> 3) << 17) | (uint32_t(kTM >> 4) << 24);
constexpr uint32_t kInstrDescBf16 = kInstrDesc | (1u << 7) | (1u << 10);
static_assert(kStages * kBBytes <= kWBytes, "bf16 plane 2 fits the w buffer");

// Shared-memory matrix descriptor of a K-major operand with 64-byte rows and
// the 64-byte swizzle: 8-row groups 512 bytes apart. Adding 2 advances K by
// 16 elements (32 bytes), adding 512 advances 128 rows.
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
                                       uint32_t accumulate,
                                       uint32_t idesc = kInstrDesc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
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

// Unit u: split fastest, then prompt tile, then row tile.
struct Unit {
  int rt, tt, tile, kb0, kb1;
};
__device__ __forceinline__ Unit unit_of(const PrefillParams& p, int u,
                                        int token_tiles, int blocks_per_split) {
  Unit x;
  const int sp = u % p.splits;
  x.tile = u / p.splits;
  x.tt = x.tile % token_tiles;
  x.rt = x.tile / token_tiles;
  x.kb0 = sp * blocks_per_split;
  x.kb1 = x.kb0 + blocks_per_split;
  return x;
}

__device__ __forceinline__ int output_of(const PrefillParams& p, int rt) {
  int j = 0;
#pragma unroll
  for (int q = 1; q < 4; ++q)
    if (q < p.n_out && rt >= p.first_tile[q])
      j = q;
  return j;
}

// One 8-block chunk of the tile's 256 raw weight rows into s.w.
__device__ __forceinline__ void load_weights(const PrefillParams& p,
                                             PrefillSmem& s, int rt,
                                             int chunk) {
  mbar_arrive_expect_tx(&s.w_full, kWBytes);
  if (p.kind == kPrefillPlain) {
    const int j = output_of(p, rt);
    tma_load_2d(s.w, &p.w_maps[j], chunk * (kWRowBytes / 8),
                (rt - p.first_tile[j]) * kRows, &s.w_full);
  } else {
    tma_load_2d(s.w, &p.w_maps[0], chunk * (kWRowBytes / 8), rt * kTM,
                &s.w_full);
    tma_load_2d(s.w + kTM * kWRowBytes, &p.w_maps[1],
                chunk * (kWRowBytes / 8), rt * kTM, &s.w_full);
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    q8_prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PrefillSmem& s = *reinterpret_cast<PrefillSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int token_tiles = (p.tokens + kTN - 1) / kTN;
  const int units = p.row_tiles * token_tiles * p.splits;
  const int bps = p.K / 32 / p.splits;  // blocks per split, a multiple of 8

  if (tid == 0) {
    mbar_init(&s.w_full, 1);
    mbar_init(&s.w_empty, 8);
    for (int i = 0; i < kStages; ++i) {
      // 8 converter warps + the producer's bytes (bf16: the producer only)
      mbar_init(&s.full[i], kBf16 ? 1 : 9);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kAccBufs; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 4);
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
  // launched behind the previous kernel (programmatic dependent launch): the
  // weight chunks, conversions and MMAs read nothing it writes; the
  // activation tiles and the epilogue wait for it
  allow_dependents();

  if (warp == 0) {
    // ---- activation tiles
    if (lane == 0) {
      grid_dependency_wait();
      Ring b;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const Unit x = unit_of(p, u, token_tiles, bps);
        for (int kb = x.kb0; kb < x.kb1; ++kb) {
          if (!mbar_wait(&s.empty[b.slot], b.phase ^ 1, kErrPrefillWait))
            goto done;
          const int row = p.x_row0 + x.tt * kTN;
          if constexpr (kBf16) {
            uint64_t* bar = &s.full[b.slot];
            mbar_arrive_expect_tx(bar, kAPartBytes + 3 * kBBytes);
            // weight tile: 256 rows (SwiGLU: 128 gate then 128 up rows)
            if (p.kind == kPrefillPlain) {
              const int j = output_of(p, x.rt);
              const int r0 = (x.rt - p.first_tile[j]) * kRows;
              tma_load_2d(s.a_hi[b.slot], &p.w_maps[j], kb * 32, r0, bar);
              tma_load_2d(s.a_hi[b.slot] + kTM * 64, &p.w_maps[j], kb * 32,
                          r0 + kTM, bar);
            } else {
              tma_load_2d(s.a_hi[b.slot], &p.w_maps[0], kb * 32, x.rt * kTM,
                          bar);
              tma_load_2d(s.a_hi[b.slot] + kTM * 64, &p.w_maps[1], kb * 32,
                          x.rt * kTM, bar);
            }
            tma_load_2d(s.b[b.slot], &p.x_map, kb * 32, row, bar);
            tma_load_2d(s.a_lo[b.slot], &p.x_map, kb * 32,
                        row + p.x_plane_rows, bar);
            tma_load_2d(s.w + b.slot * kBBytes, &p.x_map, kb * 32,
                        row + 2 * p.x_plane_rows, bar);
          } else {
            mbar_arrive_expect_tx(&s.full[b.slot], kBBytes);
            tma_load_2d(s.b[b.slot], &p.x_map, kb * 32, row, &s.full[b.slot]);
          }
          b.next(kStages);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue
    if (lane == 0) {
      Ring st;
      int j = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
        const Unit x = unit_of(p, u, token_tiles, bps);
        const int buf = j % kAccBufs;
        if (!mbar_wait(&s.acc_empty[buf], ((j / kAccBufs) & 1) ^ 1,
                       kErrPrefillWait))
          goto done;
        tc_fence_after();
        const uint32_t d0 = tmem + uint32_t(buf * 2 * kTN);
        const uint32_t d1 = d0 + kTN;
        for (int kb = x.kb0; kb < x.kb1; ++kb) {
          if (!mbar_wait(&s.full[st.slot], st.phase, kErrPrefillWait))
            goto done;
          tc_fence_after();
          const uint64_t hi = sw64_desc(s.a_hi[st.slot]);
          const uint64_t lo = sw64_desc(s.a_lo[st.slot]);
          const uint64_t xb = sw64_desc(s.b[st.slot]);
          const uint32_t acc = kb != x.kb0;
          if constexpr (kBf16) {
            const uint64_t x2 = sw64_desc(s.w + st.slot * kBBytes);
            const uint64_t planes[3] = {xb, lo, x2};
#pragma unroll
            for (int q = 0; q < 3; ++q) {
              tc_mma(d0, hi, planes[q], q ? 1 : acc, kInstrDescBf16);
              tc_mma(d0, hi + 2, planes[q] + 2, 1, kInstrDescBf16);
              tc_mma(d1, hi + 512, planes[q], q ? 1 : acc, kInstrDescBf16);
              tc_mma(d1, hi + 514, planes[q] + 2, 1, kInstrDescBf16);
            }
            tc_commit(&s.empty[st.slot]);
            st.next(kStages);
            continue;
          }
          tc_mma(d0, hi, xb, acc);
          tc_mma(d0, hi + 2, xb + 2, 1);
          tc_mma(d0, lo, xb, 1);
          tc_mma(d0, lo + 2, xb + 2, 1);
          tc_mma(d1, hi + 512, xb, acc);
          tc_mma(d1, hi + 514, xb + 2, 1);
          tc_mma(d1, lo + 512, xb, 1);
          tc_mma(d1, lo + 514, xb + 2, 1);
          tc_commit(&s.empty[st.slot]);
          st.next(kStages);
        }
        tc_commit(&s.acc_full[buf]);
      }
    }
  } else if (warp < 10) {
    // ---- converters: thread owns weight row r of the tile (Q8_0 only)
    if constexpr (kBf16)
      goto done;
    const int r = (warp - 2) * 32 + lane;
    const bool loader = warp == 2 && lane == 0;
    const int swz = (r >> 1) & 3;  // 64-byte swizzle of row r
    Ring a;
    uint32_t w_phase = 0;
    if (loader && int(blockIdx.x) < units) {
      const Unit x = unit_of(p, blockIdx.x, token_tiles, bps);
      load_weights(p, s, x.rt, x.kb0 / 8);
    }
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const Unit x = unit_of(p, u, token_tiles, bps);
      for (int chunk = x.kb0 / 8; chunk < x.kb1 / 8; ++chunk) {
        if (!mbar_wait(&s.w_full, w_phase, kErrPrefillWait))
          goto done;
        uint32_t raw[68];
        {
          const uint4* row =
              reinterpret_cast<const uint4*>(s.w + r * kWRowBytes);
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
          mbar_arrive(&s.w_empty);
        if (loader) {
          // the next chunk (of this tile, or of this CTA's next unit) once
          // every converter warp holds this one in registers
          int nu = u, next = chunk + 1;
          if (next == x.kb1 / 8) {
            nu = u + gridDim.x;
            if (nu < units)
              next = unit_of(p, nu, token_tiles, bps).kb0 / 8;
          }
          if (nu < units) {
            if (!mbar_wait(&s.w_empty, w_phase, kErrPrefillWait))
              goto done;
            load_weights(p, s, unit_of(p, nu, token_tiles, bps).rt, next);
          }
        }
        w_phase ^= 1;
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
          // block blk: d at byte 34 blk, codes at 34 blk + 2
          const int o = 34 * blk;
          const uint32_t dw = raw[o / 4];
          const uint16_t dbits = (o % 4) ? uint16_t(dw >> 16) : uint16_t(dw);
          const __half2 d2 = __half2half2(__ushort_as_half(dbits));
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int c = o + 2 + 4 * i;
            const uint32_t codes =
                (c % 4) ? __funnelshift_r(raw[c / 4], raw[c / 4 + 1], 16)
                        : raw[c / 4];
            uint32_t q[2];
            codes_to_half2(codes, q[0], q[1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const __half2 qv = *reinterpret_cast<const __half2*>(&q[h]);
              const __half2 wh = __hmul2(qv, d2);
              const __half2 wl = __hfma2(qv, d2, __hneg2(wh));
              hi[2 * i + h] = *reinterpret_cast<const uint32_t*>(&wh);
              lo[2 * i + h] = *reinterpret_cast<const uint32_t*>(&wl);
            }
          }
          if (!mbar_wait(&s.empty[a.slot], a.phase ^ 1, kErrPrefillWait))
            goto done;
          uint8_t* dh = s.a_hi[a.slot] + r * 64;
          uint8_t* dl = s.a_lo[a.slot] + r * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            *reinterpret_cast<uint4*>(dh + ((c ^ swz) * 16)) =
                make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2],
                           hi[4 * c + 3]);
            *reinterpret_cast<uint4*>(dl + ((c ^ swz) * 16)) =
                make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2],
                           lo[4 * c + 3]);
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0)
            mbar_arrive(&s.full[a.slot]);
          a.next(kStages);
        }
      }
    }
  } else {
    // ---- epilogue: thread owns TMEM lane r of both accumulators
    grid_dependency_wait();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int j = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      const Unit x = unit_of(p, u, token_tiles, bps);
      const int buf = j % kAccBufs;
      if (!mbar_wait(&s.acc_full[buf], (j / kAccBufs) & 1, kErrPrefillWait))
        goto done;
      tc_fence_after();
      const uint32_t base = tmem + (uint32_t(quarter * 32) << 16) +
                            uint32_t(buf * 2 * kTN);
      const int tok0 = x.tt * kTN;
      const int ntok = min(kTN, p.tokens - tok0);
      // releases the accumulator pair once its last columns are in registers
      const auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
          mbar_arrive(&s.acc_empty[buf]);
      };
      if (p.kind == kPrefillSwiGLU) {
        const int row = x.rt * kTM + r;
        const bool valid = row < p.o[0].rows;
        float* out = p.o[0].out;
        const int ld = p.o[0].ld;
        for (int c = 0; c < kTN / 32; ++c) {
          uint32_t g[32], v[32];
          tc_ld32(base + c * 32, g);
          tc_ld32(base + kTN + c * 32, v);
          // lane i holds the row scale of prompt row c * 32 + i
          const int tl = c * 32 + lane;
          const float lane_scale =
              tl < ntok ? (p.scale ? p.scale[tok0 + tl] : 1.0F) : 0.f;
          tc_wait_ld();
          if (c == kTN / 32 - 1)
            release();
          // independent per prompt row: activation, store, |h| bits
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float sc = __shfl_sync(0xffffffffu, lane_scale, i);
            const float gv = __uint_as_float(g[i]) * sc;
            const float uv = __uint_as_float(v[i]) * sc;
            // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
            // with the hardware exponential and reciprocal (a few ulp in
            // FP32): h is rounded to FP16 before the down projection reads
            // it, and the correctly rounded forms cost the epilogue three
            // times the stores' time
            const float sig = __fdividef(1.0F, 1.0F + __expf(-gv));
            const float h = (gv * sig) * uv;
            if (valid && c * 32 + i < ntok)
              out[size_t(tok0 + c * 32 + i) * ld + row] = h;
            g[i] = valid ? __float_as_uint(fabsf(h)) : 0u;
          }
          if (!p.row_max)
            continue;
          // max |h| over the warp's 32 rows per prompt row (non-negative
          // floats order as their bit patterns); lane i keeps row i's
          unsigned mine = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const unsigned m = __reduce_max_sync(0xffffffffu, g[i]);
            mine = lane == i ? m : mine;
          }
          if (tl < ntok)
            atomicMax(p.row_max + tok0 + tl, mine);
        }
        continue;
      }
      if (p.splits > 1) {
        // FP32 partial [prompt row][256 rows] of unit u
        float* part = p.partial + size_t(u) * (kRows * kTN);
#pragma unroll 1
        for (int acc = 0; acc < 2; ++acc) {
          for (int c = 0; c < kTN / 32; ++c) {
            uint32_t v[32];
            tc_ld32(base + acc * kTN + c * 32, v);
            tc_wait_ld();
            if (acc == 1 && c == kTN / 32 - 1)
              release();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              __stcg(part + (c * 32 + i) * kRows + acc * kTM + r,
                     __uint_as_float(v[i]));
          }
        }
        continue;
      }
      const int jo = output_of(p, x.rt);
      float* out = p.o[jo].out;
      const int ld = p.o[jo].ld, rows = p.o[jo].rows;
      const int row0 = (x.rt - p.first_tile[jo]) * kRows;
#pragma unroll 1
      for (int acc = 0; acc < 2; ++acc) {
        const int row = row0 + acc * kTM + r;
        for (int c = 0; c < kTN / 32; ++c) {
          uint32_t v[32];
          tc_ld32(base + acc * kTN + c * 32, v);
          const int tl = c * 32 + lane;
          const float lane_scale =
              tl < ntok ? (p.scale ? p.scale[tok0 + tl] : 1.0F) : 0.f;
          tc_wait_ld();
          if (acc == 1 && c == kTN / 32 - 1)
            release();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = c * 32 + i;
            const float sc = __shfl_sync(0xffffffffu, lane_scale, i);
            if (row < rows && t < ntok)
              out[size_t(tok0 + t) * ld + row] = __uint_as_float(v[i]) * sc;
          }
        }
      }
    }
  }
done:
  // lanes of the producer and MMA warps arrive here at different times: the
  // warp converges before the CTA barrier, which must count every warp once
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(
        tmem));
  }
}

// Split tiles: out[t][row] = scale[t] * sum over splits, in split order, of
// the FP32 partials (four rows per thread).
struct ReduceParams {
  const float* partial;
  const float* scale;
  int splits, token_tiles, tokens, n_out;
  int first_tile[5];
  float* out[4];
  int rows[4];
  int ld[4];
};

__global__ void __launch_bounds__(256)
    prefill_split_reduce_kernel(const __grid_constant__ ReduceParams p) {
  grid_dependency_wait();
  allow_dependents();
  const int quads = kRows / 4;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // tile, t, row quad
  const int tile = e / (kTN * quads);
  const int t = (e / quads) % kTN, q = e % quads;
  const int tt = tile % p.token_tiles, rt = tile / p.token_tiles;
  const int tok = tt * kTN + t;
  if (rt >= p.first_tile[p.n_out] || tok >= p.tokens)
    return;
  int j = 0;
#pragma unroll
  for (int o = 1; o < 4; ++o)
    if (o < p.n_out && rt >= p.first_tile[o])
      j = o;
  const float4* src = reinterpret_cast<const float4*>(
      p.partial + size_t(tile) * p.splits * (kRows * kTN) + t * kRows) + q;
  float4 sum = __ldcg(src);
  for (int sp = 1; sp < p.splits; ++sp) {
    const float4 v = __ldcg(src + size_t(sp) * (kRows * kTN / 4));
    sum.x += v.x;
    sum.y += v.y;
    sum.z += v.z;
    sum.w += v.w;
  }
  const float sc = p.scale ? p.scale[tok] : 1.0F;
  const int row = (rt - p.first_tile[j]) * kRows + 4 * q;
  float* out = p.out[j] + size_t(tok) * p.ld[j];
  const float v[4] = {sum.x * sc, sum.y * sc, sum.z * sc, sum.w * sc};
  if (row + 4 <= p.rows[j] && reinterpret_cast<uintptr_t>(out + row) % 16 == 0) {
    *reinterpret_cast<float4*>(out + row) = make_float4(v[0], v[1], v[2], v[3]);
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (row + i < p.rows[j])
      out[row + i] = v[i];
}

}  // namespace

cudaError_t launch_q8_prefill(PrefillParams p, const void* x, int x_rows,
                              cudaStream_t stream, int* splits, bool pdl) {
  int device = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess)
    return e;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int smem = int(sizeof(PrefillSmem)) + 1024;
  const auto kernel =
      p.bf16 ? q8_prefill_tc_kernel<true> : q8_prefill_tc_kernel<false>;
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
  if (e != cudaSuccess)
    return e;
  if (p.K <= 0 || p.K % 256 || p.tokens <= 0 || !x ||
      (!p.scale && !p.bf16) || x_rows < p.x_row0 + p.tokens)
    return cudaErrorInvalidValue;
  p.x_plane_rows = x_rows;
  // weight maps: Q8_0 rows in 8-block chunks, or bf16 [rows][K] tiles
  const auto weight_map = [&](CUtensorMap* map, const uint8_t* w, int rows,
                              int box_rows) {
    return p.bf16 ? cached_activation_map(map, w, rows, p.K, kTM, 32)
                  : cached_q8_rows(map, w, size_t(p.K / 32) * 34, rows,
                                   kWRowBytes, box_rows);
  };
  const int token_tiles = (p.tokens + kTN - 1) / kTN;
  p.splits = 1;
  if (p.kind == kPrefillPlain) {
    if (p.n_out < 1 || p.n_out > 4)
      return cudaErrorInvalidValue;
    int tiles = 0;
    for (int j = 0; j < p.n_out; ++j) {
      if (!p.o[j].w || !p.o[j].out || p.o[j].rows <= 0)
        return cudaErrorInvalidValue;
      p.first_tile[j] = tiles;
      tiles += (p.o[j].rows + kRows - 1) / kRows;
      e = weight_map(&p.w_maps[j], p.o[j].w, p.o[j].rows, kRows);
      if (e != cudaSuccess)
        return e;
    }
    for (int j = p.n_out; j < 5; ++j)
      p.first_tile[j] = tiles;
    p.row_tiles = tiles;
    // split K when the tiles leave SMs idle: fewest waves x K range
    if (p.keep_splits && p.n_out != 1)
      return cudaErrorInvalidValue;
    if (p.partial) {
      const int stages = p.K / 256, all = tiles * token_tiles;
      long best = long((all + sms - 1) / sms) * stages;
      for (int sp = 2; sp <= 8; sp *= 2) {
        if (stages % sp || all * sp > kPrefillMaxSplitUnits)
          continue;
        const long cost = long((all * sp + sms - 1) / sms) * (stages / sp);
        if (cost < best) {
          best = cost;
          p.splits = sp;
        }
      }
    }
  } else {
    if (!p.o[0].w || !p.o[1].w || !p.o[0].out ||
        p.o[0].rows != p.o[1].rows || p.o[0].rows <= 0)
      return cudaErrorInvalidValue;
    p.n_out = 2;
    p.row_tiles = (p.o[0].rows + kTM - 1) / kTM;
    for (int j = 0; j < 2; ++j) {
      e = weight_map(&p.w_maps[j], p.o[j].w, p.o[j].rows, kTM);
      if (e != cudaSuccess)
        return e;
    }
  }
  e = cached_activation_map(&p.x_map, x, p.bf16 ? 3 * x_rows : x_rows, p.K,
                            kTN, 32);
  if (e != cudaSuccess)
    return e;
  const int units = p.row_tiles * token_tiles * p.splits;
  e = launch_kernel(kernel, dim3(units < sms ? units : sms),
                    dim3(kThreads), smem, stream, pdl, p);
  if (splits)
    *splits = p.splits;
  if (e != cudaSuccess || p.splits == 1 || p.keep_splits)
    return e;
  ReduceParams r{};
  r.partial = p.partial;
  r.scale = p.scale;
  r.splits = p.splits;
  r.token_tiles = token_tiles;
  r.tokens = p.tokens;
  r.n_out = p.n_out;
  for (int j = 0; j < 5; ++j)
    r.first_tile[j] = p.first_tile[j];
  for (int j = 0; j < p.n_out; ++j) {
    r.out[j] = p.o[j].out;
    r.rows[j] = p.o[j].rows;
    r.ld[j] = p.o[j].ld;
  }
  const long threads = long(p.row_tiles) * token_tiles * kTN * (kRows / 4);
  return launch_kernel(prefill_split_reduce_kernel,
                       dim3(unsigned((threads + 255) / 256)), dim3(256), 0,
                       stream, pdl, r);
}

}  // namespace lfm3
