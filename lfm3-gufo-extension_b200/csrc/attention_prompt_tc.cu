// Prompt attention of the full-attention layers on the tcgen05 tensor cores.
//
// The reference's WmmaAttn (hip/ops.hip:1355-1561) arithmetic: Q carries the
// softmax scale in base-2 units (rsqrt(128) log2 e) before its FP16
// rounding, S accumulates in FP32, probabilities round to FP16 once and the
// denominator adds the rounded values, O accumulates in FP32; long histories
// split their keys into spans whose (max, sum, output) the combine kernel
// merges (hip/ops.hip:1692-1709, prompt_combine_kernel).
//
// A CTA owns one KV group and 128 / G queries of it: the G heads' query rows
// (head-major) make the M = 128 rows of every MMA, so each key tile serves
// the whole group. Per tile j of 64 keys:
//   S_j = Q K_j^T   M128 N64, 8 K16 steps, into one of two FP32 buffers in
//                   tensor memory; S_{j+2} is issued as soon as the softmax
//                   has read S_j, so scores never wait for P V
//   softmax         thread r owns row r (its tensor-memory lane): reads S_j,
//                   masks causally and writes its P row (fp16) into one of
//                   two shared buffers
//   O += P_j V_j    M128 N160, 4 K16 steps; B is V_j read as an MN-major
//                   operand straight from the TMA tile (no transpose) plus a
//                   block of ones, so columns 128..159 of the accumulator
//                   sum the rounded probabilities (the softmax denominator)
// A row's probabilities are taken against a reference maximum m, not the
// exact running maximum: m moves (and the row's O and denominator are
// rescaled in tensor memory) only when a tile's maximum passes it by more
// than kRescaleSlack, so rescales, which must wait for the previous P V,
// are rare. P = 2^(s - m) <= 2^8 is still rounded to FP16 once; O / l is
// the same quantity the reference normalises.
// Warp roles: warps 0-3 softmax and epilogue, warp 4 the TMA producer (K and
// V tiles of 64 keys from the F16 cache, four stages, 64-byte swizzle),
// warp 5 tensor-memory allocation and (one thread) every MMA; the MMA
// commits release the K and V stages and the P buffers. Every wait is
// bounded: a pipeline that stops reports kErrPrefillWait, the warps skip to
// the end, the copies and MMAs in flight are waited for and the tensor
// memory is freed.
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"
#include "tensor_map.hpp"

namespace lfm3 {
namespace {

constexpr int kRowsTc = 128;  // query rows per CTA (M)
constexpr int kKeysTc = 64;   // keys per tile
constexpr int kStagesTc = 4;
constexpr int kThreadsTc = 6 * 32;
constexpr int kMinSpanTc = 1024, kMaxSpansTc = 8;  // as the mma.sync kernel
// A row's probabilities are taken against a reference maximum that moves
// (rescaling O) only when the running maximum passes it by more than this
// (base 2): P <= 2^8 stays well inside FP16.
constexpr float kRescaleSlack = 8.0F;
// tensor memory: S buffers at columns 0 and 64; O at 128 .. 255 and the
// softmax denominators (P times a block of ones) at 256 .. 287
constexpr uint32_t kColO = 128, kColL = 256, kColumns = 512;
constexpr uint32_t kIdescS = tc::f16_idesc(kRowsTc, kKeysTc);
constexpr uint32_t kIdescO = tc::f16_idesc(kRowsTc, kHeadDim + 32, true);
constexpr uint32_t kChunkBytes = kKeysTc * 64;  // 64 keys x 32 dims
constexpr uint32_t kTileBytes = 4 * kChunkBytes;

struct __align__(1024) PromptTcSmem {
  uint8_t q[4][kRowsTc * 64];             // Q rows, 4 chunks of 32 dims
  uint8_t k[kStagesTc][4][kChunkBytes];   // K tiles [key][32 dims] x 4
  // V tiles [key][32 dims] x 4, then a block of ones: P V and the row
  // sums of the rounded P in one MMA (N = 160)
  uint8_t v[kStagesTc][5][kChunkBytes];
  uint8_t p[2][2][kRowsTc * 64];          // P [row][key], 2 chunks of keys
  uint64_t k_full[kStagesTc], k_empty[kStagesTc];
  uint64_t v_full[kStagesTc], v_empty[kStagesTc];
  uint64_t s_full[2], s_empty[2], p_full[2], p_empty[2];
  uint64_t q_full, mma_idle;
  uint32_t tmem_base;
};

struct PromptTcArgs {
  alignas(64) CUtensorMap kmap;  // K ring rows [position + n][kv_heads * 128]
  alignas(64) CUtensorMap vmap;
  const float* q;  // [rows][ldq], normalised and rotated
  int ldq;
  const float* gate;
  int ldg;
  float* out;      // [rows][heads * 128]
  float* partial;  // spans > 1: [spans][rows][heads][130]
  int n, heads, kv_heads, group, position, span, spans;
};

__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(__half a, __half b) {
  const __half2 h = __halves2half2(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreadsTc, 1)
    prompt_attention_tc_kernel(const __grid_constant__ PromptTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  PromptTcSmem& s = *reinterpret_cast<PromptTcSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int QB = kRowsTc / a.group;  // queries per CTA
  const int q0 = blockIdx.x * QB, grp = blockIdx.y, split = blockIdx.z;
  const int P = a.position;
  const int nq = min(QB, a.n - q0);
  const int first_key = split * a.span, span_last = first_key + a.span - 1;
  const int last_key = min(P + q0 + nq - 1, span_last);
  const int tiles =
      first_key <= last_key ? (last_key - first_key) / kKeysTc + 1 : 0;
  if (tid == 0) {
    for (int i = 0; i < kStagesTc; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 4);
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.p_empty[i], 1);
    }
    mbar_init(&s.q_full, 4);
    mbar_init(&s.mma_idle, 1);
    fence_barrier_init();
  }
  if (warp == 5)
    tc::alloc(&s.tmem_base, kColumns);
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = s.tmem_base;
  bool ok = true;

  if (warp == 4) {
    // ---- producer: K and V tiles of 64 keys (this pass's keys were
    // written into the ring by the previous kernel)
    grid_dependency_wait();
    allow_dependents();
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < tiles && ok; ++j) {
        const int st = j % kStagesTc;
        const uint32_t reuse = ((j / kStagesTc) - 1) & 1;
        const int key0 = first_key + j * kKeysTc;
        if (j >= kStagesTc &&
            !mbar_wait(&s.k_empty[st], reuse, kErrPrefillWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(s.k[st][c], &a.kmap, grp * kHeadDim + c * 32, key0,
                      &s.k_full[st]);
        if (j >= kStagesTc &&
            !mbar_wait(&s.v_empty[st], reuse, kErrPrefillWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(s.v[st][c], &a.vmap, grp * kHeadDim + c * 32, key0,
                      &s.v_full[st]);
        ++issued;
      }
      // no copy may still be landing when the block exits (error paths;
      // a K tile whose V was never issued has landed by the V wait above)
      for (int j = max(0, issued - kStagesTc); j < issued; ++j) {
        mbar_wait(&s.k_full[j % kStagesTc], (j / kStagesTc) & 1,
                  kErrPrefillWait);
        mbar_wait(&s.v_full[j % kStagesTc], (j / kStagesTc) & 1,
                  kErrPrefillWait);
      }
    }
  } else if (warp == 5) {
    // ---- MMA issue (one thread): S_0, then per tile S_{j+1} ahead of
    // P_j V_j
    if (lane == 0 && tiles > 0) {
      const auto scores = [&](int i) {
        const int st = i % kStagesTc, b = i & 1;
        if (!mbar_wait(&s.k_full[st], (i / kStagesTc) & 1, kErrPrefillWait) ||
            (i >= 2 &&
             !mbar_wait(&s.s_empty[b], ((i >> 1) - 1) & 1, kErrPrefillWait)))
          return false;
        tc::fence_after();
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16)
          tc::mma(tmem + b * kKeysTc, tc::sw64_desc(s.q[k16 / 2]) + (k16 % 2) * 2,
                  tc::sw64_desc(s.k[st][k16 / 2]) + (k16 % 2) * 2, kIdescS,
                  k16 > 0);
        tc::commit(&s.k_empty[st]);
        tc::commit(&s.s_full[b]);
        return true;
      };
      ok = mbar_wait(&s.q_full, 0, kErrPrefillWait) && scores(0) &&
           (tiles < 2 || scores(1));
      for (int j = 0; j < tiles && ok; ++j) {
        const int st = j % kStagesTc, b = j & 1;
        if ((j + 2 < tiles && !scores(j + 2)) ||
            !mbar_wait(&s.v_full[st], (j / kStagesTc) & 1, kErrPrefillWait) ||
            !mbar_wait(&s.p_full[b], (j >> 1) & 1, kErrPrefillWait)) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int k16 = 0; k16 < 4; ++k16)
          tc::mma(tmem + kColO, tc::sw64_desc(s.p[b][k16 / 2]) + (k16 % 2) * 2,
                  tc::sw64_mn_desc(s.v[st][0], kChunkBytes) + k16 * 64, kIdescO,
                  j > 0 || k16 > 0);
        tc::commit(&s.v_empty[st]);
        tc::commit(&s.p_empty[b]);
      }
      // every MMA issued has finished before the tensor memory is freed
      tc::commit(&s.mma_idle);
      mbar_wait(&s.mma_idle, 0, kErrPrefillWait);
    }
  } else {
    // ---- softmax and epilogue: thread t owns row t (head t / QB of the
    // group, query q0 + t % QB) and tensor-memory lane t
    const int t = tid;
    const int head = grp * a.group + t / QB;
    const int row = q0 + t % QB;
    const bool live = row < a.n;
    const int qpos = P + row;
    const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
    grid_dependency_wait();
    allow_dependents();
    {
      // Q row, scaled in base-2 units, FP16, into the K-major operand
      const float scale = 0.0883883476483184405F * 1.44269504088896341F;
      const float* qr =
          a.q + size_t(live ? row : 0) * a.ldq + size_t(head) * kHeadDim;
#pragma unroll
      for (int piece = 0; piece < 16; ++piece) {
        float4 lo = make_float4(0, 0, 0, 0), hi = lo;
        if (live) {
          lo = *reinterpret_cast<const float4*>(qr + piece * 8);
          hi = *reinterpret_cast<const float4*>(qr + piece * 8 + 4);
        }
        const uint4 packed = make_uint4(
            pack2(__float2half_rn(lo.x * scale), __float2half_rn(lo.y * scale)),
            pack2(__float2half_rn(lo.z * scale), __float2half_rn(lo.w * scale)),
            pack2(__float2half_rn(hi.x * scale), __float2half_rn(hi.y * scale)),
            pack2(__float2half_rn(hi.z * scale),
                  __float2half_rn(hi.w * scale)));
        *reinterpret_cast<uint4*>(s.q[piece / 4] +
                                  tc::sw64_offset(t, piece % 4)) = packed;
      }
      // the ones blocks of the V stages (fp16 1.0), 128 bytes a thread
#pragma unroll
      for (int i = 0; i < kStagesTc * kChunkBytes / (16 * 128); ++i) {
        const int byte = (i * 128 + t) * 16;
        *reinterpret_cast<uint4*>(s.v[byte / kChunkBytes][4] +
                                  byte % kChunkBytes) =
            make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.q_full);
    }
    // a warp's lanes give up together: the tensor-memory loads and stores
    // below are warp-wide
    const auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, kErrPrefillWait));
    };
    float m = -INFINITY;
    for (int j = 0; j < tiles && ok; ++j) {
      const int b = j & 1;
      const int key0 = first_key + j * kKeysTc;
      if (!wait_all(&s.s_full[b], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc::fence_after();
      uint32_t sv[64];
      tc::ld32(lane_base + b * kKeysTc, *reinterpret_cast<uint32_t(*)[32]>(sv));
      tc::ld32(lane_base + b * kKeysTc + 32,
               *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
      tc::wait_ld();
      tc::fence_before();
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.s_empty[b]);
      // causal mask (keys key0 + i with i <= lim are in), running maximum
      // (base 2) over 8 independent chains
      const int lim = min(last_key, qpos) - key0;
      if (lim < kKeysTc - 1) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i > lim)
            sv[i] = __float_as_uint(-INFINITY);
      }
      float tops[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        tops[i] = __uint_as_float(sv[i]);
#pragma unroll
      for (int i = 8; i < 64; ++i)
        tops[i % 8] = fmaxf(tops[i % 8], __uint_as_float(sv[i]));
      const float top = fmaxf(fmaxf(fmaxf(tops[0], tops[1]), fmaxf(tops[2], tops[3])),
                              fmaxf(fmaxf(tops[4], tops[5]), fmaxf(tops[6], tops[7])));
      // the reference maximum m moves only when the row's maximum passes
      // it by more than the slack (always on its first finite tile)
      const bool move = top > m + kRescaleSlack;
      const float alpha = move ? exp2f(m - top) : 1.0F;
      if (move)
        m = top;
      const float shift = m == -INFINITY ? 0.0F : m;
      // probabilities rounded to FP16 (exp2 by ex2.approx.ftz: an output
      // below 2^-126 that it flushes rounds to zero in FP16 all the same);
      // the tensor cores add the rounded values into the denominator
      uint32_t pw[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const __half2 h =
            __floats2half2_rn(ex2_ftz(__uint_as_float(sv[2 * i]) - shift),
                              ex2_ftz(__uint_as_float(sv[2 * i + 1]) - shift));
        pw[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      // P_{j-2} V_{j-2} has finished reading this P buffer
      if (j >= 2 && !wait_all(&s.p_empty[b], ((j >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int piece = 0; piece < 8; ++piece)
        *reinterpret_cast<uint4*>(s.p[b][piece / 4] +
                                  tc::sw64_offset(t, piece % 4)) =
            make_uint4(pw[4 * piece], pw[4 * piece + 1], pw[4 * piece + 2],
                       pw[4 * piece + 3]);
      // rescale this row of O and its denominator when m moved, once
      // P_{j-1} V_{j-1} has landed
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0F)) {
        if (!wait_all(&s.p_empty[b ^ 1], ((j - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int c = 0; c < 5; ++c) {
          uint32_t ov[32];
          tc::ld32(lane_base + kColO + c * 32, ov);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tc::st32(lane_base + kColO + c * 32, ov);
        }
        tc::wait_st();
      }
      fence_proxy_async();
      tc::fence_before();
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.p_full[b]);
    }
    // ---- epilogue: the row's output (or, with spans, its maximum, sum and
    // unnormalised output for the combine kernel)
    if (ok && tiles > 0 &&
        !wait_all(&s.p_empty[(tiles - 1) & 1], ((tiles - 1) >> 1) & 1))
      ok = false;
    tc::fence_after();
    if (ok) {
      float l = 0;
      if (tiles > 0) {  // CTA-uniform
        uint32_t lv[32];
        tc::ld32(lane_base + kColL, lv);
        tc::wait_ld();
        l = __uint_as_float(lv[0]);
      }
      float* part = a.partial + ((size_t(split) * a.n + row) * a.heads + head) *
                                    (kHeadDim + 2);
      if (live && a.spans > 1) {
        part[0] = m;
        part[1] = l;
      }
      const float gs =
          live && a.spans == 1 ? 1 + expf(-a.gate[size_t(row) * a.ldg + head])
                               : 1.0F;
      float* dst = a.spans > 1
                       ? part + 2
                       : a.out + (size_t(row) * a.heads + head) * kHeadDim;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          ov[i] = 0;
        if (tiles > 0) {  // CTA-uniform
          tc::ld32(lane_base + kColO + c * 32, ov);
          tc::wait_ld();
        }
        if (live)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float o = __uint_as_float(ov[i]);
            dst[c * 32 + i] = a.spans > 1 ? o : (o / l) / gs;
          }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after();
    tc::dealloc(tmem, kColumns);
  }
}

int plan_spans_tc(int keys, int* span) {
  *span = max(kMinSpanTc, (keys + kMaxSpansTc - 1) / kMaxSpansTc);
  return (keys + *span - 1) / *span;
}

}  // namespace

cudaError_t launch_prompt_attention_tc(const float* q, int ldq,
                                       const __half* ring_k,
                                       const __half* ring_v, const float* gate,
                                       int ldg, float* out, int n, int heads,
                                       int kv_heads, int position,
                                       int capacity, float* scratch,
                                       cudaStream_t stream, bool pdl) {
  if (n <= 0)
    return cudaSuccess;
  if (kv_heads <= 0 || heads % kv_heads || position + n > capacity ||
      !ring_k || !ring_v || ldq % 4)
    return cudaErrorInvalidValue;
  const int group = heads / kv_heads;
  if (group != 2 && group != 4 && group != 8)
    return cudaErrorInvalidValue;
  PromptTcArgs a{};
  // The maps end at the pass's last key: a tile reaching past it reads
  // zeros, never the ring slots this pass has not written (a zero
  // probability times a NaN there would still be NaN).
  const int keys = position + n;
  if (cudaError_t e = encode_activation_map(&a.kmap, ring_k, keys,
                                            kv_heads * kHeadDim, kKeysTc, 32))
    return e;
  if (cudaError_t e = encode_activation_map(&a.vmap, ring_v, keys,
                                            kv_heads * kHeadDim, kKeysTc, 32))
    return e;
  a.q = q;
  a.ldq = ldq;
  a.gate = gate;
  a.ldg = ldg;
  a.out = out;
  a.partial = scratch;
  a.n = n;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.group = group;
  a.position = position;
  a.spans = plan_spans_tc(position + n, &a.span);
  if (a.spans > 1 && !scratch)
    return cudaErrorInvalidValue;
  const int queries = kRowsTc / group;
  const dim3 grid((n + queries - 1) / queries, kv_heads, a.spans);
  const int smem = int(sizeof(PromptTcSmem)) + 1024;
  if (cudaError_t e = ensure_dynamic_smem(
          reinterpret_cast<const void*>(prompt_attention_tc_kernel), smem))
    return e;
  cudaError_t e = launch_kernel(prompt_attention_tc_kernel, grid,
                                dim3(kThreadsTc), smem, stream, pdl, a);
  if (e != cudaSuccess || a.spans == 1)
    return e;
  return launch_prompt_combine(scratch, gate, ldg, out, n, heads, a.spans,
                               stream, pdl);
}

}  // namespace lfm3
