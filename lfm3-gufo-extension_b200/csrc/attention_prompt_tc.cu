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
// the whole group. Per tile of 64 keys:
//   S = Q K^T     M128 N64, 8 K16 steps, FP32 in tensor memory
//   softmax       thread r owns row r (its tensor-memory lane): reads S,
//                 masks causally, rescales its O row in tensor memory when
//                 the row maximum moves, writes its P row (fp16) to shared
//                 memory; the four softmax warps also transpose the V tile
//                 into the K-major operand layout
//   O += P V      M128 N128, 4 K16 steps, FP32 in tensor memory
// Warp roles: warps 0-3 softmax and epilogue, warp 4 the TMA producer (K and
// V tiles of 64 keys from the F16 cache, two stages, 64-byte swizzle),
// warp 5 tensor-memory allocation and (one thread) every MMA. Every
// handover is an mbarrier and every wait is bounded: a pipeline that stops
// reports kErrPrefillWait, the warps skip to the end and the tensor memory
// is freed.
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"
#include "tensor_map.hpp"

namespace lfm3 {
namespace {

constexpr int kRowsTc = 128;  // query rows per CTA (M)
constexpr int kKeysTc = 64;   // keys per tile
constexpr int kStagesTc = 2;
constexpr int kThreadsTc = 6 * 32;
constexpr int kMinSpanTc = 1024, kMaxSpansTc = 8;  // as the mma.sync kernel
constexpr uint32_t kColS = 0, kColO = 128, kColumns = 256;
constexpr uint32_t kIdescS = tc::f16_idesc(kRowsTc, kKeysTc);
constexpr uint32_t kIdescO = tc::f16_idesc(kRowsTc, kHeadDim);
constexpr uint32_t kStageBytes = 2 * 4 * kKeysTc * 64;  // K and V of a tile

struct __align__(1024) PromptTcSmem {
  uint8_t q[4][kRowsTc * 64];             // Q rows, 4 chunks of 32 dims
  uint8_t k[kStagesTc][4][kKeysTc * 64];  // K tiles [key][dim]
  uint8_t v[kStagesTc][4][kKeysTc * 64];  // V tiles [key][dim]
  uint8_t vt[2][kHeadDim * 64];           // V^T [dim][key], 2 chunks of keys
  uint8_t p[2][kRowsTc * 64];             // P [row][key], 2 chunks of keys
  uint64_t kv_full[kStagesTc], kv_empty[kStagesTc];
  uint64_t q_full, s_full, s_empty, p_full, o_done, mma_idle;
  uint32_t tmem_base;
};

struct PromptTcArgs {
  alignas(64) CUtensorMap kmap;  // the K ring [capacity][kv_heads * 128]
  alignas(64) CUtensorMap vmap;
  const float* q;  // [rows][ldq], normalised and rotated
  int ldq;
  const float* gate;
  int ldg;
  float* out;      // [rows][heads * 128]
  float* partial;  // spans > 1: [spans][rows][heads][130]
  int n, heads, kv_heads, group, position, span, spans;
};

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
  const int span_first = split * a.span, span_last = span_first + a.span - 1;
  const int first_key = span_first;
  const int last_key = min(P + q0 + nq - 1, span_last);
  const int tiles =
      first_key <= last_key ? (last_key - first_key) / kKeysTc + 1 : 0;
  if (tid == 0) {
    for (int i = 0; i < kStagesTc; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 4);
    }
    mbar_init(&s.q_full, 4);
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_empty, 4);
    mbar_init(&s.p_full, 4);
    mbar_init(&s.o_done, 1);
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
        if (j >= kStagesTc &&
            !mbar_wait(&s.kv_empty[st], ((j / kStagesTc) - 1) & 1,
                       kErrPrefillWait)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.kv_full[st], kStageBytes);
        ++issued;
        const int key0 = first_key + j * kKeysTc;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int x = grp * kHeadDim + c * 32;
          tma_load_2d(s.k[st][c], &a.kmap, x, key0, &s.kv_full[st]);
          tma_load_2d(s.v[st][c], &a.vmap, x, key0, &s.kv_full[st]);
        }
      }
      // no copy may still be landing when the block exits (error paths)
      for (int j = max(0, issued - kStagesTc); j < issued; ++j)
        mbar_wait(&s.kv_full[j % kStagesTc], (j / kStagesTc) & 1,
                  kErrPrefillWait);
    }
  } else if (warp == 5) {
    // ---- MMA issue (one thread)
    if (lane == 0 && tiles > 0) {
      ok = mbar_wait(&s.q_full, 0, kErrPrefillWait);
      for (int j = 0; j < tiles && ok; ++j) {
        const int st = j % kStagesTc;
        if (!mbar_wait(&s.kv_full[st], (j / kStagesTc) & 1,
                       kErrPrefillWait) ||
            (j > 0 && !mbar_wait(&s.s_empty, (j - 1) & 1, kErrPrefillWait))) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16)
          tc::mma(tmem + kColS,
                  tc::sw64_desc(s.q[k16 / 2]) + (k16 % 2) * 2,
                  tc::sw64_desc(s.k[st][k16 / 2]) + (k16 % 2) * 2, kIdescS,
                  k16 > 0);
        tc::commit(&s.s_full);
        if (!mbar_wait(&s.p_full, j & 1, kErrPrefillWait)) {
          ok = false;
          break;
        }
        tc::fence_after();
#pragma unroll
        for (int k16 = 0; k16 < 4; ++k16)
          tc::mma(tmem + kColO, tc::sw64_desc(s.p[k16 / 2]) + (k16 % 2) * 2,
                  tc::sw64_desc(s.vt[k16 / 2]) + (k16 % 2) * 2, kIdescO,
                  j > 0 || k16 > 0);
        tc::commit(&s.o_done);
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
    float m = -INFINITY, l = 0;
    for (int j = 0; j < tiles && ok; ++j) {
      const int st = j % kStagesTc;
      const int key0 = first_key + j * kKeysTc;
      if (!wait_all(&s.s_full, j & 1) ||
          !wait_all(&s.kv_full[st], (j / kStagesTc) & 1)) {
        ok = false;
        break;
      }
      tc::fence_after();
      uint32_t sv[64];
      tc::ld32(lane_base + kColS, *reinterpret_cast<uint32_t(*)[32]>(sv));
      tc::ld32(lane_base + kColS + 32,
               *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
      tc::wait_ld();
      tc::fence_before();
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.s_empty);
      // causal mask, running maximum (base 2)
      float top = -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int key = key0 + i;
        const bool in = key <= last_key && key <= qpos;
        const float x = in ? __uint_as_float(sv[i]) : -INFINITY;
        sv[i] = __float_as_uint(x);
        top = fmaxf(top, x);
      }
      const float next = fmaxf(m, top);
      const float shift = next == -INFINITY ? 0.0F : next;
      const float alpha = exp2f(m - shift);
      m = next;
      // probabilities rounded to FP16; the denominator adds the rounded
      uint32_t pw[32];
      float local = 0;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const __half p0 = __float2half_rn(exp2f(__uint_as_float(sv[2 * i]) - shift));
        const __half p1 =
            __float2half_rn(exp2f(__uint_as_float(sv[2 * i + 1]) - shift));
        local += __half2float(p0) + __half2float(p1);
        pw[i] = pack2(p0, p1);
      }
      l = l * alpha + local;
      // the previous tile's P V has finished with P, V^T and O
      if (j > 0 && !wait_all(&s.o_done, (j - 1) & 1)) {
        ok = false;
        break;
      }
      tc::fence_after();
#pragma unroll
      for (int piece = 0; piece < 8; ++piece)
        *reinterpret_cast<uint4*>(s.p[piece / 4] +
                                  tc::sw64_offset(t, piece % 4)) =
            make_uint4(pw[4 * piece], pw[4 * piece + 1], pw[4 * piece + 2],
                       pw[4 * piece + 3]);
      {
        // V^T: thread t transposes the 8 x 8 block of keys 8 kb .. 8 kb + 7
        // and dimensions 8 db .. 8 db + 7. Keys past last_key (ring slots
        // this pass has not written, whatever they hold) become zeros: a
        // zero probability times a NaN would still be NaN.
        const int kb = t / 16, db = t % 16;
        uint4 rows[8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
          rows[r] = key0 + 8 * kb + r <= last_key
                        ? *reinterpret_cast<const uint4*>(
                              s.v[st][db / 4] +
                              tc::sw64_offset(8 * kb + r, db % 4))
                        : make_uint4(0, 0, 0, 0);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(rows);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          // dimension 8 db + d: keys 8 kb + 2 i and 8 kb + 2 i + 1
          const uint32_t sel = (d & 1) ? 0x7632u : 0x5410u;
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[i] = __byte_perm(w[(2 * i) * 4 + d / 2],
                               w[(2 * i + 1) * 4 + d / 2], sel);
          *reinterpret_cast<uint4*>(s.vt[kb / 4] +
                                    tc::sw64_offset(8 * db + d, kb % 4)) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      // rescale this row of O when its maximum moved
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0F)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
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
      if (lane == 0) {
        mbar_arrive(&s.p_full);
        mbar_arrive(&s.kv_empty[st]);
      }
    }
    // ---- epilogue: the row's output (or, with spans, its maximum, sum and
    // unnormalised output for the combine kernel)
    if (ok && tiles > 0 && !wait_all(&s.o_done, (tiles - 1) & 1))
      ok = false;
    tc::fence_after();
    if (ok) {
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
  if (cudaError_t e = cached_activation_map(&a.kmap, ring_k, capacity,
                                            kv_heads * kHeadDim, kKeysTc, 32))
    return e;
  if (cudaError_t e = cached_activation_map(&a.vmap, ring_v, capacity,
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
