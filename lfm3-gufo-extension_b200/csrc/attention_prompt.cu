// Prompt-pass attention kernels: per-head norms + RoPE + F16 K/V rows, the
// causal GQA attention on the tensor cores, the key-span combine and the
// sliding-ring store.
//
// Attention CTA: one KV group, 16 query rows, one warp per query head of the
// group (so every K/V tile read serves G heads). Keys stream through shared
// memory in tiles of 64 with cp.async double buffering; S = Q K^T and
// O += P V run as m16n8k16 MMAs with fragments loaded by ldmatrix from
// XOR-swizzled tiles. As in WmmaAttn (hip/ops.hip:1355-1561), Q carries the
// softmax scale in base-2 units before its FP16 rounding, probabilities round
// to FP16 once and the denominator adds the rounded values, and the
// accumulation stays FP32. Long histories split their keys into spans whose
// partial (max, sum, output) a combine kernel merges (hip/ops.hip:1692-1709).
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kQ = 16;       // queries per CTA
constexpr int kKeys = 64;    // keys per tile
constexpr int kMinSpan = 1024, kMaxSpans = 8;

// ---- prompt heads ----------------------------------------------------------
// Block = one head of one row, 64 threads (one RoPE pair each).
__global__ void prompt_heads_kernel(float* q, float* k, const float* v,
                                    int ldq, int ldk, const float* q_norm,
                                    const float* k_norm, const float* freq,
                                    const float* factors, __half* k16,
                                    __half* v16, int heads, int kv_heads,
                                    int position, float eps) {
  const int head = blockIdx.x, row = blockIdx.y, i = threadIdx.x;
  grid_dependency_wait();
  allow_dependents();
  const bool is_key = head >= heads;
  const int kvh = head - heads;
  float* x = is_key ? k + size_t(row) * ldk + size_t(kvh) * kHeadDim
                    : q + size_t(row) * ldq + size_t(head) * kHeadDim;
  const float* w = is_key ? k_norm : q_norm;
  const float x0 = x[i], x1 = x[i + 64];
  __shared__ float partial[2];
  float squares = warp_sum(x0 * x0 + x1 * x1);
  if (i % 32 == 0)
    partial[i / 32] = squares;
  __syncthreads();
  squares = partial[0] + partial[1];
  const float inv = 1.0F / sqrtf(squares / 128.0F + eps);
  const float a = (x0 * inv) * w[i], b = (x1 * inv) * w[i + 64];
  float angle = float(position + row) * freq[i];
  if (factors)
    angle /= factors[i];
  float sn, cs;
  sincosf(angle, &sn, &cs);
  const float r0 = a * cs - b * sn, r1 = b * cs + a * sn;
  x[i] = r0;
  x[i + 64] = r1;
  if (!is_key)
    return;
  const size_t stride = size_t(kv_heads) * kHeadDim;
  const size_t o = size_t(row) * stride + size_t(kvh) * kHeadDim;
  k16[o + i] = __float2half_rn(r0);
  k16[o + i + 64] = __float2half_rn(r1);
  const float* vr = v + size_t(row) * ldk + size_t(kvh) * kHeadDim;
  v16[o + i] = __float2half_rn(vr[i]);
  v16[o + i + 64] = __float2half_rn(vr[i + 64]);
}

// ---- attention -----------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4],
                                                  uint32_t addr) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src,
                                           bool valid) {
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_one() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Byte offset of 16-byte piece `piece` of key row `key` in a swizzled tile.
__device__ __forceinline__ uint32_t tile_offset(int key, int piece) {
  return uint32_t(key * 256 + ((piece ^ (key & 7)) * 16));
}

struct PromptArgs {
  const float* q;
  int ldq;
  const __half* k16;
  const __half* v16;
  const __half* ring_k;
  const __half* ring_v;
  const float* gate;
  int ldg;
  float* out;
  float* partial;
  int n, heads, kv_heads, position, capacity, window, span, spans;
};

template <int G>
__global__ void __launch_bounds__(G * 32)
    prompt_attention_kernel(const __grid_constant__ PromptArgs a) {
  extern __shared__ __align__(128) uint8_t tiles_raw[];
  uint8_t(*sk)[kKeys * 256] = reinterpret_cast<uint8_t(*)[kKeys * 256]>(tiles_raw);
  uint8_t(*sv)[kKeys * 256] =
      reinterpret_cast<uint8_t(*)[kKeys * 256]>(tiles_raw + 2 * kKeys * 256);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int g = lane / 4, cq = lane % 4;
  const int q0 = blockIdx.x * kQ, grp = blockIdx.y, split = blockIdx.z;
  const int head = grp * G + warp;
  const size_t stride = size_t(a.kv_heads) * kHeadDim;
  const int P = a.position;
  const int span_first = split * a.span, span_last = span_first + a.span - 1;
  const int nq = min(kQ, a.n - q0);
  // key range of the CTA
  const int first_key = [&] {
    const int lo = a.window > 0 ? P + q0 + 1 - a.window : 0;
    return max(max(lo, 0), span_first);
  }();
  const int last_key = min(P + q0 + nq - 1, span_last);
  grid_dependency_wait();
  allow_dependents();

  // Q fragments: 16 queries x 128 dims, scaled, FP16
  const float scale = 0.0883883476483184405F * 1.44269504088896341F;
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = q0 + g + 8 * h;
      const float* qr = a.q + size_t(min(row, a.n - 1)) * a.ldq +
                        size_t(head) * kHeadDim + ks * 16 + 2 * cq;
      const bool live = row < a.n;
      const float2 lo = live ? *reinterpret_cast<const float2*>(qr)
                             : make_float2(0, 0);
      const float2 hi = live ? *reinterpret_cast<const float2*>(qr + 8)
                             : make_float2(0, 0);
      qa[ks][h] = pack_half2(lo.x * scale, lo.y * scale);
      qa[ks][2 + h] = pack_half2(hi.x * scale, hi.y * scale);
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[j][e] = 0;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0, 0};
  const int qpos[2] = {P + q0 + g, P + q0 + g + 8};

  const auto key_row = [&](int t, const __half* chunk, const __half* ring) {
    return t >= P ? chunk + size_t(t - P) * stride + size_t(grp) * kHeadDim
                  : ring + size_t(t % a.capacity) * stride +
                        size_t(grp) * kHeadDim;
  };
  const auto load_tile = [&](int buf, int base) {
    // 64 keys x 16 pieces of K and of V
    for (int c = tid; c < kKeys * 16; c += G * 32) {
      const int key = c / 16, piece = c % 16, t = base + key;
      const bool valid = t <= last_key;
      const int ts = valid ? t : first_key;
      cp_async16(smem_addr(sk[buf]) + tile_offset(key, piece),
                 key_row(ts, a.k16, a.ring_k) + piece * 8, valid);
      cp_async16(smem_addr(sv[buf]) + tile_offset(key, piece),
                 key_row(ts, a.v16, a.ring_v) + piece * 8, valid);
    }
    cp_async_commit();
  };

  if (first_key <= last_key && nq > 0) {
    const int tiles = (last_key - first_key) / kKeys + 1;
    load_tile(0, first_key);
    for (int it = 0; it < tiles; ++it) {
      const int base = first_key + it * kKeys, buf = it & 1;
      if (it + 1 < tiles) {
        load_tile(buf ^ 1, base + kKeys);
        cp_async_wait_one();
      } else {
        cp_async_wait_all();
      }
      __syncthreads();
      // S = Q K^T, 16 x 64
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sc[j][e] = 0;
      const uint32_t kbase = smem_addr(sk[buf]);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          // two key n-tiles (2jp, 2jp+1) x dims ks*16..+16
          const int mat = lane / 8, r8 = lane % 8;
          const int key = (2 * jp + (mat / 2)) * 8 + r8;
          const int piece = ks * 2 + (mat % 2);
          uint32_t b[4];
          ldmatrix_x4(b, kbase + tile_offset(key, piece));
          mma_f16(sc[2 * jp], qa[ks], b[0], b[1]);
          mma_f16(sc[2 * jp + 1], qa[ks], b[2], b[3]);
        }
      }
      // mask (only tiles that reach past a bound), online softmax (base 2)
      float top[2] = {-INFINITY, -INFINITY};
      const bool inside = base + kKeys - 1 <= last_key &&
                          base + kKeys - 1 <= P + q0 && base >= span_first &&
                          (a.window <= 0 || base > P + q0 + nq - 1 - a.window);
      if (inside) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            top[e >> 1] = fmaxf(top[e >> 1], sc[j][e]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = base + j * 8 + 2 * cq + (e & 1);
            const int qp = qpos[e >> 1];
            const bool ok = t <= last_key && t <= qp &&
                            (a.window <= 0 || t > qp - a.window) &&
                            t >= span_first;
            sc[j][e] = ok ? sc[j][e] : -INFINITY;
            top[e >> 1] = fmaxf(top[e >> 1], sc[j][e]);
          }
      }
      float alpha[2], shift[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        top[h] = fmaxf(top[h], __shfl_xor_sync(0xffffffffu, top[h], 1));
        top[h] = fmaxf(top[h], __shfl_xor_sync(0xffffffffu, top[h], 2));
        const float next = fmaxf(m[h], top[h]);
        shift[h] = next == -INFINITY ? 0 : next;
        alpha[h] = exp2f(m[h] - shift[h]);
        m[h] = next;
      }
      uint32_t pa[4][4];  // P as A fragments of 4 k-steps (16 keys each)
      float local[2] = {0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half p0 = __float2half_rn(exp2f(sc[j][0] - shift[0]));
        const __half p1 = __float2half_rn(exp2f(sc[j][1] - shift[0]));
        const __half p2 = __float2half_rn(exp2f(sc[j][2] - shift[1]));
        const __half p3 = __float2half_rn(exp2f(sc[j][3] - shift[1]));
        local[0] += __half2float(p0) + __half2float(p1);
        local[1] += __half2float(p2) + __half2float(p3);
        const __half2 top2 = __halves2half2(p0, p1);
        const __half2 bot2 = __halves2half2(p2, p3);
        const int kk = j / 2, hi = j % 2;
        pa[kk][hi * 2 + 0] = *reinterpret_cast<const uint32_t*>(&top2);
        pa[kk][hi * 2 + 1] = *reinterpret_cast<const uint32_t*>(&bot2);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        local[h] += __shfl_xor_sync(0xffffffffu, local[h], 1);
        local[h] += __shfl_xor_sync(0xffffffffu, local[h], 2);
        l[h] = l[h] * alpha[h] + local[h];
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha[0];
        o[j][1] *= alpha[0];
        o[j][2] *= alpha[1];
        o[j][3] *= alpha[1];
      }
      // O += P V
      const uint32_t vbase = smem_addr(sv[buf]);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {
          // dims n-tiles 2jp, 2jp+1 (16 dims = 2 pieces), keys kk*16..+16
          const int mat = lane / 8, r8 = lane % 8;
          const int key = kk * 16 + (mat % 2) * 8 + r8;
          const int piece = 2 * jp + mat / 2;
          uint32_t b[4];
          ldmatrix_x4_trans(b, vbase + tile_offset(key, piece));
          mma_f16(o[2 * jp], pa[kk], b[0], b[1]);
          mma_f16(o[2 * jp + 1], pa[kk], b[2], b[3]);
        }
      }
      __syncthreads();
    }
  }
  // ---- output rows q0 + g (e < 2) and q0 + g + 8
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = q0 + g + 8 * h;
    if (row >= a.n)
      continue;
    if (a.spans > 1) {
      float* part = a.partial +
                    ((size_t(split) * a.n + row) * a.heads + head) *
                        (kHeadDim + 2);
      if (cq == 0) {
        part[0] = m[h];
        part[1] = l[h];
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        part[2 + j * 8 + 2 * cq] = o[j][2 * h];
        part[2 + j * 8 + 2 * cq + 1] = o[j][2 * h + 1];
      }
      continue;
    }
    const float gs = 1 + expf(-a.gate[size_t(row) * a.ldg + head]);
    float* out = a.out + (size_t(row) * a.heads + head) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      out[j * 8 + 2 * cq] = (o[j][2 * h] / l[h]) / gs;
      out[j * 8 + 2 * cq + 1] = (o[j][2 * h + 1] / l[h]) / gs;
    }
  }
}

__global__ void prompt_combine_kernel(const float* __restrict__ partial,
                                      const float* __restrict__ gate, int ldg,
                                      float* out, int n, int heads,
                                      int spans) {
  const int rh = blockIdx.x, d = threadIdx.x;
  const int row = rh / heads, head = rh % heads;
  grid_dependency_wait();
  allow_dependents();
  const auto part = [&](int s) {
    return partial + ((size_t(s) * n + row) * heads + head) * (kHeadDim + 2);
  };
  float maximum = -INFINITY;
  for (int s = 0; s < spans; ++s)
    maximum = fmaxf(maximum, part(s)[0]);
  float sum = 0, acc = 0;
  for (int s = 0; s < spans; ++s) {
    const float* pp = part(s);
    const float w = pp[0] == -INFINITY ? 0.0F : exp2f(pp[0] - maximum);
    sum = fmaf(pp[1], w, sum);
    acc = fmaf(pp[2 + d], w, acc);
  }
  out[size_t(rh) * kHeadDim + d] =
      (acc / sum) / (1 + expf(-gate[size_t(row) * ldg + head]));
}

__global__ void store_kv_kernel(const __half* k, const __half* v, __half* ck,
                                __half* cv, int n, int stride, int position,
                                int capacity) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  grid_dependency_wait();
  allow_dependents();
  const int kept = min(n, capacity), first = n - kept;
  if (i >= size_t(kept) * stride)
    return;
  const size_t src = size_t(first) * stride + i;
  const size_t dst =
      size_t((position + first + int(i / stride)) % capacity) * stride +
      i % stride;
  ck[dst] = k[src];
  cv[dst] = v[src];
}

int plan_spans(int keys, int window, int* span) {
  if (window > 0) {
    *span = keys;
    return 1;
  }
  *span = max(kMinSpan, (keys + kMaxSpans - 1) / kMaxSpans);
  return (keys + *span - 1) / *span;
}

}  // namespace

cudaError_t launch_prompt_heads(float* q, float* k, const float* v, int ldq,
                                int ldk, const float* q_norm,
                                const float* k_norm, const float* freq,
                                const float* factors, __half* k16, __half* v16,
                                int n, int heads, int kv_heads, int position,
                                float eps, cudaStream_t stream, bool pdl) {
  if (n <= 0)
    return cudaSuccess;
  return launch_kernel(prompt_heads_kernel, dim3(heads + kv_heads, n),
                       dim3(64), 0, stream, pdl, q, k, v, ldq, ldk, q_norm,
                       k_norm, freq, factors, k16, v16, heads, kv_heads,
                       position, eps);
}

size_t prompt_attention_scratch_floats(int heads, int rows, int keys) {
  int span;
  const int spans = plan_spans(keys, 0, &span);
  return spans > 1 ? size_t(spans) * rows * heads * (kHeadDim + 2) : 0;
}

cudaError_t launch_prompt_attention(const float* q, int ldq, const __half* k16,
                                    const __half* v16, const __half* ring_k,
                                    const __half* ring_v, const float* gate,
                                    int ldg, float* out, int n, int heads,
                                    int kv_heads, int position, int capacity,
                                    int window, float* scratch,
                                    cudaStream_t stream, bool pdl) {
  if (kv_heads <= 0 || heads % kv_heads || n <= 0)
    return n == 0 ? cudaSuccess : cudaErrorInvalidValue;
  PromptArgs a{q,    ldq,   k16,       v16,      ring_k,   ring_v,
               gate, ldg,   out,       scratch,  n,        heads,
               kv_heads, position, capacity, window, 0, 1};
  a.spans = plan_spans(position + n, window, &a.span);
  if (a.spans > 1 && !scratch)
    return cudaErrorInvalidValue;
  const dim3 grid((n + kQ - 1) / kQ, kv_heads, a.spans);
  constexpr int kSmem = 4 * kKeys * 256;
  const int group = heads / kv_heads;
  if (group != 2 && group != 4 && group != 8)
    return cudaErrorInvalidValue;
  for (const void* kernel :
       {reinterpret_cast<const void*>(prompt_attention_kernel<2>),
        reinterpret_cast<const void*>(prompt_attention_kernel<4>),
        reinterpret_cast<const void*>(prompt_attention_kernel<8>)})
    if (const cudaError_t e = ensure_dynamic_smem(kernel, kSmem))
      return e;
  cudaError_t e = launch_kernel(
      group == 2   ? prompt_attention_kernel<2>
      : group == 4 ? prompt_attention_kernel<4>
                   : prompt_attention_kernel<8>,
      grid, dim3(32 * group), kSmem, stream, pdl, a);
  if (e != cudaSuccess || a.spans == 1)
    return e;
  return launch_kernel(prompt_combine_kernel, dim3(n * heads), dim3(kHeadDim),
                       0, stream, pdl, static_cast<const float*>(scratch), gate,
                       ldg, out, n, heads, a.spans);
}

cudaError_t launch_prompt_combine(const float* partial, const float* gate,
                                  int ldg, float* out, int n, int heads,
                                  int spans, cudaStream_t stream, bool pdl) {
  return launch_kernel(prompt_combine_kernel, dim3(n * heads), dim3(kHeadDim),
                       0, stream, pdl, partial, gate, ldg, out, n, heads,
                       spans);
}

cudaError_t launch_store_kv(const __half* k16, const __half* v16,
                            __half* ring_k, __half* ring_v, int n, int stride,
                            int position, int capacity, cudaStream_t stream,
                            bool pdl) {
  if (n <= 0)
    return cudaSuccess;
  const size_t count = size_t(min(n, capacity)) * stride;
  return launch_kernel(store_kv_kernel, dim3(unsigned((count + 255) / 256)),
                       dim3(256), 0, stream, pdl, k16, v16, ring_k, ring_v, n,
                       stride, position, capacity);
}

}  // namespace lfm3
