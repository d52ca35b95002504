/* Deterministic synthetic LFM3 weights; see include/lfm3_synth.h.
 *
 * Tensor names, shapes and the tied output follow weights.cpp:54-93 of the
 * reference. The Q8_0 encoding restates llama.cpp's quantize_row_q8_0_ref
 * (ggml-quants.c, the rule the reference's GGUF checkpoints were made with):
 * d = amax / 127, id = d ? 1 / d : 0, qs = roundf(x * id), d stored as fp16.
 */
#define _POSIX_C_SOURCE 200809L
#include "lfm3_synth.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

uint16_t lfm3_float_to_half(float value) {
  uint32_t x;
  memcpy(&x, &value, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, mag = x & 0x7fffffffu;
  if (mag >= 0x7f800000u)
    return (uint16_t)(sign | 0x7c00u | (mag > 0x7f800000u ? 0x200u : 0u));
  if (mag >= 0x477ff000u) /* 65520 and above round to infinity */
    return (uint16_t)(sign | 0x7c00u);
  if (mag < 0x38800000u) { /* below 2^-14: half subnormal or zero */
    if (mag < 0x33000000u) /* at most 2^-25: rounds to (even) zero */
      return (uint16_t)sign;
    const uint32_t e = mag >> 23, m = (mag & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126 - e; /* value / 2^-24 = m >> shift */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1u)))
      ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t h = ((mag >> 23) - 112) << 10 | ((mag >> 13) & 0x3ffu);
  const uint32_t rem = mag & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
    ++h;
  return (uint16_t)(sign | h);
}

float lfm3_half_to_float(uint16_t bits) {
  const uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  const uint32_t e = (bits >> 10) & 0x1fu, m = bits & 0x3ffu;
  uint32_t x;
  if (e == 0x1f)
    x = sign | 0x7f800000u | (m << 13);
  else if (e)
    x = sign | ((e + 112) << 23) | (m << 13);
  else if (!m)
    x = sign;
  else {
    /* subnormal: m * 2^-24 */
    float f = (float)m * 5.9604644775390625e-8f;
    memcpy(&x, &f, 4);
    x |= sign;
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint16_t float_to_bf16(float value) {
  uint32_t u;
  memcpy(&u, &value, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float bf16_to_float(uint16_t bits) {
  const uint32_t u = (uint32_t)bits << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

size_t lfm3_row_bytes(uint32_t type, uint32_t cols) {
  switch (type) {
    case LFM3_F32:
      return (size_t)cols * 4;
    case LFM3_F16:
    case LFM3_BF16:
      return (size_t)cols * 2;
    case LFM3_Q8_0:
      return cols % LFM3_Q8_BLOCK ? 0
                                  : (size_t)cols / LFM3_Q8_BLOCK *
                                        LFM3_Q8_BLOCK_BYTES;
    default:
      return 0;
  }
}

void lfm3_synth_default_config(lfm3_config* c) {
  memset(c, 0, sizeof(*c));
  c->hidden = 2048;
  c->intermediate = 8192;
  c->vocab = 65536;
  c->context = 262144;
  c->heads = 16;
  c->head_dim = 128;
  c->window = 256;
  c->conv_width = 7;
  c->eps = 1e-5f;
  c->theta = 1e6f;
  c->theta_swa = 1e4f;
  lfm3_synth_set_layers(c, "CCSGCCSGCCSGCCSGCCSGCCGC", 4);
}

int lfm3_synth_set_layers(lfm3_config* c, const char* pattern,
                          uint32_t kv_heads) {
  const size_t n = pattern ? strlen(pattern) : 0;
  if (!n || n > LFM3_MAX_LAYERS)
    return -1;
  for (size_t i = 0; i < n; ++i) {
    switch (pattern[i]) {
      case 'C':
        c->layer_type[i] = LFM3_CONV;
        c->kv_heads[i] = 0;
        break;
      case 'S':
        c->layer_type[i] = LFM3_SLIDING_ATTENTION;
        c->kv_heads[i] = kv_heads;
        break;
      case 'G':
        c->layer_type[i] = LFM3_FULL_ATTENTION;
        c->kv_heads[i] = kv_heads;
        break;
      default:
        return -1;
    }
  }
  c->n_layers = (uint32_t)n;
  return 0;
}

/* ---- generation ---------------------------------------------------------- */

enum { KIND_MATRIX, KIND_NORM, KIND_CONV, KIND_ROPE };

typedef struct job {
  lfm3_tensor* tensor;
  uint32_t id, kind;
} job;

typedef struct plan {
  job jobs[4 + LFM3_MAX_LAYERS * 17];
  size_t count;
  uint64_t seed;
  float jitter;
  double sigma; /* standard deviation of the four-uniform sum */
  /* work queue of (job, first row) chunks */
  atomic_size_t next;
  size_t chunk_rows;
  size_t* chunk_job; /* job index of chunk i */
  size_t* chunk_row; /* first row of chunk i */
  size_t chunks;
} plan;

static uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

/* Approximately N(0, 1): Irwin-Hall sum of four 16-bit uniforms, centred
 * and divided by its exact standard deviation. Only exact integer steps and
 * correctly rounded double operations, so any IEEE machine agrees. */
static double unit_normal(uint64_t seed, uint32_t id, uint64_t index,
                          double sigma) {
  const uint64_t h =
      splitmix64(seed ^ ((uint64_t)id * 0xd1b54a32d192ed03ULL) ^
                 splitmix64(index + ((uint64_t)id << 40)));
  const int64_t s = (int64_t)(h & 0xffff) + (int64_t)((h >> 16) & 0xffff) +
                    (int64_t)((h >> 32) & 0xffff) + (int64_t)(h >> 48);
  return (double)(2 * s - 4 * 65535) * 0.5 / sigma;
}

static void fill_rows(const plan* p, const job* j, size_t row0, size_t rows) {
  lfm3_tensor* t = j->tensor;
  const size_t cols = t->cols;
  const size_t row_bytes = lfm3_row_bytes(t->type, t->cols);
  unsigned char* base = (unsigned char*)t->data;
  float* values = (float*)malloc(cols * sizeof(float));
  for (size_t r = row0; r < row0 + rows; ++r) {
    for (size_t c = 0; c < cols; ++c) {
      const uint64_t index = (uint64_t)r * cols + c;
      switch (j->kind) {
        case KIND_MATRIX:
          values[c] = bf16_to_float(float_to_bf16(
              (float)(0.02 * unit_normal(p->seed, j->id, index, p->sigma))));
          break;
        case KIND_CONV:
          values[c] = (float)(0.02 * unit_normal(p->seed, j->id, index, p->sigma));
          break;
        case KIND_NORM:
          values[c] =
              p->jitter == 0.0f
                  ? 1.0f
                  : (float)(1.0 + (double)p->jitter *
                                      unit_normal(p->seed, j->id, index, p->sigma));
          break;
        case KIND_ROPE:
          values[c] = c < cols / 2 ? 1.0f : 1e30f;
          break;
      }
    }
    unsigned char* out = base + r * row_bytes;
    switch (t->type) {
      case LFM3_F32:
        memcpy(out, values, cols * 4);
        break;
      case LFM3_BF16:
        for (size_t c = 0; c < cols; ++c) {
          const uint16_t b = float_to_bf16(values[c]);
          memcpy(out + 2 * c, &b, 2);
        }
        break;
      case LFM3_Q8_0:
        for (size_t b = 0; b < cols / LFM3_Q8_BLOCK; ++b) {
          const float* x = values + b * LFM3_Q8_BLOCK;
          float amax = 0.0f;
          for (int i = 0; i < LFM3_Q8_BLOCK; ++i)
            amax = fmaxf(amax, fabsf(x[i]));
          const float d = amax / 127.0f;
          const float id = d != 0.0f ? 1.0f / d : 0.0f;
          unsigned char* block = out + b * LFM3_Q8_BLOCK_BYTES;
          const uint16_t dh = lfm3_float_to_half(d);
          memcpy(block, &dh, 2);
          for (int i = 0; i < LFM3_Q8_BLOCK; ++i)
            block[2 + i] = (unsigned char)(int8_t)roundf(x[i] * id);
        }
        break;
    }
  }
  free(values);
}

static void* worker(void* arg) {
  plan* p = (plan*)arg;
  for (;;) {
    const size_t i = atomic_fetch_add(&p->next, 1);
    if (i >= p->chunks)
      return NULL;
    const job* j = &p->jobs[p->chunk_job[i]];
    const size_t row0 = p->chunk_row[i];
    size_t rows = j->tensor->rows - row0;
    if (rows > p->chunk_rows)
      rows = p->chunk_rows;
    fill_rows(p, j, row0, rows);
  }
}

static int valid_config(const lfm3_config* c) {
  if (!c->n_layers || c->n_layers > LFM3_MAX_LAYERS || !c->hidden ||
      !c->intermediate || !c->vocab || !c->heads || c->head_dim != 128 ||
      c->conv_width < 2 || c->conv_width > 32 || !c->window || !c->context)
    return 0;
  for (uint32_t i = 0; i < c->n_layers; ++i) {
    const uint32_t t = c->layer_type[i], h = c->kv_heads[i];
    if (t > LFM3_SLIDING_ATTENTION)
      return 0;
    if ((t == LFM3_CONV) != (h == 0))
      return 0;
    if (h && (h > c->heads || c->heads % h))
      return 0;
  }
  return 1;
}

int lfm3_synth_generate(const lfm3_config* c, uint64_t seed,
                        uint32_t matrix_type, float norm_jitter, int threads,
                        lfm3_synth_model* out) {
  memset(out, 0, sizeof(*out));
  if (!valid_config(c) ||
      (matrix_type != LFM3_Q8_0 && matrix_type != LFM3_BF16))
    return -1;
  if (matrix_type == LFM3_Q8_0 &&
      (c->hidden % 32 || c->intermediate % 32 ||
       (c->heads * c->head_dim) % 32))
    return -1;
  lfm3_weights* w = &out->weights;
  w->config = *c;
  plan* p = (plan*)calloc(1, sizeof(plan));
  if (!p)
    return -2;
  p->seed = seed;
  p->jitter = norm_jitter;
  /* variance of the sum of four discrete uniforms on [0, 65535] */
  p->sigma = sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  uint32_t id = 0;
#define ADD(t_, type_, cols_, rows_, kind_)                             \
  do {                                                                  \
    (t_).type = (type_);                                                \
    (t_).cols = (cols_);                                                \
    (t_).rows = (rows_);                                                \
    (t_).bytes = lfm3_row_bytes((type_), (cols_)) * (size_t)(rows_);    \
    p->jobs[p->count].tensor = &(t_);                                   \
    p->jobs[p->count].id = id++;                                        \
    p->jobs[p->count].kind = (kind_);                                   \
    ++p->count;                                                         \
  } while (0)
  const uint32_t H = c->hidden, F = c->intermediate, D = c->head_dim;
  ADD(w->embedding, matrix_type, H, c->vocab, KIND_MATRIX);
  ADD(w->output_norm, LFM3_F32, H, 1, KIND_NORM);
  ADD(w->rope_freqs, LFM3_F32, D / 2, 1, KIND_ROPE);
  for (uint32_t i = 0; i < c->n_layers; ++i) {
    lfm3_layer* l = &w->layers[i];
    ADD(l->norm, LFM3_F32, H, 1, KIND_NORM);
    ADD(l->ffn_norm, LFM3_F32, H, 1, KIND_NORM);
    ADD(l->post_norm, LFM3_F32, H, 1, KIND_NORM);
    ADD(l->post_ffn_norm, LFM3_F32, H, 1, KIND_NORM);
    ADD(l->gate, matrix_type, H, F, KIND_MATRIX);
    ADD(l->up, matrix_type, H, F, KIND_MATRIX);
    ADD(l->down, matrix_type, F, H, KIND_MATRIX);
    if (c->layer_type[i] == LFM3_CONV) {
      ADD(l->conv, LFM3_F32, c->conv_width, H, KIND_CONV);
      ADD(l->in_proj, matrix_type, H, 3 * H, KIND_MATRIX);
      ADD(l->out_proj, matrix_type, H, H, KIND_MATRIX);
    } else {
      const uint32_t kv = c->kv_heads[i] * D;
      ADD(l->q, matrix_type, H, c->heads * D, KIND_MATRIX);
      ADD(l->k, matrix_type, H, kv, KIND_MATRIX);
      ADD(l->v, matrix_type, H, kv, KIND_MATRIX);
      ADD(l->q_norm, LFM3_F32, D, 1, KIND_NORM);
      ADD(l->k_norm, LFM3_F32, D, 1, KIND_NORM);
      ADD(l->attn_gate, matrix_type, H, c->heads, KIND_MATRIX);
      ADD(l->attn_out, matrix_type, c->heads * D, H, KIND_MATRIX);
    }
  }
#undef ADD
  /* one allocation, every tensor 256-byte aligned (upload.cpp:12) */
  size_t total = 0;
  for (size_t i = 0; i < p->count; ++i)
    total += (p->jobs[i].tensor->bytes + 255) / 256 * 256;
  void* storage = NULL;
  if (posix_memalign(&storage, 4096, total ? total : 256)) {
    free(p);
    return -2;
  }
  size_t offset = 0;
  for (size_t i = 0; i < p->count; ++i) {
    p->jobs[i].tensor->data = (unsigned char*)storage + offset;
    offset += (p->jobs[i].tensor->bytes + 255) / 256 * 256;
  }
  w->output = w->embedding; /* tied (weights.cpp:55-57) */
  out->storage = storage;
  out->storage_bytes = total;
  /* chunked work queue */
  p->chunk_rows = 64;
  size_t chunks = 0;
  for (size_t i = 0; i < p->count; ++i)
    chunks += (p->jobs[i].tensor->rows + p->chunk_rows - 1) / p->chunk_rows;
  p->chunk_job = (size_t*)malloc(chunks * sizeof(size_t));
  p->chunk_row = (size_t*)malloc(chunks * sizeof(size_t));
  if (!p->chunk_job || !p->chunk_row) {
    free(p->chunk_job);
    free(p->chunk_row);
    free(p);
    lfm3_synth_free(out);
    return -2;
  }
  size_t k = 0;
  for (size_t i = 0; i < p->count; ++i)
    for (size_t r = 0; r < p->jobs[i].tensor->rows; r += p->chunk_rows) {
      p->chunk_job[k] = i;
      p->chunk_row[k] = r;
      ++k;
    }
  p->chunks = chunks;
  atomic_init(&p->next, 0);
  if (threads <= 0) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    threads = n > 0 ? (int)n : 1;
  }
  if (threads > 256)
    threads = 256;
  pthread_t pool[256];
  int started = 0;
  for (int t = 1; t < threads; ++t)
    if (pthread_create(&pool[started], NULL, worker, p) == 0)
      ++started;
  worker(p);
  for (int t = 0; t < started; ++t)
    pthread_join(pool[t], NULL);
  free(p->chunk_job);
  free(p->chunk_row);
  free(p);
  return 0;
}

void lfm3_synth_free(lfm3_synth_model* m) {
  free(m->storage);
  memset(m, 0, sizeof(*m));
}
