/* CPU oracle for the LFM3 backbone step — TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's FP32 scalar oracle
 * (reference.cpp:9-168). Each function names the reference lines it follows
 * and keeps their arithmetic in the same order and precision (float
 * products and sums, powf/cosf/sinf/expf/sqrtf), so that, compiled with
 * -ffp-contract=off like oracle/_ref, it reproduces the reference bit for
 * bit. Only the matrix-vector product is restructured: eight rows advance
 * together and threads split the rows, while each row's sum still runs over
 * k = 0..K-1 in order (reference.cpp:9-19), so results are independent of
 * the thread count.
 *
 * Row decoding follows weights.cpp:101-126 (DecodeRow): F32 copy, F16 and
 * BF16 widening, Q8_0 as d * q per 32-element block with d the fp16 scale.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / the
 * reference arm may load this code, as the checker or the timed CPU
 * baseline. The product path never calls it.
 */
#include "lfm3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define MAX_THREADS 64

static float half_to_float(uint16_t bits) {
  const uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  const uint32_t e = (bits >> 10) & 0x1fu, m = bits & 0x3ffu;
  uint32_t x;
  float f;
  if (e == 0x1f)
    x = sign | 0x7f800000u | (m << 13);
  else if (e)
    x = sign | ((e + 112) << 23) | (m << 13);
  else if (!m)
    x = sign;
  else {
    f = (float)m * 5.9604644775390625e-8f;
    memcpy(&x, &f, 4);
    x |= sign;
  }
  memcpy(&f, &x, 4);
  return f;
}

/* Round-to-nearest-even to the nearest fp16 value (overflow to infinity),
 * back in float: the value an F16 K/V ring holds. */
static float round_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = x & 0x80000000u, ax = x & 0x7fffffffu;
  uint16_t h;
  if (ax >= 0x7f800000u)
    h = (uint16_t)((sign >> 16) | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  else if (ax >= 0x477ff000u) /* rounds to >= 65520: infinity */
    h = (uint16_t)((sign >> 16) | 0x7c00u);
  else if (ax < 0x38800000u) { /* below 2^-14: subnormal or zero */
    float a;
    memcpy(&a, &ax, 4);
    const float q = a * 16777216.0f; /* units of 2^-24, exact */
    h = (uint16_t)((sign >> 16) | (uint16_t)nearbyintf(q));
  } else {
    const uint32_t e = (ax >> 23) - 112, m = ax & 0x7fffffu;
    uint32_t v = (e << 10) | (m >> 13);
    const uint32_t rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (v & 1)))
      ++v;
    h = (uint16_t)((sign >> 16) | v);
  }
  return half_to_float(h);
}

/* ---- thread pool for Mat ------------------------------------------------ */

typedef struct mat_task {
  const lfm3_tensor* t;
  const float* x;
  float* y;
} mat_task;

/* Workers wake on a new generation, take their share of rows and report
 * back; the caller takes share 0. */
typedef struct pool {
  int threads; /* participants, the caller included */
  pthread_t th[MAX_THREADS];
  pthread_mutex_t mu;
  pthread_cond_t wake, done;
  unsigned generation;
  int pending, quit;
  mat_task task;
} pool;

/* Rows [r0, r1) of y = t x, each as reference.cpp:13-17: decode the row,
 * then sum += row[k] * x[k] for k in order. */
static void mat_rows(const lfm3_tensor* t, const float* x, float* y,
                     uint32_t r0, uint32_t r1) {
  const size_t row_bytes = t->bytes / t->rows;
  const uint32_t K = t->cols;
  const unsigned char* base = (const unsigned char*)t->data;
  for (uint32_t r = r0; r < r1; r += 8) {
    const uint32_t n = r1 - r < 8 ? r1 - r : 8;
    float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const unsigned char* rows[8];
    for (uint32_t i = 0; i < 8; ++i)
      rows[i] = base + (size_t)(r + (i < n ? i : 0)) * row_bytes;
    switch (t->type) {
      case LFM3_Q8_0:
        for (uint32_t b = 0; b < K / 32; ++b) {
          float d[8];
          for (uint32_t i = 0; i < 8; ++i) {
            uint16_t h;
            memcpy(&h, rows[i] + (size_t)b * 34, 2);
            d[i] = half_to_float(h);
          }
          for (uint32_t j = 0; j < 32; ++j) {
            const float xk = x[b * 32 + j];
            for (uint32_t i = 0; i < 8; ++i) {
              const float w =
                  (float)(int8_t)rows[i][(size_t)b * 34 + 2 + j] * d[i];
              sum[i] += w * xk;
            }
          }
        }
        break;
      case LFM3_BF16:
        for (uint32_t k = 0; k < K; ++k) {
          const float xk = x[k];
          for (uint32_t i = 0; i < 8; ++i) {
            uint16_t h;
            memcpy(&h, rows[i] + (size_t)k * 2, 2);
            const uint32_t u = (uint32_t)h << 16;
            float w;
            memcpy(&w, &u, 4);
            sum[i] += w * xk;
          }
        }
        break;
      case LFM3_F16:
        for (uint32_t k = 0; k < K; ++k) {
          const float xk = x[k];
          for (uint32_t i = 0; i < 8; ++i) {
            uint16_t h;
            memcpy(&h, rows[i] + (size_t)k * 2, 2);
            sum[i] += half_to_float(h) * xk;
          }
        }
        break;
      default: /* F32 */
        for (uint32_t k = 0; k < K; ++k) {
          const float xk = x[k];
          for (uint32_t i = 0; i < 8; ++i) {
            float w;
            memcpy(&w, rows[i] + (size_t)k * 4, 4);
            sum[i] += w * xk;
          }
        }
        break;
    }
    for (uint32_t i = 0; i < n; ++i)
      y[r + i] = sum[i];
  }
}

static void mat_share(pool* p, int index) {
  const mat_task* task = &p->task;
  const uint32_t rows = task->t->rows;
  /* chunks of 8 rows, dealt contiguously */
  const uint32_t groups = (rows + 7) / 8;
  const uint32_t g0 = (uint32_t)((uint64_t)groups * index / p->threads);
  const uint32_t g1 = (uint32_t)((uint64_t)groups * (index + 1) / p->threads);
  const uint32_t r0 = g0 * 8, r1 = g1 * 8 < rows ? g1 * 8 : rows;
  if (r0 < r1)
    mat_rows(task->t, task->x, task->y, r0, r1);
}

typedef struct worker_arg {
  pool* p;
  int index;
} worker_arg;

static void* worker(void* arg) {
  worker_arg* a = (worker_arg*)arg;
  pool* p = a->p;
  unsigned seen = 0;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    while (p->generation == seen && !p->quit)
      pthread_cond_wait(&p->wake, &p->mu);
    if (p->quit) {
      pthread_mutex_unlock(&p->mu);
      return NULL;
    }
    seen = p->generation;
    pthread_mutex_unlock(&p->mu);
    mat_share(p, a->index);
    pthread_mutex_lock(&p->mu);
    if (--p->pending == 0)
      pthread_cond_signal(&p->done);
    pthread_mutex_unlock(&p->mu);
  }
}

/* ---- oracle ------------------------------------------------------------- */

typedef struct layer_state {
  float *conv, *k, *v;
  uint32_t capacity;
} layer_state;

struct lfm3_oracle {
  const lfm3_weights* w;
  uint32_t context, position;
  int kv_half; /* round stored K/V through fp16 (lfm3_oracle_set_kv_half) */
  layer_state states[LFM3_MAX_LAYERS];
  /* per-step scratch */
  float *x, *z, *out, *p, *conv, *q, *kk, *vv, *gate, *a, *ff_gate, *ff_up,
      *scores, *hidden;
  pool* pool;
  worker_arg* args;
};

static void mat(lfm3_oracle* o, const lfm3_tensor* t, const float* x,
                float* y) {
  if (!o->pool || t->rows < 64) {
    mat_rows(t, x, y, 0, t->rows);
    return;
  }
  pool* p = o->pool;
  pthread_mutex_lock(&p->mu);
  p->task.t = t;
  p->task.x = x;
  p->task.y = y;
  p->pending = p->threads - 1;
  ++p->generation;
  pthread_cond_broadcast(&p->wake);
  pthread_mutex_unlock(&p->mu);
  mat_share(p, 0);
  pthread_mutex_lock(&p->mu);
  while (p->pending)
    pthread_cond_wait(&p->done, &p->mu);
  pthread_mutex_unlock(&p->mu);
}

/* reference.cpp:20-27 */
static void norm(float* x, uint32_t n, const lfm3_tensor* w, float eps) {
  float sum = 0;
  for (uint32_t i = 0; i < n; ++i)
    sum += x[i] * x[i];
  const float scale = 1 / sqrtf(sum / (float)n + eps);
  const float* weight = (const float*)w->data;
  for (uint32_t i = 0; i < n; ++i)
    x[i] = x[i] * scale * weight[i];
}

/* reference.cpp:28-43 */
static void rope(float* x, uint32_t size, const lfm3_config* c,
                 uint32_t position, int swa, const lfm3_tensor* factors) {
  const uint32_t D = c->head_dim;
  const float theta = swa ? c->theta_swa : c->theta;
  for (uint32_t h = 0; h < size; h += D) {
    for (uint32_t i = 0; i < D / 2; ++i) {
      float angle = (float)position * powf(theta, -2.0F * (float)i / (float)D);
      if (!swa)
        angle /= ((const float*)factors->data)[i];
      const float a = x[h + i], b = x[h + i + D / 2];
      x[h + i] = a * cosf(angle) - b * sinf(angle);
      x[h + i + D / 2] = b * cosf(angle) + a * sinf(angle);
    }
  }
}

void lfm3_oracle_destroy(lfm3_oracle* o) {
  if (!o)
    return;
  if (o->pool) {
    pool* p = o->pool;
    pthread_mutex_lock(&p->mu);
    p->quit = 1;
    pthread_cond_broadcast(&p->wake);
    pthread_mutex_unlock(&p->mu);
    for (int i = 1; i < p->threads; ++i)
      pthread_join(p->th[i], NULL);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->wake);
    pthread_cond_destroy(&p->done);
    free(p);
  }
  free(o->args);
  for (uint32_t i = 0; i < LFM3_MAX_LAYERS; ++i) {
    free(o->states[i].conv);
    free(o->states[i].k);
    free(o->states[i].v);
  }
  free(o->x);
  free(o->z);
  free(o->out);
  free(o->p);
  free(o->conv);
  free(o->q);
  free(o->kk);
  free(o->vv);
  free(o->gate);
  free(o->a);
  free(o->ff_gate);
  free(o->ff_up);
  free(o->scores);
  free(o->hidden);
  free(o);
}

/* reference.cpp:45-63 */
lfm3_oracle* lfm3_oracle_create(const lfm3_weights* w, uint32_t context,
                                int threads) {
  const lfm3_config* c = &w->config;
  if (!context || context > c->context)
    return NULL;
  lfm3_oracle* o = (lfm3_oracle*)calloc(1, sizeof(*o));
  if (!o)
    return NULL;
  o->w = w;
  o->context = context;
  int ok = 1;
  for (uint32_t i = 0; i < c->n_layers; ++i) {
    layer_state* s = &o->states[i];
    if (c->layer_type[i] == LFM3_CONV) {
      s->conv = (float*)calloc((size_t)c->hidden * (c->conv_width - 1), 4);
      ok = ok && s->conv;
    } else {
      s->capacity = c->layer_type[i] == LFM3_SLIDING_ATTENTION
                        ? (context < c->window ? context : c->window)
                        : context;
      const size_t n = (size_t)s->capacity * c->kv_heads[i] * c->head_dim;
      s->k = (float*)calloc(n, 4);
      s->v = (float*)calloc(n, 4);
      ok = ok && s->k && s->v;
    }
  }
  const size_t H = c->hidden, A = (size_t)c->heads * c->head_dim;
  o->x = (float*)calloc(H, 4);
  o->z = (float*)calloc(H, 4);
  o->out = (float*)calloc(H > c->vocab ? H : c->vocab, 4);
  o->p = (float*)calloc(3 * H, 4);
  o->conv = (float*)calloc(H, 4);
  o->q = (float*)calloc(A, 4);
  o->kk = (float*)calloc(A, 4);
  o->vv = (float*)calloc(A, 4);
  o->gate = (float*)calloc(c->heads, 4);
  o->a = (float*)calloc(A, 4);
  o->ff_gate = (float*)calloc(c->intermediate, 4);
  o->ff_up = (float*)calloc(c->intermediate, 4);
  o->scores = (float*)calloc((size_t)context + 1, 4);
  o->hidden = (float*)calloc(H, 4);
  ok = ok && o->x && o->z && o->out && o->p && o->conv && o->q && o->kk &&
       o->vv && o->gate && o->a && o->ff_gate && o->ff_up && o->scores &&
       o->hidden;
  if (ok && threads > 1) {
    if (threads > MAX_THREADS)
      threads = MAX_THREADS;
    o->pool = (pool*)calloc(1, sizeof(pool));
    o->args = (worker_arg*)calloc((size_t)threads, sizeof(worker_arg));
    ok = o->pool && o->args;
    if (ok) {
      pool* p = o->pool;
      pthread_mutex_init(&p->mu, NULL);
      pthread_cond_init(&p->wake, NULL);
      pthread_cond_init(&p->done, NULL);
      p->threads = 1;
      for (int i = 1; i < threads; ++i) {
        o->args[i].p = p;
        o->args[i].index = i;
        if (pthread_create(&p->th[i], NULL, worker, &o->args[i]) != 0)
          break; /* run with the workers that started */
        p->threads = i + 1;
      }
    }
  }
  if (!ok) {
    lfm3_oracle_destroy(o);
    return NULL;
  }
  return o;
}

/* reference.cpp:64-71 */
void lfm3_oracle_reset(lfm3_oracle* o) {
  const lfm3_config* c = &o->w->config;
  o->position = 0;
  for (uint32_t i = 0; i < c->n_layers; ++i) {
    layer_state* s = &o->states[i];
    if (s->conv)
      memset(s->conv, 0, (size_t)c->hidden * (c->conv_width - 1) * 4);
    if (s->k) {
      const size_t n = (size_t)s->capacity * c->kv_heads[i] * c->head_dim;
      memset(s->k, 0, n * 4);
      memset(s->v, 0, n * 4);
    }
  }
}

uint32_t lfm3_oracle_position(const lfm3_oracle* o) { return o->position; }

void lfm3_oracle_set_kv_half(lfm3_oracle* o, int on) { o->kv_half = on != 0; }

float lfm3_oracle_round_half(float value) { return round_half(value); }

const float* lfm3_oracle_hidden(const lfm3_oracle* o) { return o->hidden; }

/* reference.cpp:72-168 */
int lfm3_oracle_step(lfm3_oracle* o, uint32_t token, float* logits) {
  const lfm3_weights* w = o->w;
  const lfm3_config* c = &w->config;
  if (token >= c->vocab || o->position >= o->context)
    return -1;
  const uint32_t H = c->hidden, D = c->head_dim, L = c->conv_width;
  float* x = o->x;
  /* DecodeRow(embedding, token) */
  {
    const lfm3_tensor* e = &w->embedding;
    const unsigned char* row =
        (const unsigned char*)e->data + (size_t)token * (e->bytes / e->rows);
    for (uint32_t k = 0; k < H; ++k) {
      if (e->type == LFM3_Q8_0) {
        uint16_t h;
        memcpy(&h, row + (size_t)(k / 32) * 34, 2);
        x[k] = (float)(int8_t)row[(size_t)(k / 32) * 34 + 2 + k % 32] *
               half_to_float(h);
      } else if (e->type == LFM3_BF16) {
        uint16_t h;
        memcpy(&h, row + 2 * (size_t)k, 2);
        const uint32_t u = (uint32_t)h << 16;
        memcpy(&x[k], &u, 4);
      } else if (e->type == LFM3_F16) {
        uint16_t h;
        memcpy(&h, row + 2 * (size_t)k, 2);
        x[k] = half_to_float(h);
      } else {
        memcpy(&x[k], row + 4 * (size_t)k, 4);
      }
    }
  }
  for (uint32_t il = 0; il < c->n_layers; ++il) {
    const lfm3_layer* l = &w->layers[il];
    layer_state* state = &o->states[il];
    float* z = o->z;
    memcpy(z, x, (size_t)H * 4);
    norm(z, H, &l->norm, c->eps);
    float* out = o->out;
    if (c->layer_type[il] == LFM3_CONV) {
      float* p = o->p;
      mat(o, &l->in_proj, z, p);
      const float* weight = (const float*)l->conv.data;
      for (uint32_t ch = 0; ch < H; ++ch) {
        float* history = state->conv + (size_t)ch * (L - 1);
        const float bx = p[ch] * p[2 * H + ch];
        float sum = 0;
        for (uint32_t t = 0; t < L; ++t)
          sum += weight[ch * L + t] * (t + 1 == L ? bx : history[t]);
        for (uint32_t t = 1; t < L - 1; ++t)
          history[t - 1] = history[t];
        if (L > 1)
          history[L - 2] = bx;
        o->conv[ch] = sum * p[H + ch];
      }
      mat(o, &l->out_proj, o->conv, out);
    } else {
      const uint32_t kvh = c->kv_heads[il];
      float *q = o->q, *k = o->kk, *v = o->vv, *gate = o->gate;
      mat(o, &l->q, z, q);
      mat(o, &l->k, z, k);
      mat(o, &l->v, z, v);
      mat(o, &l->attn_gate, z, gate);
      for (uint32_t h = 0; h < c->heads; ++h)
        norm(q + (size_t)h * D, D, &l->q_norm, c->eps);
      for (uint32_t h = 0; h < kvh; ++h)
        norm(k + (size_t)h * D, D, &l->k_norm, c->eps);
      const int swa = c->layer_type[il] == LFM3_SLIDING_ATTENTION;
      rope(q, c->heads * D, c, o->position, swa, &w->rope_freqs);
      rope(k, kvh * D, c, o->position, swa, &w->rope_freqs);
      const size_t stride = (size_t)kvh * D;
      const size_t slot = o->position % state->capacity;
      memcpy(state->k + slot * stride, k, stride * 4);
      memcpy(state->v + slot * stride, v, stride * 4);
      if (o->kv_half)
        for (size_t i = 0; i < stride; ++i) {
          state->k[slot * stride + i] = round_half(state->k[slot * stride + i]);
          state->v[slot * stride + i] = round_half(state->v[slot * stride + i]);
        }
      const uint32_t first =
          swa && o->position + 1 > c->window ? o->position + 1 - c->window : 0;
      float* scores = o->scores;
      for (uint32_t h = 0; h < c->heads; ++h) {
        const uint32_t kh = h / (c->heads / kvh);
        float max = -INFINITY;
        for (uint32_t t = first; t <= o->position; ++t) {
          float score = 0;
          const float* key =
              state->k + (size_t)(t % state->capacity) * stride + kh * D;
          for (uint32_t d = 0; d < D; ++d)
            score += q[h * D + d] * key[d];
          scores[t - first] = score / sqrtf((float)D);
          max = fmaxf(max, scores[t - first]);
        }
        float den = 0;
        const uint32_t count = o->position + 1 - first;
        for (uint32_t i = 0; i < count; ++i) {
          scores[i] = expf(scores[i] - max);
          den += scores[i];
        }
        for (uint32_t d = 0; d < D; ++d) {
          float sum = 0;
          for (uint32_t t = first; t <= o->position; ++t)
            sum += (scores[t - first] / den) *
                   state->v[(size_t)(t % state->capacity) * stride + kh * D +
                            d];
          o->a[h * D + d] = sum / (1 + expf(-gate[h]));
        }
      }
      mat(o, &l->attn_out, o->a, out);
    }
    if (l->post_norm.data)
      norm(out, H, &l->post_norm, c->eps);
    for (uint32_t i = 0; i < H; ++i)
      x[i] += out[i];
    memcpy(z, x, (size_t)H * 4);
    norm(z, H, &l->ffn_norm, c->eps);
    mat(o, &l->gate, z, o->ff_gate);
    mat(o, &l->up, z, o->ff_up);
    for (uint32_t i = 0; i < c->intermediate; ++i)
      o->ff_gate[i] =
          (o->ff_gate[i] / (1 + expf(-o->ff_gate[i]))) * o->ff_up[i];
    mat(o, &l->down, o->ff_gate, out);
    if (l->post_ffn_norm.data)
      norm(out, H, &l->post_ffn_norm, c->eps);
    for (uint32_t i = 0; i < H; ++i)
      x[i] += out[i];
  }
  if (logits) {
    norm(x, H, &w->output_norm, c->eps);
    memcpy(o->hidden, x, (size_t)H * 4);
    mat(o, &w->output, x, logits);
  }
  ++o->position;
  return 0;
}
