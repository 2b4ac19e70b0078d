/*
 * Oracle: CPU restatement of potpori's per-shard Qwen3 forward (TEST INFRASTRUCTURE ONLY;
 * see oracle.h for what may load it and which reference lines each part follows).
 *
 * Arithmetic follows src/qwen/tiny.rs:9-132 operation for operation in F32: every sum is a
 * sequential left-to-right sum of rounded products (no fused multiply-add; the build passes
 * -ffp-contract=off), the norm divides by the RMS and then multiplies by the weight, softmax
 * subtracts the row maximum, divides each probability by the total and then multiplies by
 * the value. Matrices are kept as BF16 bits and decoded exactly to F32 on use. The
 * vectorisation below runs independent (row, token) sums side by side; it never reorders
 * the terms of one sum.
 */
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NMAT 7
#define NNORM 4
enum { W_Q, W_K, W_V, W_O, W_G, W_U, W_D };
enum { N_ATTN, N_QN, N_KN, N_FFN };

typedef struct or_layer {
  uint16_t *mat[NMAT];
  float *norm[NNORM];
  int mat_set[NMAT], norm_set[NNORM];
  float *kc, *vc; /* [capacity][kv_dim], src/qwen/model.rs:265-266 */
} or_layer;

struct or_shard {
  or_config c;
  int lb, le, first, last, capacity, chunk, rope_mode;
  uint16_t *embed; /* [vocab][hidden] (first || last), model.rs:231-238 */
  float *final_norm;
  int embed_set, final_norm_set;
  or_layer *L;
  float *rope_cos, *rope_sin; /* [capacity][head_dim/2] */
};

static const char *MAT_NAMES[NMAT] = {"self_attn.q_proj", "self_attn.k_proj",
                                      "self_attn.v_proj", "self_attn.o_proj",
                                      "mlp.gate_proj",    "mlp.up_proj",
                                      "mlp.down_proj"};
static const char *NORM_NAMES[NNORM] = {"input_layernorm", "self_attn.q_norm",
                                        "self_attn.k_norm", "post_attention_layernorm"};

static int g_threads = 0;

void or_set_threads(int32_t n) {
  g_threads = n > 0 ? n : 0;
  if (g_threads) omp_set_num_threads(g_threads);
}
int32_t or_get_threads(void) { return g_threads ? g_threads : omp_get_max_threads(); }

static inline float bf16_to_f32(uint16_t b) {
  union { uint32_t u; float f; } v;
  v.u = (uint32_t)b << 16;
  return v.f;
}
/* Round to nearest even, as half::bf16::from_f32 (hf.rs:248-253). NaN stays NaN. */
static inline uint16_t f32_to_bf16(float f) {
  union { uint32_t u; float f; } v;
  v.f = f;
  if ((v.u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((v.u >> 16) | 0x40);
  uint32_t rounding = 0x7fffu + ((v.u >> 16) & 1u);
  return (uint16_t)((v.u + rounding) >> 16);
}

/* ---------------------------------------------------------------------------------------
 * Seeded generator. Tensor element i of tensor `name` under `seed`:
 *   key  = mix(seed * G ^ fnv1a64(name))
 *   r_j  = mix(key + (3i + j + 1) * G), j = 0,1,2        (64 random bits each)
 *   S    = sum of the twelve 16-bit fields of r_0..r_2    (Irwin-Hall, 12 terms)
 *   v    = (float)(S - 393210) * (std * 2^-16)             (one f32 rounding)
 *   bf16 = round-to-nearest-even(v)
 * mix is the splitmix64 finaliser and G = 0x9E3779B97F4A7C15. Integer steps and one IEEE
 * multiply, so the CUDA generator reproduces it bit for bit.
 * ------------------------------------------------------------------------------------- */
#define GOLDEN 0x9E3779B97F4A7C15ull
static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
uint64_t or_name_hash(const char *name) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (const unsigned char *p = (const unsigned char *)name; *p; ++p) {
    h ^= *p;
    h *= 0x100000001b3ull;
  }
  return h;
}
static inline uint16_t gen_one(uint64_t key, int64_t i, float scale) {
  int32_t s = 0;
  for (int j = 0; j < 3; ++j) {
    uint64_t r = mix64(key + (uint64_t)(3 * i + j + 1) * GOLDEN);
    s += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) + (int32_t)((r >> 32) & 0xffff) +
         (int32_t)(r >> 48);
  }
  volatile float v = (float)(s - 393210) * scale;
  return f32_to_bf16(v);
}
void or_gen_bf16(uint64_t seed, const char *name, int64_t start, int64_t count, float std,
                 uint16_t *out) {
  uint64_t key = mix64(seed * GOLDEN ^ or_name_hash(name));
  float scale = std * (1.0f / 65536.0f);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < count; ++i) out[i] = gen_one(key, start + i, scale);
}

/* ------------------------------------------------------------------------------------- */

static int q_dim(const or_config *c) { return c->n_heads * c->head_dim; }
static int kv_dim(const or_config *c) { return c->n_kv_heads * c->head_dim; }

static void mat_shape(const or_config *c, int which, int64_t *rows, int64_t *cols) {
  switch (which) {
    case W_Q: *rows = q_dim(c); *cols = c->hidden; break;
    case W_K:
    case W_V: *rows = kv_dim(c); *cols = c->hidden; break;
    case W_O: *rows = c->hidden; *cols = q_dim(c); break;
    case W_G:
    case W_U: *rows = c->intermediate; *cols = c->hidden; break;
    default: *rows = c->hidden; *cols = c->intermediate; break;
  }
}
static int64_t norm_len(const or_config *c, int which) {
  return (which == N_QN || which == N_KN) ? c->head_dim : c->hidden;
}

static void build_rope(or_shard *s) {
  int half = s->c.head_dim / 2;
  for (int p = 0; p < s->capacity; ++p)
    for (int i = 0; i < half; ++i) {
      float cs, sn;
      if (s->rope_mode == OR_ROPE_F32) {
        /* tiny.rs:29-30 */
        float angle = (float)p / powf(s->c.rope_theta, 2.0f * (float)i / (float)s->c.head_dim);
        sn = sinf(angle);
        cs = cosf(angle);
      } else {
        double angle =
            (double)p * pow((double)s->c.rope_theta, -2.0 * (double)i / (double)s->c.head_dim);
        cs = (float)cos(angle);
        sn = (float)sin(angle);
      }
      s->rope_cos[(size_t)p * half + i] = cs;
      s->rope_sin[(size_t)p * half + i] = sn;
    }
}

or_shard *or_shard_create(const or_config *cfg, int32_t lb, int32_t le, int32_t capacity,
                          int32_t chunk) {
  /* model.rs:206-217 */
  if (!cfg || lb < 0 || lb >= le || le > cfg->layers || capacity <= 0 || chunk < 0 ||
      chunk > capacity || cfg->head_dim % 2 || cfg->n_kv_heads <= 0 ||
      cfg->n_heads % cfg->n_kv_heads)
    return NULL;
  or_shard *s = (or_shard *)calloc(1, sizeof(or_shard));
  s->c = *cfg;
  s->lb = lb;
  s->le = le;
  s->first = lb == 0;
  s->last = le == cfg->layers;
  s->capacity = capacity;
  s->chunk = chunk;
  s->rope_mode = OR_ROPE_F64;
  int nl = le - lb;
  s->L = (or_layer *)calloc((size_t)nl, sizeof(or_layer));
  for (int l = 0; l < nl; ++l) {
    for (int w = 0; w < NMAT; ++w) {
      int64_t r, c;
      mat_shape(cfg, w, &r, &c);
      s->L[l].mat[w] = (uint16_t *)calloc((size_t)(r * c), 2);
    }
    for (int w = 0; w < NNORM; ++w) s->L[l].norm[w] = (float *)calloc((size_t)norm_len(cfg, w), 4);
    s->L[l].kc = (float *)calloc((size_t)capacity * kv_dim(cfg), 4);
    s->L[l].vc = (float *)calloc((size_t)capacity * kv_dim(cfg), 4);
  }
  if (s->first || s->last) s->embed = (uint16_t *)calloc((size_t)cfg->vocab_size * cfg->hidden, 2);
  if (s->last) s->final_norm = (float *)calloc((size_t)cfg->hidden, 4);
  s->rope_cos = (float *)malloc((size_t)capacity * (cfg->head_dim / 2) * 4);
  s->rope_sin = (float *)malloc((size_t)capacity * (cfg->head_dim / 2) * 4);
  build_rope(s);
  return s;
}

void or_shard_set_rope_mode(or_shard *s, int32_t mode) {
  s->rope_mode = mode;
  build_rope(s);
}

void or_shard_destroy(or_shard *s) {
  if (!s) return;
  for (int l = 0; l < s->le - s->lb; ++l) {
    for (int w = 0; w < NMAT; ++w) free(s->L[l].mat[w]);
    for (int w = 0; w < NNORM; ++w) free(s->L[l].norm[w]);
    free(s->L[l].kc);
    free(s->L[l].vc);
  }
  free(s->L);
  free(s->embed);
  free(s->final_norm);
  free(s->rope_cos);
  free(s->rope_sin);
  free(s);
}

static int store(void *dst, int is_norm, int32_t dtype, const void *data, int64_t n) {
  if (is_norm) {
    float *d = (float *)dst;
    for (int64_t i = 0; i < n; ++i)
      d[i] = dtype == OR_F32 ? ((const float *)data)[i] : bf16_to_f32(((const uint16_t *)data)[i]);
  } else {
    uint16_t *d = (uint16_t *)dst;
    if (dtype == OR_BF16)
      memcpy(d, data, (size_t)n * 2);
    else
      for (int64_t i = 0; i < n; ++i) d[i] = f32_to_bf16(((const float *)data)[i]);
  }
  return OR_OK;
}

int or_shard_set_tensor(or_shard *s, const char *name, int32_t dtype, const void *data,
                        int64_t elements) {
  const or_config *c = &s->c;
  if (!strcmp(name, "model.embed_tokens.weight")) {
    if (!s->embed) return OR_OK; /* not this shard's parameter */
    if (elements != (int64_t)c->vocab_size * c->hidden) return OR_E_INVALID;
    s->embed_set = 1;
    return store(s->embed, 0, dtype, data, elements);
  }
  if (!strcmp(name, "model.norm.weight")) {
    if (!s->final_norm) return OR_OK;
    if (elements != c->hidden) return OR_E_INVALID;
    s->final_norm_set = 1;
    return store(s->final_norm, 1, dtype, data, elements);
  }
  int layer, off = 0;
  if (sscanf(name, "model.layers.%d.%n", &layer, &off) != 1 || off == 0) return OR_E_INVALID;
  if (layer < s->lb || layer >= s->le) return OR_OK;
  or_layer *L = &s->L[layer - s->lb];
  const char *rest = name + off;
  for (int w = 0; w < NMAT; ++w) {
    char full[96];
    snprintf(full, sizeof full, "%s.weight", MAT_NAMES[w]);
    if (!strcmp(rest, full)) {
      int64_t r, cc;
      mat_shape(c, w, &r, &cc);
      if (elements != r * cc) return OR_E_INVALID;
      L->mat_set[w] = 1;
      return store(L->mat[w], 0, dtype, data, elements);
    }
  }
  for (int w = 0; w < NNORM; ++w) {
    char full[96];
    snprintf(full, sizeof full, "%s.weight", NORM_NAMES[w]);
    if (!strcmp(rest, full)) {
      if (elements != norm_len(c, w)) return OR_E_INVALID;
      L->norm_set[w] = 1;
      return store(L->norm[w], 1, dtype, data, elements);
    }
  }
  return OR_E_INVALID;
}

int or_shard_init_random(or_shard *s, uint64_t seed, float std) {
  const or_config *c = &s->c;
  char name[128];
  if (s->embed) {
    or_gen_bf16(seed, "model.embed_tokens.weight", 0, (int64_t)c->vocab_size * c->hidden, std,
                s->embed);
    s->embed_set = 1;
  }
  if (s->final_norm) {
    for (int i = 0; i < c->hidden; ++i) s->final_norm[i] = 1.0f;
    s->final_norm_set = 1;
  }
  for (int l = s->lb; l < s->le; ++l) {
    or_layer *L = &s->L[l - s->lb];
    for (int w = 0; w < NMAT; ++w) {
      int64_t r, cc;
      mat_shape(c, w, &r, &cc);
      snprintf(name, sizeof name, "model.layers.%d.%s.weight", l, MAT_NAMES[w]);
      or_gen_bf16(seed, name, 0, r * cc, std, L->mat[w]);
      L->mat_set[w] = 1;
    }
    for (int w = 0; w < NNORM; ++w) {
      for (int64_t i = 0; i < norm_len(c, w); ++i) L->norm[w][i] = 1.0f;
      L->norm_set[w] = 1;
    }
  }
  return OR_OK;
}

int or_shard_fill_kv(or_shard *s, uint64_t seed, int32_t rows) {
  if (rows < 0 || rows > s->capacity) return OR_E_INVALID;
  int kv = kv_dim(&s->c);
  for (int l = 0; l < s->le - s->lb; ++l) {
    uint64_t key = mix64(seed * GOLDEN ^ (uint64_t)(l + 1));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)rows * kv; ++i) {
      s->L[l].kc[i] = bf16_to_f32(gen_one(key, 2 * i, 1.0f / 65536.0f));
      s->L[l].vc[i] = bf16_to_f32(gen_one(key, 2 * i + 1, 1.0f / 65536.0f));
    }
  }
  return OR_OK;
}

int or_shard_missing(const or_shard *s, char *buf, int64_t len) {
  int n = 0;
  if (buf && len > 0) buf[0] = 0;
#define MISSING(str)                                                        \
  do {                                                                      \
    if (buf && (int64_t)strlen(buf) + 80 < len) {                           \
      strcat(buf, str);                                                     \
      strcat(buf, ";");                                                     \
    }                                                                       \
    ++n;                                                                    \
  } while (0)
  if (s->embed && !s->embed_set) MISSING("model.embed_tokens.weight");
  if (s->final_norm && !s->final_norm_set) MISSING("model.norm.weight");
  for (int l = s->lb; l < s->le; ++l) {
    const or_layer *L = &s->L[l - s->lb];
    char nm[128];
    for (int w = 0; w < NMAT; ++w)
      if (!L->mat_set[w]) {
        snprintf(nm, sizeof nm, "model.layers.%d.%s.weight", l, MAT_NAMES[w]);
        MISSING(nm);
      }
    for (int w = 0; w < NNORM; ++w)
      if (!L->norm_set[w]) {
        snprintf(nm, sizeof nm, "model.layers.%d.%s.weight", l, NORM_NAMES[w]);
        MISSING(nm);
      }
  }
#undef MISSING
  return n;
}

void or_shard_reset(or_shard *s) {
  /* runtime/cuda.rs:181-189: every KV buffer back to zeros. */
  size_t n = (size_t)s->capacity * kv_dim(&s->c);
  for (int l = 0; l < s->le - s->lb; ++l) {
    memset(s->L[l].kc, 0, n * 4);
    memset(s->L[l].vc, 0, n * 4);
  }
}

/* ---------------------------------------------------------------------------------------
 * Arithmetic (tiny.rs:14-37)
 * ------------------------------------------------------------------------------------- */

#define LANES 8
/* out[r][n] = sum_k W[n][k] * x[r][k], each sum sequential in k (tiny.rs:14-19).
 * xt is x transposed and padded to `mp` lanes: xt[k*mp + r]. */
static void project(const uint16_t *W, int64_t rows_n, int64_t cols_k, const float *xt, int mp,
                    int m, float *out, int64_t out_stride) {
  int64_t nb = (rows_n + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    float acc[4][16];
    int64_t n0 = b * 4;
    int cnt = (int)(rows_n - n0 < 4 ? rows_n - n0 : 4);
    for (int j = 0; j < 4; ++j)
      for (int r = 0; r < mp; ++r) acc[j][r] = 0.0f;
    const uint16_t *w0 = W + n0 * cols_k;
    if (cnt == 4 && mp == 8) {
      for (int64_t k = 0; k < cols_k; ++k) {
        const float *xk = xt + k * 8;
        float a0 = bf16_to_f32(w0[k]), a1 = bf16_to_f32(w0[cols_k + k]);
        float a2 = bf16_to_f32(w0[2 * cols_k + k]), a3 = bf16_to_f32(w0[3 * cols_k + k]);
        for (int r = 0; r < 8; ++r) {
          acc[0][r] += a0 * xk[r];
          acc[1][r] += a1 * xk[r];
          acc[2][r] += a2 * xk[r];
          acc[3][r] += a3 * xk[r];
        }
      }
    } else {
      for (int64_t k = 0; k < cols_k; ++k) {
        const float *xk = xt + k * mp;
        for (int j = 0; j < cnt; ++j) {
          float a = bf16_to_f32(w0[j * cols_k + k]);
          for (int r = 0; r < mp; ++r) acc[j][r] += a * xk[r];
        }
      }
    }
    for (int j = 0; j < cnt; ++j)
      for (int r = 0; r < m; ++r) out[r * out_stride + n0 + j] = acc[j][r];
  }
}

static float *transpose_pad(const float *x, int m, int64_t k, int mp) {
  float *t = (float *)calloc((size_t)k * mp, 4);
  for (int r = 0; r < m; ++r)
    for (int64_t i = 0; i < k; ++i) t[i * mp + r] = x[r * k + i];
  return t;
}

/* tiny.rs:20-23: x / sqrt(mean(x^2) + eps) * w */
static void rms_norm(const float *x, const float *w, int64_t n, float eps, float *out) {
  float ss = 0.0f;
  for (int64_t i = 0; i < n; ++i) ss += x[i] * x[i];
  float rms = sqrtf(ss / (float)n + eps);
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] / rms * w[i];
}

/* tiny.rs:24-37: per-head norm, then rotate-half at absolute position p. */
static void norm_rope_heads(float *v, int heads, const float *w, const or_shard *s, int p) {
  int hd = s->c.head_dim, half = hd / 2;
  float tmp[1024];
  for (int h = 0; h < heads; ++h) {
    float *head = v + (int64_t)h * hd;
    rms_norm(head, w, hd, s->c.rms_norm_eps, tmp);
    memcpy(head, tmp, (size_t)hd * 4);
    const float *cs = s->rope_cos + (size_t)p * half, *sn = s->rope_sin + (size_t)p * half;
    for (int i = 0; i < half; ++i) {
      float a = head[i], b = head[i + half];
      head[i] = a * cs[i] - b * sn[i];
      head[i + half] = b * cs[i] + a * sn[i];
    }
  }
}

static int mp_for(int m) { return m <= 8 ? 8 : 16; }

int or_shard_forward(or_shard *s, int32_t pos, int32_t m, const int32_t *tokens,
                     const float *hidden, float *out, float *taps) {
  const or_config *c = &s->c;
  /* model.rs:373-395 */
  if (m <= 0 || m > 16 || pos < 0 || (int64_t)pos + m > s->capacity) return OR_E_INVALID;
  if (s->chunk != 0 && m != 1 && m != s->chunk) return OR_E_INVALID;
  if (s->first) {
    if (!tokens) return OR_E_INVALID;
    for (int i = 0; i < m; ++i)
      if (tokens[i] < 0 || tokens[i] >= c->vocab_size) return OR_E_INVALID;
  } else {
    if (!hidden) return OR_E_INVALID;
    for (int64_t i = 0; i < (int64_t)m * c->hidden; ++i)
      if (!isfinite(hidden[i])) return OR_E_INVALID;
  }
  if (or_shard_missing(s, NULL, 0)) return OR_E_MISSING;

  const int H = c->hidden, Q = q_dim(c), KV = kv_dim(c), I = c->intermediate, hd = c->head_dim;
  const int groups = c->n_heads / c->n_kv_heads;
  const int mp = mp_for(m);
  float *x = (float *)malloc((size_t)m * H * 4);
  float *nrm = (float *)malloc((size_t)m * H * 4);
  float *q = (float *)malloc((size_t)m * Q * 4);
  float *k = (float *)malloc((size_t)m * KV * 4);
  float *v = (float *)malloc((size_t)m * KV * 4);
  float *att = (float *)malloc((size_t)m * Q * 4);
  float *o = (float *)malloc((size_t)m * H * 4);
  float *g = (float *)malloc((size_t)m * I * 4);
  float *u = (float *)malloc((size_t)m * I * 4);

  if (s->first) /* model.rs:239-241, tiny.rs:39-42 */
    for (int r = 0; r < m; ++r)
      for (int i = 0; i < H; ++i) x[(int64_t)r * H + i] = bf16_to_f32(s->embed[(int64_t)tokens[r] * H + i]);
  else
    memcpy(x, hidden, (size_t)m * H * 4);

  for (int l = s->lb; l < s->le; ++l) {
    or_layer *L = &s->L[l - s->lb];
    for (int r = 0; r < m; ++r) rms_norm(x + (int64_t)r * H, L->norm[N_ATTN], H, c->rms_norm_eps, nrm + (int64_t)r * H);
    float *nt = transpose_pad(nrm, m, H, mp);
    project(L->mat[W_Q], Q, H, nt, mp, m, q, Q);
    project(L->mat[W_K], KV, H, nt, mp, m, k, KV);
    project(L->mat[W_V], KV, H, nt, mp, m, v, KV);
    free(nt);
    for (int r = 0; r < m; ++r) {
      norm_rope_heads(q + (int64_t)r * Q, c->n_heads, L->norm[N_QN], s, pos + r);
      norm_rope_heads(k + (int64_t)r * KV, c->n_kv_heads, L->norm[N_KN], s, pos + r);
      /* KV written at absolute positions (model.rs:282-302); V is the raw projection. */
      memcpy(L->kc + (int64_t)(pos + r) * KV, k + (int64_t)r * KV, (size_t)KV * 4);
      memcpy(L->vc + (int64_t)(pos + r) * KV, v + (int64_t)r * KV, (size_t)KV * 4);
    }
    /* tiny.rs:77-101, keys 0..=p visible to the row at absolute position p. */
    const float scale = sqrtf((float)hd);
#pragma omp parallel for schedule(dynamic) collapse(2)
    for (int r = 0; r < m; ++r)
      for (int h = 0; h < c->n_heads; ++h) {
        int p = pos + r;
        int kvh = h / groups;
        const float *qh = q + (int64_t)r * Q + (int64_t)h * hd;
        float *scores = (float *)malloc((size_t)(p + 1) * 4);
        float mx = -INFINITY;
        for (int j = 0; j <= p; ++j) {
          const float *kj = L->kc + (int64_t)j * KV + (int64_t)kvh * hd;
          float d = 0.0f;
          for (int i = 0; i < hd; ++i) d += qh[i] * kj[i];
          scores[j] = d / scale;
          mx = fmaxf(mx, scores[j]);
        }
        float total = 0.0f;
        for (int j = 0; j <= p; ++j) {
          scores[j] = expf(scores[j] - mx);
          total += scores[j];
        }
        float *ah = att + (int64_t)r * Q + (int64_t)h * hd;
        for (int i = 0; i < hd; ++i) ah[i] = 0.0f;
        for (int j = 0; j <= p; ++j) {
          const float *vj = L->vc + (int64_t)j * KV + (int64_t)kvh * hd;
          float w = scores[j] / total;
          for (int i = 0; i < hd; ++i) ah[i] += w * vj[i];
        }
        free(scores);
      }
    float *at = transpose_pad(att, m, Q, mp);
    project(L->mat[W_O], H, Q, at, mp, m, o, H);
    free(at);
    for (int64_t i = 0; i < (int64_t)m * H; ++i) x[i] += o[i]; /* model.rs:303 */
    for (int r = 0; r < m; ++r) rms_norm(x + (int64_t)r * H, L->norm[N_FFN], H, c->rms_norm_eps, nrm + (int64_t)r * H);
    nt = transpose_pad(nrm, m, H, mp);
    project(L->mat[W_G], I, H, nt, mp, m, g, I);
    project(L->mat[W_U], I, H, nt, mp, m, u, I);
    free(nt);
    for (int64_t i = 0; i < (int64_t)m * I; ++i) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i]; /* tiny.rs:111-115 */
    float *gt = transpose_pad(g, m, I, mp);
    project(L->mat[W_D], H, I, gt, mp, m, o, H);
    free(gt);
    for (int64_t i = 0; i < (int64_t)m * H; ++i) x[i] += o[i]; /* model.rs:305 */
    if (taps) memcpy(taps + (int64_t)(l - s->lb) * m * H, x, (size_t)m * H * 4);
  }

  int status = OR_OK;
  if (s->last) { /* model.rs:307-319, tiny.rs:124-131 */
    for (int r = 0; r < m; ++r) rms_norm(x + (int64_t)r * H, s->final_norm, H, c->rms_norm_eps, nrm + (int64_t)r * H);
    float *nt = transpose_pad(nrm, m, H, mp);
    project(s->embed, c->vocab_size, H, nt, mp, m, out, c->vocab_size);
    free(nt);
  } else {
    memcpy(out, x, (size_t)m * H * 4);
  }
  free(x); free(nrm); free(q); free(k); free(v); free(att); free(o); free(g); free(u);
  return status;
}

int or_argmax(const float *row, int64_t n, int32_t *index) {
  if (n <= 0) return 0;
  for (int64_t i = 0; i < n; ++i)
    if (!isfinite(row[i])) return 0;
  int64_t best = 0;
  float bv = -INFINITY;
  for (int64_t i = 0; i < n; ++i)
    if (row[i] > bv) {
      bv = row[i];
      best = i;
    }
  *index = (int32_t)best;
  return 1;
}

void or_top2(const float *row, int64_t n, float *top1, float *top2) {
  float a = -INFINITY, b = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    if (row[i] > a) {
      b = a;
      a = row[i];
    } else if (row[i] > b) {
      b = row[i];
    }
  }
  *top1 = a;
  *top2 = b;
}
