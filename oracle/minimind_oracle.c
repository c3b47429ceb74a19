/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle. Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load this; the
 * product path (libminimind_cuda.so and the C++ runtime) never links it.
 *
 * A plain-C restatement of the reference's fp32 CPU decode step
 * (lvyufeng/minimind-orangepi, the `#if !MINIMIND_USE_ASCEND` fall-through),
 * written to reproduce its arithmetic operation for operation so that it is
 * bit-identical to the reference built by oracle/build_ref.sh:
 *   - sequential fp32 sums, same association of every product;
 *   - powf/cosf/sinf/expf/sqrtf exactly where the reference calls the float
 *     overloads of std::pow/std::cos/std::sin/std::exp/std::sqrt.
 * Each function cites the reference lines it follows (paths relative to the
 * reference project root).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MMO_API __attribute__((visibility("default")))

typedef struct {
  int64_t hidden, layers, vocab, nq, nkv, hd, inter, max_pos;
  float eps, theta;
  int64_t use_moe, experts, moe_inter; /* top-1 MoE MLP (runtime_loader.cpp:76,84-86) */
} mmo_config;

typedef struct {
  float *input_norm, *post_norm, *q_norm, *k_norm;
  float *qkv;     /* fused [q;k;v] rows, language_model.cpp:95-119 */
  float *o;       /* [hidden][nq*hd] */
  float *gate_up; /* fused [gate;up] rows */
  float *down;    /* [hidden][inter] */
  float *moe_gate;            /* [experts][hidden] router */
  float **exp_gate_up, **exp_down; /* per expert: fused [gate;up] rows, down */
} mmo_layer;

typedef struct {
  mmo_config c;
  float *embed, *final_norm, *lm_head;
  mmo_layer *layer;
  float *rope_cos, *rope_sin; /* [max_pos][hd/2], decoder_layer.cpp:97-122 */
} mmo_model;

typedef struct {
  int64_t tokens, cap;
  float *keys, *values; /* [tokens][nkv][hd], decoder_layer.cpp:354-359 */
} mmo_cache;

typedef struct {
  int64_t position;
  mmo_cache *cache;
} mmo_state;

static char g_err[256];
/* smallest router top-2 margin (top1 - top2, relative to |top1|) over the
 * layers of the last mmo_forward_token call; INFINITY for dense models */
static float g_router_margin = INFINITY;
MMO_API float mmo_last_router_margin(void) { return g_router_margin; }
MMO_API const char *mmo_last_error(void) { return g_err; }

/* ---------------------------------------------------------------- kernels */

/* decoder_layer.cpp:32-42 rms_norm_inplace: values[i] *= scale * weight[i] */
MMO_API void mmo_rms_norm_inplace(float *v, const float *w, int64_t n, float eps) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum += v[i] * v[i];
  const float scale = 1.0f / sqrtf(sum / (float)n + eps);
  for (int64_t i = 0; i < n; ++i) v[i] *= scale * w[i];
}

/* language_model.cpp:24-38 rms_norm (final norm): out[i] = in[i] * scale * w[i] */
MMO_API void mmo_rms_norm_final(const float *in, const float *w, int64_t n, float eps, float *out) {
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum += in[i] * in[i];
  const float scale = 1.0f / sqrtf(sum / (float)n + eps);
  for (int64_t i = 0; i < n; ++i) out[i] = in[i] * scale * w[i];
}

/* decoder_layer.cpp:65-78 cpu_matvec: row-major [rows][cols], sequential sum */
MMO_API void mmo_matvec(const float *m, int64_t rows, int64_t cols, const float *x, float *y) {
  for (int64_t r = 0; r < rows; ++r) {
    float sum = 0.0f;
    const float *row = m + r * cols;
    for (int64_t c = 0; c < cols; ++c) sum += row[c] * x[c];
    y[r] = sum;
  }
}

/* decoder_layer.cpp:97-122 rope_tables: cos/sin of pos * 1/theta^(2d/hd) */
MMO_API void mmo_rope_tables(int64_t max_pos, int64_t hd, float theta, float *cos_t, float *sin_t) {
  const int64_t half = hd / 2;
  for (int64_t p = 0; p < max_pos; ++p) {
    for (int64_t d = 0; d < half; ++d) {
      const float inv_freq = 1.0f / powf(theta, (float)(d * 2) / (float)hd);
      const float angle = (float)p * inv_freq;
      cos_t[p * half + d] = cosf(angle);
      sin_t[p * half + d] = sinf(angle);
    }
  }
}

/* decoder_layer.cpp:124-153 apply_rope: rotate-half pairs (d, d+hd/2) */
MMO_API void mmo_apply_rope(float *v, int64_t heads, int64_t hd, int64_t pos, const float *cos_t, const float *sin_t) {
  const int64_t half = hd / 2;
  for (int64_t h = 0; h < heads; ++h) {
    float *b = v + h * hd;
    for (int64_t d = 0; d < half; ++d) {
      const float c = cos_t[pos * half + d], s = sin_t[pos * half + d];
      const float first = b[d], second = b[d + half];
      b[d] = first * c - second * s;
      b[d + half] = second * c + first * s;
    }
  }
}

/* decoder_layer.cpp:171-182 silu + swiglu_from_gate_up */
MMO_API void mmo_swiglu(const float *gate_up, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) {
    const float g = gate_up[i];
    out[i] = (g / (1.0f + expf(-g))) * gate_up[i + n];
  }
}

/* decoder_layer.cpp:184-234 attention_step (CPU branch): GQA softmax(q.K/sqrt(hd)).V
 * keys/values: [tokens][nkv][hd]. out: [nq][hd]. */
MMO_API void mmo_attention(const float *q, const float *keys, const float *values, int64_t tokens, int64_t nq,
                           int64_t nkv, int64_t hd, float *out) {
  const int64_t rep = nq / nkv;
  float *scores = (float *)malloc((size_t)(tokens > 0 ? tokens : 1) * sizeof(float));
  memset(out, 0, (size_t)(nq * hd) * sizeof(float));
  for (int64_t qh = 0; qh < nq; ++qh) {
    const int64_t kh = qh / rep;
    float max_score = -INFINITY;
    for (int64_t t = 0; t < tokens; ++t) {
      float dot = 0.0f;
      for (int64_t d = 0; d < hd; ++d) dot += q[qh * hd + d] * keys[(t * nkv + kh) * hd + d];
      const float score = dot / sqrtf((float)hd);
      scores[t] = score;
      max_score = score > max_score ? score : max_score; /* std::max(max_score, score) */
    }
    float denom = 0.0f;
    for (int64_t t = 0; t < tokens; ++t) {
      scores[t] = expf(scores[t] - max_score);
      denom += scores[t];
    }
    for (int64_t t = 0; t < tokens; ++t) {
      const float weight = scores[t] / denom;
      for (int64_t d = 0; d < hd; ++d) out[qh * hd + d] += weight * values[(t * nkv + kh) * hd + d];
    }
  }
  free(scores);
}

/* language_model.cpp:408-413 argmax_token: first maximum (std::max_element) */
MMO_API int32_t mmo_argmax(const float *v, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (v[best] < v[i]) best = i;
  return (int32_t)best;
}

/* ------------------------------------------------------------ model / IO */

static float *read_tensor(FILE *f, const char *name, uint64_t expect) {
  uint64_t n = 0;
  char buf[256];
  if (fread(&n, 8, 1, f) != 1 || n >= sizeof(buf) || fread(buf, 1, n, f) != n) goto bad;
  buf[n] = 0;
  if (strcmp(buf, name) != 0) {
    snprintf(g_err, sizeof g_err, "expected tensor %s, got %s", name, buf);
    return NULL;
  }
  uint64_t count = 0;
  if (fread(&count, 8, 1, f) != 1) goto bad;
  if (expect && count != expect) {
    snprintf(g_err, sizeof g_err, "%s has invalid size", name);
    return NULL;
  }
  float *v = (float *)malloc(count * sizeof(float));
  if (fread(v, 4, count, f) != count) {
    free(v);
    goto bad;
  }
  return v;
bad:
  snprintf(g_err, sizeof g_err, "failed to read %s", name);
  return NULL;
}

static float *concat2(float *a, size_t na, float *b, size_t nb) {
  float *r = (float *)malloc((na + nb) * sizeof(float));
  memcpy(r, a, na * sizeof(float));
  memcpy(r + na, b, nb * sizeof(float));
  free(a);
  free(b);
  return r;
}

static int64_t kv_get(const char *text, const char *key, int64_t fallback) {
  size_t kl = strlen(key);
  const char *p = text;
  while (p && *p) {
    while (*p == ' ' || *p == '\t') ++p;
    if (strncmp(p, key, kl) == 0) {
      const char *q = p + kl;
      while (*q == ' ' || *q == '\t') ++q;
      if (*q == '=') return strtoll(q + 1, NULL, 10);
    }
    p = strchr(p, '\n');
    if (p) ++p;
  }
  return fallback;
}

/* runtime_loader.cpp:71-88 (same keys and defaults) + runtime_loader.cpp:121-167
 * (MMRTW001 tensor order). eps/theta are explicit: the reference loader reads
 * neither and leaves the config.h defaults (1e-6, 1e6). */
MMO_API mmo_model *mmo_load(const char *dir, float eps, float theta) {
  char path[4096];
  snprintf(path, sizeof path, "%s/minimind_runtime_config.txt", dir);
  FILE *f = fopen(path, "rb");
  if (!f) {
    snprintf(g_err, sizeof g_err, "failed to open runtime config");
    return NULL;
  }
  char text[8192];
  size_t nt = fread(text, 1, sizeof(text) - 1, f);
  text[nt] = 0;
  fclose(f);
  mmo_model *m = (mmo_model *)calloc(1, sizeof(mmo_model));
  mmo_config *c = &m->c;
  c->hidden = kv_get(text, "hidden_size", 768);
  c->layers = kv_get(text, "num_hidden_layers", 8);
  c->vocab = kv_get(text, "vocab_size", 6400);
  c->nq = kv_get(text, "num_attention_heads", 8);
  c->nkv = kv_get(text, "num_key_value_heads", 4);
  c->hd = kv_get(text, "head_dim", c->hidden / c->nq);
  c->inter = kv_get(text, "intermediate_size", 2432);
  c->max_pos = kv_get(text, "max_position_embeddings", 32768);
  c->eps = eps > 0.0f ? eps : 1e-6f;
  c->theta = theta > 0.0f ? theta : 1000000.0f;
  c->use_moe = kv_get(text, "use_moe", 0);
  c->experts = kv_get(text, "num_experts", 4);
  c->moe_inter = kv_get(text, "moe_intermediate_size", c->inter);
  snprintf(path, sizeof path, "%s/weights.bin", dir);
  f = fopen(path, "rb");
  if (!f) {
    snprintf(g_err, sizeof g_err, "failed to open runtime weights");
    free(m);
    return NULL;
  }
  char magic[8];
  if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "MMRTW001", 8) != 0) {
    snprintf(g_err, sizeof g_err, "unsupported runtime weight format");
    fclose(f);
    free(m);
    return NULL;
  }
  const int64_t H = c->hidden, Q = c->nq * c->hd, KV = c->nkv * c->hd, I = c->inter;
  int ok = 1;
  ok &= (m->embed = read_tensor(f, "model.embed_tokens.weight", (uint64_t)(c->vocab * H))) != NULL;
  ok &= ok && (m->final_norm = read_tensor(f, "model.norm.weight", (uint64_t)H)) != NULL;
  ok &= ok && (m->lm_head = read_tensor(f, "lm_head.weight", (uint64_t)(c->vocab * H))) != NULL;
  m->layer = (mmo_layer *)calloc((size_t)c->layers, sizeof(mmo_layer));
  for (int64_t l = 0; ok && l < c->layers; ++l) {
    char p[128], n[256];
    snprintf(p, sizeof p, "model.layers.%lld.", (long long)l);
    mmo_layer *L = &m->layer[l];
#define RD(dst, suffix, cnt) \
  snprintf(n, sizeof n, "%s%s", p, suffix); \
  ok &= ok && ((dst) = read_tensor(f, n, (uint64_t)(cnt))) != NULL;
    float *qp = NULL, *kp = NULL, *vp = NULL, *gp = NULL, *up = NULL;
    RD(L->input_norm, "input_layernorm.weight", H);
    RD(L->post_norm, "post_attention_layernorm.weight", H);
    RD(L->q_norm, "self_attn.q_norm.weight", c->hd);
    RD(L->k_norm, "self_attn.k_norm.weight", c->hd);
    RD(qp, "self_attn.q_proj.weight", Q * H);
    RD(kp, "self_attn.k_proj.weight", KV * H);
    RD(vp, "self_attn.v_proj.weight", KV * H);
    RD(L->o, "self_attn.o_proj.weight", H * Q);
    if (c->use_moe) { /* runtime_loader.cpp:148-158; experts fused as language_model.cpp:110-116 */
      const int64_t MI = c->moe_inter;
      RD(L->moe_gate, "mlp.gate.weight", c->experts * H);
      L->exp_gate_up = (float **)calloc((size_t)c->experts, sizeof(float *));
      L->exp_down = (float **)calloc((size_t)c->experts, sizeof(float *));
      for (int64_t e = 0; ok && e < c->experts; ++e) {
        char ep[64];
        float *eg = NULL, *eu = NULL;
        snprintf(ep, sizeof ep, "mlp.experts.%lld.gate_proj.weight", (long long)e);
        RD(eg, ep, MI * H);
        snprintf(ep, sizeof ep, "mlp.experts.%lld.up_proj.weight", (long long)e);
        RD(eu, ep, MI * H);
        snprintf(ep, sizeof ep, "mlp.experts.%lld.down_proj.weight", (long long)e);
        RD(L->exp_down[e], ep, H * MI);
        if (ok) L->exp_gate_up[e] = concat2(eg, (size_t)(MI * H), eu, (size_t)(MI * H));
      }
    } else {
      RD(gp, "mlp.gate_proj.weight", I * H);
      RD(up, "mlp.up_proj.weight", I * H);
      RD(L->down, "mlp.down_proj.weight", H * I);
    }
#undef RD
    if (ok) {
      L->qkv = concat2(concat2(qp, (size_t)(Q * H), kp, (size_t)(KV * H)), (size_t)((Q + KV) * H), vp,
                       (size_t)(KV * H));
      if (!c->use_moe) L->gate_up = concat2(gp, (size_t)(I * H), up, (size_t)(I * H));
    }
  }
  fclose(f);
  if (!ok) return NULL; /* error text already set; small leak on a failed load is acceptable for a test oracle */
  const int64_t half = c->hd / 2;
  m->rope_cos = (float *)malloc((size_t)(c->max_pos * half) * sizeof(float));
  m->rope_sin = (float *)malloc((size_t)(c->max_pos * half) * sizeof(float));
  mmo_rope_tables(c->max_pos, c->hd, c->theta, m->rope_cos, m->rope_sin);
  return m;
}

MMO_API void mmo_free(mmo_model *m) {
  if (!m) return;
  for (int64_t l = 0; l < m->c.layers; ++l) {
    mmo_layer *L = &m->layer[l];
    free(L->input_norm); free(L->post_norm); free(L->q_norm); free(L->k_norm);
    free(L->qkv); free(L->o); free(L->gate_up); free(L->down); free(L->moe_gate);
    for (int64_t e = 0; L->exp_gate_up && e < m->c.experts; ++e) {
      free(L->exp_gate_up[e]);
      free(L->exp_down[e]);
    }
    free(L->exp_gate_up); free(L->exp_down);
  }
  free(m->layer); free(m->embed); free(m->final_norm); free(m->lm_head);
  free(m->rope_cos); free(m->rope_sin);
  free(m);
}

MMO_API void mmo_config_of(const mmo_model *m, mmo_config *out) { *out = m->c; }

MMO_API mmo_state *mmo_state_new(const mmo_model *m) {
  mmo_state *s = (mmo_state *)calloc(1, sizeof(mmo_state));
  s->cache = (mmo_cache *)calloc((size_t)m->c.layers, sizeof(mmo_cache));
  return s;
}

MMO_API void mmo_state_free(const mmo_model *m, mmo_state *s) {
  if (!s) return;
  for (int64_t l = 0; l < m->c.layers; ++l) {
    free(s->cache[l].keys);
    free(s->cache[l].values);
  }
  free(s->cache);
  free(s);
}

MMO_API int64_t mmo_position(const mmo_state *s) { return s->position; }

static void cache_append(mmo_cache *c, const float *k, const float *v, int64_t row) {
  if (c->tokens == c->cap) {
    c->cap = c->cap ? c->cap * 2 : 64;
    c->keys = (float *)realloc(c->keys, (size_t)(c->cap * row) * sizeof(float));
    c->values = (float *)realloc(c->values, (size_t)(c->cap * row) * sizeof(float));
  }
  memcpy(c->keys + c->tokens * row, k, (size_t)row * sizeof(float));
  memcpy(c->values + c->tokens * row, v, (size_t)row * sizeof(float));
  c->tokens += 1;
}

/* decoder_layer.cpp:312-407 run_dense_decoder_layer (dense, fused weights). */
static void decoder_layer(const mmo_model *m, const mmo_layer *L, mmo_cache *cache, float *hidden, int64_t pos) {
  const mmo_config *c = &m->c;
  const int64_t H = c->hidden, Q = c->nq * c->hd, KV = c->nkv * c->hd;
  const int64_t I = c->use_moe ? (c->moe_inter > c->inter ? c->moe_inter : c->inter) : c->inter;
  float *normed = (float *)malloc((size_t)H * sizeof(float));
  float *qkv = (float *)malloc((size_t)(Q + 2 * KV) * sizeof(float));
  float *ctx = (float *)malloc((size_t)Q * sizeof(float));
  float *attn = (float *)malloc((size_t)H * sizeof(float));
  float *gu = (float *)malloc((size_t)(2 * I) * sizeof(float));
  float *act = (float *)malloc((size_t)I * sizeof(float));
  float *mlp = (float *)malloc((size_t)H * sizeof(float));

  memcpy(normed, hidden, (size_t)H * sizeof(float));
  mmo_rms_norm_inplace(normed, L->input_norm, H, c->eps);                     /* :327 */
  mmo_matvec(L->qkv, Q + 2 * KV, H, normed, qkv);                             /* :331-335 */
  float *q = qkv, *k = qkv + Q, *v = qkv + Q + KV;
  for (int64_t h = 0; h < c->nq; ++h) mmo_rms_norm_inplace(q + h * c->hd, L->q_norm, c->hd, c->eps);  /* :342-344 */
  for (int64_t h = 0; h < c->nkv; ++h) mmo_rms_norm_inplace(k + h * c->hd, L->k_norm, c->hd, c->eps); /* :345-347 */
  mmo_apply_rope(q, c->nq, c->hd, pos, m->rope_cos, m->rope_sin);             /* :349-350 */
  mmo_apply_rope(k, c->nkv, c->hd, pos, m->rope_cos, m->rope_sin);            /* :351-352 */
  cache_append(cache, k, v, KV);                                              /* :354-359 */
  mmo_attention(q, cache->keys, cache->values, cache->tokens, c->nq, c->nkv, c->hd, ctx); /* :361 */
  mmo_matvec(L->o, H, Q, ctx, attn);                                          /* :362 */
  for (int64_t i = 0; i < H; ++i) hidden[i] = hidden[i] + attn[i];           /* :364-367 */
  memcpy(normed, hidden, (size_t)H * sizeof(float));
  mmo_rms_norm_inplace(normed, L->post_norm, H, c->eps);                      /* :369 */
  if (c->use_moe) { /* :370-389: router argmax (first max), the chosen expert's MLP, no gate weighting */
    float *router = (float *)malloc((size_t)c->experts * sizeof(float));
    mmo_matvec(L->moe_gate, c->experts, H, normed, router);
    const int64_t e = mmo_argmax(router, c->experts);
    float second = -INFINITY;
    for (int64_t k = 0; k < c->experts; ++k)
      if (k != e && router[k] > second) second = router[k];
    const float margin = (router[e] - second) / (fabsf(router[e]) + 1e-12f);
    if (margin < g_router_margin) g_router_margin = margin;
    free(router);
    const int64_t MI = c->moe_inter;
    mmo_matvec(L->exp_gate_up[e], 2 * MI, H, normed, gu);
    mmo_swiglu(gu, MI, act);
    mmo_matvec(L->exp_down[e], H, MI, act, mlp);
  } else {
    mmo_matvec(L->gate_up, 2 * I, H, normed, gu);                             /* :392-393 */
    mmo_swiglu(gu, I, act);                                                   /* :394 */
    mmo_matvec(L->down, H, I, act, mlp);                                      /* :400 */
  }
  for (int64_t i = 0; i < H; ++i) hidden[i] += mlp[i];                        /* :403-405 */
  free(normed); free(qkv); free(ctx); free(attn); free(gu); free(act); free(mlp);
}

/* language_model.cpp:297-308 forward_token: returns fp32 logits; the return
 * value is argmax_token(logits) as forward_next_token would give it
 * (language_model.cpp:317-332). Returns -1 for an out-of-vocabulary token
 * (embedding_row throws std::out_of_range, language_model.cpp:67-77). */
MMO_API int32_t mmo_forward_token(const mmo_model *m, mmo_state *s, int32_t token, float *logits_out) {
  const mmo_config *c = &m->c;
  if (token < 0 || token >= c->vocab) {
    snprintf(g_err, sizeof g_err, "token id out of vocabulary range");
    return -1;
  }
  float *hidden = (float *)malloc((size_t)c->hidden * sizeof(float));
  g_router_margin = INFINITY;
  memcpy(hidden, m->embed + (int64_t)token * c->hidden, (size_t)c->hidden * sizeof(float));
  for (int64_t l = 0; l < c->layers; ++l) decoder_layer(m, &m->layer[l], &s->cache[l], hidden, s->position);
  s->position += 1;
  float *normed = (float *)malloc((size_t)c->hidden * sizeof(float));
  mmo_rms_norm_final(hidden, m->final_norm, c->hidden, c->eps, normed);
  float *logits = logits_out ? logits_out : (float *)malloc((size_t)c->vocab * sizeof(float));
  mmo_matvec(m->lm_head, c->vocab, c->hidden, normed, logits);
  const int32_t next = mmo_argmax(logits, c->vocab);
  if (!logits_out) free(logits);
  free(hidden);
  free(normed);
  return next;
}

/* language_model.cpp:368-396 generate_stream on the CPU branch (prompt fed
 * token by token, greedy, stop on eos). Returns the number of tokens written. */
MMO_API int64_t mmo_generate(const mmo_model *m, const int32_t *prompt, int64_t n_prompt, int64_t max_new,
                             int32_t eos, int32_t *out) {
  if (n_prompt <= 0 || max_new < 0) return -1;
  mmo_state *s = mmo_state_new(m);
  int32_t next = 0;
  for (int64_t i = 0; i < n_prompt; ++i) {
    next = mmo_forward_token(m, s, prompt[i], NULL);
    if (next < 0) {
      mmo_state_free(m, s);
      return -1;
    }
  }
  int64_t n = 0;
  for (int64_t i = 0; i < max_new; ++i) {
    out[n++] = next;
    if (next == eos || i + 1 == max_new) break;
    next = mmo_forward_token(m, s, next, NULL);
  }
  mmo_state_free(m, s);
  return n;
}
