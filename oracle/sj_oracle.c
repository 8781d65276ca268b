/*
 * sj_oracle.c — CPU restatement of snapjudge's fp32 encoder forward.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the B200
 * kernels: only the tests, the smoke check and the benchmark's CPU-baseline
 * leg load it.  The product library never links or calls it.
 *
 * Every function restates the reference algorithm at the cited location
 * (paths relative to the snapjudge source tree):
 *
 *   orc_layer_norm   src/tensor.cpp:54-79    fp64 mean / population variance,
 *                                            inv = float(1/sqrt(var+eps))
 *   orc_gemm_nt      src/tensor.cpp:101-131  C = A W^T (+bias, act 0/1/2) via
 *                                            cblas_sgemm (OpenBLAS 0.3.15, the
 *                                            reference's BLAS, when loaded with
 *                                            orc_set_blas) or the plain dot-product
 *                                            loop of src/cblas_fallback.cpp:22-47
 *   orc_gelu_erf     src/tensor.cpp:96-98
 *   orc_geglu        src/tensor.cpp:133-151  gelu(z[:, :F]) * z[:, F:]
 *   orc_rope_table   src/model.cpp:173-190   fp64 angles, cast to float
 *   orc_rope         src/tensor.cpp:257-279  rotate-half, position = r % L
 *   orc_attention    src/tensor.cpp:156-228  keys [max(0,i-w), min(len,i+w+1)),
 *                                            fp64 row sum, threads over (b, h)
 *   orc_encode       src/model.cpp:222-307   emb -> LN -> layers -> final LN
 *                                            (+ optional LoRA)
 *   orc_forward_head src/model.cpp:409-535   type_emb, head layers, scorer,
 *                                            act head
 *
 * Parity is pinned in tests against the reference's own golden vectors
 * (tests/golden/tensor_ops.json of the reference) and against the reference
 * sources compiled unchanged into oracle/_ref (see oracle/Makefile).
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef void (*sgemm_fn)(int, int, int, int, int, int, float, const float*, int,
                         const float*, int, float, float*, int);
static sgemm_fn g_sgemm = NULL;

/* Load cblas_sgemm from a shared BLAS (the reference links OpenBLAS). 0 = ok. */
int orc_set_blas(const char* path) {
  void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h) return -1;
  g_sgemm = (sgemm_fn)dlsym(h, "cblas_sgemm");
  return g_sgemm ? 0 : -2;
}
int orc_has_blas(void) { return g_sgemm != NULL; }

static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n; }
static int n_threads(void) {
  if (g_threads > 0) return g_threads;
  const char* e = getenv("SNAPJUDGE_THREADS");
  if (e && *e && atoi(e) > 0) return atoi(e);
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

/* ---- elementwise ------------------------------------------------------- */
float orc_gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654757f)); }

void orc_layer_norm(const float* x, int64_t rows, int64_t D, const float* w, const float* b,
                    float eps, float* out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * D;
    float* o = out + r * D;
    double mean = 0;
    for (int64_t j = 0; j < D; ++j) mean += xr[j];
    mean /= (double)D;
    double var = 0;
    for (int64_t j = 0; j < D; ++j) {
      double d = xr[j] - mean;
      var += d * d;
    }
    var /= (double)D;
    float inv = (float)(1.0 / sqrt(var + eps));
    float meanf = (float)mean;
    for (int64_t j = 0; j < D; ++j) {
      float v = (xr[j] - meanf) * inv * (w ? w[j] : 1.0f);
      o[j] = b ? v + b[j] : v;
    }
  }
}

/* ---- GEMM ----------------------------------------------------------------- */
typedef struct {
  const float *A, *W;
  float* C;
  int64_t M, N, K, r0, r1;
} gemm_job;

static void* gemm_rows(void* p) {
  gemm_job* j = (gemm_job*)p;
  for (int64_t i = j->r0; i < j->r1; ++i)
    for (int64_t n = 0; n < j->N; ++n) {
      const float* a = j->A + i * j->K;
      const float* w = j->W + n * j->K;
      float acc = 0.0f;
      for (int64_t k = 0; k < j->K; ++k) acc += a[k] * w[k];
      j->C[i * j->N + n] = acc;
    }
  return NULL;
}

static void sgemm_nt(const float* A, const float* W, float* C, int64_t M, int64_t N,
                     int64_t K) {
  if (g_sgemm) {
    g_sgemm(101, 111, 112, (int)M, (int)N, (int)K, 1.0f, A, (int)K, W, (int)K, 0.0f, C,
            (int)N);
    return;
  }
  int nt = n_threads();
  if (nt > M) nt = (int)(M > 0 ? M : 1);
  pthread_t th[256];
  gemm_job jobs[256];
  if (nt > 256) nt = 256;
  for (int t = 0; t < nt; ++t) {
    jobs[t] = (gemm_job){A, W, C, M, N, K, M * t / nt, M * (t + 1) / nt};
    pthread_create(&th[t], NULL, gemm_rows, &jobs[t]);
  }
  for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
}

void orc_gemm_nt(const float* A, int64_t M, int64_t K, const float* W, int64_t N,
                 const float* bias, int act, float* out) {
  sgemm_nt(A, W, out, M, N, K);
  if (bias || act) {
    for (int64_t r = 0; r < M; ++r)
      for (int64_t j = 0; j < N; ++j) {
        float v = out[r * N + j];
        if (bias) v += bias[j];
        if (act == 1) v = orc_gelu_erf(v);
        else if (act == 2) v = v > 0.0f ? v : 0.0f;
        out[r * N + j] = v;
      }
  }
}

void orc_geglu(const float* A, int64_t M, int64_t K, const float* Wi, int64_t F, float* out) {
  float* tmp = (float*)malloc(sizeof(float) * (size_t)(M * 2 * F));
  sgemm_nt(A, Wi, tmp, M, 2 * F, K);
  for (int64_t r = 0; r < M; ++r)
    for (int64_t j = 0; j < F; ++j)
      out[r * F + j] = orc_gelu_erf(tmp[r * 2 * F + j]) * tmp[r * 2 * F + F + j];
  free(tmp);
}

/* ---- RoPE ---------------------------------------------------------------- */
void orc_rope_table(double theta, int Dh, int64_t L, float* cos_t, float* sin_t) {
  int64_t half = Dh / 2;
  for (int64_t pos = 0; pos < L; ++pos)
    for (int64_t d = 0; d < half; ++d) {
      double inv = 1.0 / pow(theta, 2.0 * (double)d / Dh);
      double fr = (double)pos * inv;
      cos_t[pos * half + d] = (float)cos(fr);
      sin_t[pos * half + d] = (float)sin(fr);
    }
}

void orc_rope(float* qkv, int64_t M, const float* cos_t, const float* sin_t, int64_t L,
              int64_t H, int64_t Dh) {
  int64_t half = Dh / 2;
  for (int64_t r = 0; r < M; ++r) {
    int64_t pos = r % L;
    const float* cr = cos_t + pos * half;
    const float* sr = sin_t + pos * half;
    float* row = qkv + r * 3 * H * Dh;
    for (int64_t hh = 0; hh < 2 * H; ++hh) {
      float* qk = row + hh * Dh;
      for (int64_t d = 0; d < half; ++d) {
        float x0 = qk[d], x1 = qk[d + half];
        float cs = cr[d], sn = sr[d];
        qk[d] = x0 * cs - x1 * sn;
        qk[d + half] = x1 * cs + x0 * sn;
      }
    }
  }
}

/* ---- attention ------------------------------------------------------------ */
typedef struct {
  const float *q, *k, *v;
  float* out;
  const int64_t* lens;
  int64_t B, H, L, Dh;
  int window;
  int64_t next;
  pthread_mutex_t mu;
} attn_ctx;

static void* attn_worker(void* p) {
  attn_ctx* c = (attn_ctx*)p;
  const float scale = 1.0f / sqrtf((float)c->Dh);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(c->L > 0 ? c->L : 1));
  for (;;) {
    pthread_mutex_lock(&c->mu);
    int64_t idx = c->next++;
    pthread_mutex_unlock(&c->mu);
    if (idx >= c->B * c->H) break;
    int64_t b = idx / c->H, h = idx % c->H;
    int64_t len = c->lens ? c->lens[b] : c->L;
    const float* qb = c->q + ((b * c->H + h) * c->L) * c->Dh;
    const float* kb = c->k + ((b * c->H + h) * c->L) * c->Dh;
    const float* vb = c->v + ((b * c->H + h) * c->L) * c->Dh;
    float* ob = c->out + ((b * c->H + h) * c->L) * c->Dh;
    for (int64_t i = 0; i < c->L; ++i) {
      const float* qi = qb + i * c->Dh;
      int64_t lo = 0, hi = len;
      if (c->window > 0) {
        lo = i - c->window > 0 ? i - c->window : 0;
        hi = i + c->window + 1 < len ? i + c->window + 1 : len;
      }
      float m = -INFINITY;
      for (int64_t j = lo; j < hi; ++j) {
        const float* kj = kb + j * c->Dh;
        float s = 0;
        for (int64_t d = 0; d < c->Dh; ++d) s += qi[d] * kj[d];
        scores[j] = s * scale;
        if (scores[j] > m) m = scores[j];
      }
      double l = 0;
      for (int64_t j = lo; j < hi; ++j) {
        float e = expf(scores[j] - m);
        scores[j] = e;
        l += e;
      }
      float linv = (float)(1.0 / l);
      float* oi = ob + i * c->Dh;
      for (int64_t d = 0; d < c->Dh; ++d) oi[d] = 0.0f;
      for (int64_t j = lo; j < hi; ++j) {
        float w = scores[j] * linv;
        const float* vj = vb + j * c->Dh;
        for (int64_t d = 0; d < c->Dh; ++d) oi[d] += w * vj[d];
      }
    }
  }
  free(scores);
  return NULL;
}

/* q/k/v/out: [B, H, L, Dh]; lens [B] (NULL = all L). */
void orc_attention(const float* q, const float* k, const float* v, int64_t B, int64_t H,
                   int64_t L, int64_t Dh, const int64_t* lens, int window, float* out) {
  attn_ctx c;
  c.q = q; c.k = k; c.v = v; c.out = out; c.lens = lens;
  c.B = B; c.H = H; c.L = L; c.Dh = Dh; c.window = window; c.next = 0;
  pthread_mutex_init(&c.mu, NULL);
  int nt = n_threads();
  if (nt > B * H) nt = (int)(B * H);
  if (nt < 1) nt = 1;
  if (nt > 256) nt = 256;
  pthread_t th[256];
  for (int t = 0; t < nt; ++t) pthread_create(&th[t], NULL, attn_worker, &c);
  for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
  pthread_mutex_destroy(&c.mu);
}

/* ---- encoder ---------------------------------------------------------------- */
typedef struct {
  const float* attn_norm; /* NULL on layer 0 (identity) */
  const float* wqkv;      /* [3D, D] */
  const float* wo;        /* [D, D] */
  const float* mlp_norm;  /* [D] */
  const float* wi;        /* [2F, D] */
  const float* wo2;       /* [D, F] */
  int window;             /* 0 = full attention */
  int sliding;            /* selects the sliding RoPE table */
} orc_layer;

typedef struct {
  int D, H, F, V, n_layers;
  int64_t max_pos;
  float eps;
  const float* emb;        /* [V, D] */
  const float* emb_norm;   /* [D] */
  const float* final_norm; /* [D] */
  const orc_layer* layers;
  const float *cos_full, *sin_full, *cos_slide, *sin_slide; /* [max_pos, Dh/2] */
  int lora_r;
  const float* lora_a; /* [r, D] */
  const float* lora_b; /* [D, r] */
} orc_model;

static void add_(float* a, const float* b, int64_t n) {
  for (int64_t i = 0; i < n; ++i) a[i] += b[i];
}

/* Padded batch: ids/mask [B, L] int64 (right padding).  out [B, L, D]. */
int orc_encode(const orc_model* m, const int64_t* ids, const int64_t* mask, int64_t B,
               int64_t L, float* out) {
  const int64_t D = m->D, H = m->H, Dh = D / H, F = m->F, M = B * L;
  if (B == 0) return 0;
  if (L > m->max_pos) return -1;
  int64_t* lens = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
  for (int64_t b = 0; b < B; ++b) {
    int64_t s = 0;
    for (int64_t i = 0; i < L; ++i) s += mask[b * L + i];
    lens[b] = s;
  }
  float* X = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* Y = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* E = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* qkv = (float*)malloc(sizeof(float) * (size_t)(M * 3 * D));
  float* Q = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* K = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* V = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* At = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* G = (float*)malloc(sizeof(float) * (size_t)(M * F));
  for (int64_t r = 0; r < M; ++r) {
    int64_t id = ids[r];
    if (id < 0 || id >= m->V) { /* out of vocabulary: the reference reads out of bounds */
      free(lens); free(X); free(Y); free(E); free(qkv); free(Q); free(K); free(V);
      free(At); free(G);
      return -2;
    }
    memcpy(E + r * D, m->emb + id * D, sizeof(float) * (size_t)D);
  }
  orc_layer_norm(E, M, D, m->emb_norm, NULL, m->eps, X);
  for (int li = 0; li < m->n_layers; ++li) {
    const orc_layer* ly = &m->layers[li];
    const float* Yin = X;
    if (ly->attn_norm) {
      orc_layer_norm(X, M, D, ly->attn_norm, NULL, m->eps, Y);
      Yin = Y;
    }
    orc_gemm_nt(Yin, M, D, ly->wqkv, 3 * D, NULL, 0, qkv);
    orc_rope(qkv, M, ly->sliding ? m->cos_slide : m->cos_full,
             ly->sliding ? m->sin_slide : m->sin_full, L, H, Dh);
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i) {
        const float* row = qkv + (b * L + i) * 3 * D;
        for (int64_t h = 0; h < H; ++h) {
          memcpy(Q + ((b * H + h) * L + i) * Dh, row + h * Dh, sizeof(float) * (size_t)Dh);
          memcpy(K + ((b * H + h) * L + i) * Dh, row + D + h * Dh, sizeof(float) * (size_t)Dh);
          memcpy(V + ((b * H + h) * L + i) * Dh, row + 2 * D + h * Dh,
                 sizeof(float) * (size_t)Dh);
        }
      }
    orc_attention(Q, K, V, B, H, L, Dh, lens, ly->window, At);
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i)
        for (int64_t h = 0; h < H; ++h)
          memcpy(Q + (b * L + i) * D + h * Dh, At + ((b * H + h) * L + i) * Dh,
                 sizeof(float) * (size_t)Dh);
    orc_gemm_nt(Q, M, D, ly->wo, D, NULL, 0, Y);
    add_(X, Y, M * D);
    orc_layer_norm(X, M, D, ly->mlp_norm, NULL, m->eps, Y);
    orc_geglu(Y, M, D, ly->wi, F, G);
    orc_gemm_nt(G, M, F, ly->wo2, D, NULL, 0, Y);
    add_(X, Y, M * D);
  }
  orc_layer_norm(X, M, D, m->final_norm, NULL, m->eps, out);
  if (m->lora_r > 0) {
    float* z = (float*)malloc(sizeof(float) * (size_t)(M * m->lora_r));
    orc_gemm_nt(out, M, D, m->lora_a, m->lora_r, NULL, 0, z);
    orc_gemm_nt(z, M, m->lora_r, m->lora_b, D, NULL, 0, Y);
    add_(out, Y, M * D);
    free(z);
  }
  free(lens); free(X); free(Y); free(E); free(qkv); free(Q); free(K); free(V); free(At);
  free(G);
  return 0;
}

/* ---- decision head (after the encoder) ------------------------------------- */
typedef struct {
  const float *n1w, *n1b, *n2w, *n2b;
  const float *in_w, *in_b, *out_w, *out_b; /* in_w [3D, D] */
  const float *l1w, *l1b, *l2w, *l2b;       /* l1w [4D, D] */
} orc_head_layer;

typedef struct {
  const float* type_emb; /* [3, D] */
  int n_head_layers;
  const orc_head_layer* head;
  const float *sc_ln_w, *sc_ln_b, *sc_w1, *sc_b1, *sc_w2, *sc_b2; /* b's nullable */
  const float *act_w1, *act_b1, *act_w2, *act_b2;                 /* [256, D+4], [n_act,256] */
  int n_act;
} orc_head;

/* h [B, L, D] = encoder output (modified in place: becomes the head stream).
 * marker_pos [B, K], marker_mask [B, K] (uint8), qtype [B].
 * logits [B, K], act [B, n_act]. */
int orc_forward_head(const orc_model* m, const orc_head* hd, float* h, const int64_t* mask,
                     int64_t B, int64_t L, const int64_t* marker_pos,
                     const uint8_t* marker_mask, int64_t Kmk, const int64_t* qtype,
                     float* logits, float* act) {
  const int64_t D = m->D, H = m->H, Dh = D / H, M = B * L;
  int64_t* lens = (int64_t*)malloc(sizeof(int64_t) * (size_t)B);
  for (int64_t b = 0; b < B; ++b) {
    int64_t s = 0;
    for (int64_t i = 0; i < L; ++i) s += mask[b * L + i];
    lens[b] = s;
  }
  for (int64_t b = 0; b < B; ++b) {
    const float* te = hd->type_emb + qtype[b] * D;
    for (int64_t i = 0; i < L; ++i)
      for (int64_t j = 0; j < D; ++j) h[(b * L + i) * D + j] += te[j];
  }
  float* ln = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* qkv = (float*)malloc(sizeof(float) * (size_t)(M * 3 * D));
  float* Q = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* K = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* V = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* At = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* P = (float*)malloc(sizeof(float) * (size_t)(M * D));
  float* F1 = (float*)malloc(sizeof(float) * (size_t)(M * 4 * D));
  for (int li = 0; li < hd->n_head_layers; ++li) {
    const orc_head_layer* hl = &hd->head[li];
    orc_layer_norm(h, M, D, hl->n1w, hl->n1b, 1e-5f, ln);
    orc_gemm_nt(ln, M, D, hl->in_w, 3 * D, hl->in_b, 0, qkv);
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i) {
        const float* row = qkv + (b * L + i) * 3 * D;
        for (int64_t hh = 0; hh < H; ++hh) {
          memcpy(Q + ((b * H + hh) * L + i) * Dh, row + hh * Dh, sizeof(float) * (size_t)Dh);
          memcpy(K + ((b * H + hh) * L + i) * Dh, row + D + hh * Dh,
                 sizeof(float) * (size_t)Dh);
          memcpy(V + ((b * H + hh) * L + i) * Dh, row + 2 * D + hh * Dh,
                 sizeof(float) * (size_t)Dh);
        }
      }
    orc_attention(Q, K, V, B, H, L, Dh, lens, 0, At);
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i)
        for (int64_t hh = 0; hh < H; ++hh)
          memcpy(Q + (b * L + i) * D + hh * Dh, At + ((b * H + hh) * L + i) * Dh,
                 sizeof(float) * (size_t)Dh);
    orc_gemm_nt(Q, M, D, hl->out_w, D, hl->out_b, 0, P);
    add_(h, P, M * D);
    orc_layer_norm(h, M, D, hl->n2w, hl->n2b, 1e-5f, ln);
    orc_gemm_nt(ln, M, D, hl->l1w, 4 * D, hl->l1b, 2, F1);
    orc_gemm_nt(F1, M, 4 * D, hl->l2w, D, hl->l2b, 0, P);
    add_(h, P, M * D);
  }
  /* scorer */
  float* mk = (float*)malloc(sizeof(float) * (size_t)(B * Kmk * D));
  float* s1 = (float*)malloc(sizeof(float) * (size_t)(B * Kmk * D));
  float* s2 = (float*)malloc(sizeof(float) * (size_t)(B * Kmk * D));
  float* s3 = (float*)malloc(sizeof(float) * (size_t)(B * Kmk + 1));
  for (int64_t b = 0; b < B; ++b)
    for (int64_t kk = 0; kk < Kmk; ++kk) {
      int64_t p = marker_pos[b * Kmk + kk];
      if (p < 0) p = 0;
      if (p >= L) p = L - 1;
      memcpy(mk + (b * Kmk + kk) * D, h + (b * L + p) * D, sizeof(float) * (size_t)D);
    }
  orc_layer_norm(mk, B * Kmk, D, hd->sc_ln_w, hd->sc_ln_b, m->eps, s1);
  orc_gemm_nt(s1, B * Kmk, D, hd->sc_w1, D, hd->sc_b1, 1, s2);
  orc_gemm_nt(s2, B * Kmk, D, hd->sc_w2, 1, hd->sc_b2, 0, s3);
  for (int64_t b = 0; b < B; ++b)
    for (int64_t kk = 0; kk < Kmk; ++kk) {
      float lg = s3[b * Kmk + kk];
      if (!marker_mask[b * Kmk + kk]) lg = -1e4f;
      logits[b * Kmk + kk] = lg;
    }
  /* act head */
  float* feats = (float*)malloc(sizeof(float) * (size_t)(D + 4));
  float* a1 = (float*)malloc(sizeof(float) * 256);
  float* a2 = (float*)malloc(sizeof(float) * (size_t)hd->n_act);
  double* p = (double*)malloc(sizeof(double) * (size_t)(Kmk > 0 ? Kmk : 1));
  for (int64_t b = 0; b < B; ++b) {
    const float* lg = logits + b * Kmk;
    float mx = lg[0];
    for (int64_t j = 1; j < Kmk; ++j) mx = lg[j] > mx ? lg[j] : mx;
    double s = 0;
    for (int64_t j = 0; j < Kmk; ++j) { p[j] = exp((double)(lg[j] - mx)); s += p[j]; }
    for (int64_t j = 0; j < Kmk; ++j) p[j] /= s;
    double top1 = 0, top2 = 0;
    for (int64_t j = 0; j < Kmk; ++j) {
      if (p[j] > top1) { top2 = top1; top1 = p[j]; }
      else if (p[j] > top2) top2 = p[j];
    }
    double ksum = 0;
    for (int64_t kk = 0; kk < Kmk; ++kk) ksum += marker_mask[b * Kmk + kk];
    double kf = ksum > 2.0 ? ksum : 2.0;
    double ent = 0;
    for (int64_t j = 0; j < Kmk; ++j) ent -= p[j] * log(p[j] > 1e-9 ? p[j] : 1e-9);
    ent /= log(kf);
    memcpy(feats, h + (b * L) * D, sizeof(float) * (size_t)D);
    feats[D + 0] = (float)top1;
    feats[D + 1] = (float)(top1 - top2);
    feats[D + 2] = (float)ent;
    feats[D + 3] = (float)(kf / 255.0);
    orc_gemm_nt(feats, 1, D + 4, hd->act_w1, 256, hd->act_b1, 1, a1);
    orc_gemm_nt(a1, 1, 256, hd->act_w2, hd->n_act, hd->act_b2, 0, a2);
    float amx = a2[0];
    for (int j = 1; j < hd->n_act; ++j) amx = a2[j] > amx ? a2[j] : amx;
    double as = 0;
    for (int j = 0; j < hd->n_act; ++j) { a2[j] = expf(a2[j] - amx); as += a2[j]; }
    for (int j = 0; j < hd->n_act; ++j) act[b * hd->n_act + j] = (float)(a2[j] / as);
  }
  free(lens); free(ln); free(qkv); free(Q); free(K); free(V); free(At); free(P); free(F1);
  free(mk); free(s1); free(s2); free(s3); free(feats); free(a1); free(a2); free(p);
  return 0;
}
