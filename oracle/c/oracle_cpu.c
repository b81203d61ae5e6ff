/*
 * CPU restatement of the decode-path arithmetic, multithreaded with pthreads.
 * TEST INFRASTRUCTURE / CPU BASELINE ONLY: used by tests/ (checked against the
 * NumPy oracle) and by bench.py's CPU-baseline and --impl reference legs. The
 * product path never links or calls it.
 *
 * Each function restates the reference arithmetic it names:
 *   oc_affine_linear   mx.quantized_matmul(..., mode="affine") as called at
 *                      spark_mlx_llm/ops/linear.py:180-191, evaluated per group as
 *                      scale*sum(q*x) + bias*sum(x) in fp32 like
 *                      spark_mlx_ext/_w4a16_sources.py:24-39
 *   oc_w8a16           src/kernels/w8a16_matvec.metal:40-94 (fp32 dot, * scale)
 *   oc_sdpa_int8       int8_quantized_sdpa decode (online softmax in fp32,
 *                      _int8_sdpa_sources.py:87-170) for per-token/per-head
 *                      symmetric INT8 K/V with fp16 scales
 *   oc_rms_norm        mx.fast.rms_norm (spark_mlx_llm/ops/ffn.py:99), fp32 output
 *   oc_bf16_argmax     bf16 lm_head GEMV + greedy argmax (lowest index on ties)
 *   oc_bf16_logits     the same GEMV, returning the fp32 logits
 * Outputs are fp32; the caller rounds to bf16 where the reference stores bf16.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline float bf16f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float halff(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF, u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal */
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400));
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7F800000u | (man << 13);
  } else {
    u = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ---------------------------------------------------------------- threads */
typedef void (*oc_body)(const void* ctx, long begin, long end);
typedef struct {
  oc_body body;
  const void* ctx;
  long begin, end;
} oc_chunk;

static void* oc_run(void* arg) {
  oc_chunk* c = (oc_chunk*)arg;
  c->body(c->ctx, c->begin, c->end);
  return NULL;
}

int oc_threads(void) {
  const char* env = getenv("OC_THREADS");
  long n = env ? atol(env) : sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

/* Runs body over [0, n) split into one contiguous range per thread. */
static void oc_parallel(long n, oc_body body, const void* ctx) {
  int t = oc_threads();
  if (t > n) t = (int)n;
  if (t <= 1) {
    body(ctx, 0, n);
    return;
  }
  pthread_t tid[256];
  oc_chunk chunk[256];
  for (int i = 0; i < t; ++i) {
    chunk[i].body = body;
    chunk[i].ctx = ctx;
    chunk[i].begin = n * i / t;
    chunk[i].end = n * (i + 1) / t;
    if (i > 0) pthread_create(&tid[i], NULL, oc_run, &chunk[i]);
  }
  oc_run(&chunk[0]);
  for (int i = 1; i < t; ++i) pthread_join(tid[i], NULL);
}

/* ------------------------------------------------------------ affine linear */
typedef struct {
  const float* x;
  int M;
  const uint32_t* w;
  const uint16_t *s, *b;
  int N, K, G, bits;
  float* y;
  const float* xsum;
} affine_ctx;

static void affine_rows(const void* vctx, long n0, long n1) {
  const affine_ctx* c = (const affine_ctx*)vctx;
  const int M = c->M, K = c->K, G = c->G, bits = c->bits, N = c->N;
  const int groups = K / G, per_word = 32 / bits, words_per_row = K * bits / 32;
  const uint32_t mask = (1u << bits) - 1u;
  float q[128];
  for (long n = n0; n < n1; ++n) {
    const uint32_t* wr = c->w + (size_t)n * words_per_row;
    float out[8] = {0};
    for (int g = 0; g < groups; ++g) {
      const float sc = bf16f(c->s[(size_t)n * groups + g]), bi = bf16f(c->b[(size_t)n * groups + g]);
      const int w0 = g * G / per_word;
      for (int i = 0; i < G / per_word; ++i) {
        const uint32_t word = wr[w0 + i];
        for (int j = 0; j < per_word; ++j) q[i * per_word + j] = (float)((word >> (j * bits)) & mask);
      }
      for (int m = 0; m < M; ++m) {
        const float* xm = c->x + (size_t)m * K + (size_t)g * G;
        float dot = 0.f;
        for (int k = 0; k < G; ++k) dot += q[k] * xm[k];
        out[m] += sc * dot + bi * c->xsum[(size_t)m * groups + g];
      }
    }
    for (int m = 0; m < M; ++m) c->y[(size_t)m * N + n] = out[m];
  }
}

/* y [M, N] fp32; x [M, K] fp32 (M <= 8); w [N, K*bits/32]; s, b [N, K/G] bf16 bits; G <= 128 */
void oc_affine_linear(const float* x, int M, const uint32_t* w, const uint16_t* s, const uint16_t* b, int N, int K,
                      int G, int bits, float* y) {
  const int groups = K / G;
  float* xsum = (float*)malloc(sizeof(float) * (size_t)M * groups);
  for (int m = 0; m < M; ++m)
    for (int g = 0; g < groups; ++g) {
      float acc = 0.f;
      for (int k = 0; k < G; ++k) acc += x[(size_t)m * K + (size_t)g * G + k];
      xsum[(size_t)m * groups + g] = acc;
    }
  affine_ctx ctx = {x, M, w, s, b, N, K, G, bits, y, xsum};
  oc_parallel(N, affine_rows, &ctx);
  free(xsum);
}

/* ------------------------------------------------------------------ W8A16 */
typedef struct {
  const float* x;
  int M;
  const int8_t* w;
  const float* scales;
  int N, K;
  float* y;
} w8_ctx;

static void w8_rows(const void* vctx, long n0, long n1) {
  const w8_ctx* c = (const w8_ctx*)vctx;
  for (long n = n0; n < n1; ++n) {
    const int8_t* wr = c->w + (size_t)n * c->K;
    for (int m = 0; m < c->M; ++m) {
      const float* xm = c->x + (size_t)m * c->K;
      float dot = 0.f;
      for (int k = 0; k < c->K; ++k) dot += xm[k] * (float)wr[k];
      c->y[(size_t)m * c->N + n] = dot * c->scales[n];
    }
  }
}

void oc_w8a16(const float* x, int M, const int8_t* w, const float* scales, int N, int K, float* y) {
  w8_ctx ctx = {x, M, w, scales, N, K, y};
  oc_parallel(N, w8_rows, &ctx);
}

/* ---------------------------------------------------------------- RMSNorm */
void oc_rms_norm(const float* x, const float* w, int M, int K, float eps, float* y) {
  for (int m = 0; m < M; ++m) {
    const float* xm = x + (size_t)m * K;
    double ss = 0.0;
    for (int k = 0; k < K; ++k) ss += (double)xm[k] * xm[k];
    const float r = (float)(1.0 / sqrt(ss / K + eps));
    for (int k = 0; k < K; ++k) y[(size_t)m * K + k] = xm[k] * r * w[k];
  }
}

/* ---------------------------------------------------------------- INT8 SDPA */
typedef struct {
  const float* q;
  const int8_t *k, *v;
  const uint16_t *ks, *vs;
  int B, H, KH, N, cap, D;
  float scale;
  float* out;
} sdpa_ctx;

static void sdpa_heads(const void* vctx, long i0, long i1) {
  const sdpa_ctx* c = (const sdpa_ctx*)vctx;
  const int H = c->H, D = c->D, G = c->H / c->KH;
  float acc[256];
  for (long i = i0; i < i1; ++i) {
    const int bb = (int)(i / H), h = (int)(i % H), kh = h / G;
    const float* qh = c->q + ((size_t)bb * H + h) * D;
    const size_t base = ((size_t)bb * c->KH + kh) * c->cap;
    float m = -INFINITY, l = 0.f;
    for (int d = 0; d < D; ++d) acc[d] = 0.f;
    for (int t = 0; t < c->N; ++t) {
      const int8_t* kr = c->k + (base + t) * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot += qh[d] * (float)kr[d];
      const float sc = dot * halff(c->ks[base + t]) * c->scale;
      const float nm = sc > m ? sc : m;
      const float alpha = expf(m - nm), p = expf(sc - nm);
      l = l * alpha + p;
      m = nm;
      const int8_t* vr = c->v + (base + t) * D;
      const float pv = p * halff(c->vs[base + t]);
      for (int d = 0; d < D; ++d) acc[d] = acc[d] * alpha + pv * (float)vr[d];
    }
    for (int d = 0; d < D; ++d) c->out[((size_t)bb * H + h) * D + d] = l > 0.f ? acc[d] / l : 0.f;
  }
}

/* q [B, H, D]; k, v [B, KH, cap, D] int8; ks, vs [B, KH, cap] fp16 bits; out [B, H, D]; D <= 256 */
void oc_sdpa_int8(const float* q, const int8_t* k, const uint16_t* ks, const int8_t* v, const uint16_t* vs, int B,
                  int H, int KH, int N, int cap, int D, float scale, float* out) {
  sdpa_ctx ctx = {q, k, v, ks, vs, B, H, KH, N, cap, D, scale, out};
  oc_parallel((long)B * H, sdpa_heads, &ctx);
}

/* ------------------------------------------------------------ lm_head argmax */
typedef struct {
  const float* x;
  int M;
  const uint16_t* w;
  int N, K;
  float* logits;
} head_ctx;

static void head_rows(const void* vctx, long n0, long n1) {
  const head_ctx* c = (const head_ctx*)vctx;
  for (long n = n0; n < n1; ++n) {
    const uint16_t* wr = c->w + (size_t)n * c->K;
    for (int m = 0; m < c->M; ++m) {
      const float* xm = c->x + (size_t)m * c->K;
      float dot = 0.f;
      for (int k = 0; k < c->K; ++k) dot += xm[k] * bf16f(wr[k]);
      c->logits[(size_t)m * c->N + n] = dot;
    }
  }
}

/* logits [M, N] = x [M, K] . w [N, K]^T (bf16 bits), fp32 */
void oc_bf16_logits(const float* x, int M, const uint16_t* w, int N, int K, float* logits) {
  head_ctx ctx = {x, M, w, N, K, logits};
  oc_parallel(N, head_rows, &ctx);
}

/* logits = x [M, K] . w [N, K]^T (bf16 bits); idx[m] = argmax (lowest index on ties) */
void oc_bf16_argmax(const float* x, int M, const uint16_t* w, int N, int K, int* idx, float* best) {
  float* logits = (float*)malloc(sizeof(float) * (size_t)M * N);
  head_ctx ctx = {x, M, w, N, K, logits};
  oc_parallel(N, head_rows, &ctx);
  for (int m = 0; m < M; ++m) {
    best[m] = -INFINITY;
    idx[m] = 0;
    for (int n = 0; n < N; ++n) {
      const float v = logits[(size_t)m * N + n];
      if (v > best[m]) {
        best[m] = v;
        idx[m] = n;
      }
    }
  }
  free(logits);
}
