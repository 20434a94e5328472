/*
 * C/OpenMP restatement of the routed sparse-MoE block (TEST INFRASTRUCTURE /
 * CPU BASELINE ONLY).  It is timed as the CPU baseline of bench.py and
 * checked against the NumPy oracle in tests/; the CUDA library never calls
 * it.  Activations and bf16 parameters arrive as float32 arrays holding
 * bf16 values; packed Q4 words as uint32.
 *
 * Arithmetic follows the reference block (models/flashnext, Veystrix-Core):
 *   router logits x.Wg^T rounded to bf16 (adaptive_topk.py:60);
 *   softmax(precise) in float32, top-k by logit (ties: lower id), renorm
 *     scores/sum (adaptive_topk.py:62-65, :257-262);
 *   Q4 qmv: per group scale*sum(q*x) + bias*sum(x) in float32
 *     (metal_runtime.py:1014-1029), outputs rounded to bf16;
 *   SwiGLU with MLX's bf16 sequence (metal_runtime.py:267-285);
 *   fused combine: bf16(y_s)*score_s summed in float32 in slot order,
 *     then + bf16(sg*shared) (metal_runtime.py:315-334).
 * Experts touched by several tokens are computed once for all of them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float bf16r(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return f;
  u += 0x7FFFu + ((u >> 16) & 1u);
  u &= 0xFFFF0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static float sigmoid_bf16(float z) {
  float t = bf16r((float)exp((double)fabsf(z)));
  float den = bf16r(1.0f + t);
  float s = bf16r(1.0f / den);
  return z < 0.0f ? s : bf16r(1.0f - s);
}

static float silu_mul_bf16(float g, float u) {
  float sg = sigmoid_bf16(g);
  return bf16r(bf16r(g * sg) * u);
}

typedef struct {
  const uint32_t* w;   /* [E, out, in/8] */
  const float* s;      /* [E, out, in/32] */
  const float* b;
  int experts, out, in;
} cq4;

/* out[t][r] = bf16(sum_g s*qsum + b*xsum) for rows [r0, r1) of expert e. */
static void qmv_rows(const cq4* P, int e, const float* x, int ntok, const int* toks, int ldx,
                     float* out, int ldo, int r0, int r1) {
  const int K = P->in, G = K / 32, KW = K / 8;
  const uint32_t* W = P->w + (int64_t)e * P->out * KW;
  const float* S = P->s + (int64_t)e * P->out * G;
  const float* B = P->b + (int64_t)e * P->out * G;
  for (int r = r0; r < r1; ++r) {
    for (int ti = 0; ti < ntok; ++ti) {
      const float* xr = x + (int64_t)toks[ti] * ldx;
      float acc = 0.0f;
      for (int g = 0; g < G; ++g) {
        const uint32_t* wg = W + (int64_t)r * KW + g * 4;
        const float* xg = xr + g * 32;
        float qs = 0.0f, xs = 0.0f;
        for (int j = 0; j < 32; ++j) {
          const float q = (float)((wg[j >> 3] >> (4 * (j & 7))) & 15u);
          qs += q * xg[j];
          xs += xg[j];
        }
        acc += S[(int64_t)r * G + g] * qs + B[(int64_t)r * G + g] * xs;
      }
      out[(int64_t)ti * ldo + r] = bf16r(acc);
    }
  }
}

int vx_cref_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* The whole block for T tokens.  Returns 0 on success. */
int vx_cref_block(const float* x, int T, int E, int d, int I, int Is, int k, const float* router_w,
                  cq4 gate, cq4 up, cq4 down, cq4 sgate, cq4 sup, cq4 sdown, cq4 segate, float* y) {
  if (T <= 0) return 0;
  float* logits = (float*)malloc(sizeof(float) * (size_t)T * E);
  int* inds = (int*)malloc(sizeof(int) * (size_t)T * k);
  float* wts = (float*)malloc(sizeof(float) * (size_t)T * k);
  float* yd = (float*)calloc((size_t)T * k * d, sizeof(float));
  float* shared = (float*)malloc(sizeof(float) * (size_t)T * d);
  float* sg = (float*)malloc(sizeof(float) * (size_t)T);
  int* all = (int*)malloc(sizeof(int) * (size_t)T);
  for (int t = 0; t < T; ++t) all[t] = t;

  /* router */
#pragma omp parallel for schedule(static)
  for (int e = 0; e < E; ++e)
    for (int t = 0; t < T; ++t) {
      const float* xr = x + (int64_t)t * d;
      const float* wr = router_w + (int64_t)e * d;
      float a = 0.0f;
      for (int i = 0; i < d; ++i) a += xr[i] * wr[i];
      logits[(int64_t)t * E + e] = bf16r(a);
    }
  for (int t = 0; t < T; ++t) {
    const float* l = logits + (int64_t)t * E;
    float m = -INFINITY;
    for (int e = 0; e < E; ++e) m = l[e] > m ? l[e] : m;
    float s = 0.0f;
    for (int e = 0; e < E; ++e) s += (float)exp((double)(l[e] - m));
    const float inv = 1.0f / s;
    char* taken = (char*)calloc((size_t)E, 1);
    float tot = 0.0f, sel[64];
    for (int r = 0; r < k; ++r) {
      int bi = -1;
      for (int e = 0; e < E; ++e)
        if (!taken[e] && (bi < 0 || l[e] > l[bi])) bi = e;
      taken[bi] = 1;
      inds[t * k + r] = bi;
      sel[r] = bf16r((float)exp((double)(l[bi] - m)) * inv);
      tot += sel[r];
    }
    free(taken);
    const float mass = bf16r(tot);
    for (int r = 0; r < k; ++r) wts[t * k + r] = bf16r(sel[r] / mass);
  }

  /* shared expert and its gate */
  if (sgate.w) {
    float* hs = (float*)malloc(sizeof(float) * (size_t)T * Is * 2);
#pragma omp parallel for schedule(static)
    for (int rb = 0; rb < Is; rb += 16) {
      qmv_rows(&sgate, 0, x, T, all, d, hs, Is, rb, rb + 16 < Is ? rb + 16 : Is);
      qmv_rows(&sup, 0, x, T, all, d, hs + (size_t)T * Is, Is, rb, rb + 16 < Is ? rb + 16 : Is);
    }
    for (int i = 0; i < T * Is; ++i) hs[i] = silu_mul_bf16(hs[i], hs[(size_t)T * Is + i]);
#pragma omp parallel for schedule(static)
    for (int rb = 0; rb < d; rb += 64)
      qmv_rows(&sdown, 0, hs, T, all, Is, shared, d, rb, rb + 64 < d ? rb + 64 : d);
    float* z = (float*)malloc(sizeof(float) * (size_t)T);
    qmv_rows(&segate, 0, x, T, all, d, z, 1, 0, 1);
    for (int t = 0; t < T; ++t) sg[t] = sigmoid_bf16(z[t]);
    free(z);
    free(hs);
  }

  /* routed experts, each touched expert once for all its tokens */
  int* cnt = (int*)calloc((size_t)E, sizeof(int));
  for (int i = 0; i < T * k; ++i) cnt[inds[i]]++;
  int* off = (int*)malloc(sizeof(int) * (size_t)(E + 1));
  off[0] = 0;
  for (int e = 0; e < E; ++e) off[e + 1] = off[e] + cnt[e];
  int* pairs = (int*)malloc(sizeof(int) * (size_t)T * k);
  int* fill = (int*)calloc((size_t)E, sizeof(int));
  for (int i = 0; i < T * k; ++i) pairs[off[inds[i]] + fill[inds[i]]++] = i;
  free(fill);
#pragma omp parallel for schedule(dynamic, 1)
  for (int e = 0; e < E; ++e) {
    const int n = cnt[e];
    if (!n) continue;
    int* toks = (int*)malloc(sizeof(int) * (size_t)n);
    for (int j = 0; j < n; ++j) toks[j] = pairs[off[e] + j] / k;
    float* gu = (float*)malloc(sizeof(float) * (size_t)n * I * 2);
    qmv_rows(&gate, e, x, n, toks, d, gu, I, 0, I);
    qmv_rows(&up, e, x, n, toks, d, gu + (size_t)n * I, I, 0, I);
    for (int i = 0; i < n * I; ++i) gu[i] = silu_mul_bf16(gu[i], gu[(size_t)n * I + i]);
    float* ye = (float*)malloc(sizeof(float) * (size_t)n * d);
    int* idn = (int*)malloc(sizeof(int) * (size_t)n);
    for (int j = 0; j < n; ++j) idn[j] = j;
    qmv_rows(&down, e, gu, n, idn, I, ye, d, 0, d);
    for (int j = 0; j < n; ++j) memcpy(yd + (size_t)pairs[off[e] + j] * d, ye + (size_t)j * d, sizeof(float) * d);
    free(idn);
    free(ye);
    free(gu);
    free(toks);
  }

  /* fused combine */
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int c = 0; c < d; ++c) {
      float acc = 0.0f;
      for (int s = 0; s < k; ++s) acc += yd[((size_t)t * k + s) * d + c] * wts[t * k + s];
      float r = bf16r(acc);
      if (sgate.w) r = bf16r(r + bf16r(sg[t] * shared[(size_t)t * d + c]));
      y[(size_t)t * d + c] = r;
    }
  free(pairs);
  free(off);
  free(cnt);
  free(all);
  free(sg);
  free(shared);
  free(yd);
  free(wts);
  free(inds);
  free(logits);
  return 0;
}
