/*
 * CPU restatement of the MoE block's expert half -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline and
 * --impl reference legs may load this library, and only as the checker or
 * the timed CPU baseline.  The product path (livglm_b200/csrc) never links or
 * calls it.
 *
 * Restates, with the MXFP4 weights decoded on the fly from the checkpoint
 * bytes (the way the reference's native path reads them, never a
 * dequantised copy):
 *   routed experts   ExpertSSD.__call__       src/glm53flash/expert_ssd.py:159-188
 *     gate = bf16(x @ Wg_e.T), up = bf16(x @ Wu_e.T)        (mx.gather_qmm, mxfp4)
 *     act  = limited SwiGLU, each op rounded to bf16         expert_ssd.py:103-107
 *     y    = bf16(act @ Wd_e.T)
 *   shared expert    DenseMLP.__call__         src/glm53flash/layers.py:160-171
 *     the same chain on bf16 weights
 *   merge            ExpertSSDMoE.__call__     src/glm53flash/moe.py:199-201
 *     out = ((0 + y0*w0) + y1*w1) + ... + shared, in f32
 * Weight bytes: U8 [rows, cols/2] E2M1 nibbles (low nibble = even column),
 * U8 [rows, cols/32] UE8M0 scales (value = E2M1 * 2^(s-127), 255 = NaN);
 * expert_source.py:210-215 reads them byte-preserving.
 *
 * The dot products sum in f32 over 8 interleaved partial sums (element i
 * into partial i % 8, partials added in index order): a fixed order the
 * compiler can keep in vector registers without reassociating.  MLX leaves
 * the order unspecified, so results agree with other restatements (the NumPy
 * oracle, the GPU kernels) to within f32 rounding before each bf16 rounding.
 *
 * Work is grouped by expert (each weight row is decoded once per call and
 * applied to every route of that expert) and spread over OpenMP threads.
 * Build: oracle/build_oracle.py (gcc -O3 -ffp-contract=off -fopenmp).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float oracle_sigmoidf1(float v); /* router_ref.c: the canonical sigmoid */
int oracle_router(const uint16_t *x, const float *w, const float *bias, int M, int d, int E, int G,
                  int topk_group, int k, int norm, float scale, float *logits, float *choice,
                  float *weights, uint32_t *indices);
void oracle_dispatch(const uint32_t *indices, int64_t slots, int E, int32_t *counts, int32_t *offsets,
                     int32_t *perm);

static float f32_of_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t bits_of_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float bf16f(uint16_t h) { return f32_of_bits((uint32_t)h << 16); }
/* round to nearest even bf16; NaN stays NaN */
static uint16_t to_bf16(float f) {
  uint32_t u = bits_of_f32(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static float rbf16(float f) { return bf16f(to_bf16(f)); }

static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
static float e8m0(uint8_t s) {
  if (s == 255) return f32_of_bits(0x7FC00000u);
  if (s == 0) return f32_of_bits(0x00400000u); /* 2^-127 */
  return f32_of_bits((uint32_t)s << 23);
}
/* one MXFP4 row of n values */
static void decode_row(const uint8_t *packed, const uint8_t *scale, int n, float *out) {
  for (int b = 0; b < n / 32; ++b) {
    const float s = e8m0(scale[b]);
    const uint8_t *p = packed + b * 16;
    float *o = out + b * 32;
    for (int i = 0; i < 16; ++i) {
      o[2 * i] = kE2M1[p[i] & 15] * s;
      o[2 * i + 1] = kE2M1[p[i] >> 4] * s;
    }
  }
}
static void decode_bf16_row(const uint16_t *w, int n, float *out) {
  for (int i = 0; i < n; ++i) out[i] = bf16f(w[i]);
}
/* built for AVX2 and for the x86-64 baseline, picked at run time */
__attribute__((target_clones("avx2", "default")))
static float dot8(const float *a, const float *b, int n) { /* n % 8 == 0 */
  float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int i = 0; i < n; i += 8)
    for (int l = 0; l < 8; ++l) p[l] = p[l] + a[i + l] * b[i + l];
  return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}
/* expert_ssd.py:103-107 on bf16 values, each op rounded to bf16 */
static uint16_t swiglu(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = g < limit ? g : limit;
    u = u > -limit ? (u < limit ? u : limit) : -limit;
  }
  const float s = rbf16(oracle_sigmoidf1(g));
  const float a = rbf16(g * s);
  return to_bf16(a * u);
}

/* The chain gate/up -> SwiGLU -> down for n_routes rows of xf (f32 copies of
 * bf16 tokens, row stride d) through one expert, outputs bf16 rows of y
 * (row i at y + out_rows[i] * d).  Weight rows come from row(kind, r, buf). */
typedef void (*row_fn)(const void *ctx, int kind, int r, float *buf);

struct mx_ctx {
  const uint8_t *gp, *gs, *up, *us, *dp, *ds;
  int d, F;
};
static void mx_row(const void *c_, int kind, int r, float *buf) {
  const struct mx_ctx *c = (const struct mx_ctx *)c_;
  if (kind == 0) decode_row(c->gp + (size_t)r * (c->d / 2), c->gs + (size_t)r * (c->d / 32), c->d, buf);
  else if (kind == 1) decode_row(c->up + (size_t)r * (c->d / 2), c->us + (size_t)r * (c->d / 32), c->d, buf);
  else decode_row(c->dp + (size_t)r * (c->F / 2), c->ds + (size_t)r * (c->F / 32), c->F, buf);
}
struct bf_ctx {
  const uint16_t *wg, *wu, *wd;
  int d, F;
};
static void bf_row(const void *c_, int kind, int r, float *buf) {
  const struct bf_ctx *c = (const struct bf_ctx *)c_;
  if (kind == 0) decode_bf16_row(c->wg + (size_t)r * c->d, c->d, buf);
  else if (kind == 1) decode_bf16_row(c->wu + (size_t)r * c->d, c->d, buf);
  else decode_bf16_row(c->wd + (size_t)r * c->F, c->F, buf);
}

/* groups[g] = (ctx, first route, route count); routes r of a group read
 * xf[rows[r]] and write y[out_rows[r]].  Two passes, each a parallel loop
 * over (group, block of 16 weight rows). */
struct group {
  const void *ctx;
  int first, count;
};
static void run_groups(const struct group *groups, int n_groups, row_fn row, const float *xf,
                       const int32_t *rows, const int32_t *out_rows, int d, int F, float limit, uint16_t *y,
                       float *actf /* [routes][F] */) {
  const int RB = 16;
  const int nb_up = (F + RB - 1) / RB, nb_dn = (d + RB - 1) / RB;
  /* gate/up + SwiGLU: act of every route, f32 copies of bf16 values */
#pragma omp parallel
  {
    float *wg = (float *)malloc(sizeof(float) * (size_t)d);
    float *wu = (float *)malloc(sizeof(float) * (size_t)d);
#pragma omp for schedule(dynamic, 1)
    for (long long it = 0; it < (long long)n_groups * nb_up; ++it) {
      const struct group *g = &groups[it / nb_up];
      const int f0 = (int)(it % nb_up) * RB;
      if (!g->count) continue;
      for (int f = f0; f < f0 + RB && f < F; ++f) {
        row(g->ctx, 0, f, wg);
        row(g->ctx, 1, f, wu);
        for (int r = g->first; r < g->first + g->count; ++r) {
          const float *x = xf + (size_t)rows[r] * d;
          const float gv = rbf16(dot8(x, wg, d)), uv = rbf16(dot8(x, wu, d));
          actf[(size_t)r * F + f] = bf16f(swiglu(gv, uv, limit));
        }
      }
    }
    free(wg);
    free(wu);
  }
  /* down */
#pragma omp parallel
  {
    float *wd = (float *)malloc(sizeof(float) * (size_t)F);
#pragma omp for schedule(dynamic, 1)
    for (long long it = 0; it < (long long)n_groups * nb_dn; ++it) {
      const struct group *g = &groups[it / nb_dn];
      const int c0 = (int)(it % nb_dn) * RB;
      if (!g->count) continue;
      for (int c = c0; c < c0 + RB && c < d; ++c) {
        row(g->ctx, 2, c, wd);
        for (int r = g->first; r < g->first + g->count; ++r)
          y[(size_t)out_rows[r] * d + c] = to_bf16(dot8(actf + (size_t)r * F, wd, F));
      }
    }
    free(wd);
  }
}

/* Routed experts: y[t*k + j] (bf16 [M*k, d]) for expert indices[t*k + j];
 * banks expert-major ([E][F][d/2], [E][F][d/32], [E][d][F/2], [E][d][F/32]). */
int oracle_experts(const uint16_t *x, int M, int d, int F, int E, int k, const uint32_t *indices,
                   const uint8_t *gp, const uint8_t *gs, const uint8_t *upk, const uint8_t *us,
                   const uint8_t *dp, const uint8_t *ds, float limit, uint16_t *y) {
  if (M < 0 || d % 32 || F % 32 || E < 1 || E > 4096 || k < 1) return 1;
  const int64_t R = (int64_t)M * k;
  for (int64_t s = 0; s < R; ++s)
    if (indices[s] >= (uint32_t)E) return 2;
  float *xf = (float *)malloc(sizeof(float) * ((size_t)M * d + 1));
  int32_t *counts = (int32_t *)malloc(sizeof(int32_t) * E), *offsets = (int32_t *)malloc(sizeof(int32_t) * (E + 1));
  int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * (R + 1)), *rows = (int32_t *)malloc(sizeof(int32_t) * (R + 1));
  float *actf = (float *)malloc(sizeof(float) * ((size_t)R * F + 1));
  struct mx_ctx *ctx = (struct mx_ctx *)malloc(sizeof(struct mx_ctx) * E);
  struct group *groups = (struct group *)malloc(sizeof(struct group) * E);
  for (size_t i = 0; i < (size_t)M * d; ++i) xf[i] = bf16f(x[i]);
  oracle_dispatch(indices, R, E, counts, offsets, perm);
  for (int64_t p = 0; p < R; ++p) rows[p] = perm[p] / k;
  const size_t gpe = (size_t)F * (d / 2), gse = (size_t)F * (d / 32), dpe = (size_t)d * (F / 2), dse = (size_t)d * (F / 32);
  for (int e = 0; e < E; ++e) {
    ctx[e] = (struct mx_ctx){gp + e * gpe, gs + e * gse, upk + e * gpe, us + e * gse, dp + e * dpe, ds + e * dse, d, F};
    groups[e] = (struct group){&ctx[e], offsets[e], counts[e]};
  }
  run_groups(groups, E, mx_row, xf, rows, perm, d, F, limit, y, actf);
  free(xf); free(counts); free(offsets); free(perm); free(rows); free(actf); free(ctx); free(groups);
  return 0;
}

/* Shared expert: ys [M, d] bf16 from bf16 weights [Fs,d], [Fs,d], [d,Fs]. */
int oracle_shared(const uint16_t *x, int M, int d, int Fs, const uint16_t *wg, const uint16_t *wu,
                  const uint16_t *wd, float limit, uint16_t *ys) {
  if (M < 0 || d % 8 || Fs % 8) return 1;
  float *xf = (float *)malloc(sizeof(float) * ((size_t)M * d + 1));
  int32_t *rows = (int32_t *)malloc(sizeof(int32_t) * ((size_t)M + 1));
  float *actf = (float *)malloc(sizeof(float) * ((size_t)M * Fs + 1));
  for (size_t i = 0; i < (size_t)M * d; ++i) xf[i] = bf16f(x[i]);
  for (int t = 0; t < M; ++t) rows[t] = t;
  struct bf_ctx ctx = {wg, wu, wd, d, Fs};
  struct group g = {&ctx, 0, M};
  run_groups(&g, 1, bf_row, xf, rows, rows, d, Fs, limit, ys, actf);
  free(xf); free(rows); free(actf);
  return 0;
}

/* The whole block, ExpertSSDMoE.__call__ (moe.py:96-201) for bf16 rows:
 * router, routed experts, shared expert (Fs = 0: none), merge -> out f32 [M, d];
 * weights_out / indices_out [M, k] optional. */
int oracle_moe_layer(const uint16_t *x, int M, int d, int F, int Fs, int E, int G, int topk_group, int k,
                     int norm, float scale, float limit, const float *router_w, const float *router_b,
                     const uint8_t *gp, const uint8_t *gs, const uint8_t *upk, const uint8_t *us,
                     const uint8_t *dp, const uint8_t *ds, const uint16_t *swg, const uint16_t *swu,
                     const uint16_t *swd, float *out, float *weights_out, uint32_t *indices_out) {
  if (M < 0) return 1;
  if (M == 0) return 0;
  float *logits = (float *)malloc(sizeof(float) * (size_t)M * E);
  float *w = (float *)malloc(sizeof(float) * (size_t)M * k);
  uint32_t *idx = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)M * k);
  uint16_t *y = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)M * k * d);
  uint16_t *ys = Fs > 0 ? (uint16_t *)malloc(sizeof(uint16_t) * (size_t)M * d) : NULL;
  int rc = oracle_router(x, router_w, router_b, M, d, E, G, topk_group, k, norm, scale, logits, NULL, w, idx);
  if (!rc) rc = oracle_experts(x, M, d, F, E, k, idx, gp, gs, upk, us, dp, ds, limit, y);
  if (!rc && Fs > 0) rc = oracle_shared(x, M, d, Fs, swg, swu, swd, limit, ys);
  if (!rc) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < M; ++t)
      for (int c = 0; c < d; ++c) {
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) acc = acc + bf16f(y[((size_t)t * k + j) * d + c]) * w[(size_t)t * k + j];
        if (ys) acc = acc + bf16f(ys[(size_t)t * d + c]);
        out[(size_t)t * d + c] = acc;
      }
    if (weights_out) memcpy(weights_out, w, sizeof(float) * (size_t)M * k);
    if (indices_out) memcpy(indices_out, idx, sizeof(uint32_t) * (size_t)M * k);
  }
  free(logits); free(w); free(idx); free(y); free(ys);
  return rc;
}
