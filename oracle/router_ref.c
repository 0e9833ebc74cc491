/*
 * CPU oracle for the GLM MoE router -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker.  The product path
 * (livglm_b200/csrc) never links or calls it.
 *
 * Restates TopKRouter.__call__ of kg36/livglm, src/glm53flash/moe.py:36-63:
 *   rows    = x.reshape(-1, d).astype(f32)                      moe.py:37
 *   logits  = rows @ W.T                                        moe.py:38
 *   scores  = sigmoid(logits)                                   moe.py:39
 *   choice  = scores + e_score_correction_bias                  moe.py:40-43
 *   group   = sum of the two largest choices per group          moe.py:45-47
 *   keep the topk_group best groups, others -> -inf             moe.py:48-57
 *   indices = argsort(choice)[..., -k:]  (ascending, best last) moe.py:58
 *   weights = scores[indices]; w /= (sum(w) + 1e-20); w *= s    moe.py:59-62
 *
 * MLX leaves the fp32 summation order of the matmul and the sum, the exp
 * inside sigmoid, and the tie order of argsort unspecified.  This build pins
 * them (the "canonical router arithmetic"); the CUDA router implements the
 * same definitions, so indices and weights compare bit-for-bit:
 *
 *  (1) logit[t,e]: 32 partial sums p[0..31].  Partial l accumulates, with
 *      fmaf in increasing element order, the 8-element chunks c = l, l+32,
 *      l+64, ... (elements 8c..8c+7) of x[t]*W[e].  Then a butterfly:
 *      for off in 16,8,4,2,1: p[l] = p[l] + p[l^off]; the logit is p[0].
 *      Requires d % 8 == 0.
 *  (2) sigmoid(v) = 1 / (1 + own_exp(-v)), IEEE division.  own_exp is a
 *      Cody-Waite reduction by ln 2 (split into a 12-bit-short high part and
 *      the remainder) and a degree-8 Taylor polynomial in Horner form with
 *      fmaf, scaled by 2^n in two power-of-two steps.
 *  (3) Ties in every argsort follow a stable ascending sort (numpy
 *      kind="stable"): among equal values the lower index sorts first, so
 *      the last-k slice prefers the higher index.
 *  (4) sum(w) is sequential over the k selected routes in output order.
 *
 * Build: see oracle/build_oracle.py (gcc -O2 -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define LOG2E_F   0x1.715476p+0f
#define LN2_HI_F  0x1.62ep-1f      /* ln2 with the low 12 mantissa bits cleared */
#define LN2_LO_F  0x1.0bfbe8p-15f  /* float32(ln2 - LN2_HI_F) */
#define RND_MAGIC 0x1.8p23f        /* adding/subtracting rounds to an integer */

static float pow2i(int n) { /* 2^n for -126 <= n <= 127 */
  uint32_t u = (uint32_t)(n + 127) << 23;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

float oracle_expf1(float x) {
  if (x > 89.0f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  float t = fmaf(x, LOG2E_F, RND_MAGIC);
  float n = t - RND_MAGIC;
  float r = fmaf(n, -LN2_HI_F, x);
  r = fmaf(n, -LN2_LO_F, r);
  float p = 0x1.a01a02p-16f;           /* 1/8! */
  p = fmaf(p, r, 0x1.a01a02p-13f);     /* 1/7! */
  p = fmaf(p, r, 0x1.6c16c2p-10f);     /* 1/6! */
  p = fmaf(p, r, 0x1.111112p-7f);      /* 1/5! */
  p = fmaf(p, r, 0x1.555556p-5f);      /* 1/4! */
  p = fmaf(p, r, 0x1.555556p-3f);      /* 1/3! */
  p = fmaf(p, r, 0x1.0p-1f);           /* 1/2! */
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  int n1 = ni >> 1; /* floor(n/2) */
  int n2 = ni - n1;
  return (p * pow2i(n1)) * pow2i(n2);
}

float oracle_sigmoidf1(float v) {
  float e = oracle_expf1(-v);
  return 1.0f / (1.0f + e);
}

void oracle_expf(const float *x, float *y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = oracle_expf1(x[i]);
}

void oracle_sigmoidf(const float *x, float *y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = oracle_sigmoidf1(x[i]);
}

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* (value, index) total order of a stable ascending sort. */
static int after(float a, int ia, float b, int ib) {
  return a > b || (a == b && ia > ib);
}

float oracle_router_logit(const uint16_t *x, const float *w, int d) {
  float p[32];
  int chunks = d / 8;
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int c = l; c < chunks; c += 32)
      for (int q = 0; q < 8; ++q) {
        int i = 8 * c + q;
        acc = fmaf(bf16_to_f32(x[i]), w[i], acc);
      }
    p[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float nxt[32];
    for (int l = 0; l < 32; ++l) nxt[l] = p[l] + p[l ^ off];
    memcpy(p, nxt, sizeof p);
  }
  return p[0];
}

/*
 * Returns 0 on success, -1 on a geometry the reference rejects
 * (model_config.py:142-176: E % G, 1 <= g <= G, E/G >= 2, 1 <= k <= E) or
 * d % 8 != 0, or E > 4096 (scratch limit of this oracle).
 * logits/scores may be NULL.
 */
int oracle_router(const uint16_t *x, const float *w, const float *bias, int M,
                  int d, int E, int G, int g, int k, int norm, float scale,
                  float *logits, float *scores_out, float *weights,
                  uint32_t *indices) {
  if (d % 8 || G < 1 || E % G || g < 1 || g > G || E / G < 2 || k < 1 ||
      k > E || E > 4096)
    return -1;
  int per = E / G;
  /* tokens are independent; each (token, expert) sum keeps its own order */
#pragma omp parallel for schedule(static)
  for (int t = 0; t < M; ++t) {
    float scores[4096], choice[4096], gscore[4096];
    int gsel[4096];
    const uint16_t *xt = x + (int64_t)t * d;
    for (int e = 0; e < E; ++e) {
      float lg = oracle_router_logit(xt, w + (int64_t)e * d, d);
      if (logits) logits[(int64_t)t * E + e] = lg;
      scores[e] = oracle_sigmoidf1(lg);
      choice[e] = scores[e] + bias[e];
      if (scores_out) scores_out[(int64_t)t * E + e] = scores[e];
    }
    for (int gi = 0; gi < G; ++gi) {
      /* two largest of the group under the stable order */
      int b1 = -1, b2 = -1;
      for (int j = 0; j < per; ++j) {
        int e = gi * per + j;
        if (b1 < 0 || after(choice[e], e, choice[b1], b1)) {
          b2 = b1;
          b1 = e;
        } else if (b2 < 0 || after(choice[e], e, choice[b2], b2)) {
          b2 = e;
        }
      }
      gscore[gi] = choice[b2] + choice[b1];
      gsel[gi] = 0;
    }
    for (int s = 0; s < g; ++s) {
      int best = -1;
      for (int gi = 0; gi < G; ++gi)
        if (!gsel[gi] && (best < 0 || after(gscore[gi], gi, gscore[best], best)))
          best = gi;
      gsel[best] = 1;
    }
    for (int e = 0; e < E; ++e)
      if (!gsel[e / per]) choice[e] = -INFINITY;
    uint32_t *it = indices + (int64_t)t * k;
    float *wt = weights + (int64_t)t * k;
    unsigned char taken[4096];
    memset(taken, 0, (size_t)E);
    for (int s = 0; s < k; ++s) {
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!taken[e] && (best < 0 || after(choice[e], e, choice[best], best)))
          best = e;
      taken[best] = 1;
      it[k - 1 - s] = (uint32_t)best;
    }
    for (int j = 0; j < k; ++j) wt[j] = scores[it[j]];
    if (norm) {
      float sum = wt[0];
      for (int j = 1; j < k; ++j) sum = sum + wt[j];
      float denom = sum + 0x1.79ca1p-67f; /* float32(1e-20) */
      for (int j = 0; j < k; ++j) wt[j] = wt[j] / denom;
    }
    for (int j = 0; j < k; ++j) wt[j] = wt[j] * scale;
  }
  return 0;
}

/*
 * Dispatch contract (the reference has no explicit permutation; it compacts
 * first occurrences, expert_ssd.py:162-170): a stable counting sort of the
 * route slots s = t*k + j by expert id.
 *   counts[e]  = #slots routed to e
 *   offsets[e] = sum of counts below e, offsets[E] = M*k
 *   perm[offsets[e] + r] = the r-th slot (increasing) routed to e
 */
void oracle_dispatch(const uint32_t *indices, int64_t slots, int E,
                     int32_t *counts, int32_t *offsets, int32_t *perm) {
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t s = 0; s < slots; ++s) counts[indices[s]]++;
  offsets[0] = 0;
  for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t fill[4096];
  for (int e = 0; e < E; ++e) fill[e] = offsets[e];
  for (int64_t s = 0; s < slots; ++s) perm[fill[indices[s]]++] = (int32_t)s;
}
