// Fused decode MoE block for 1..4 tokens: one persistent cooperative kernel.
//
// Every CTA (one per SM) runs a single bulk-copy ring: one producer warp
// issues the copies, eight consumer warps work on every stage.  The ring
// carries, in this order, everything the CTA reads from HBM:
//
//   phase 1  router rows (f32)      -> logits            (moe.py:37-38)
//            shared gate/up rows    -> shared act        (layers.py:160-171)
//            routed gate/up rows    -> routed act        (expert_ssd.py:96-107)
//   phase 2  shared down rows       -> shared y          (layers.py:160-171)
//            routed down rows       -> routed y          (expert_ssd.py:96-107)
//            then the weighted merge of this CTA's output rows (moe.py:199-201)
//
// Two grid-wide counters order the phases.  The producer warp of every CTA
// adds its router rows to `logits` once its consumers wrote them, waits until
// all E logits exist and computes the routing (sigmoid, bias, group-limited
// top-k, weights, the stable dispatch of the M*k routes) itself, so no CTA
// waits for another one's tables.  Each CTA adds one to `act` when its
// phase-1 results are written; consumers wait for all CTAs before the down
// phase while the producer keeps streaming down weights into the ring.  The
// last CTA to finish resets the counters, so every call starts from zero.
// All CTAs must be resident at once: the kernel is launched cooperatively
// with one CTA per SM, and every wait gives up after kWaitLimitNs with a
// status word.
//
// Work split: router rows e = b, b+P, ...; gate/up chunks j = b, b+P, ...
// over the shared chunks followed by the routed chunks of the active experts
// (expert-major); down rows [r_lo, r_hi) of CTA b for the shared expert and
// every active expert, so the merge of those rows is local and in route order.
//
// Latency: with the ring streaming, one L2 round trip costs microseconds, so
// every global read off the ring (x, bias, logits, act) is issued as one batch
// of independent loads, and the dot products interleave 4-8 independent
// accumulation chains per thread (two consumer warps per SM sub-partition
// cannot hide dependent-FMA latency otherwise).
//
// Arithmetic.  Router: the canonical fp32 order (32 lane partials, butterfly)
// that the CPU checker restates, so routing is bit-exact.  MXFP4 rows: E2M1
// pairs -> f16x2 (cvt.rn.f16x2.e2m1x2, exact) times f16 activations with
// packed f16x2 FMAs over 8-product chains, each chain's two halves summed in
// f32 and scaled by the E8M0 group scale in f32.  Activation rows are scaled
// by a power of two so that max|v| < 2^8 (chains stay below 2^14, no f16
// overflow) and the scale is undone exactly in f32.  bf16 rows (shared
// expert): mixed fma.rn.f32.bf16 into f32.
#pragma once
#include "decode_kernels.cuh"
#include "pipeline.cuh"

namespace lg {
namespace layer {

constexpr int kWarps = 8;                  // consumer warps; all of them work on every stage
constexpr int kConsumers = kWarps * 32;
constexpr int kCtl = 4;                    // control warps: copy issue, routing (one token each)
constexpr int kThreads = kConsumers + kCtl * 32;
constexpr int kBarCons = 1;                // named barrier over the consumer warps
constexpr int kBarCtl = 2;                 // named barrier over the control warps
constexpr int kNRed = 4;                   // cross-warp reduction buffers
constexpr int kMaxStages = 8;
constexpr int kGuRows = 8;      // routed gate/up rows per chunk (one token: one row pair per warp)
constexpr int kXcg = 4;         // one token: column groups per lane (d <= 32 * 32 * kXcg)
static_assert(kGuRows == kWarps, "one token: each consumer warp owns one row pair of a chunk");
constexpr int kShGuRows = 2;    // shared gate/up rows per chunk
constexpr int kShDnRows = 8;    // shared down rows per chunk (warp per row)
constexpr int kDnRowsMax = 32;  // routed down rows per chunk (16 row sets x 2)
constexpr int kMaxRoutes = 32;  // M * k
constexpr int kMaxExperts = 256;
constexpr int kMaxGroups = 32;

// status sites (LG_ERR_TIMEOUT | site << 8)
constexpr int kSiteFull = 7 << 8, kSiteEmpty = 8 << 8, kSiteDrain = 9 << 8;
constexpr int kSiteLogits = 10 << 8, kSiteAct = 11 << 8, kSiteTable = 12 << 8;
constexpr int kSiteSync = 13 << 8;   // with LG_ERR_WORKSPACE: grid counters were not zero on entry
constexpr int kSiteRed = 14 << 8;
constexpr int kSiteRoute = 15 << 8;  // with LG_ERR_INVALID_ARG: a routed expert id outside [0, E)
constexpr int kSiteActS = 16 << 8;

// grid counters in the workspace (zero between calls)
constexpr int kSyncLogits = 0;  // router rows written
constexpr int kSyncGu = 1;      // CTAs done with the routed gate/up rows
constexpr int kSyncExit = 2;    // CTAs done
constexpr int kSyncShGu = 3;    // CTAs done with the shared gate/up rows
constexpr int kSyncComb = 8;    // one token: per output block, down rows finished
constexpr int kMaxGrid = 1024;
constexpr int kSyncWords = kSyncComb + kMaxGrid;

// one token, phase 2: the CTA owns output block b (rows [b*d/P, (b+1)*d/P))
// of the shared down rows and an even slice of the routed down rows, routes
// concatenated; the last CTA to finish a block's rows combines it
constexpr int kDn1Rows = 32;  // routed down rows per chunk (two per half-warp)
constexpr int kDcg = 3;       // routed down column groups per half-warp lane (F <= 1536)
constexpr int kScg = 6;       // shared down 8-column words per lane (Fs <= 1536)
constexpr int kMaxComb = 64;  // output blocks one CTA may complete

struct Args {
  int M, d, F, Fs, E, k, G, g, norm;
  float scale, limit;
  const uint16_t* x;
  const float *Wr, *bias;
  const uint8_t *gate_p, *gate_s, *up_p, *up_s, *down_p, *down_s;
  long long gate_ps, gate_ss, up_ps, up_ss, down_ps, down_ss;
  const uint16_t *sh_gate, *sh_up, *sh_down;
  float* logits;    // [M, E] workspace
  float* w_out;     // [M, k] or NULL
  uint32_t* i_out;  // [M, k] or NULL
  uint16_t* act;    // [M*k, F] workspace, route-position order
  uint16_t* act_s;  // [M, Fs] workspace
  uint16_t* y;      // [M*k, d] workspace, slot order (one token: routed down rows)
  uint16_t* ys;     // [M, d] workspace (one token: shared down rows)
  float* out;       // [M, d]
  int* status;
  unsigned* sync;   // grid counters, kSync* below
};

// Host-computed shared-memory plan (all offsets in bytes from the dynamic base).
struct Plan {
  int stages, stage_bytes;
  int x_off;     // union: x (phase 1) / act (phase 2)
  int y_off;     // y rows [M*k + TT][rows_max] f32
  int rpr;       // router rows per router chunk
  int unit;      // down-partition row unit (rows * F/32 is a multiple of 16)
  int sub_rows;  // routed down rows per chunk
  int sh_rows;   // shared down rows per chunk
  int rows_max;  // most down rows of one CTA
  int act_off;   // one token: staged act_s [Fs] then act [rr_max][F], bf16
  int rr_max;    // one token: most routes in one CTA's routed down slice
  int yb_off;    // one token: this CTA's routed then shared down rows, bf16
  int yb_rows;   // one token: most routed down rows of one CTA
};

// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Every CTA polls the same counter word: poll slowly, or the waiters' loads
// on that one L2 line slow the weight stream sharing its L2 slice.
constexpr unsigned kPollNs = 512;
// bounded wait until *p >= target
__device__ __forceinline__ bool spin_geq(const unsigned* p, unsigned target, int* status, int site) {
  if (ld_acquire(p) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire(p) < target) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicExch(status, 6 | site);
      return false;
    }
    __nanosleep(kPollNs);
  }
  return true;
}

// try_wait that may suspend the thread in the barrier for up to `hint_ns`
// (instead of a busy poll that takes issue slots and shared-memory bandwidth
// from the warps doing work).  Keep the hint short: a waiter suspended with a
// long hint was observed to resume microseconds after the phase completed.
constexpr unsigned kSleepHintNs = 200;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* b, unsigned parity, unsigned hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait by one lane, then every lane of the warp observes the completed
// phase itself (each gets the acquire).  Returns the same result in all lanes.
__device__ __forceinline__ bool wait_warp(uint64_t* b, unsigned parity, int* status, int site, int lane) {
  unsigned good = 1u;
  if (lane == 0 && !mbar_try_wait_sleep(b, parity, kSleepHintNs)) {
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait_sleep(b, parity, kSleepHintNs)) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(status, 6 | site);
        good = 0u;
        break;
      }
    }
  }
  good = __shfl_sync(0xffffffffu, good, 0);
  // the phase is complete, so this returns at once; the cap only bounds it
  for (int n = 0; good && n < (1 << 20) && !mbar_try_wait(b, parity); ++n) {
  }
  return good != 0u;
}
// Every lane tests the phase itself (one instruction when it is already
// complete, the usual case in a deep ring); otherwise the bounded wait_warp.
__device__ __forceinline__ bool wait_all(uint64_t* b, unsigned parity, int* status, int site, int lane) {
  if (__all_sync(0xffffffffu, mbar_try_wait(b, parity))) return true;
  return wait_warp(b, parity, status, site, lane);
}

__device__ __forceinline__ uint4 lds128(const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const unsigned char* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ unsigned fold4(const uint4& v) { return v.x ^ v.y ^ v.z ^ v.w; }
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
// volatile: keeps the conversions in program order, so the scheduler does not
// hoist every row's converted weights at once (which spills registers)
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm volatile("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
               "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
               "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
               "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
               : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
               : "r"(w));
}
// Same conversion, free for the scheduler to interleave with the FMA pipe
// (used where the working set is small enough not to spill).
__device__ __forceinline__ void e2m1x8_to_f16x2_nv(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}
__device__ __forceinline__ float f16x2_sum(uint32_t h) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  return __fadd_rn(f.x, f.y);
}

// NR x NC MXFP4 groups w[r][c] (16 packed bytes = 32 E2M1 values each)
// against TP activation rows: part[r][c][q] = the 32 products of group (r, c)
// with activation row q, column group c.  Activation words (8 f16) of row q,
// group c are at x[c][q] + wq * xs, wq = 0..3.  Each (r, c, q) accumulates in
// two f16x2 chains of 8 products (words 0-1, words 2-3); all NR*NC*TP chains
// are interleaved.
template <int NR, int NC, int TP>
__device__ __forceinline__ void mx_dot(const uint4 (&w)[NR][NC], const uint4* const (&x)[NC][TP], int xs,
                                       float (&part)[NR][NC][TP]) {
  uint32_t ch[NR][NC][TP][2];
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int q = 0; q < TP; ++q) { ch[r][c][q][0] = 0u; ch[r][c][q][1] = 0u; }
#pragma unroll
  for (int wq = 0; wq < 4; ++wq) {
    uint4 xv[NC][TP];
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int q = 0; q < TP; ++q) xv[c][q] = x[c][q][wq * xs];
    uint32_t h[NR][NC][4];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int c = 0; c < NC; ++c) e2m1x8_to_f16x2(word_of(w[r][c], wq), h[r][c]);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
          for (int q = 0; q < TP; ++q)
            ch[r][c][q][wq >> 1] = hfma2(h[r][c][j], word_of(xv[c][q], j), ch[r][c][q][wq >> 1]);
  }
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int q = 0; q < TP; ++q) part[r][c][q] = __fadd_rn(f16x2_sum(ch[r][c][q][0]), f16x2_sum(ch[r][c][q][1]));
}

// NV bf16 groups w[v] (4 uint4 = 32 values each) against TP bf16 activation
// groups (words at x[q] + wq * xs): part[v][q], one f32 chain per word.
template <int NV, int TP>
__device__ __forceinline__ void bf_dot(const uint4 (&w)[NV][4], const uint4* const (&x)[TP], int xs,
                                       float (&part)[NV][TP]) {
  float ch[NV][4][TP];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int wq = 0; wq < 4; ++wq)
#pragma unroll
      for (int q = 0; q < TP; ++q) ch[v][wq][q] = 0.f;
  uint4 xv[4][TP];
#pragma unroll
  for (int wq = 0; wq < 4; ++wq)
#pragma unroll
    for (int q = 0; q < TP; ++q) xv[wq][q] = x[q][wq * xs];
#pragma unroll
  for (int e = 0; e < 4; ++e)
#pragma unroll
    for (int wq = 0; wq < 4; ++wq)
#pragma unroll
      for (int v = 0; v < NV; ++v)
#pragma unroll
        for (int q = 0; q < TP; ++q)
          ch[v][wq][q] = fma_bf16(word_of(w[v][wq], e), word_of(xv[wq][q], e), ch[v][wq][q]);
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int q = 0; q < TP; ++q)
      part[v][q] = __fadd_rn(__fadd_rn(ch[v][0][q], ch[v][1][q]), __fadd_rn(ch[v][2][q], ch[v][3][q]));
}

// mx_dot with the activation words in registers: groups w[r][C0 + c] against
// xv[C0 + c][wq] (one activation row), same chains and order as mx_dot.
template <int NR, int C0, int NC, int NW>
__device__ __forceinline__ void mx_dot_reg(const uint4 (&w)[NR][NW], const uint4 (&xv)[NW][4], float (&part)[NR][NC]) {
  uint32_t ch[NR][NC][2];
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c) { ch[r][c][0] = 0u; ch[r][c][1] = 0u; }
#pragma unroll
  for (int wq = 0; wq < 4; ++wq) {
    uint32_t h[NR][NC][4];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int c = 0; c < NC; ++c) e2m1x8_to_f16x2_nv(word_of(w[r][C0 + c], wq), h[r][c]);
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int c = 0; c < NC; ++c)
          ch[r][c][wq >> 1] = hfma2(h[r][c][e], word_of(xv[C0 + c][wq], e), ch[r][c][wq >> 1]);
  }
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c) part[r][c] = __fadd_rn(f16x2_sum(ch[r][c][0]), f16x2_sum(ch[r][c][1]));
}

// Reduce V values over SEG lanes (aligned segments of a warp) by halving:
// afterwards lane l holds in v[0] the segment total of value index
// (l % SEG) / (SEG / V).  Deterministic order.
template <int N, int O>
struct Halve {
  template <int V>
  static __device__ __forceinline__ void run(float (&v)[V], int lane) {
    if constexpr (O >= 1) {
      if constexpr (N > 1) {
        const bool upper = (lane & O) != 0;
#pragma unroll
        for (int i = 0; i < N / 2; ++i) {
          const float send = upper ? v[i] : v[i + N / 2];
          const float keep = upper ? v[i + N / 2] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, O));
        }
        Halve<N / 2, O / 2>::run(v, lane);
      } else {
        v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], O));
        Halve<1, O / 2>::run(v, lane);
      }
    }
  }
};
template <int V, int SEG>
__device__ __forceinline__ void reduce_scatter(float (&v)[V], int lane) {
  static_assert(V <= SEG && (V & (V - 1)) == 0, "V must be a power of two <= SEG");
  Halve<V, SEG / 2>::run(v, lane);
}

// power-of-two activation scale: max|v| * 2^-shift < 2^8
__device__ __forceinline__ int act_shift(float amax) {
  const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127;
  if (amax == 0.0f) return 0;
  const int s = e - 7;
  return s < -120 ? -120 : (s > 120 ? 120 : s);
}
__device__ __forceinline__ float absmax8_bf16(const uint4& u) {
  float m = fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y))));
  return fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
}
__device__ __forceinline__ uint4 bf16x8_to_f16x8_scaled(const uint4& u, float s) {
  return make_uint4(bf16x2_to_f16x2_scaled(u.x, s), bf16x2_to_f16x2_scaled(u.y, s), bf16x2_to_f16x2_scaled(u.z, s),
                    bf16x2_to_f16x2_scaled(u.w, s));
}

// ---------------------------------------------------------------------------
// Routing of one CTA, computed by the producer warp from the global logits.
// Restates TopKRouter.__call__ (moe.py:39-62) with the stable (value, index)
// order of the CPU checker; results go to shared memory.
struct alignas(16) Tables {
  int ae[kMaxRoutes];    // active experts, ascending id
  int ap0[kMaxRoutes];   // first route position of active expert
  int an[kMaxRoutes];    // routes of active expert
  int perm[kMaxRoutes];  // route position -> slot t*k + j
  int sel[kMaxRoutes];   // slot -> expert
  float w[kMaxRoutes];   // slot -> route weight
  int n_active;
  float bias[kMaxExperts];
  float sc[kDecodeMaxTokens][kMaxExperts];  // sigmoid scores, per token
  alignas(16) float ch[kDecodeMaxTokens][kMaxExperts];  // choice scores (masked), per token (16-byte rows)
  int ix[kDecodeMaxTokens][kMaxExperts];    // candidate indices, per token
};

// Top two (value, index) pairs under the stable order: merge (w1, j1, w2, j2)
// into (v1, i1, v2, i2).
__device__ __forceinline__ void top2_merge(float& v1, int& i1, float& v2, int& i2, float w1, int j1, float w2, int j2) {
  if (after(w1, j1, v1, i1)) {
    if (after(v1, i1, w2, j2)) { v2 = v1; i2 = i1; } else { v2 = w2; i2 = j2; }
    v1 = w1; i1 = j1;
  } else if (after(w1, j1, v2, i2)) {
    v2 = w1; i2 = j1;
  }
}

// Routing of token t by one warp.  Lane l owns the contiguous experts
// l*V .. l*V+V-1 (V = E/32) in registers.  Same results as the checker's
// sequential scans for the stable (value, index) order (for non-NaN scores):
// group top-2 by a merge over the group's lanes, kept groups by rank, then k
// rounds of a warp argmax done with two redux.sync reductions (largest score
// key, then largest index among equal keys).
// Returns false (doing nothing) for E % 32 != 0, E > 256, or groups that do
// not span a power-of-two number of whole lanes.
__device__ __forceinline__ bool warp_routing_ok(const Args& a) {
  const int E = a.E, per = E / a.G, V = E >> 5;
  if ((E & 31) || V < 1 || V > kMaxExperts / 32) return false;
  const int L = per / V;  // lanes per group
  return a.g >= a.G || (per % V == 0 && L >= 1 && (L & (L - 1)) == 0);
}

// order-preserving key of a choice score (0 = no candidate, NaN lowest)
__device__ __forceinline__ unsigned score_key(float v) {
  const unsigned u = __float_as_uint(v);
  if (v != v) return 1u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __noinline__ bool route_token_warp(const Args& a, Tables& T, int t, int lane, bool write_out) {
  if (!warp_routing_ok(a)) return false;
  constexpr int VM = kMaxExperts / 32;
  const int E = a.E, G = a.G, k = a.k, per = E / G, V = E >> 5;
  const bool grouped = a.g < G;
  const int L = per / V;  // lanes per group
  float* sc = T.sc[t];
  const float ninf = __uint_as_float(0xff800000u);
  const int e0 = lane * V;
  float cv[VM];
  {
    float lg[VM];
#pragma unroll
    for (int q = 0; q < VM; ++q) lg[q] = q < V ? __ldcg(a.logits + static_cast<size_t>(t) * E + e0 + q) : 0.f;
#pragma unroll
    for (int q = 0; q < VM; ++q) {
      cv[q] = ninf;
      if (q < V) {
        const float sg = own_sigmoidf(lg[q]);
        sc[e0 + q] = sg;
        cv[q] = __fadd_rn(sg, T.bias[e0 + q]);
      }
    }
  }
  if (grouped) {
    // group score: the two best of the group's experts, summed (second + best)
    float v1 = 0.f, v2 = 0.f;
    int i1 = -1, i2 = -1;
#pragma unroll
    for (int q = 0; q < VM; ++q)
      if (q < V) top2_merge(v1, i1, v2, i2, cv[q], e0 + q, 0.f, -1);
#pragma unroll 1
    for (int off = 1; off < L; off <<= 1) {
      const float w1 = __shfl_xor_sync(0xffffffffu, v1, off), w2 = __shfl_xor_sync(0xffffffffu, v2, off);
      const int j1 = __shfl_xor_sync(0xffffffffu, i1, off), j2 = __shfl_xor_sync(0xffffffffu, i2, off);
      top2_merge(v1, i1, v2, i2, w1, j1, w2, j2);
    }
    const float gsc = __fadd_rn(v2, v1);
    const int gi = lane / L;
    int rank = 0;
#pragma unroll 1
    for (int gj = 0; gj < G; ++gj) {
      const float sj = __shfl_sync(0xffffffffu, gsc, gj * L);
      rank += after(sj, gj, gsc, gi) ? 1 : 0;
    }
    if (rank >= a.g) {
#pragma unroll
      for (int q = 0; q < VM; ++q) cv[q] = ninf;
    }
  }
  __syncwarp();  // sigmoid scores in shared memory for the weight lookup
  // top-k: round s takes the best remaining candidate of the warp
  unsigned taken = 0u;
  float wj = 0.f;
#pragma unroll 1
  for (int s = 0; s < k; ++s) {
    float bv = 0.f;
    int bi = -1;
#pragma unroll
    for (int q = 0; q < VM; ++q)
      if (q < V && !((taken >> q) & 1u) && after(cv[q], e0 + q, bv, bi)) {
        bv = cv[q];
        bi = e0 + q;
      }
    const unsigned key = bi < 0 ? 0u : score_key(bv);
    const unsigned m = __reduce_max_sync(0xffffffffu, key);
    const unsigned wi = __reduce_max_sync(0xffffffffu, key == m && bi >= 0 ? static_cast<unsigned>(bi) + 1u : 0u);
    const int i = static_cast<int>(wi) - 1;
    if (i >= 0 && i - e0 >= 0 && i - e0 < V) taken |= 1u << (i - e0);
    if (lane == k - 1 - s) wj = i >= 0 ? sc[i] : 0.f;
    if (lane == 0) T.sel[t * k + (k - 1 - s)] = i;
  }
  // weights: sequential sum over the k routes in output order
  float denom = 1.f;
  if (a.norm) {
    float sum = __shfl_sync(0xffffffffu, wj, 0);
#pragma unroll 1
    for (int j = 1; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wj, j));
    denom = __fadd_rn(sum, 0x1.79ca1p-67f);
  }
  __syncwarp();
  if (lane < k) {
    const float w = __fmul_rn(a.norm ? __fdiv_rn(wj, denom) : wj, a.scale);
    T.w[t * k + lane] = w;
    if (write_out && a.w_out) a.w_out[static_cast<size_t>(t) * k + lane] = w;
    if (write_out && a.i_out) a.i_out[static_cast<size_t>(t) * k + lane] = static_cast<uint32_t>(T.sel[t * k + lane]);
  }
  __syncwarp();
  return true;
}

// Routing of token t by the kCtl control warps, one thread per expert
// (E <= kCtl*32, groups of a power-of-two size <= 32 experts).  Same results
// as the checker's sequential scans for the stable (value, index) order:
// group score = second + best of the group (a merge over the group's lanes),
// a group is kept when fewer than topk_group groups come after it, and expert
// e is chosen in place k-1-r when r < k candidates come after it.  Named
// barrier kBarCtl separates the steps; every control thread must call this.
__device__ __forceinline__ bool block_routing_ok(const Args& a) {
  const int per = a.E / a.G;
  return a.E <= kCtl * 32 && a.E % a.G == 0 && per <= 32 && (per & (per - 1)) == 0 && a.k <= kMaxRoutes;
}
__device__ __forceinline__ void route_token_block(const Args& a, Tables& T, int t, int tid, bool write_out) {
  const int E = a.E, G = a.G, k = a.k, per = E / G;
  const bool grouped = a.g < G;
  const bool live = tid < E;
  const float ninf = __uint_as_float(0xff800000u);
  float* sc = T.sc[t];
  float* cm = T.ch[t];                          // masked choice scores
  float* gs = reinterpret_cast<float*>(T.ix[t]);  // group scores
  const int e = tid;
  float c = ninf;
  if (live) {
    const float sg = own_sigmoidf(__ldcg(a.logits + static_cast<size_t>(t) * E + e));
    sc[e] = sg;
    c = __fadd_rn(sg, T.bias[e]);
  }
  if (grouped) {
    // best two of the group: merge over the group's `per` lanes
    float v1 = live ? c : 0.f, v2 = 0.f;
    int i1 = live ? e : -1, i2 = -1;
#pragma unroll 1
    for (int off = 1; off < per; off <<= 1) {
      const float w1 = __shfl_xor_sync(0xffffffffu, v1, off), w2 = __shfl_xor_sync(0xffffffffu, v2, off);
      const int j1 = __shfl_xor_sync(0xffffffffu, i1, off), j2 = __shfl_xor_sync(0xffffffffu, i2, off);
      top2_merge(v1, i1, v2, i2, w1, j1, w2, j2);
    }
    if (live && (e % per) == 0) gs[e / per] = __fadd_rn(v2, v1);
    named_sync(kBarCtl, kCtl * 32);
    if (live) {
      const int gi = e / per;
      const float mine = gs[gi];
      int rank = 0;
#pragma unroll 4
      for (int gj = 0; gj < G; ++gj) {
        const float v = gs[gj];
        rank += (v > mine) | ((v == mine) & (gj > gi));  // after(v, gj, mine, gi)
      }
      if (rank >= a.g) c = ninf;
    }
  }
  if (live) cm[e] = c;
  named_sync(kBarCtl, kCtl * 32);
  if (live) {
    // candidates after this one, four per 16-byte broadcast load
    int rank = 0;
    const float4* cm4 = reinterpret_cast<const float4*>(cm);
#pragma unroll 8
    for (int q = 0; q < (E >> 2); ++q) {
      const float4 v = cm4[q];
      const int ej = 4 * q;
      rank += (v.x > c) | ((v.x == c) & (ej > e));
      rank += (v.y > c) | ((v.y == c) & (ej + 1 > e));
      rank += (v.z > c) | ((v.z == c) & (ej + 2 > e));
      rank += (v.w > c) | ((v.w == c) & (ej + 3 > e));
    }
    for (int ej = E & ~3; ej < E; ++ej) rank += (cm[ej] > c) | ((cm[ej] == c) & (ej > e));
    if (rank < k) T.sel[t * k + (k - 1 - rank)] = e;
  }
  named_sync(kBarCtl, kCtl * 32);
  // weights: sequential sum over the k routes in output order
  if (tid < k) {
    const float wj = sc[T.sel[t * k + tid]];
    float denom = 1.f;
    if (a.norm) {
      float sum = sc[T.sel[t * k]];
      for (int j = 1; j < k; ++j) sum = __fadd_rn(sum, sc[T.sel[t * k + j]]);
      denom = __fadd_rn(sum, 0x1.79ca1p-67f);
    }
    const float w = __fmul_rn(a.norm ? __fdiv_rn(wj, denom) : wj, a.scale);
    T.w[t * k + tid] = w;
    if (write_out && a.w_out) a.w_out[static_cast<size_t>(t) * k + tid] = w;
    if (write_out && a.i_out) a.i_out[static_cast<size_t>(t) * k + tid] = static_cast<uint32_t>(T.sel[t * k + tid]);
  }
  named_sync(kBarCtl, kCtl * 32);
}

// Same routing by one warp for all tokens, scanning shared memory: the path
// for group sizes that do not divide 32.
__device__ __noinline__ void route_tokens_scan(const Args& a, Tables& T, int lane, bool write_out) {
  const int E = a.E, G = a.G, k = a.k, per = E / G;
  const float ninf = __uint_as_float(0xff800000u);
  for (int t = 0; t < a.M; ++t) {
    for (int e = lane; e < E; e += 32) {
      const float s = own_sigmoidf(__ldcg(a.logits + static_cast<size_t>(t) * E + e));
      T.sc[0][e] = s;
      T.ch[0][e] = __fadd_rn(s, T.bias[e]);
    }
    __syncwarp();
    if (a.g < G) {
      float gsc = 0.f;
      if (lane < G) {
        int b1 = -1, b2 = -1;
        for (int j = 0; j < per; ++j) {
          const int e = lane * per + j;
          if (b1 < 0 || after(T.ch[0][e], e, T.ch[0][b1], b1)) { b2 = b1; b1 = e; }
          else if (b2 < 0 || after(T.ch[0][e], e, T.ch[0][b2], b2)) { b2 = e; }
        }
        gsc = __fadd_rn(T.ch[0][b2], T.ch[0][b1]);
      }
      bool kept = false;
      for (int s = 0; s < a.g; ++s) {
        float v = gsc;
        int i = (lane < G && !kept) ? lane : -1;
        warp_best(v, i);
        if (lane == i) kept = true;
      }
      const unsigned keep = __ballot_sync(0xffffffffu, kept);
      __syncwarp();
      for (int e = lane; e < E; e += 32)
        if (!((keep >> (e / per)) & 1u)) T.ch[0][e] = ninf;
      __syncwarp();
    }
    unsigned taken = 0u;
    for (int s = 0; s < k; ++s) {
      float v = 0.f;
      int i = -1;
      for (int q = 0; lane + 32 * q < E; ++q) {
        const int e = lane + 32 * q;
        if (!((taken >> q) & 1u) && (i < 0 || after(T.ch[0][e], e, v, i))) { v = T.ch[0][e]; i = e; }
      }
      warp_best(v, i);
      if (i >= 0 && (i & 31) == lane) taken |= 1u << (i >> 5);
      if (lane == 0) T.sel[t * k + (k - 1 - s)] = i;
    }
    __syncwarp();
    const float wj = lane < k ? T.sc[0][T.sel[t * k + lane]] : 0.f;
    float denom = 1.f;
    if (a.norm) {
      float sum = __shfl_sync(0xffffffffu, wj, 0);
      for (int j = 1; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wj, j));
      denom = __fadd_rn(sum, 0x1.79ca1p-67f);
    }
    if (lane < k) {
      const float w = __fmul_rn(a.norm ? __fdiv_rn(wj, denom) : wj, a.scale);
      T.w[t * k + lane] = w;
      if (write_out && a.w_out) a.w_out[static_cast<size_t>(t) * k + lane] = w;
      if (write_out && a.i_out) a.i_out[static_cast<size_t>(t) * k + lane] = static_cast<uint32_t>(T.sel[t * k + lane]);
    }
    __syncwarp();
  }
}

// Stable counting sort of the S = M*k route slots by expert (S <= 32: lane =
// slot): route positions, active experts in ascending id, their first
// position and route count.
__device__ __forceinline__ void dispatch_routes(const Args& a, Tables& T, int lane) {
  const int S = a.M * a.k;
  // every selected expert must be a real one before any copy uses it
  const bool bad = __any_sync(0xffffffffu, lane < S && (T.sel[lane] < 0 || T.sel[lane] >= a.E));
  if (bad) {
    if (lane == 0) {
      atomicExch(a.status, 1 | kSiteRoute);
      T.n_active = 0;
    }
    __syncwarp();
    return;
  }
  const bool valid = lane < S;
  const int e = valid ? T.sel[lane] : 0x40000000 + lane;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  int below = 0, act_below = 0;
  const unsigned leaders = __ballot_sync(0xffffffffu, valid && rank == 0);
  for (int j = 0; j < S; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e, j);
    below += ej < e;
    act_below += ((leaders >> j) & 1u) && ej < e;
  }
  if (valid) {
    T.perm[below + rank] = lane;
    if (rank == 0) {
      T.ae[act_below] = e;
      T.ap0[act_below] = below;
      T.an[act_below] = __popc(peers);
    }
  }
  if (lane == 0) T.n_active = __popc(leaders);
  __syncwarp();
}

// Down rows [r_lo, r_hi) of CTA b: the d rows in units of pl.unit, split
// evenly over the P CTAs.
struct DownRange {
  int r_lo, r_hi, rows, n_sdp, n_sub;
  __device__ __forceinline__ DownRange(const Args& a, const Plan& pl, int b, int P) {
    const int nunits = a.d / pl.unit;
    r_lo = pl.unit * static_cast<int>((static_cast<long long>(b) * nunits) / P);
    r_hi = pl.unit * static_cast<int>((static_cast<long long>(b + 1) * nunits) / P);
    rows = r_hi - r_lo;
    n_sdp = a.Fs > 0 ? (rows + pl.sh_rows - 1) / pl.sh_rows : 0;
    n_sub = (rows + pl.sub_rows - 1) / pl.sub_rows;
  }
};

// One token: CTA b's shared down rows [sr_lo, sr_hi) (its output block) and
// routed down rows [u_lo, u_hi) of the routes concatenated (route p has rows
// [p*d, (p+1)*d)), split evenly in units of pl.unit rows.
// (32-bit arithmetic: d <= 4096, P <= kMaxGrid, M*k*d/unit <= 2^17, so every
// product stays below 2^31.)
struct Down1 {
  int sr_lo, sr_hi, u_lo, u_hi;
  __device__ __forceinline__ Down1(const Args& a, const Plan& pl, int b, int P) {
    const unsigned d = a.d, p = P, nu = static_cast<unsigned>(a.M * a.k) * d / pl.unit;
    sr_lo = static_cast<int>(b * d / p);
    sr_hi = static_cast<int>((b + 1) * d / p);
    u_lo = pl.unit * static_cast<int>(b * nu / p);
    u_hi = pl.unit * static_cast<int>((b + 1) * nu / p);
  }
};
// output block holding row r: the largest c with c*d/P <= r
__device__ __forceinline__ int out_block(int r, int d, int P) {
  return static_cast<int>((static_cast<unsigned>(r + 1) * P - 1u) / static_cast<unsigned>(d));
}
__device__ __forceinline__ int block_lo(int c, int d, int P) {
  return static_cast<int>(static_cast<unsigned>(c) * d / static_cast<unsigned>(P));
}

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(kThreads, 1) layer_kernel(Args a, Plan pl) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ __align__(8) uint64_t tbl;     // routing tables ready
  __shared__ __align__(8) uint64_t lgdone;  // this CTA's logits written
  __shared__ __align__(8) uint64_t xbar;    // x copied in
  __shared__ __align__(8) uint64_t abar;    // act / act_s copied in (one token: act)
  __shared__ __align__(8) uint64_t sbar;    // one token: act_s copied in
  __shared__ Tables T;
  __shared__ float red[kNRed][kWarps][32];
  __shared__ int red_cnt[kNRed], red_gen[kNRed];
  __shared__ int s_go;
  __shared__ unsigned rel_sink[kConsumers];
  __shared__ float tok_mult[TT], tok_inv[TT];
  __shared__ float rscale[kMaxRoutes], rinv[kMaxRoutes];
  __shared__ int s_nact, s_fail, s_afail;
  __shared__ int s_ncomb, s_comb[kMaxComb], s_ncb, s_cb[kMaxComb], s_cr[kMaxComb];

  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, b = blockIdx.x;
  const int M = a.M, d = a.d, F = a.F, Fs = a.Fs, E = a.E, k = a.k;
  const int G = d >> 5, G2 = F >> 5, G2s = Fs >> 5;
  const int S = pl.stages, R = M * k;
  constexpr int GR = kGuRows;
  const int nrb = F / GR, n_sh = Fs / kShGuRows;
  // chunk sequence: router rows, shared gate/up, routed gate/up, shared down,
  // routed down (expert-major); the routed parts follow the routing tables
  const int nrr = b < E ? (E - b + P - 1) / P : 0;
  const int n_rt = (nrr + pl.rpr - 1) / pl.rpr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kWarps); }
    mbar_init(&tbl, 1);
    mbar_init(&lgdone, kWarps * (n_rt > 0 ? n_rt : 1));
    mbar_init(&xbar, 1);
    mbar_init(&abar, 1);
    mbar_init(&sbar, 1);
    mbar_fence_init();
    T.n_active = 0;
    s_afail = 0;
  }
  if (threadIdx.x < kNRed) { red_cnt[threadIdx.x] = 0; red_gen[threadIdx.x] = 0; }
  __syncthreads();

  // ============================ control warps ============================
  // warp kWarps issues the copies (lane 0) and builds the dispatch; the four
  // control warps route one token each
  if (warp_id >= kWarps) {
    const int cw = warp_id - kWarps;
    bool ok = true;
    int it = 0;
    bool signaled = n_rt == 0;
    // this CTA's logits are written: publish them to the grid
    auto signal_logits = [&]() {
      __threadfence();
      atomicAdd(a.sync + kSyncLogits, static_cast<unsigned>(nrr));
      signaled = true;
    };
    // lane 0: bounded wait until stage `it` is free (its previous chunk
    // released by every consumer warp), publishing the logits meanwhile
    auto stage_free = [&]() -> bool {
      if (!ok) return false;
      if (it < S) return true;
      const unsigned par = ((it / S) - 1) & 1;
      unsigned long long t0 = 0;
      while (!mbar_try_wait_sleep(&empty[it % S], par, kSleepHintNs)) {
        if (!signaled && mbar_try_wait(&lgdone, 0)) signal_logits();
        const unsigned long long t = globaltimer_ns();
        if (!t0) t0 = t;
        else if (t - t0 > kWaitLimitNs) {
          atomicExch(a.status, 6 | kSiteEmpty);
          ok = false;
          return false;
        }
      }
      return true;
    };
    if (cw == 0 && lane == 0) {
      // the tokens' hidden states first (bf16 rows, contiguous)
      mbar_arrive_expect_tx(&xbar, static_cast<unsigned>(M) * d * 2u);
      bulk_g2s(smem + pl.x_off + static_cast<size_t>(TT) * d * 2, a.x, static_cast<unsigned>(M) * d * 2u, &xbar);
      const unsigned rrow = static_cast<unsigned>(d) * 4u;
      for (int rc = 0; rc < n_rt; ++rc, ++it) {
        if (!stage_free()) continue;
        const int r0 = rc * pl.rpr, nr = min(pl.rpr, nrr - r0);
        unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[it % S], rrow * nr);
        for (int r = 0; r < nr; ++r)
          bulk_g2s(st + r * rrow, a.Wr + static_cast<size_t>(b + P * (r0 + r)) * d, rrow, &full[it % S]);
      }
      const unsigned shb = kShGuRows * static_cast<unsigned>(d) * 2u;
      for (int j = b; j < n_sh; j += P, ++it) {
        if (!stage_free()) continue;
        unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[it % S], 2 * shb);
        bulk_g2s(st, a.sh_gate + static_cast<size_t>(j) * kShGuRows * d, shb, &full[it % S]);
        bulk_g2s(st + shb, a.sh_up + static_cast<size_t>(j) * kShGuRows * d, shb, &full[it % S]);
      }
      // publish this CTA's logits, then wait for every logit row
      if (ok && !signaled) {
        if (mbar_wait(&lgdone, 0, a.status, kSiteLogits)) signal_logits();
        else ok = false;
      }
      s_go = (ok && spin_geq(a.sync + kSyncLogits, static_cast<unsigned>(E), a.status, kSiteLogits)) ? 1 : 0;
    }
    if (cw == 1) {  // score-correction bias, one batch of loads
      float bv[kMaxExperts / 32];
#pragma unroll
      for (int q = 0; q < kMaxExperts / 32; ++q) bv[q] = lane + 32 * q < E ? a.bias[lane + 32 * q] : 0.f;
#pragma unroll
      for (int q = 0; q < kMaxExperts / 32; ++q) T.bias[lane + 32 * q] = bv[q];
    }
    named_sync(kBarCtl, kCtl * 32);
    const bool go = s_go != 0;
    const bool blk = block_routing_ok(a), scan = !blk && !warp_routing_ok(a);
    if (go) {
      // the logits were acquired by the counter poll before the barrier and
      // are read through L2 (ld.global.cg)
      if (blk) {
        for (int t = 0; t < M; ++t) route_token_block(a, T, t, cw * 32 + lane, b == 0);
      } else if (!scan) {
        if (cw < M) route_token_warp(a, T, cw, lane, b == 0);
      } else if (cw == 0) {
        route_tokens_scan(a, T, lane, b == 0);
      }
    }
    named_sync(kBarCtl, kCtl * 32);
    if constexpr (TT == 1) {
      // one token: control warp 1 stages act_s and this CTA's act rows once
      // every CTA has written them (plain arrive on failure, with s_afail set)
      if (cw == 1 && lane == 0) {
        const Down1 dn(a, pl, b, P);
        unsigned char* as = smem + pl.act_off;
        if (Fs > 0) {
          if (go && spin_geq(a.sync + kSyncShGu, static_cast<unsigned>(P), a.status, kSiteActS)) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(&sbar, static_cast<unsigned>(Fs) * 2u);
            bulk_g2s(as, a.act_s, static_cast<unsigned>(Fs) * 2u, &sbar);
          } else {
            s_afail = 1;
            mbar_arrive(&sbar);
          }
        }
        if (dn.u_hi > dn.u_lo) {
          const int p_lo = dn.u_lo / d, np = (dn.u_hi - 1) / d - p_lo + 1;
          const unsigned bytes = static_cast<unsigned>(np) * F * 2u;
          if (go && spin_geq(a.sync + kSyncGu, static_cast<unsigned>(P), a.status, kSiteAct)) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbar_arrive_expect_tx(&abar, bytes);
            bulk_g2s(as + static_cast<size_t>(Fs) * 2, a.act + static_cast<size_t>(p_lo) * F, bytes, &abar);
          } else {
            s_afail = 1;
            mbar_arrive(&abar);
          }
        }
        // the copies land before this warp (and so the CTA) can leave
        if (Fs > 0) mbar_wait(&sbar, 0, a.status, kSiteDrain);
        if (dn.u_hi > dn.u_lo) mbar_wait(&abar, 0, a.status, kSiteDrain);
      }
    }
    if (cw != 0) return;
    if (go) dispatch_routes(a, T, lane);
    else ok = false;
    __syncwarp();
    if (lane == 0) mbar_arrive(&tbl);
    if (lane == 0) {
      const int n_r = T.n_active * nrb;
      const unsigned pk = GR * static_cast<unsigned>(d) / 2u, sk = GR * static_cast<unsigned>(G);
      int j = b;
      while (j < n_sh) j += P;
      for (; j < n_sh + n_r; j += P, ++it) {
        if (!stage_free()) continue;
        const int jr = j - n_sh;
        const int ai = jr / nrb;
        const long long e = T.ae[ai];
        const size_t f0 = static_cast<size_t>(jr - ai * nrb) * GR;
        unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
        uint64_t* fb = &full[it % S];
        mbar_arrive_expect_tx(fb, 2 * pk + 2 * sk);
        bulk_g2s(st, a.gate_p + e * a.gate_ps + f0 * (d / 2), pk, fb);
        bulk_g2s(st + pk, a.up_p + e * a.up_ps + f0 * (d / 2), pk, fb);
        bulk_g2s(st + 2 * pk, a.gate_s + e * a.gate_ss + f0 * G, sk, fb);
        bulk_g2s(st + 2 * pk + sk, a.up_s + e * a.up_ss + f0 * G, sk, fb);
      }
      // down weights need nothing from the gate/up phase
      if constexpr (TT == 1) {
        const Down1 dn(a, pl, b, P);
        if (Fs > 0) {
          for (int r0 = dn.sr_lo; r0 < dn.sr_hi; r0 += kShDnRows, ++it) {
            if (!stage_free()) continue;
            const int nr = min(kShDnRows, dn.sr_hi - r0);
            const unsigned bytes = static_cast<unsigned>(nr) * Fs * 2u;
            unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
            mbar_arrive_expect_tx(&full[it % S], bytes);
            bulk_g2s(st, a.sh_down + static_cast<size_t>(r0) * Fs, bytes, &full[it % S]);
          }
        }
        // one token: route p is active expert p (none if the routing failed)
        for (int u = T.n_active == R ? dn.u_lo : dn.u_hi; u < dn.u_hi; ++it) {
          const int p = u / d, r0 = u - p * d, nr = min(kDn1Rows, min(dn.u_hi, (p + 1) * d) - u);
          u += nr;
          if (!stage_free()) continue;
          const long long e = T.ae[p];
          const unsigned pb = static_cast<unsigned>(nr) * (F / 2), sb = static_cast<unsigned>(nr) * G2;
          unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
          uint64_t* fb = &full[it % S];
          mbar_arrive_expect_tx(fb, pb + sb);
          bulk_g2s(st, a.down_p + e * a.down_ps + static_cast<size_t>(r0) * (F / 2), pb, fb);
          bulk_g2s(st + pb, a.down_s + e * a.down_ss + static_cast<size_t>(r0) * G2, sb, fb);
        }
      } else {
      const DownRange dr(a, pl, b, P);
      for (int pc = 0; pc < dr.n_sdp; ++pc, ++it) {
        if (!stage_free()) continue;
        const int r0 = dr.r_lo + pc * pl.sh_rows, nr = min(pl.sh_rows, dr.r_hi - r0);
        const unsigned bytes = static_cast<unsigned>(nr) * Fs * 2u;
        unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
        mbar_arrive_expect_tx(&full[it % S], bytes);
        bulk_g2s(st, a.sh_down + static_cast<size_t>(r0) * Fs, bytes, &full[it % S]);
      }
      for (int ai = 0; ai < T.n_active; ++ai) {
        const long long e = T.ae[ai];
        for (int sc = 0; sc < dr.n_sub; ++sc, ++it) {
          if (!stage_free()) continue;
          const int r0 = dr.r_lo + sc * pl.sub_rows, nr = min(pl.sub_rows, dr.r_hi - r0);
          const unsigned pb = static_cast<unsigned>(nr) * (F / 2), sb = static_cast<unsigned>(nr) * G2;
          unsigned char* st = smem + static_cast<size_t>(it % S) * pl.stage_bytes;
          uint64_t* fb = &full[it % S];
          mbar_arrive_expect_tx(fb, pb + sb);
          bulk_g2s(st, a.down_p + e * a.down_ps + static_cast<size_t>(r0) * (F / 2), pb, fb);
          bulk_g2s(st + pb, a.down_s + e * a.down_ss + static_cast<size_t>(r0) * G2, sb, fb);
        }
      }
      }
      if (!ok) {  // copies already issued land before the CTA leaves
        for (int q = (it > S ? it - S : 0); q < it; ++q)
          mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteDrain);
      }
    }
    return;
  }

  // =============================== consumers ==============================
  const int wg = warp_id, ct = threadIdx.x;
  uint4* xh = reinterpret_cast<uint4*>(smem + pl.x_off);  // f16 [t][wq][c], scaled
  uint4* xb = xh + TT * 4 * G;                             // bf16 [t][d], as copied
  float* ysm = reinterpret_cast<float*>(smem + pl.y_off);  // [R + TT][rows_max]
  const int d8 = d >> 3;

  // ---- stage x: f16 copy scaled so max|x| < 2^8, in the [t][wq][c] order ----
  bool ok = wait_warp(&xbar, 0, a.status, kSiteFull, lane);
  if (wg < M) {
    unsigned m = 0u;
#pragma unroll 1
    for (int u = lane; u < d8; u += 32) m = max(m, __float_as_uint(absmax8_bf16(xb[wg * d8 + u])));
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) {
      tok_mult[wg] = pow2i(act_shift(__uint_as_float(m)));
      tok_inv[wg] = __fdiv_rn(1.0f, tok_mult[wg]);
    }
  }
  named_sync(kBarCons, kConsumers);
#pragma unroll 1
  for (int i4 = ct; i4 < M * d8; i4 += kConsumers) {
    const int t = i4 / d8, i8 = i4 - t * d8;
    xh[(t * 4 + (i8 & 3)) * G + (i8 >> 2)] = bf16x8_to_f16x8_scaled(xb[i4], tok_inv[t]);
  }
  named_sync(kBarCons, kConsumers);

  int it = 0;
  // Cross-warp reductions without a CTA barrier: use u of buffer rb waits
  // until the previous use was finished, every warp adds its partials, and
  // the warp that arrives last finishes the chunk and frees the buffer.
  int rchunk = 0;
  auto red_begin = [&](int rb, int use) {
    if (lane == 0) {
      for (int n = 0; *reinterpret_cast<volatile int*>(&red_gen[rb]) != use; ++n) {
        if (n > (1 << 24)) {
          atomicExch(a.status, 6 | kSiteRed);
          ok = false;
          break;
        }
        __nanosleep(32);
      }
      __threadfence_block();
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  };
  auto red_arrive = [&](int rb, int use) -> bool {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&red_cnt[rb], 1) == kWarps * (use + 1) - 1;
      if (last) __threadfence_block();
    }
    return __shfl_sync(0xffffffffu, last, 0) != 0;
  };
  auto red_end = [&](int rb, int use) {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      atomicExch(&red_gen[rb], use + 1);
    }
  };
  const int c0 = ct & 127, rs = ct >> 7;  // gate/up: column-group lane, row set 0..1
  const int CI = (G + 127) >> 7;
  auto release = [&](int s) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  };
  // Early release: the slice a thread copied out of the stage must be in its
  // registers before the stage goes back to the producer.  A store of a value
  // computed from every copied word sits before the release, which orders
  // prior stores; without it the loads were observed executing after lane
  // 0's arrive (the compiler is free to sink them, they only feed registers).
  auto release_after = [&](int s, unsigned dep) {
    *reinterpret_cast<volatile unsigned*>(&rel_sink[ct]) = dep;  // volatile: never elided
    release(s);
  };

  // ---------------------------- phase 1 ----------------------------
  // router rows: warp -> row, canonical lane partials + butterfly
  for (int rc = 0; rc < n_rt; ++rc, ++it) {
    const int s = it % S;
    if (ok) ok = wait_warp(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
    const int r0 = rc * pl.rpr, nr = min(pl.rpr, nrr - r0);
    const float* ws = reinterpret_cast<const float*>(smem + static_cast<size_t>(s) * pl.stage_bytes);
    for (int r = wg; ok && r < nr; r += kWarps) {
      const float* wrow = ws + static_cast<size_t>(r) * d;
      float acc[TT];
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[t] = 0.f;
      for (int c8 = lane; c8 < (d >> 3); c8 += 32) {
        const float4 w0 = *reinterpret_cast<const float4*>(wrow + 8 * c8);
        const float4 w1 = *reinterpret_cast<const float4*>(wrow + 8 * c8 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          if (t < M) {
            const uint4 u = xb[t * d8 + c8];
            const float xv[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                                 bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[t] = __fmaf_rn(xv[q], wv[q], acc[t]);
          }
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = __fadd_rn(acc[t], __shfl_xor_sync(0xffffffffu, acc[t], off));
      if (lane == 0) {
        const int e = b + P * (r0 + r);
#pragma unroll
        for (int t = 0; t < TT; ++t)
          if (t < M) a.logits[static_cast<size_t>(t) * E + e] = acc[t];
      }
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[s]);
      mbar_arrive(&lgdone);  // release: this warp's logits are written
    }
  }

  // shared gate/up, rows 2j and 2j+1: thread -> row rs (gate and up),
  // column groups c0 + 128*ci
  int j = b;
  for (; j < n_sh; j += P, ++it) {
    const int s = it % S;
    if (ok) ok = wait_warp(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    const unsigned char* grow = st + static_cast<size_t>(rs) * d * 2;
    const unsigned char* urow = st + static_cast<size_t>(kShGuRows + rs) * d * 2;
    float acc[2][TT];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[h][t] = 0.f;
    const bool early = CI == 1;
    uint4 wv[2][4];
    if (early) {
      unsigned dep = 0u;
      if (ok && c0 < G) {
#pragma unroll
        for (int wq = 0; wq < 4; ++wq) {
          wv[0][wq] = lds128(grow + c0 * 64 + 16 * wq);
          wv[1][wq] = lds128(urow + c0 * 64 + 16 * wq);
          dep ^= fold4(wv[0][wq]) ^ fold4(wv[1][wq]);
        }
      }
      release_after(s, dep);
    }
    if (ok) {
      for (int ci = 0; ci < CI; ++ci) {
        const int c = c0 + 128 * ci;
        if (c >= G) break;
        if (!early) {
#pragma unroll
          for (int wq = 0; wq < 4; ++wq) {
            wv[0][wq] = lds128(grow + c * 64 + 16 * wq);
            wv[1][wq] = lds128(urow + c * 64 + 16 * wq);
          }
        }
        const uint4* xp[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) xp[t] = xb + min(t, M - 1) * d8 + c * 4;
        float part[2][TT];
        bf_dot<2, TT>(wv, xp, 1, part);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int t = 0; t < TT; ++t) acc[h][t] = __fadd_rn(acc[h][t], part[h][t]);
      }
    }
    if (!early) release(s);
    float v[2 * TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      v[t] = acc[0][t];
      v[TT + t] = acc[1][t];
    }
    reduce_scatter<2 * TT, 32>(v, lane);
    const int rb = rchunk % kNRed, use = rchunk / kNRed;
    ++rchunk;
    red_begin(rb, use);
    if ((lane & (32 / (2 * TT) - 1)) == 0) red[rb][wg][lane / (32 / (2 * TT))] = v[0];
    if (red_arrive(rb, use)) {
      if (ok && lane < kShGuRows * TT) {
        const int r = lane / TT, t = lane - (lane / TT) * TT;
        if (t < M) {
          float g = 0.f, u = 0.f;
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            g = __fadd_rn(g, red[rb][r * 4 + w4][t]);
            u = __fadd_rn(u, red[rb][r * 4 + w4][TT + t]);
          }
          a.act_s[static_cast<size_t>(t) * Fs + j * kShGuRows + r] = swiglu_bf16(round_bf16(g), round_bf16(u), a.limit);
        }
      }
      red_end(rb, use);
    }
  }

  // this CTA's act_s rows are written: publish them
  __threadfence();
  named_sync(kBarCons, kConsumers);
  if (ct == 0) atomicAdd(a.sync + kSyncShGu, 1u);
  // routing tables from the producer warp; one agreed active-expert count
  if (ok) ok = wait_warp(&tbl, 0, a.status, kSiteTable, lane);
  named_sync(kBarCons, kConsumers);
  if (ct == 0) s_nact = T.n_active;
  named_sync(kBarCons, kConsumers);
  const int n_act = s_nact;

  if constexpr (TT == 1) {
    // One token: warp wg owns gate row and up row f0 + wg of every chunk, so
    // each row's sum stays inside the warp, and the token's activation words
    // stay in registers for the whole loop.  Lane l covers the column groups
    // 4*q(l) + ((i + l) & 3), i = 0..3: every 16-byte weight load is
    // conflict-free and the lane's four scale bytes are one 32-bit word.
    // The next chunk's loads are in flight while this chunk's sums are
    // reduced; finished (gate, up) sums wait in lane (n % 32) and become
    // activations 32 at a time.
    const int ql = (lane & ~7) | ((lane & 3) << 1) | ((lane >> 2) & 1);
    int cg[kXcg];
#pragma unroll
    for (int i = 0; i < kXcg; ++i) cg[i] = 4 * ql + ((i + lane) & 3);
    uint4 xr[kXcg][4];
#pragma unroll
    for (int i = 0; i < kXcg; ++i)
#pragma unroll
      for (int wq = 0; wq < 4; ++wq) xr[i][wq] = cg[i] < G ? xh[wq * G + cg[i]] : make_uint4(0u, 0u, 0u, 0u);
    const int nend = n_sh + n_act * nrb;
    const size_t pk = static_cast<size_t>(GR) * (d >> 1);
    const size_t rowb = static_cast<size_t>(wg) * (d >> 1);
    const bool has_sc = 4 * ql < G;
    int s = it % S, ph = (it / S) & 1;
    int ai = 0, fc = 0;
    if (j < nend) {
      ai = (j - n_sh) / nrb;
      fc = (j - n_sh) - ai * nrb;
    }
    uint4 w[2][kXcg];
    uint32_t sw[2];
    // wait for stage s and issue this lane's loads (not waited for here)
    auto fetch = [&]() {
      if (ok) ok = wait_all(&full[s], ph, a.status, kSiteFull, lane);
      const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int i = 0; i < kXcg; ++i)
          w[h][i] = ok && cg[i] < G ? lds128(st + h * pk + rowb + 16 * cg[i]) : make_uint4(0u, 0u, 0u, 0u);
        sw[h] = ok && has_sc ? lds32(st + 2 * pk + (h * GR + wg) * G + 4 * ql) : 0u;
      }
    };
    auto loaded = [&]() {
      unsigned dep = sw[0] ^ sw[1];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < kXcg; ++i) dep ^= fold4(w[h][i]);
      return dep;
    };
    float pg = 0.f, pu = 0.f;
    int pidx = 0, npend = 0;
    const float m = tok_mult[0];
    auto flush = [&]() {
      if (ok && lane < npend) a.act[pidx] = swiglu_bf16(round_bf16(__fmul_rn(pg, m)), round_bf16(__fmul_rn(pu, m)), a.limit);
      npend = 0;
    };
    if (j < nend) {
      fetch();
      release_after(s, loaded());
    }
    // warps wg and wg + 4 share a scheduler: start the second half later so
    // one warp's conversions overlap the other's waits and reductions
    if (wg >= kWarps / 2) __nanosleep(300);
    while (j < nend) {
      float v[2] = {0.f, 0.f};
      {
        float scl[2][kXcg];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < kXcg; ++i) scl[h][i] = e8m0_to_f32((sw[h] >> (8 * ((i + lane) & 3))) & 0xffu);
        float part[2][2];
        mx_dot_reg<2, 0, 2, kXcg>(w, xr, part);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 2; ++c) v[h] = __fmaf_rn(part[h][c], scl[h][c], v[h]);
        mx_dot_reg<2, 2, 2, kXcg>(w, xr, part);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 2; ++c) v[h] = __fmaf_rn(part[h][c], scl[h][2 + c], v[h]);
      }
      const int idx = T.ap0[ai] * F + fc * GR + wg;
      // next chunk: stage, expert and row block without divisions
      j += P;
      ++it;
      if (++s == S) { s = 0; ph ^= 1; }
      fc += P;
      while (fc >= nrb) { fc -= nrb; ++ai; }
      const bool more = j < nend;
      if (more) fetch();
      reduce_scatter<2, 32>(v, lane);  // lanes 0-15: gate sum, 16-31: up sum
      const float gs = __shfl_sync(0xffffffffu, v[0], 0), us = __shfl_sync(0xffffffffu, v[0], 16);
      if (more) release_after(s, loaded());
      if (lane == npend) {
        pg = gs;
        pu = us;
        pidx = idx;
      }
      if (++npend == 32) flush();
    }
    flush();
  } else {
  // routed gate/up: thread -> rows rs*4 .. rs*4+3 of the chunk's 8, gate and up
  {
    const int n_r = n_act * nrb;
    const size_t pk = static_cast<size_t>(kGuRows) * (d >> 1);
    for (; j < n_sh + n_r; j += P, ++it) {
      const int s = it % S;
      if (ok) ok = wait_warp(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
      const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
      const int jr = j - n_sh;
      const int ai = jr / nrb;
      const int f0 = (jr - ai * nrb) * kGuRows;
      const int p0 = T.ap0[ai], n = T.an[ai];
      int tok[TT];
#pragma unroll
      for (int q = 0; q < TT; ++q) tok[q] = T.perm[p0 + (q < n ? q : 0)] / k;
      float acc[8][TT];  // row-vector v = h*4 + r: h gate/up, row rs*4 + r
#pragma unroll
      for (int v = 0; v < 8; ++v)
#pragma unroll
        for (int q = 0; q < TT; ++q) acc[v][q] = 0.f;
      constexpr int TP = TT < 2 ? TT : 2;  // tokens per pass
      const bool early = CI == 1;
      uint4 w[8][1];
      float scl[8];
      auto load_slice = [&](int c) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int Rw = rs * 4 + r;
            w[h * 4 + r][0] = lds128(st + h * pk + static_cast<size_t>(Rw) * (d >> 1) + 16 * c);
            scl[h * 4 + r] = e8m0_to_f32(st[2 * pk + h * kGuRows * G + Rw * G + c]);
          }
      };
      if (early) {
        unsigned dep = 0u;
        if (ok && c0 < G) {
          load_slice(c0);
#pragma unroll
          for (int v = 0; v < 8; ++v) dep ^= fold4(w[v][0]) ^ __float_as_uint(scl[v]);
        }
        release_after(s, dep);
      }
      if (ok) {
        for (int ci = 0; ci < CI; ++ci) {
          const int c = c0 + 128 * ci;
          if (c >= G) break;
          if (!early) load_slice(c);
#pragma unroll
          for (int q0 = 0; q0 < TT; q0 += TP) {
            if (q0 >= n) break;
            const uint4* xp[1][TP];
#pragma unroll
            for (int tq = 0; tq < TP; ++tq) xp[0][tq] = xh + (tok[q0 + tq] * 4) * G + c;
            float part[8][1][TP];
            mx_dot<8, 1, TP>(w, xp, G, part);
#pragma unroll
            for (int v = 0; v < 8; ++v)
#pragma unroll
              for (int tq = 0; tq < TP; ++tq) acc[v][q0 + tq] = __fmaf_rn(part[v][0][tq], scl[v], acc[v][q0 + tq]);
          }
        }
      }
      if (!early) release(s);
      float vv[8 * TT];  // index (r*2 + h)*TT + q
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q = 0; q < TT; ++q) vv[(r * 2 + h) * TT + q] = acc[h * 4 + r][q];
      reduce_scatter<8 * TT, 32>(vv, lane);
      const int rb = rchunk % kNRed, use = rchunk / kNRed;
      ++rchunk;
      red_begin(rb, use);
      if ((lane & (32 / (8 * TT) - 1)) == 0) red[rb][wg][lane / (32 / (8 * TT))] = vv[0];
      if (red_arrive(rb, use)) {
        if (ok && lane < kGuRows * TT) {
          const int Rw = lane / TT, q = lane - (lane / TT) * TT;
          if (q < n) {
            const int set = Rw >> 2, r = Rw & 3;
            float g = 0.f, u = 0.f;
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              g = __fadd_rn(g, red[rb][set * 4 + w4][(r * 2) * TT + q]);
              u = __fadd_rn(u, red[rb][set * 4 + w4][(r * 2 + 1) * TT + q]);
            }
            int tq = tok[0];
#pragma unroll
            for (int qq = 1; qq < TT; ++qq)
              if (q == qq) tq = tok[qq];
            const float m = tok_mult[tq];
            a.act[static_cast<size_t>(p0 + q) * F + f0 + Rw] =
                swiglu_bf16(round_bf16(__fmul_rn(g, m)), round_bf16(__fmul_rn(u, m)), a.limit);
          }
        }
        red_end(rb, use);
      }
    }
  }
  }

  if constexpr (TT == 1) {
    // ---------------------- one token, phase 2 ----------------------
    // this CTA's act rows are written: publish them (control warp 1 stages
    // the rows this CTA needs once every CTA has)
    __threadfence();
    named_sync(kBarCons, kConsumers);
    if (ct == 0) atomicAdd(a.sync + kSyncGu, 1u);
    const Down1 dn(a, pl, b, P);
    const unsigned char* as = smem + pl.act_off;
    // finished rows wait here (routed, then shared) until the end of phase 2:
    // a global store before a stage release would hold the release up
    uint16_t* yb = reinterpret_cast<uint16_t*>(smem + pl.yb_off);
    uint16_t* ysb = yb + pl.yb_rows;
    // shared down: warp wg owns row r0 + wg of each chunk, act_s in registers
    if (Fs > 0 && dn.sr_hi > dn.sr_lo) {
      if (ok) ok = wait_warp(&sbar, 0, a.status, kSiteActS, lane) && *reinterpret_cast<volatile int*>(&s_afail) == 0;
      const int fs8 = Fs >> 3;
      uint4 xs[kScg];
#pragma unroll
      for (int i = 0; i < kScg; ++i)
        xs[i] = lane + 32 * i < fs8 ? reinterpret_cast<const uint4*>(as)[lane + 32 * i] : make_uint4(0u, 0u, 0u, 0u);
      for (int r0 = dn.sr_lo; r0 < dn.sr_hi; r0 += kShDnRows, ++it) {
        const int s = it % S;
        if (ok) ok = wait_all(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
        const int nr = min(kShDnRows, dn.sr_hi - r0);
        const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes + static_cast<size_t>(wg) * Fs * 2;
        uint4 wv[kScg];
        unsigned dep = 0u;
#pragma unroll
        for (int i = 0; i < kScg; ++i) {
          wv[i] = ok && wg < nr && lane + 32 * i < fs8 ? lds128(st + 16 * (lane + 32 * i)) : make_uint4(0u, 0u, 0u, 0u);
          dep ^= fold4(wv[i]);
        }
        release_after(s, dep);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < kScg; ++i) {
          acc = fma_bf16(wv[i].x, xs[i].x, acc);
          acc = fma_bf16(wv[i].y, xs[i].y, acc);
          acc = fma_bf16(wv[i].z, xs[i].z, acc);
          acc = fma_bf16(wv[i].w, xs[i].w, acc);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0 && wg < nr) ysb[r0 - dn.sr_lo + wg] = f32_to_bf16(acc);
      }
    }
    // routed down: chunks of up to kDn1Rows rows of one route; half-warp hh of
    // warp wg owns rows 4*wg + 2*hh + {0, 1}, lane hl the column groups
    // hl + 16*cc with the route's activations in registers
    if (dn.u_hi > dn.u_lo && n_act == R) {
      if (ok) ok = wait_warp(&abar, 0, a.status, kSiteAct, lane) && *reinterpret_cast<volatile int*>(&s_afail) == 0;
      const uint4* av = reinterpret_cast<const uint4*>(as + static_cast<size_t>(Fs) * 2);  // bf16 [route][F]
      const int p_lo = dn.u_lo / d;
      const int hl = lane & 15, hh = lane >> 4, f8 = F >> 3;
      int cgd[kDcg];
#pragma unroll
      for (int cc = 0; cc < kDcg; ++cc) cgd[cc] = hl + 16 * cc;
      uint4 xr[kDcg][4];
      float rsc = 1.f;
      // the route's act row: power-of-two scale from its max, f16 copy of
      // this lane's column groups (both half-warps hold the same row)
      auto load_route = [&](int p) {
        const uint4* row = av + static_cast<size_t>(p - p_lo) * f8;
        unsigned m = 0u;
#pragma unroll
        for (int cc = 0; cc < kDcg; ++cc)
#pragma unroll
          for (int wq = 0; wq < 4; ++wq)
            if (cgd[cc] < G2) m = max(m, __float_as_uint(absmax8_bf16(row[cgd[cc] * 4 + wq])));
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
        rsc = pow2i(act_shift(__uint_as_float(m)));
        const float inv = __fdiv_rn(1.0f, rsc);
#pragma unroll
        for (int cc = 0; cc < kDcg; ++cc)
#pragma unroll
          for (int wq = 0; wq < 4; ++wq)
            xr[cc][wq] = cgd[cc] < G2 ? bf16x8_to_f16x8_scaled(row[cgd[cc] * 4 + wq], inv) : make_uint4(0u, 0u, 0u, 0u);
      };
      uint4 w[2][kDcg];
      uint32_t sw[2][kDcg];
      int s = it % S, ph = (it / S) & 1;
      auto fetch = [&](int nrr) {
        if (ok) ok = wait_all(&full[s], ph, a.status, kSiteFull, lane);
        const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
        const size_t pb = static_cast<size_t>(nrr) * (F >> 1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = 4 * wg + 2 * hh + h;
#pragma unroll
          for (int cc = 0; cc < kDcg; ++cc) {
            const bool in = ok && row < nrr && cgd[cc] < G2;
            w[h][cc] = in ? lds128(st + static_cast<size_t>(row) * (F >> 1) + 16 * cgd[cc]) : make_uint4(0u, 0u, 0u, 0u);
            sw[h][cc] = in ? lds32(st + pb + static_cast<size_t>(row) * G2 + 4 * ((hl >> 2) + 4 * cc)) : 0u;
          }
        }
      };
      auto loaded = [&]() {
        unsigned dep = 0u;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int cc = 0; cc < kDcg; ++cc) dep ^= fold4(w[h][cc]) ^ sw[h][cc];
        return dep;
      };
      int u = dn.u_lo;
      int p = u / d, r0 = u - p * d, nr = min(kDn1Rows, min(dn.u_hi, (p + 1) * d) - u);
      fetch(nr);
      release_after(s, loaded());
      int pcur = -1;
      while (u < dn.u_hi) {
        if (p != pcur) {
          load_route(p);
          pcur = p;
        }
        float v[2] = {0.f, 0.f};
        {
          float part[2][kDcg];
          mx_dot_reg<2, 0, kDcg, kDcg>(w, xr, part);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int cc = 0; cc < kDcg; ++cc)
              v[h] = __fmaf_rn(part[h][cc], e8m0_to_f32((sw[h][cc] >> (8 * (hl & 3))) & 0xffu), v[h]);
        }
        const int cu = u - dn.u_lo, cnr = nr;
        const float crs = rsc;
        u += nr;
        ++it;
        if (++s == S) { s = 0; ph ^= 1; }
        const bool more = u < dn.u_hi;
        if (more) {
          p = u / d;
          r0 = u - p * d;
          nr = min(kDn1Rows, min(dn.u_hi, (p + 1) * d) - u);
          fetch(nr);
        }
        reduce_scatter<2, 16>(v, lane);  // half-warp lanes 0-7: row 0, 8-15: row 1
        if (more) release_after(s, loaded());
        if ((hl & 7) == 0) {
          const int row = 4 * wg + 2 * hh + (hl >> 3);
          if (row < cnr) yb[cu + row] = f32_to_bf16(__fmul_rn(v[0], crs));
        }
      }
    }
    // publish this CTA's rows, then count them per output block (one atomic
    // per block, in parallel); the CTA completing a block merges it: routes
    // in slot order, then the shared row
    named_sync(kBarCons, kConsumers);
    if (ok && n_act == R)
      for (int i = ct; i < dn.u_hi - dn.u_lo; i += kConsumers) {
        const int u = dn.u_lo + i, pp = u / d;
        a.y[static_cast<size_t>(T.perm[pp]) * d + (u - pp * d)] = yb[i];
      }
    if (ok && Fs > 0)
      for (int i = ct; i < dn.sr_hi - dn.sr_lo; i += kConsumers) a.ys[dn.sr_lo + i] = ysb[i];
    __threadfence();
    if (ct == 0) {
      int nc = 0;
      auto add = [&](int c, int rows) {
        if (nc < kMaxComb) {
          s_cb[nc] = c;
          s_cr[nc] = rows;
        }
        ++nc;
      };
      if (Fs > 0 && dn.sr_hi > dn.sr_lo) add(b, dn.sr_hi - dn.sr_lo);
      for (int uu = dn.u_lo; uu < dn.u_hi;) {
        const int pp = uu / d, end = min(dn.u_hi, (pp + 1) * d) - pp * d;
        for (int rr = uu - pp * d; rr < end;) {
          const int c = out_block(rr, d, P), chi = min(end, block_lo(c + 1, d, P));
          add(c, chi - rr);
          rr = chi;
        }
        uu = pp * d + end;
      }
      if (nc > kMaxComb) {
        atomicExch(a.status, 2 | kSiteSync);
        nc = kMaxComb;
      }
      s_ncb = nc;
      s_ncomb = 0;
    }
    named_sync(kBarCons, kConsumers);
    if (ct < s_ncb) {
      const int c = s_cb[ct], rows = s_cr[ct];
      const unsigned target =
          static_cast<unsigned>(R + (Fs > 0 ? 1 : 0)) * static_cast<unsigned>(block_lo(c + 1, d, P) - block_lo(c, d, P));
      if (atomicAdd(a.sync + kSyncComb + c, static_cast<unsigned>(rows)) + rows == target) {
        __threadfence();
        s_comb[atomicAdd(&s_ncomb, 1)] = c;
      }
    }
    named_sync(kBarCons, kConsumers);
    for (int q = 0; q < s_ncomb; ++q) {
      const int c = s_comb[q], lo = block_lo(c, d, P), hi = block_lo(c + 1, d, P);
      for (int r = lo + ct; r < hi; r += kConsumers) {
        float sacc = 0.f;
        for (int jj = 0; jj < k; ++jj)
          sacc = __fadd_rn(sacc, __fmul_rn(bf16_to_f32(__ldcg(a.y + static_cast<size_t>(jj) * d + r)), T.w[jj]));
        if (Fs > 0) sacc = __fadd_rn(sacc, bf16_to_f32(__ldcg(a.ys + r)));
        if (ok) a.out[r] = sacc;
      }
      if (ct == 0) atomicExch(a.sync + kSyncComb + c, 0u);
    }
  } else {
  // ------------------------- phase 1 -> phase 2 -------------------------
  named_sync(kBarCons, kConsumers);
  if (ct == 0) {
    __threadfence();
    atomicAdd(a.sync + kSyncGu, 1u);
    s_fail = (ok && spin_geq(a.sync + kSyncGu, static_cast<unsigned>(P), a.status, kSiteAct)) ? 0 : 1;
    __threadfence();
  }
  named_sync(kBarCons, kConsumers);
  if (s_fail) ok = false;
  // act (f16 in place, scaled per route so max|v| < 2^8) and act_s (bf16),
  // both row-major as written, copied into the union area in one batch
  uint4* xa = reinterpret_cast<uint4*>(smem + pl.x_off);  // f16 [p][F]
  uint4* xs = xa + R * (F >> 3);                           // bf16 [t][Fs]
  const int f8 = F >> 3, fs8 = Fs >> 3;
  if (ct == 0 && ok) {
    asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes of other CTAs -> async-proxy reads
    mbar_arrive_expect_tx(&abar, static_cast<unsigned>(R) * F * 2u + static_cast<unsigned>(M) * Fs * 2u);
    bulk_g2s(xa, a.act, static_cast<unsigned>(R) * F * 2u, &abar);
    if (Fs > 0) bulk_g2s(xs, a.act_s, static_cast<unsigned>(M) * Fs * 2u, &abar);
  }
  if (ok) ok = wait_warp(&abar, 0, a.status, kSiteAct, lane);
#pragma unroll 1
  for (int p = wg; p < R; p += kWarps) {
    unsigned m = 0u;
#pragma unroll 1
    for (int u = lane; u < f8; u += 32) m = max(m, __float_as_uint(absmax8_bf16(xa[p * f8 + u])));
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) {
      rscale[p] = pow2i(act_shift(__uint_as_float(m)));
      rinv[p] = __fdiv_rn(1.0f, rscale[p]);
    }
  }
  named_sync(kBarCons, kConsumers);
#pragma unroll 1
  for (int i4 = ct; i4 < R * f8; i4 += kConsumers) xa[i4] = bf16x8_to_f16x8_scaled(xa[i4], rinv[i4 / f8]);
  named_sync(kBarCons, kConsumers);

  // ---------------------------- phase 2 ----------------------------
  const DownRange dr(a, pl, b, P);
  const int r_lo = dr.r_lo, rows = dr.rows;
  // shared down: warp -> row, lanes over column groups
  const int CIs = (G2s + 31) >> 5;
  for (int pc = 0; pc < dr.n_sdp; ++pc, ++it) {
    const int s = it % S;
    if (ok) ok = wait_warp(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
    const int rl0 = pc * pl.sh_rows, nr = min(pl.sh_rows, rows - rl0);
    const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
    float acc[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) acc[t] = 0.f;
    if (ok && wg < nr) {
      const unsigned char* wrow = st + static_cast<size_t>(wg) * Fs * 2;
      for (int ci = 0; ci < CIs; ++ci) {
        const int c = lane + 32 * ci;
        if (c < G2s) {
          uint4 wv[1][4];
#pragma unroll
          for (int wq = 0; wq < 4; ++wq) wv[0][wq] = lds128(wrow + c * 64 + 16 * wq);
          const uint4* xp[TT];
#pragma unroll
          for (int t = 0; t < TT; ++t) xp[t] = xs + min(t, M - 1) * fs8 + c * 4;
          float part[1][TT];
          bf_dot<1, TT>(wv, xp, 1, part);
#pragma unroll
          for (int t = 0; t < TT; ++t) acc[t] = __fadd_rn(acc[t], part[0][t]);
        }
      }
    }
    release(s);
    reduce_scatter<TT, 32>(acc, lane);
    if (ok && wg < nr && (lane & (32 / TT - 1)) == 0) {
      const int t = lane / (32 / TT);
      if (t < M) ysm[static_cast<size_t>(R + t) * pl.rows_max + rl0 + wg] = round_bf16(acc[0]);
    }
  }

  // routed down: 16 column-group lanes (3 groups each) x 16 row sets of two rows
  {
    const int cd = ct & 15, rd = ct >> 4;
    const int CI2 = (G2 + 15) >> 4;
    const int NB = (CI2 + 2) / 3;  // blocks of three column groups
    for (int ai = 0; ai < n_act; ++ai) {
      const int p0 = T.ap0[ai], n = T.an[ai];
      for (int sc = 0; sc < dr.n_sub; ++sc, ++it) {
        const int s = it % S;
        if (ok) ok = wait_warp(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
        const unsigned char* st = smem + static_cast<size_t>(s) * pl.stage_bytes;
        const int rl0 = sc * pl.sub_rows, nr = min(pl.sub_rows, rows - rl0);
        const size_t pb = static_cast<size_t>(nr) * (F >> 1);
        float acc[2][TT];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q = 0; q < TT; ++q) acc[h][q] = 0.f;
        constexpr int TP = TT < 2 ? TT : 2;
        const bool early = NB == 1;
        uint4 w[2][3];
        float scl[2][3];
        auto load_slice = [&](int cb) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int cc = 0; cc < 3; ++cc) {
              const int row = rd + 16 * h, c = cd + 16 * (cb * 3 + cc);
              const bool in = row < nr && c < G2;
              w[h][cc] = in ? lds128(st + static_cast<size_t>(row) * (F >> 1) + 16 * c) : make_uint4(0u, 0u, 0u, 0u);
              scl[h][cc] = in ? e8m0_to_f32(st[pb + row * G2 + c]) : 0.f;
            }
        };
        if (early) {
          unsigned dep = 0u;
          if (ok) {
            load_slice(0);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int cc = 0; cc < 3; ++cc) dep ^= fold4(w[h][cc]) ^ __float_as_uint(scl[h][cc]);
          }
          release_after(s, dep);
        }
        if (ok) {
          for (int cb = 0; cb < NB; ++cb) {
            if (!early) load_slice(cb);
#pragma unroll
            for (int q0 = 0; q0 < TT; q0 += TP) {
              if (q0 >= n) break;
              const uint4* xp[3][TP];
#pragma unroll
              for (int cc = 0; cc < 3; ++cc) {
                const int c = min(cd + 16 * (cb * 3 + cc), G2 - 1);
#pragma unroll
                for (int tq = 0; tq < TP; ++tq) xp[cc][tq] = xa + (p0 + min(q0 + tq, n - 1)) * f8 + c * 4;
              }
              float part[2][3][TP];
              mx_dot<2, 3, TP>(w, xp, 1, part);
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int cc = 0; cc < 3; ++cc)
#pragma unroll
                  for (int tq = 0; tq < TP; ++tq)
                    acc[h][q0 + tq] = __fmaf_rn(part[h][cc][tq], scl[h][cc], acc[h][q0 + tq]);
            }
          }
        }
        if (!early) release(s);
        float v[2 * TT];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q = 0; q < TT; ++q) v[h * TT + q] = acc[h][q];
        reduce_scatter<2 * TT, 16>(v, lane);
        if (ok && (lane & (16 / (2 * TT) - 1)) == 0) {
          const int vi = (lane & 15) / (16 / (2 * TT));
          const int h = vi / TT, q = vi - (vi / TT) * TT;
          const int row = rd + 16 * h;
          if (row < nr && q < n)
            ysm[static_cast<size_t>(T.perm[p0 + q]) * pl.rows_max + rl0 + row] =
                round_bf16(__fmul_rn(v[0], rscale[p0 + q]));
        }
      }
    }
  }

  // ---- merge this CTA's rows: routes in j order, then the shared row ----
  named_sync(kBarCons, kConsumers);
  if (ok) {
    for (int o = ct; o < M * rows; o += kConsumers) {
      const int t = o / rows, rl = o - t * rows;
      float sacc = 0.f;
      for (int q = 0; q < k; ++q) {
        const int sl = t * k + q;
        sacc = __fadd_rn(sacc, __fmul_rn(ysm[static_cast<size_t>(sl) * pl.rows_max + rl], T.w[sl]));
      }
      if (Fs > 0) sacc = __fadd_rn(sacc, ysm[static_cast<size_t>(R + t) * pl.rows_max + rl]);
      a.out[static_cast<size_t>(t) * d + r_lo + rl] = sacc;
    }
  }
  }
  // The last CTA out checks that the counters saw exactly this call (a
  // workspace that was not zeroed before its first use fails here, once) and
  // resets them for the next call.
  if (ct == 0) {
    __threadfence();
    if (atomicAdd(a.sync + kSyncExit, 1u) == static_cast<unsigned>(P) - 1u) {
      const unsigned nl = atomicExch(a.sync + kSyncLogits, 0u), na = atomicExch(a.sync + kSyncGu, 0u);
      const unsigned ns = atomicExch(a.sync + kSyncShGu, 0u);
      atomicExch(a.sync + kSyncExit, 0u);
      if (nl != static_cast<unsigned>(E) || na != static_cast<unsigned>(P) || ns != static_cast<unsigned>(P))
        atomicExch(a.status, 3 | kSiteSync);
    }
  }
}

}  // namespace layer
}  // namespace lg
