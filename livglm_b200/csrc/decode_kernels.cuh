// Decode-shape kernels (M <= kDecodeMaxTokens tokens per call), chained with
// programmatic dependent launch (PDL):
//
//   router_logits_decode_kernel    one warp per expert; canonical fp32 order
//   router_select_dispatch_kernel  one CTA: sigmoid/bias/group-limited top-k,
//                                  weights, counts/offsets/perm/active
//   gate_up_decode_kernel          MXFP4 gate+up rows x routed tokens, SwiGLU;
//                                  bf16 shared expert rows in dedicated CTAs
//   down_decode_kernel             MXFP4 down rows x routed activations, bf16
//                                  shared down; the last unit to finish a row
//                                  block writes the f32 combine (moe.py:199-201)
//
// Dot products: E2M1 pairs are converted with cvt.rn.f16x2.e2m1x2 and
// multiplied into f32 accumulators with the mixed-precision
// fma.rn.f32.f16 (bf16 for the bf16 shared weights).  Activations enter as
// f16: bf16 -> f16 is exact for 2^-17 <= |v| < 2^15, and each activation row
// is scaled by a power of two when its max |v| reaches 2^15 (undone exactly
// in f32 afterwards); magnitudes below 2^-17 round onto the f16 subnormal grid
// (absolute error <= 2^-25 per element).
#pragma once
#include "common.cuh"

namespace lg {

constexpr int kDecodeMaxTokens = 4;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float fma_f16(uint32_t a, uint32_t b, float c) {
  asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.f16 %0, a0, b0, %0;\n\tfma.rn.f32.f16 %0, a1, b1, %0;\n\t}"
      : "+f"(c) : "r"(a), "r"(b));
  return c;
}
__device__ __forceinline__ float fma_bf16(uint32_t a, uint32_t b, float c) {
  asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a0, b0, %0;\n\tfma.rn.f32.bf16 %0, a1, b1, %0;\n\t}"
      : "+f"(c) : "r"(a), "r"(b));
  return c;
}
// Dot of 8 E2M1 values (one word) with 8 f16 activations (one uint4).
__device__ __forceinline__ float dot8_e2m1_f16(uint32_t w, const uint4& x, float acc) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3) : "r"(w));
  acc = fma_f16(h0, x.x, acc);
  acc = fma_f16(h1, x.y, acc);
  acc = fma_f16(h2, x.z, acc);
  acc = fma_f16(h3, x.w, acc);
  return acc;
}
__device__ __forceinline__ float dot8_bf16(const uint4& w, const uint4& x, float acc) {
  acc = fma_bf16(w.x, x.x, acc);
  acc = fma_bf16(w.y, x.y, acc);
  acc = fma_bf16(w.z, x.z, acc);
  acc = fma_bf16(w.w, x.w, acc);
  return acc;
}

// power-of-two prescale of an activation row: shift such that max|v|*2^-shift < 2^15
__device__ __forceinline__ int f16_shift_for(float amax) {
  const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xffu) - 127;  // floor(log2)
  return e >= 15 ? e - 14 : 0;
}
__device__ __forceinline__ uint32_t bf16x2_to_f16x2_scaled(uint32_t w, float s) {
  const float lo = __fmul_rn(bf16lo(w), s), hi = __fmul_rn(bf16hi(w), s);
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

struct DecodeArgs {
  int M, d, F, Fs, E, k, G, g, norm;
  float scale, limit;
  const uint16_t* x;
  const float *Wr, *bias;
  const uint8_t *gate_p, *gate_s, *up_p, *up_s, *down_p, *down_s;
  long long gate_ps, gate_ss, up_ps, up_ss, down_ps, down_ss;
  const uint16_t *sh_gate, *sh_up, *sh_down;
  float* logits;
  float* weights;
  uint32_t* indices;
  int *counts, *offsets, *perm, *active;
  uint16_t *act, *act_s, *y, *ys;
  unsigned* tickets;  // down combine tickets, one per combine block
  float* out;
  int gu_shared_ctas, down_shared_ctas;
  int lpr_down, lpr_down_s;  // lanes per row in the down kernel (routed / shared)
  int cb_rows;               // rows per combine block
};

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(256) router_logits_decode_kernel(DecodeArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x * 8 + warp;
  const bool live = e < a.E;
  const float* wrow = a.Wr + static_cast<size_t>(live ? e : 0) * a.d;
  if (live) {  // router weights do not depend on earlier kernels: pull them into L2 now
    for (int line = lane; line < a.d / 32; line += 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow + 32 * line));
  }
  pdl_wait();
  pdl_trigger();
  if (!live) return;
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.f;
  const int chunks = a.d >> 3;
#pragma unroll 4
  for (int c = lane; c < chunks; c += 32) {
    const float4* wp = reinterpret_cast<const float4*>(wrow + 8 * c);
    const float4 w0 = wp[0], w1 = wp[1];
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t < a.M) {
        const uint4 u = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(t) * a.d + 8 * c);
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
#pragma unroll
    for (int t = 0; t < TT; ++t)
      if (t < a.M) a.logits[static_cast<size_t>(t) * a.E + e] = acc[t];
  }
}

// ---------------------------------------------------------------------------
// One CTA of 256 threads.  Per token: scores/choices per expert, group top-2
// sums via in-group ranks, kept groups via group ranks, top-k via expert
// ranks under the stable (value, index) order, then normalised weights.
// Then the dispatch tables for all M*k slots, and zeroed combine tickets.
// Shared memory: sc[E] ch[E] gtop1[G] gtop2[G] gs[G] keep[G] + small arrays.
__global__ void __launch_bounds__(256) router_select_dispatch_kernel(DecodeArgs a, int n_tickets) {
  extern __shared__ float sm[];
  const int E = a.E, G = a.G, k = a.k, M = a.M;
  float* sc = sm;
  float* ch = sc + E;
  float* gt1 = ch + E;
  float* gt2 = gt1 + G;
  float* gs = gt2 + G;
  int* keep = reinterpret_cast<int*>(gs + G);
  int* sel_e = keep + G;                  // [M*k] selected experts, slot order
  float* sel_w = reinterpret_cast<float*>(sel_e + kDecodeMaxTokens * 32);
  int* cnt = reinterpret_cast<int*>(sel_w + 32);  // [E]
  int* offs = cnt + E;                            // [E + 1]
  int* nz = offs + E + 1;                         // [E + 1] exclusive count of nonzero experts
  const int tid = threadIdx.x;
  pdl_trigger();
  pdl_wait();
  for (int i = tid; i < n_tickets; i += blockDim.x) a.tickets[i] = 0u;
  const int per = E / G;
  const float ninf = __uint_as_float(0xff800000u);
  for (int t = 0; t < M; ++t) {
    for (int e = tid; e < E; e += blockDim.x) {
      const float s = own_sigmoidf(__ldcg(a.logits + static_cast<size_t>(t) * E + e));
      sc[e] = s;
      ch[e] = __fadd_rn(s, a.bias[e]);
    }
    __syncthreads();
    if (a.g < G) {
      for (int e = tid; e < E; e += blockDim.x) {
        const int g0 = (e / per) * per;
        const float v = ch[e];
        int r = 0;
        for (int j = 0; j < per; ++j) r += after(ch[g0 + j], g0 + j, v, e);
        if (r == 0) gt1[e / per] = v;
        if (r == 1) gt2[e / per] = v;
      }
      __syncthreads();
      for (int gi = tid; gi < G; gi += blockDim.x) gs[gi] = __fadd_rn(gt2[gi], gt1[gi]);
      __syncthreads();
      for (int gi = tid; gi < G; gi += blockDim.x) {
        int r = 0;
        for (int j = 0; j < G; ++j) r += after(gs[j], j, gs[gi], gi);
        keep[gi] = r < a.g;
      }
      __syncthreads();
      for (int e = tid; e < E; e += blockDim.x)
        if (!keep[e / per]) ch[e] = ninf;
      __syncthreads();
    }
    for (int e = tid; e < E; e += blockDim.x) {
      const float v = ch[e];
      int r = 0;
      for (int j = 0; j < E; ++j) r += after(ch[j], j, v, e);
      if (r < k) {
        sel_e[t * k + (k - 1 - r)] = e;
        sel_w[k - 1 - r] = sc[e];
      }
    }
    __syncthreads();
    if (tid < 32) {
      const float wj = (tid < k) ? sel_w[tid] : 0.f;
      float denom = 0.f;
      if (a.norm) {
        float sum = __shfl_sync(0xffffffffu, wj, 0);
        for (int j = 1; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wj, j));
        denom = __fadd_rn(sum, 0x1.79ca1p-67f);
      }
      if (tid < k) {
        float w = a.norm ? __fdiv_rn(wj, denom) : wj;
        w = __fmul_rn(w, a.scale);
        a.weights[static_cast<size_t>(t) * k + tid] = w;
        a.indices[static_cast<size_t>(t) * k + tid] = static_cast<uint32_t>(sel_e[t * k + tid]);
      }
    }
    __syncthreads();
  }
  // dispatch tables: counts, exclusive offsets, nonzero ranks, stable perm
  const int S = M * k;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) atomicAdd(cnt + sel_e[s], 1);
  __syncthreads();
  if (tid < 32) {  // one warp scans E counts in 32-wide chunks
    int run_c = 0, run_n = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + tid;
      const int c = e < E ? cnt[e] : 0;
      int ic = c, in = c > 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int vc = __shfl_up_sync(0xffffffffu, ic, off), vn = __shfl_up_sync(0xffffffffu, in, off);
        if (tid >= off) { ic += vc; in += vn; }
      }
      if (e < E) { offs[e] = run_c + ic - c; nz[e] = run_n + in - (c > 0); }
      run_c += __shfl_sync(0xffffffffu, ic, 31);
      run_n += __shfl_sync(0xffffffffu, in, 31);
    }
    if (tid == 0) { offs[E] = run_c; nz[E] = run_n; }
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    a.counts[e] = cnt[e];
    a.offsets[e] = offs[e];
    if (cnt[e] > 0) a.active[1 + nz[e]] = e;
  }
  if (tid == 0) { a.offsets[E] = offs[E]; a.active[0] = nz[E]; }
  for (int s = tid; s < S; s += blockDim.x) {
    const int e = sel_e[s];
    int r = 0;
    for (int j = 0; j < s; ++j) r += sel_e[j] == e;
    a.perm[offs[e] + r] = s;
  }
}

// ---------------------------------------------------------------------------
// Gate/up.  CTAs [0, gu_shared_ctas) stream the shared expert's bf16 rows
// (they need no routing, so they start while the router still runs); the
// others stream routed (expert, row) units.  A warp owns one row pair (gate
// row f and up row f) at a time; lane l owns the 32-column groups
// c = l, l+32, ...: one 16-byte packed load and one scale byte per group
// (four 16-byte loads per group for bf16 rows).
// Shared memory: activations of all M tokens, [t][i][w][lane] uint4 so that
// lane l reads group c = l + 32i, word w (8 values) conflict-free.
template <int TT>
__global__ void __launch_bounds__(256) gate_up_decode_kernel(DecodeArgs a) {
  extern __shared__ uint4 gu_xs[];
  __shared__ unsigned amax_bits[TT];
  __shared__ float tok_scale[TT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = a.d, G = K >> 5, KI = (G + 31) >> 5;
  const bool shared_cta = static_cast<int>(blockIdx.x) < a.gu_shared_ctas;
  const int M = a.M;
  // ---- stage the M token rows (x is complete: the router waited on it) ----
  if (threadIdx.x < TT) amax_bits[threadIdx.x] = 0u;
  __syncthreads();
  const int n4 = M * G * 4;  // uint4 per row: G groups x 4 words
  for (int i4 = threadIdx.x; i4 < n4; i4 += blockDim.x) {
    const int t = i4 / (G * 4), rem = i4 - t * G * 4, c = rem >> 2, w = rem & 3;
    const uint4 u = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(t) * K + 32 * c + 8 * w);
    gu_xs[((t * KI + (c >> 5)) * 4 + w) * 32 + (c & 31)] = u;
    if (!shared_cta) {
      float m = fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y))));
      m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
      atomicMax(amax_bits + t, __float_as_uint(m));
    }
  }
  __syncthreads();
  if (shared_cta) {
    pdl_trigger();
    const int units = a.Fs;
    const int wpc = blockDim.x >> 5;
    const int nw = a.gu_shared_ctas * wpc;
    for (int f = blockIdx.x * wpc + warp; f < units; f += nw) {
      float ag[TT], au[TT];
#pragma unroll
      for (int t = 0; t < TT; ++t) { ag[t] = 0.f; au[t] = 0.f; }
      const uint16_t* gr = a.sh_gate + static_cast<size_t>(f) * K;
      const uint16_t* ur = a.sh_up + static_cast<size_t>(f) * K;
      for (int i = 0; i < KI; ++i) {
        const int c = lane + 32 * i;
        if (c < G) {
          uint4 wg[4], wu[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            wg[w] = ldg_nc_v4(gr + 32 * c + 8 * w);
            wu[w] = ldg_nc_v4(ur + 32 * c + 8 * w);
          }
#pragma unroll
          for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int t = 0; t < TT; ++t)
              if (t < M) {
                const uint4 xv = gu_xs[((t * KI + i) * 4 + w) * 32 + lane];
                ag[t] = dot8_bf16(wg[w], xv, ag[t]);
                au[t] = dot8_bf16(wu[w], xv, au[t]);
              }
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          ag[t] = __fadd_rn(ag[t], __shfl_xor_sync(0xffffffffu, ag[t], off));
          au[t] = __fadd_rn(au[t], __shfl_xor_sync(0xffffffffu, au[t], off));
        }
      if (lane < TT && lane < M) {
        float g = ag[0], u = au[0];
#pragma unroll
        for (int t = 1; t < TT; ++t)
          if (lane == t) { g = ag[t]; u = au[t]; }
        a.act_s[static_cast<size_t>(lane) * a.Fs + f] = swiglu_bf16(round_bf16(g), round_bf16(u), a.limit);
      }
    }
    return;
  }
  // ---- routed: convert the staged rows to f16 in place (prescaled) ----
  if (threadIdx.x < TT) {
    const int sh = f16_shift_for(__uint_as_float(amax_bits[threadIdx.x]));
    tok_scale[threadIdx.x] = pow2i(sh);  // result multiplier
    amax_bits[threadIdx.x] = static_cast<unsigned>(sh);
  }
  __syncthreads();
  for (int i4 = threadIdx.x; i4 < n4; i4 += blockDim.x) {
    const int t = i4 / (G * 4), rem = i4 - t * G * 4, c = rem >> 2, w = rem & 3;
    uint4& v = gu_xs[((t * KI + (c >> 5)) * 4 + w) * 32 + (c & 31)];
    const float s = pow2i(-static_cast<int>(amax_bits[t]));
    v = make_uint4(bf16x2_to_f16x2_scaled(v.x, s), bf16x2_to_f16x2_scaled(v.y, s),
                   bf16x2_to_f16x2_scaled(v.z, s), bf16x2_to_f16x2_scaled(v.w, s));
  }
  __syncthreads();
  pdl_wait();  // routing tables written by the router
  pdl_trigger();
  const int n_active = __ldcg(a.active);
  const long long units = static_cast<long long>(n_active) * a.F;
  const int wpc = blockDim.x >> 5;
  const int routed_ctas = gridDim.x - a.gu_shared_ctas;
  const int nw = routed_ctas * wpc;
  const int gw = (blockIdx.x - a.gu_shared_ctas) * wpc + warp;
  for (long long u = gw; u < units; u += nw) {
    const int ai = static_cast<int>(u / a.F);
    const int f = static_cast<int>(u - static_cast<long long>(ai) * a.F);
    const int e = __ldcg(a.active + 1 + ai);
    const int p0 = __ldcg(a.offsets + e);
    const int n = __ldcg(a.offsets + e + 1) - p0;
    int tok[TT];
#pragma unroll
    for (int j = 0; j < TT; ++j) tok[j] = j < n ? __ldcg(a.perm + p0 + j) / a.k : 0;
    const uint8_t* gp = a.gate_p + e * a.gate_ps + static_cast<size_t>(f) * (K >> 1);
    const uint8_t* up = a.up_p + e * a.up_ps + static_cast<size_t>(f) * (K >> 1);
    const uint8_t* gsc = a.gate_s + e * a.gate_ss + static_cast<size_t>(f) * G;
    const uint8_t* usc = a.up_s + e * a.up_ss + static_cast<size_t>(f) * G;
    float ag[TT], au[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) { ag[t] = 0.f; au[t] = 0.f; }
    constexpr int kPre = 4;  // groups per lane loaded ahead (K <= 4096 in one batch)
    for (int i0 = 0; i0 < KI; i0 += kPre) {
      uint4 pg[kPre], pu[kPre];
      uint32_t sg[kPre], su[kPre];
#pragma unroll
      for (int q = 0; q < kPre; ++q) {
        const int c = lane + 32 * (i0 + q);
        if (i0 + q < KI && c < G) {
          pg[q] = ldg_nc_v4(gp + 16 * c);
          pu[q] = ldg_nc_v4(up + 16 * c);
          sg[q] = gsc[c];
          su[q] = usc[c];
        }
      }
#pragma unroll
      for (int q = 0; q < kPre; ++q) {
        const int i = i0 + q;
        const int c = lane + 32 * i;
        if (i < KI && c < G) {
          float gg[TT], gu[TT];
#pragma unroll
          for (int t = 0; t < TT; ++t) { gg[t] = 0.f; gu[t] = 0.f; }
          const uint32_t wg4[4] = {pg[q].x, pg[q].y, pg[q].z, pg[q].w};
          const uint32_t wu4[4] = {pu[q].x, pu[q].y, pu[q].z, pu[q].w};
#pragma unroll
          for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int j = 0; j < TT; ++j)
              if (j < n) {
                const uint4 xv = gu_xs[((tok[j] * KI + i) * 4 + w) * 32 + lane];
                gg[j] = dot8_e2m1_f16(wg4[w], xv, gg[j]);
                gu[j] = dot8_e2m1_f16(wu4[w], xv, gu[j]);
              }
          const float s_g = e8m0_to_f32(sg[q]), s_u = e8m0_to_f32(su[q]);
#pragma unroll
          for (int j = 0; j < TT; ++j) {
            ag[j] = __fmaf_rn(gg[j], s_g, ag[j]);
            au[j] = __fmaf_rn(gu[j], s_u, au[j]);
          }
        }
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int j = 0; j < TT; ++j) {
        ag[j] = __fadd_rn(ag[j], __shfl_xor_sync(0xffffffffu, ag[j], off));
        au[j] = __fadd_rn(au[j], __shfl_xor_sync(0xffffffffu, au[j], off));
      }
    if (lane < TT && lane < n) {
      float g = ag[0], uu = au[0];
      int tj = tok[0];
#pragma unroll
      for (int j = 1; j < TT; ++j)
        if (lane == j) { g = ag[j]; uu = au[j]; tj = tok[j]; }
      const float m = tok_scale[tj];
      a.act[static_cast<size_t>(p0 + lane) * a.F + f] =
          swiglu_bf16(round_bf16(__fmul_rn(g, m)), round_bf16(__fmul_rn(uu, m)), a.limit);
    }
  }
}

// ---------------------------------------------------------------------------
// Down + combine.  A unit is 2 row-iterations of one warp: 32/LPR rows per
// iteration, LPR lanes per row, each lane G/LPR groups of the row.  Routed
// units cover (active expert, row block); CTAs [0, down_shared_ctas) cover the
// shared expert's bf16 rows.  After writing its rows a unit takes a ticket on
// its combine block; the unit that completes a block sums, for every token,
// the k routed rows in route order plus the shared row into `out`.
// Shared memory: f16 activations of all M*k routes ([p][q4][grp] uint4, with
// per-route power-of-two prescale) or the M shared rows (bf16, [t][q4][grp]).
template <int TT>
__global__ void __launch_bounds__(256) down_decode_kernel(DecodeArgs a) {
  extern __shared__ uint4 dn_xs[];
  __shared__ float rscale[kDecodeMaxTokens * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool shared_cta = static_cast<int>(blockIdx.x) < a.down_shared_ctas;
  const int M = a.M, k = a.k, d = a.d;
  const int K = shared_cta ? a.Fs : a.F;
  const int G = K >> 5;
  const int LPR = shared_cta ? a.lpr_down_s : a.lpr_down;
  const int slots = 32 / LPR;
  const int rows_per_unit = 2 * slots;
  const int nblk = d / rows_per_unit;
  const int sub = lane & (LPR - 1), slot = lane / LPR;
  const int per_lane = (G + LPR - 1) / LPR;
  pdl_wait();  // activations from the gate/up kernel
  pdl_trigger();
  const int n_active = __ldcg(a.active);
  const int R = shared_cta ? M : M * k;  // staged rows
  const uint16_t* src = shared_cta ? a.act_s : a.act;
  // stage: bf16 rows -> [r][q4][grp] uint4 (shared: bf16 kept; routed: f16 prescaled)
  for (int r = warp; r < R; r += blockDim.x >> 5) {
    if (shared_cta) {
      for (int v = lane; v < G * 4; v += 32) {
        const int grp = v >> 2, q4 = v & 3;
        dn_xs[(r * 4 + q4) * G + grp] = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * K + 32 * grp + 8 * q4));
      }
    } else {
      float m = 0.f;
      for (int v = lane; v < G * 4; v += 32) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * K + 8 * v));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y)))));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const int sh = f16_shift_for(m);
      const float s = pow2i(-sh);
      if (lane == 0) rscale[r] = pow2i(sh);
      for (int v = lane; v < G * 4; v += 32) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * K + 8 * v));
        dn_xs[(r * 4 + (v & 3)) * G + (v >> 2)] =
            make_uint4(bf16x2_to_f16x2_scaled(u.x, s), bf16x2_to_f16x2_scaled(u.y, s),
                       bf16x2_to_f16x2_scaled(u.z, s), bf16x2_to_f16x2_scaled(u.w, s));
      }
    }
  }
  __syncthreads();
  const int wpc = blockDim.x >> 5;
  const int my_ctas = shared_cta ? a.down_shared_ctas : gridDim.x - a.down_shared_ctas;
  const int cta_i = shared_cta ? blockIdx.x : blockIdx.x - a.down_shared_ctas;
  const int nw = my_ctas * wpc;
  const long long units = shared_cta ? static_cast<long long>(nblk) : static_cast<long long>(n_active) * nblk;
  const int cb = a.cb_rows;
  const unsigned expected = static_cast<unsigned>(n_active) * (cb / (2 * (32 / a.lpr_down))) +
                            (a.Fs > 0 ? static_cast<unsigned>(cb / (2 * (32 / a.lpr_down_s))) : 0u);
  for (long long u = cta_i * wpc + warp; u < units; u += nw) {
    const int ai = shared_cta ? 0 : static_cast<int>(u / nblk);
    const int rb = static_cast<int>(u - static_cast<long long>(ai) * nblk);
    const int e = shared_cta ? 0 : __ldcg(a.active + 1 + ai);
    const int p0 = shared_cta ? 0 : __ldcg(a.offsets + e);
    const int n = shared_cta ? M : __ldcg(a.offsets + e + 1) - p0;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int row = rb * rows_per_unit + it * slots + slot;
      float acc[TT];
#pragma unroll
      for (int j = 0; j < TT; ++j) acc[j] = 0.f;
      if (shared_cta) {
        const uint16_t* wr = a.sh_down + static_cast<size_t>(row) * K;
        for (int q = 0; q < per_lane; ++q) {
          const int grp = sub + LPR * q;
          if (grp < G) {
            uint4 wv[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) wv[w] = ldg_nc_v4(wr + 32 * grp + 8 * w);
#pragma unroll
            for (int w = 0; w < 4; ++w)
#pragma unroll
              for (int j = 0; j < TT; ++j)
                if (j < n) acc[j] = dot8_bf16(wv[w], dn_xs[(j * 4 + w) * G + grp], acc[j]);
          }
        }
      } else {
        const uint8_t* wp = a.down_p + e * a.down_ps + static_cast<size_t>(row) * (K >> 1);
        const uint8_t* ws = a.down_s + e * a.down_ss + static_cast<size_t>(row) * G;
        constexpr int kPre = 4;
        for (int q0 = 0; q0 < per_lane; q0 += kPre) {
          uint4 pk[kPre];
          uint32_t sc[kPre];
#pragma unroll
          for (int q = 0; q < kPre; ++q) {
            const int grp = sub + LPR * (q0 + q);
            if (q0 + q < per_lane && grp < G) { pk[q] = ldg_nc_v4(wp + 16 * grp); sc[q] = ws[grp]; }
          }
#pragma unroll
          for (int q = 0; q < kPre; ++q) {
            const int grp = sub + LPR * (q0 + q);
            if (q0 + q < per_lane && grp < G) {
              const uint32_t w4[4] = {pk[q].x, pk[q].y, pk[q].z, pk[q].w};
              float gsum[TT];
#pragma unroll
              for (int j = 0; j < TT; ++j) gsum[j] = 0.f;
#pragma unroll
              for (int w = 0; w < 4; ++w)
#pragma unroll
                for (int j = 0; j < TT; ++j)
                  if (j < n) gsum[j] = dot8_e2m1_f16(w4[w], dn_xs[((p0 + j) * 4 + w) * G + grp], gsum[j]);
              const float s = e8m0_to_f32(sc[q]);
#pragma unroll
              for (int j = 0; j < TT; ++j) acc[j] = __fmaf_rn(gsum[j], s, acc[j]);
            }
          }
        }
      }
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1)
#pragma unroll
        for (int j = 0; j < TT; ++j) acc[j] = __fadd_rn(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], off));
      if (sub < TT && sub < n) {
        float v = acc[0];
#pragma unroll
        for (int j = 1; j < TT; ++j)
          if (sub == j) v = acc[j];
        if (shared_cta) {
          a.ys[static_cast<size_t>(sub) * d + row] = f32_to_bf16(v);
        } else {
          const int p = p0 + sub;
          a.y[static_cast<size_t>(__ldcg(a.perm + p)) * d + row] = f32_to_bf16(__fmul_rn(v, rscale[p]));
        }
      }
    }
    // ---- combine-block ticket ----
    __syncwarp();
    unsigned ticket = 0;
    const int blk = (rb * rows_per_unit) / cb;
    if (lane == 0) {
      __threadfence();
      ticket = atomicAdd(a.tickets + blk, 1u);
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket == expected - 1) {
      __threadfence();
      for (int o = lane; o < cb * M; o += 32) {
        const int t = o / cb, row = blk * cb + (o - t * cb);
        float s = 0.f;
        for (int j = 0; j < k; ++j) {
          const float wj = __ldcg(a.weights + static_cast<size_t>(t) * k + j);
          const unsigned short yb = __ldcg(reinterpret_cast<const unsigned short*>(a.y) + (static_cast<size_t>(t) * k + j) * d + row);
          s = __fadd_rn(s, __fmul_rn(bf16_to_f32(yb), wj));
        }
        if (a.Fs > 0) s = __fadd_rn(s, bf16_to_f32(__ldcg(reinterpret_cast<const unsigned short*>(a.ys) + static_cast<size_t>(t) * d + row)));
        a.out[static_cast<size_t>(t) * d + row] = s;
      }
      if (lane == 0) a.tickets[blk] = 0u;
    }
  }
}

}  // namespace lg
