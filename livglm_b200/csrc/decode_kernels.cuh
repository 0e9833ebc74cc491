// Decode-shape kernels (M <= kDecodeMaxTokens tokens per call), chained with
// programmatic dependent launch (PDL):
//
//   router_logits_decode_kernel    one warp per expert; canonical fp32 order
//   router_select_dispatch_kernel  one CTA: sigmoid/bias/group-limited top-k,
//                                  weights, counts/offsets/perm/active
//   (gate/up and down: stream_kernels.cuh)
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
  int* status;               // device status word (0 = ok)
  int lpr_down;              // lanes per row in the down kernel (routed rows)
};

// ---------------------------------------------------------------------------
// Token staging for hidden states the caller keeps in page-locked host memory:
// copies n 16-byte words from the host mapping into the workspace, so the
// chain's kernels read the tokens from HBM and the host read happens once, in
// a kernel that joins the PDL chain (a copy-engine memcpy in front of the chain
// would wait for the previous layer to drain and leave the chain cold).  The
// source is read after griddepcontrol.wait: work before it on the stream may
// still be writing the host buffer.
__global__ void __launch_bounds__(256) stage_tokens_kernel(const uint4* src, uint4* dst, int n) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------------------
// Router logits for decode: CTA = kRouterExperts warps = kRouterExperts
// experts.  The CTA's router-weight rows (contiguous) are bulk-copied into
// shared memory before griddepcontrol.wait, so they stream while the previous
// kernel on the stream finishes; only x is read after the wait.  Lane l forms
// the canonical partial over chunks l, l+32, ... then the xor butterfly.
constexpr int kRouterExperts = 1;
template <int TT>
__global__ void __launch_bounds__(kRouterExperts * 32) router_logits_decode_kernel(DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char rsm[];
  __shared__ __align__(8) uint64_t wbar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = blockIdx.x * kRouterExperts;
  const int ne = min(kRouterExperts, a.E - e0);
  const float* ws = reinterpret_cast<const float*>(rsm);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(&wbar))), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const unsigned row = static_cast<unsigned>(a.d) * 4u;
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&wbar));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(row * ne) : "memory");
    for (int r = 0; r < ne; ++r)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
                       "r"(static_cast<uint32_t>(__cvta_generic_to_shared(rsm + r * row))),
                   "l"(a.Wr + static_cast<size_t>(e0 + r) * a.d), "r"(row), "r"(bar)
                   : "memory");
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  // bounded wait for the weight rows
  {
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&wbar));
    uint32_t done = 0;
    unsigned long long t0 = 0;
    for (;;) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(done) : "r"(bar) : "memory");
      if (done) break;
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (!t0) t0 = t;
      else if (t - t0 > 2000000000ull) { if (a.status) atomicExch(a.status, 6 | (7 << 8)); return; }
    }
  }
  if (warp >= ne) return;
  const int e = e0 + warp;
  const float* wrow = ws + static_cast<size_t>(warp) * a.d;
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.f;
  const int chunks = a.d >> 3;
#pragma unroll 4
  for (int c = lane; c < chunks; c += 32) {
    const float4 w0 = *reinterpret_cast<const float4*>(wrow + 8 * c);
    const float4 w1 = *reinterpret_cast<const float4*>(wrow + 8 * c + 4);
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
  extern __shared__ __align__(16) float sm[];
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
#pragma unroll 8
        for (int j = 0; j < per; ++j) {
          const float u = ch[g0 + j];
          r += (u > v) | ((u == v) & (g0 + j > e));  // after(u, g0 + j, v, e), both indices valid
        }
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
      // candidates after this one (after(u, j, v, e) with both indices valid),
      // four per 16-byte broadcast load when the row allows it
      const float v = ch[e];
      int r = 0;
      int j0 = 0;
      if ((E & 3) == 0) {
        const float4* ch4 = reinterpret_cast<const float4*>(ch);
#pragma unroll 8
        for (int q = 0; q < (E >> 2); ++q) {
          const float4 u = ch4[q];
          const int j = 4 * q;
          r += (u.x > v) | ((u.x == v) & (j > e));
          r += (u.y > v) | ((u.y == v) & (j + 1 > e));
          r += (u.z > v) | ((u.z == v) & (j + 2 > e));
          r += (u.w > v) | ((u.w == v) & (j + 3 > e));
        }
        j0 = E;
      }
      for (int j = j0; j < E; ++j) r += (ch[j] > v) | ((ch[j] == v) & (j > e));
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

}  // namespace lg
