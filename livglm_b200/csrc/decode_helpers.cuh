// Helpers of the CUDA-core decode kernels (sm_100a): bounded warp-wide
// mbarrier waits with a short suspend hint, shared-memory load shorthands,
// E2M1 -> f16x2 conversion with packed f16x2 FMA chains, a deterministic
// reduce-scatter over lane segments, and the power-of-two activation scaling
// that keeps f16 chains in range.
#pragma once
#include "decode_kernels.cuh"
#include "pipeline.cuh"

namespace lg {
namespace dh {

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


}  // namespace dh
}  // namespace lg
