// Shared device helpers for the GLM MoE block kernels (sm_100a).
//
// The router arithmetic here is the "canonical router arithmetic" that the
// CPU checker restates operation for operation: every floating-point step is
// an explicit round-to-nearest intrinsic so that nvcc cannot contract or
// reorder it.  Reference semantics: kg36/livglm src/glm53flash/moe.py:36-63.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lg {

constexpr int kWarp = 32;

__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// ---- own exp / sigmoid ----------------------------------------------------
// exp(x): Cody-Waite reduction x = n*ln2 + r with ln2 split into a high part
// whose low 12 mantissa bits are zero (n*LN2_HI is exact for |n| < 2^12) and
// the float32 remainder, then the degree-8 Taylor polynomial of e^r in Horner
// form, then scaling by 2^n as two power-of-two multiplies.
__device__ __forceinline__ float pow2i(int n) {  // -126 <= n <= 127
  return __uint_as_float(static_cast<uint32_t>(n + 127) << 23);
}
__device__ __forceinline__ float own_expf(float x) {
  if (x > 89.0f) return __uint_as_float(0x7f800000u);
  if (x < -104.0f) return 0.0f;
  const float kMagic = 0x1.8p23f;
  float t = __fmaf_rn(x, 0x1.715476p+0f, kMagic);
  float n = __fsub_rn(t, kMagic);
  float r = __fmaf_rn(n, -0x1.62ep-1f, x);
  r = __fmaf_rn(n, -0x1.0bfbe8p-15f, r);
  float p = 0x1.a01a02p-16f;
  p = __fmaf_rn(p, r, 0x1.a01a02p-13f);
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1.0p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = static_cast<int>(n);
  int n1 = ni >> 1;
  int n2 = ni - n1;
  return __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(n2));
}
__device__ __forceinline__ float own_sigmoidf(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, own_expf(-v)));
}

// limited SwiGLU with the bf16 rounding points of the MLX graph
// (expert_ssd.py:103-107): every op's result is rounded to bf16.
__device__ __forceinline__ uint16_t swiglu_bf16(float g, float u, float limit) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  float s = round_bf16(own_sigmoidf(g));
  float a = round_bf16(__fmul_rn(g, s));
  return f32_to_bf16(__fmul_rn(a, u));
}
// bf16(g * bf16(sigmoid(g))) of a bf16 g, the first two roundings of
// swiglu_bf16 after the clip; tabulated for all 65536 bf16 bit patterns.
__device__ __forceinline__ uint16_t silu_bf16(float g) {
  return f32_to_bf16(__fmul_rn(g, round_bf16(own_sigmoidf(g))));
}
// swiglu_bf16 with the silu factor read from such a table (same result).
__device__ __forceinline__ uint16_t swiglu_bf16_tab(float g, float u, float limit, const uint16_t* __restrict__ silu) {
  if (limit > 0.0f) {
    g = fminf(g, limit);
    u = fminf(fmaxf(u, -limit), limit);
  }
  const float a = bf16_to_f32(__ldg(silu + f32_to_bf16(g)));
  return f32_to_bf16(__fmul_rn(a, u));
}

// ---- MXFP4 (OCP MX, group 32) -------------------------------------------
// E8M0 scale byte s -> 2^(s-127); 255 is NaN; 0 is the subnormal 2^-127.
__device__ __forceinline__ float e8m0_to_f32(uint32_t s) {
  return s == 0u ? __uint_as_float(0x00400000u)
                 : (s == 255u ? __uint_as_float(0x7fc00000u) : __uint_as_float(s << 23));
}

// Eight E2M1 nibbles of one little-endian word -> eight floats.  Nibble 2i
// (the low nibble of byte i) is the earlier column, as in the checkpoint's
// U8 [rows, cols/2] layout (expert_source.py:189-229).
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t w, float (&v)[8]) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  float2 f0 = __half22float2(*reinterpret_cast<__half2*>(&h0));
  float2 f1 = __half22float2(*reinterpret_cast<__half2*>(&h1));
  float2 f2 = __half22float2(*reinterpret_cast<__half2*>(&h2));
  float2 f3 = __half22float2(*reinterpret_cast<__half2*>(&h3));
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  v[4] = f2.x; v[5] = f2.y; v[6] = f3.x; v[7] = f3.y;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// (value, index) order of a stable ascending sort; idx < 0 marks "none".
__device__ __forceinline__ bool after(float a, int ia, float b, int ib) {
  if (ib < 0) return ia >= 0;
  if (ia < 0) return false;
  return a > b || (a == b && ia > ib);
}
__device__ __forceinline__ void warp_best(float& v, int& i) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, off);
    int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (after(ov, oi, v, i)) { v = ov; i = oi; }
  }
}

}  // namespace lg
