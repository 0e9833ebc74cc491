// Fifth-generation tensor core (tcgen05) primitives for sm_100a, and the
// activation split that lets a block-scaled MXFP4 MMA take bf16 activations.
//
// Operands live in shared memory in the canonical K-major layout with the
// 128-byte swizzle: row r of a tile at (r / 8) * 1024 + (r % 8) * 128 bytes,
// 16-byte chunk c of the row stored at chunk c ^ (r % 8), tile base 1024-byte
// aligned.  One such atom column holds 128 bytes of K per row: 256 E2M1
// values (four K=64 MMAs of kind::mxf4) or 64 bf16 values (four K=16 MMAs of
// kind::f16); the descriptor of the i-th MMA starts 32 * i bytes in.
//
// Scale factors (UE8M0, one per 32 values of a row) sit in tensor memory:
// for an M=128 operand the scales of row 32q + l are in lane l of every
// sub-partition (replicated), 32-bit column q, byte s = scale index s of the
// MMA; for a 32-row B operand one column, lane l = row l.
//
// Activation split (kind::mxf4 needs E2M1 on both sides): a bf16 vector is
// written as a sum of T terms, each term a row of E2M1 values with one UE8M0
// scale per 32-value block: the first term's scale maps the block's largest
// magnitude into [0, 6], each later term's scale is 4x smaller, and each term
// takes the round-to-nearest E2M1 of the residual, so the residual after t
// terms is at most 2^(s0 - 2(t-1)).  A bf16 value's residual stays a multiple
// of its own ulp, so values down to about 2^-(2T-7) of the block max come out
// exact (T = 16: the whole block for ordinary data).
// The MMA then sums the terms as separate B rows (N = T columns of the
// accumulator); products of E2M1 values and power-of-two scales are exact.
#pragma once
#include <cstdint>

#include <cuda_fp16.h>

namespace lg {
namespace umma {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), version 1 (sm_100).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;          // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version
  d |= static_cast<uint64_t>(2) << 61;          // 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::mxf4 with UE8M0 block-32 scales: A and B E2M1
// (format 1), K-major, f32 accumulate, M rows, N columns.
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Scale-factor ids of a block-scaled instruction descriptor (A: bits 29-30,
// B: bits 4-5): the byte of the tensor-memory column where the MMA's first
// scale sits, 0 or 2 for two block-32 scales per row.
__host__ __device__ constexpr uint32_t idesc_sf_ids(int id) {
  return (static_cast<uint32_t>(id) << 29) | (static_cast<uint32_t>(id) << 4);
}

// Instruction descriptor, kind::f16 with bf16 A and B (format 1), f32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of (row, byte) in a 128-byte-swizzled K-major tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int row, int byte) {
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15)));
}

// Tensor memory allocation: whole warp; the address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes made visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                         uint32_t sfb, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d), "l"(a), "l"(b),
      "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u)
      : "memory");
}
// The MMAs issued so far by this thread arrive on the mbarrier when done.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void st_32x32b_x1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v));
}
// 32 lanes x 32 consecutive columns of 32 bits (this warp's sub-partition).
__device__ __forceinline__ void st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]));
}
// 32 lanes x 8 / 16 consecutive columns of 32 bits (this warp's sub-partition).
__device__ __forceinline__ void st_32x32b_x8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]));
}
__device__ __forceinline__ void st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 columns of 32 bits (this warp's sub-partition), no wait.
__device__ __forceinline__ void ld_32x32b_x16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 8 columns of 32 bits (this warp's sub-partition), no wait.
__device__ __forceinline__ void ld_32x32b_x8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32 bits (this warp's sub-partition), then wait.
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- activation split --------------------------------------------------------

// UE8M0 exponent e (biased byte e + 127) of the smallest power of two with
// 6 * 2^e >= a, for a normal a >= 2^-100.
__device__ __forceinline__ int term_exponent(float a) {
  const uint32_t u = __float_as_uint(a);
  const int e0 = static_cast<int>((u >> 23) & 0xFFu) - 127;  // floor(log2 a)
  const bool low = (u & 0x7FFFFFu) <= 0x400000u;              // a / 2^e0 <= 1.5
  const int e = low ? e0 - 2 : e0 - 1;
  return e > 126 ? 126 : e;
}

// The split of a 32-value block held by a half-warp, two values per lane
// (lane i of the half: values 2i, 2i+1).  split_base reduces the block's
// largest magnitude once and returns the first term's exponent s0 (*live is
// false for a block below 2^-100, whose terms are all zero with scale byte
// 127); term t then uses the fixed exponent s0 - 2t: a residual is at most one
// grid step of the previous term, 2^(s0 - 2(t-1)), which the next term's range
// 6 * 2^(s0 - 2t) covers, so no term saturates and no further reduction is
// needed.
__device__ __forceinline__ int split_base(float r0, float r1, bool* live) {
  float a = fmaxf(fabsf(r0), fabsf(r1));
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  *live = a >= 0x1p-100f;
  return *live ? term_exponent(a) : 0;
}
// Round two f32 values to E2M1 (hardware round-to-nearest-even, saturating
// at 6): the byte's low nibble holds `lo`.
__device__ __forceinline__ uint32_t e2m1x2_rn(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 b;\n\tcvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\tcvt.u32.u8 %0, b;\n\t}" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// E2M1 byte -> the two values as f32 (low nibble first).
__device__ __forceinline__ void e2m1x2_to_f32(uint32_t byte, float& lo, float& hi) {
  uint32_t h;
  asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}" : "=r"(h) : "r"(byte));
  lo = __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
  hi = __half2float(__ushort_as_half(static_cast<unsigned short>(h >> 16)));
}

// One term at exponent s (|s| <= 126): the E2M1 byte of the lane's pair; the
// residual pair loses the term's value.
__device__ __forceinline__ uint32_t split_step(float& r0, float& r1, int s) {
  const float inv = __int_as_float((127 - s) << 23), sc = __int_as_float((127 + s) << 23);
  const uint32_t byte = e2m1x2_rn(r0 * inv, r1 * inv);
  float q0, q1;
  e2m1x2_to_f32(byte, q0, q1);
  r0 = __fsub_rn(r0, q0 * sc);
  r1 = __fsub_rn(r1, q1 * sc);
  return byte;
}

// Exponent of term t, kept >= -126 (a live block reaches that only after
// its residual is below 2^-120; E2M1 saturates at 6 there).
__device__ __forceinline__ int term_scale(int s0, int t) {
  const int s = s0 - 2 * t;
  return s < -126 ? -126 : s;
}

}  // namespace umma
}  // namespace lg
