// Self-check of the tcgen05 building blocks in umma.cuh on one 128-row tile:
//   y[r] = sum_k W[r][k] * x[k]        (one token, K up to 4096)
// kind 0: W MXFP4 (E2M1 packed, low nibble = even column; UE8M0 per 32),
//         x split into T E2M1 terms (B rows 0..T-1 of a 32-row operand),
//         kind::mxf4 block-scaled MMAs, y = sum of the T accumulator columns;
//         the terms and their scales are also written out for checking.
// kind 1: W bf16, x bf16 as B row 0 of a 16-row operand, kind::f16 MMAs.
// One CTA of 128 threads; K is walked one 128-byte atom column at a time
// (256 E2M1 or 64 bf16 values per row), four MMAs per column.  Every wait is
// bounded; on a timeout the status word is set and no result is written.
#include <cstdint>
#include <cstdio>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "umma.cuh"
#include "grouped_dq.cuh"

namespace {

using namespace lg::umma;

constexpr int kRows = 128, kBRowsMx = 32, kBRowsBf = 16, kAtom = 128;
constexpr uint32_t kTmemCols = 64, kColD = 0, kColSfa = 32, kColSfb = 48;

__device__ bool wait_bar(uint64_t* bar, uint32_t parity) {
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    if (done) return true;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 1000000000ull) return false;
  }
}

__global__ void __launch_bounds__(128, 1) tile_kernel(int kind, const uint8_t* w, const uint8_t* wscale,
                                                      const uint16_t* x, int K, int T, float* y, uint8_t* terms,
                                                      uint8_t* tscales, int* status) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ uint8_t sfb[kBRowsMx][8];
  unsigned char* sa = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  unsigned char* sb = sa + kRows * kAtom;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool mx = kind == 0 || kind == 2;
  const bool packed = kind == 2;  // two MMAs per scale column, told apart by the scale-factor ids
  const int brows = mx ? kBRowsMx : kBRowsBf;
  const int per_col = mx ? 256 : 64;  // K values per atom column
  const int ncol = K / per_col;
  for (int i = tid; i < brows * kAtom / 16; i += 128) reinterpret_cast<uint4*>(sb)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(&tslot, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tslot, lanes = tbase + (static_cast<uint32_t>(warp * 32) << 16);
  const uint32_t idesc = mx ? idesc_mxf4(kRows, kBRowsMx) : idesc_bf16(kRows, kBRowsBf);
  bool ok = true;
  for (int c = 0; c < ncol && ok; ++c) {
    // A: this atom column of the 128 rows, swizzled
    for (int i = tid; i < kRows * 8; i += 128) {
      const int r = i >> 3, ch = i & 7;
      const size_t row_bytes = mx ? static_cast<size_t>(K) / 2 : static_cast<size_t>(K) * 2;
      const uint4 v = *reinterpret_cast<const uint4*>(w + r * row_bytes + static_cast<size_t>(c) * kAtom + ch * 16);
      *reinterpret_cast<uint4*>(sa + sw128_offset(r, ch * 16)) = v;
    }
    if (mx) {
      // B: T terms of this column's 8 blocks, one block per half-warp
      const int blk = warp * 2 + (lane >> 4), hl = lane & 15;
      const int k0 = c * 256 + blk * 32 + 2 * hl;
      float r0 = __uint_as_float(static_cast<uint32_t>(x[k0]) << 16), r1 = __uint_as_float(static_cast<uint32_t>(x[k0 + 1]) << 16);
      bool live;
      const int s0 = split_base(r0, r1, &live);
      for (int t = 0; t < T; ++t) {
        const uint32_t sc = live ? static_cast<uint32_t>(127 + term_scale(s0, t)) : 127u;
        const uint32_t byte = live ? split_step(r0, r1, term_scale(s0, t)) : 0u;
        sb[sw128_offset(t, blk * 16 + hl)] = static_cast<uint8_t>(byte);
        terms[static_cast<size_t>(t) * (K / 2) + c * 128 + blk * 16 + hl] = static_cast<uint8_t>(byte);
        if (hl == 0) {
          sfb[t][blk] = static_cast<uint8_t>(sc);
          tscales[static_cast<size_t>(t) * (K / 32) + c * 8 + blk] = static_cast<uint8_t>(sc);
        }
      }
      if (hl == 0)
        for (int t = T; t < kBRowsMx; ++t) sfb[t][blk] = 127;
    } else {
      if (tid < 8) *reinterpret_cast<uint4*>(sb + sw128_offset(0, tid * 16)) =
                       *reinterpret_cast<const uint4*>(x + static_cast<size_t>(c) * 64 + tid * 8);
    }
    fence_async_smem();
    __syncthreads();
    if (mx) {
      // scale factors of MMA i (blocks 2i, 2i+1 of this column) into tensor memory:
      // one column group per MMA, or (packed) MMAs 2j and 2j+1 in the low and
      // high halves of column group j
      for (int i = 0; i < 4; ++i) {
        const int col = packed ? 4 * (i >> 1) : 4 * i, shift = packed ? 16 * (i & 1) : 0;
        if (packed && (i & 1)) continue;  // written together with MMA i - 1
        for (int q = 0; q < 4; ++q) {
          const int r = 32 * q + lane;
          const uint8_t* s = wscale + static_cast<size_t>(r) * (K / 32) + c * 8 + 2 * i;
          uint32_t v = static_cast<uint32_t>(s[0]) | (static_cast<uint32_t>(s[1]) << 8);
          if (packed) v |= (static_cast<uint32_t>(s[2]) | (static_cast<uint32_t>(s[3]) << 8)) << 16;
          st_32x32b_x1(lanes + kColSfa + col + q, v << shift);
        }
        uint32_t vb = static_cast<uint32_t>(sfb[lane][2 * i]) | (static_cast<uint32_t>(sfb[lane][2 * i + 1]) << 8);
        if (packed)
          vb |= (static_cast<uint32_t>(sfb[lane][2 * i + 2]) | (static_cast<uint32_t>(sfb[lane][2 * i + 3]) << 8)) << 16;
        st_32x32b_x1(lanes + kColSfb + col, vb << shift);
      }
      wait_st();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (tid == 0) {
      const uint64_t da = desc_sw128(smem_addr(sa)), db = desc_sw128(smem_addr(sb));
      for (int i = 0; i < 4; ++i) {
        const bool acc = c > 0 || i > 0;
        if (packed)  // scale-factor ids 0 / 2 pick the low / high half of the column
          mma_mxf4(tbase + kColD, da + 2 * i, db + 2 * i, idesc | idesc_sf_ids(2 * (i & 1)),
                   tbase + kColSfa + 4 * (i >> 1), tbase + kColSfb + 4 * (i >> 1), acc);
        else if (mx)
          mma_mxf4(tbase + kColD, da + 2 * i, db + 2 * i, idesc, tbase + kColSfa + 4 * i, tbase + kColSfb + 4 * i, acc);
        else
          mma_bf16(tbase + kColD, da + 2 * i, db + 2 * i, idesc, acc);
      }
      commit(&bar);
    }
    ok = wait_bar(&bar, static_cast<uint32_t>(c & 1));
    fence_after_sync();
    ok = __syncthreads_and(ok) != 0;  // one verdict for the CTA; smem and scales are rewritten next
  }
  if (ok) {
    uint32_t d[32];
    ld_32x32b_x32(lanes + kColD, d);
    float s = 0.f;
    if (mx) {
      for (int t = 0; t < T; ++t) s = __fadd_rn(s, __uint_as_float(d[t]));
    } else {
      s = __uint_as_float(d[0]);
    }
    y[warp * 32 + lane] = s;
  } else if (tid == 0) {
    atomicExch(status, 1);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, kTmemCols);
}

}  // namespace

extern "C" int lg_umma_selftest_tile(int kind, const uint8_t* w, const uint8_t* wscale, const uint16_t* x, int K,
                                     int terms, float* y, uint8_t* terms_out, uint8_t* term_scales_out, int* status,
                                     void* stream) {
  if (kind < 0 || kind > 2) return 1;
  if (kind != 1 && (K < 256 || K > 4096 || K % 256 || terms < 1 || terms > 32 || !wscale || !terms_out || !term_scales_out))
    return 1;
  if (kind == 1 && (K < 64 || K > 4096 || K % 64)) return 1;
  if (!w || !x || !y || !status) return 1;
  const int smem = kRows * kAtom + kBRowsMx * kAtom + 1024;
  cudaError_t e = cudaFuncSetAttribute(tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return 2;
  tile_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(kind, w, wscale, x, K, terms, y, terms_out,
                                                                     term_scales_out, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// ---- MMA issue rate ---------------------------------------------------------------
// Throughput of back-to-back tcgen05.mma on resident shared-memory operands,
// one CTA per SM, one issuing thread: kind 0 = kind::mxf4 block32 (M=128, K=64
// per MMA, scale factors 1.0), kind 1 = kind::f16 bf16 (M=128, K=16).  Each
// group of 64 MMAs is committed to an mbarrier and waited for (bounded), so at
// most 64 are queued.  cycles_out[b] = clock64 cycles CTA b spent issuing.
namespace {
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int kind, int N, int groups, long long* cycles_out,
                                                          int* status) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tslot;
  unsigned char* sa = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  unsigned char* sb = sa + kRows * kAtom;
  const int tid = threadIdx.x, warp = tid >> 5;
  // operands: E2M1 bytes 0x22 (1.0, 1.0) or bf16 1/64; any finite values do
  for (int i = tid; i < (kRows + 256) * kAtom / 4; i += 128)
    reinterpret_cast<uint32_t*>(sa)[i] = kind == 0 ? 0x22222222u : 0x3C803C80u;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc(&tslot, 512);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tbase = tslot, lanes = tbase + (static_cast<uint32_t>(warp * 32) << 16);
  if (kind == 0) {  // scale factors 1.0 (127): A in columns 256..263, B in 264..279
    for (int c = 0; c < 24; ++c) st_32x32b_x1(lanes + 256 + c, 0x7F7F7F7Fu);
    wait_st();
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  if (tid == 0) {
    fence_async_smem();
    const uint64_t da = desc_sw128(smem_addr(sa)), db = desc_sw128(smem_addr(sb));
    const uint32_t id = kind == 0 ? idesc_mxf4(kRows, N) : idesc_bf16(kRows, N);
    bool ok = true;
    const long long c0 = clock64();
    for (int g = 0; g < groups && ok; ++g) {
      for (int i = 0; i < 64; ++i) {
        const int m = i & 3;
        if (kind == 0)
          mma_mxf4(tbase, da + 2 * m, db + 2 * m, id | idesc_sf_ids(2 * (m & 1)), tbase + 256 + 4 * (m >> 1),
                   tbase + 264 + 8 * (m >> 1), i > 0 || g > 0);
        else
          mma_bf16(tbase, da + 2 * m, db + 2 * m, id, i > 0 || g > 0);
      }
      commit(&bar);
      ok = wait_bar(&bar, static_cast<uint32_t>(g & 1));
    }
    cycles_out[blockIdx.x] = clock64() - c0;
    if (!ok) atomicExch(status, 1);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 512);
}
}  // namespace

extern "C" int lg_umma_mma_rate(int kind, int N, int groups, int ctas, long long* cycles_out, int* status,
                                void* stream) {
  if ((kind != 0 && kind != 1) || N < 16 || N > 256 || N % 16 || groups < 1 || groups > 100000 || ctas < 1 ||
      ctas > 1024 || !cycles_out || !status)
    return 1;
  const int smem = (kRows + 256) * kAtom + 1024;
  if (cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 2;
  mma_rate_kernel<<<ctas, 128, smem, static_cast<cudaStream_t>(stream)>>>(kind, N, groups, cycles_out, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// ---- E2M1 -> bf16 widening of the bf16 grouped GEMMs (grouped_dq.cuh) ------------
// out[i] = the eight bf16 values of words[i] under scale byte scales[i], by the
// same choice of table or f32 path as the converter warps.
namespace {
__global__ void widen_kernel(const uint32_t* words, const uint8_t* scales, int n, uint4* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t S = scales[i];
  out[i] = lg::gdq::lut_exact(S) ? lg::gdq::widen8(words[i], lg::gdq::make_lut(S)) : lg::gdq::widen8_slow(words[i], S);
}
}  // namespace

extern "C" int lg_dq_widen_selftest(const uint32_t* words, const uint8_t* scales, int n, void* out, void* stream) {
  if (!words || !scales || !out || n < 1 || n > (1 << 24)) return 1;
  widen_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(words, scales, n,
                                                                               static_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
