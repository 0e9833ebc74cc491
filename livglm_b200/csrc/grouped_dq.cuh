// Batched routed experts on the fifth-generation tensor core with the MXFP4
// weights widened to bf16 in shared memory (sm_100a).
//
// The routed half of grouped_tc.cuh's products, for calls whose experts see
// many routes each (kg36/livglm src/glm53flash/expert_ssd.py:159-188: MXFP4
// gather_qmm gate/up, limited SwiGLU, down):
//
//   routed gate/up   act[p]   = swiglu(bf16(Wg_e x_t), bf16(Wu_e x_t))
//   routed down      y[s(p)]  = bf16(Wd_e act[p])
//
// as kind::f16 MMAs on bf16 operands.  The A operand is the weights: worker
// warps load each stage's checkpoint bytes (E2M1 nibbles, 64 values = 32 bytes
// a row) from global memory into registers and widen them to bf16 -- an E2M1
// value times a power-of-two scale is exact in bf16 -- straight into the
// MMA's 128-byte-swizzled K-major layout.  The B operand is bf16 rows in
// dispatch order: the tokens gathered once per call (gather_rows_kernel) or
// act.  The products are then exactly those of a dequantised matmul, with no
// activation split, and one stage of 64 K values serves up to 256 routes, so
// a weight block is read once per 256 routes and a route row once per 256
// weight rows: the traffic from L2 that bounds narrow tiles shrinks by 3-4x.
// The cost: four MMAs (K = 16) per 64 values of K where kind::mxf4 needs one
// (K = 64), which only large route counts amortise; grouped_tc.cuh keeps the
// smaller batches.
//
// Work item: (expert e, row block rb, route chunk).  Gate/up: 128 gate rows
// and the 128 up rows with the same indices, two accumulators of N columns
// (N = the chunk's routes rounded up to 32, at most 256), so SwiGLU is local to
// a thread (lane = row, column = route).  Down: 256 rows of Wd in two
// accumulators.  An expert's routes split into ceil(count / 256) chunks of
// equal size.  Items are ordered (expert, row block, chunk), chunk fastest; one
// persistent CTA per SM walks items b, b + P, ...
//
// Warps: 0 TMA producer of the B rows (also prefetches the weight bytes into
// L2 a few stages ahead), 1 MMA issuer (one lane), 2-17 workers in two
// groups that take alternate stages (thread u widens A row u % 256 of the
// stages ks % 2 == u / 256, loading its 32 packed bytes a stage straight from
// global memory a few stages ahead) and, between items, run the
// epilogue of the previous item (tcgen05.ld of the two accumulators; 512
// tensor-memory columns, single-buffered): after converting the first stages
// of item i they wait for item i - 1's accumulators, write its outputs and
// release the tensor memory, so the MMAs of item i start on converted stages.
// SwiGLU reads bf16(g * bf16(sigmoid(g))) from a table of all bf16 g
// (silu_table_kernel, same arithmetic as swiglu_bf16).  Every wait is
// bounded: a timeout records 6 | site in the status word; a worker that gave
// up skips its remaining waits and work, the workers agree on failures at the
// next epilogue's named barrier and leave together, and the CTA leaves after
// its copies and MMAs in flight have landed.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "umma.cuh"
#include "down_tc.cuh"
#include "grouped_tc.cuh"

namespace lg {
namespace gdq {

constexpr int kBProdWarp = 0, kMmaWarp = 1, kWorkWarp0 = 2, kWorkWarps = 16;
constexpr int kThreads = 32 * (kWorkWarp0 + kWorkWarps);
constexpr int kWorkThreads = 32 * kWorkWarps;
constexpr int kGroupWarps = kWorkWarps / 2;  // two worker groups take alternate stages
constexpr int kNMax = 256;          // routes per item (MMA N)
constexpr int kBoxRows = 32;        // B rows per TMA box; N is a multiple of it
constexpr int kBBytes = kNMax * 128;
constexpr int kConvBytes = 32768;   // converted slot: 2 x 128 rows x 64 bf16 (two A operands)
constexpr int kBStages = 4, kConvSlots = 3;
constexpr int kConvOff = kBStages * kBBytes;
constexpr int kSmemBytes = kConvOff + kConvSlots * kConvBytes;  // from the 1024-aligned base
constexpr int kPrefetch = 16;       // stages between an L2 prefetch of weight bytes and their load
constexpr int kWorkBar = 3;         // named barrier of the worker warps
constexpr int kSiteBFull = 50 << 8, kSiteBEmpty = 51 << 8, kSiteConv = 52 << 8, kSiteAccFull = 53 << 8,
              kSiteAccEmpty = 54 << 8, kSiteDrain = 55 << 8, kSiteConvEmpty = 56 << 8;

struct Args {
  int d, F, E, R;
  int ks_count;         // stages (64 values of K) per item
  int rb_count;         // row blocks per expert
  int rb_rows;          // bank rows per row block: 128 (gate/up) or 256 (down)
  int acc1_rows;        // row offset of accumulator 1 within the block: 0 (up bank) or 128 (down)
  float limit;
  const int* offsets;      // [E + 1] dispatch offsets
  const int* perm;         // [R] route slot of dispatch position p
  const int* chunk_start;  // [E + 1] route chunks of experts before e
  const uint8_t* pk0;      // packed bank of accumulator 0 rows (gate or down)
  const uint8_t* pk1;      // of accumulator 1 rows (up or down)
  long long pk0_stride, pk1_stride;  // bytes between experts
  int pk_row;              // packed bytes per row: K / 2
  const uint8_t* sc0;      // scale bank of accumulator 0 rows (gate or down)
  const uint8_t* sc1;      // of accumulator 1 rows (up or down)
  long long sc0_stride, sc1_stride;  // bytes between experts
  int sc_row;              // scale bytes per row: K / 32
  const uint16_t* silu;    // [65536] silu_bf16 of every bf16 bit pattern
  uint16_t* act;           // [R][F] gate/up output, dispatch order
  uint16_t* y;             // [R][d] down output, slot order
  int* status;
};

// ---- operands in dispatch order --------------------------------------------------
// xp[p] = x[perm[p] / k] for every dispatched position p; d % 8 == 0.  A warp
// per row: one perm read, then the row's 16-byte words with eight loads in
// flight per lane.
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x, int d, int k,
                                                          const int* __restrict__ perm,
                                                          const int* __restrict__ offsets, int E,
                                                          uint16_t* __restrict__ xp) {
  const int n = offsets[E];
  const int per_row = d / 8;
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += warps) {
    const int t = __ldg(perm + p) / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * d);
    uint4* dst = reinterpret_cast<uint4*>(xp + static_cast<size_t>(p) * d);
    for (int c0 = 0; c0 < per_row; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < per_row) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < per_row) dst[c] = v[u];
      }
    }
  }
}

// The shared expert's one-"expert" tables: offsets {0, M}, chunk_start {0, ceil(M / 256)}.
__global__ void shared_table_kernel(int M, int nch, int* __restrict__ tab) {
  if (threadIdx.x == 0) {
    tab[0] = 0;
    tab[1] = M;
    tab[2] = 0;
    tab[3] = nch;
  }
}

// tab[b] = silu_bf16 of the bf16 value with bits b.
__global__ void __launch_bounds__(256) silu_table_kernel(uint16_t* __restrict__ tab) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < 65536) tab[b] = silu_bf16(bf16_to_f32(static_cast<uint32_t>(b)));
}

// ---- E2M1 -> bf16 -------------------------------------------------------------------
// Byte tables for prmt: the bf16 bits of E2M1 magnitude code c (0..7: 0, 0.5,
// 1, 1.5, 2, 3, 4, 6) times 2^(S - 127): hi / lo bytes of codes 0-3 in (ha, la),
// of codes 4-7 in (hb, lb).  Exact for 2 <= S <= 252 (every nonzero result a
// normal bf16); the scale only shifts the exponent field, added to both
// 16-bit halves of a word at once.
struct Lut {
  uint32_t ha, hb, la, lb;
};
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ Lut make_lut(uint32_t S) {
  const uint32_t dd = (S - 127u) * 0x00800080u;  // (S - 127) << 7 in both halves
  const uint32_t w01 = (0x3F00u + (S - 127u) * 0x80u) << 16;  // codes 0 (zero), 1
  const uint32_t w23 = 0x3FC03F80u + dd, w45 = 0x40404000u + dd, w67 = 0x40C04080u + dd;
  return Lut{prmt(w01, w23, 0x7531u), prmt(w45, w67, 0x7531u), prmt(w01, w23, 0x6420u), prmt(w45, w67, 0x6420u)};
}
// Eight E2M1 values (one word, nibble i = value i) -> four bf16x2 words.
__device__ __forceinline__ uint4 widen8(uint32_t w, const Lut& t) {
  const uint32_t m0 = w & 0x77777777u, m1 = m0 >> 16;
  uint32_t hi0 = prmt(t.ha, t.hb, m0), lo0 = prmt(t.la, t.lb, m0);
  uint32_t hi1 = prmt(t.ha, t.hb, m1), lo1 = prmt(t.la, t.lb, m1);
  // sign bit of value i (bit 4i + 3) -> bit 7 of byte i of the hi bytes
  const uint32_t w4 = w << 4;
  hi0 |= prmt(w4, w, 0x5140u) & 0x80808080u;
  hi1 |= prmt(w4, w, 0x7362u) & 0x80808080u;
  return make_uint4(prmt(lo0, hi0, 0x5140u), prmt(lo0, hi0, 0x7362u), prmt(lo1, hi1, 0x5140u),
                    prmt(lo1, hi1, 0x7362u));
}
// Scale bytes the tables widen exactly.
__device__ __forceinline__ bool lut_exact(uint32_t S) { return S >= 2u && S <= 252u; }
// The same for any scale byte, through f32 (scale 255 is NaN; 0 is 2^-127).
__device__ __forceinline__ uint4 widen8_slow(uint32_t w, uint32_t S) {
  const float s = S == 255u ? __uint_as_float(0x7FC00000u)
                            : (S == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(S << 23));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t n = (w >> (8 * i + 4 * h)) & 0xFu;
      const uint32_t c = n & 7u;
      const float mag =
          c < 4u ? 0.5f * static_cast<float>(c) : static_cast<float>(1u << ((c >> 1) - 1u)) * (c & 1u ? 1.5f : 1.f);
      v[h] = (n & 8u ? -mag : mag) * s;
    }
    o[i] = static_cast<uint32_t>(f32_to_bf16(v[0])) | (static_cast<uint32_t>(f32_to_bf16(v[1])) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- route chunks --------------------------------------------------------------------
// chunk_start[e] = route chunks (ceil(count / kNMax)) of experts before e; one CTA.
__global__ void __launch_bounds__(1024) chunk_table_kernel(const int* __restrict__ offsets, int E,
                                                           int* __restrict__ chunk_start) {
  __shared__ int part[32];
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  const int n = e < E ? (offsets[e + 1] - offsets[e] + kNMax - 1) / kNMax : 0;
  int v = n;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) part[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (blockDim.x >> 5) ? part[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    part[lane] = w;
  }
  __syncthreads();
  const int incl = v + (warp > 0 ? part[warp - 1] : 0);
  if (e < E) chunk_start[e + 1] = incl;
  if (e == 0) chunk_start[0] = 0;
}

struct Item {
  int e, rb, p0;
  int nt;  // routes in the chunk (>= 1)
  int n;   // nt rounded up to kBoxRows: MMA N and B rows loaded
};
constexpr int kChunkMajorMin = 4;  // chunks of an expert from which its items go chunk-major

// Item i: expert e owns items [RB * cs[e], RB * cs[e + 1]), ordered (chunk,
// row block), row block fastest, when the expert has kChunkMajorMin chunks or
// more, else (row block, chunk), chunk fastest.  A routed expert's count c splits into
// nch = ceil(c / 256) chunks of cs = ceil(c / nch) rounded up to 32 routes
// (cs <= 256, and every chunk is nonempty: (nch - 1) * 256 < c); the shared
// expert's chunk count comes from the host (shared_chunks), also with no
// empty chunk.
__device__ __forceinline__ bool item_of(const Args& a, const int* cs, int i, Item& it) {
  const int RB = a.rb_count;
  if (i >= RB * cs[a.E]) return false;
  int lo = 0, hi = a.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (RB * cs[mid] <= i) lo = mid;
    else hi = mid;
  }
  const int nch = cs[lo + 1] - cs[lo];
  const int local = i - RB * cs[lo];
  // An expert of many chunks goes chunk-major: consecutive items (co-scheduled
  // CTAs) take every row block of one route chunk, so the chunk's B rows are
  // read from HBM once and then served by L2 however many chunks the expert
  // has.  With few chunks, row-block-major keeps a weight block's re-reads
  // adjacent instead.
  const bool chunk_major = nch >= kChunkMajorMin;
  const int j = chunk_major ? local / RB : local % nch;
  const int rb = chunk_major ? local - j * RB : local / nch;
  const int cnt = a.offsets[lo + 1] - a.offsets[lo];
  const int csz = ((cnt + nch - 1) / nch + kBoxRows - 1) / kBoxRows * kBoxRows;
  it.e = lo;
  it.rb = rb;
  it.p0 = a.offsets[lo] + j * csz;
  it.nt = min(csz, cnt - j * csz);
  it.n = (it.nt + kBoxRows - 1) / kBoxRows * kBoxRows;
  return true;
}

// ---- the kernel ----------------------------------------------------------------------
__device__ __forceinline__ void prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// mA0 / mA1: 3-D [E][rows][bytes] packed banks of the accumulator 0 / 1 rows
// (L2 prefetches only); mB: 2-D [R][K * 2 bytes] B rows, 128-byte x 32-row
// boxes with the 128-byte swizzle.
// Shared memory: a ring of kBStages B stages and kConvSlots widened A slots,
// both freed by the MMAs' commit.  The packed weight bytes never pass
// through shared memory: each worker loads its row's 32 bytes of a stage
// from global memory into registers one of its stages (two stages) early.
// kBf16A: the shared expert -- bf16 weight rows loaded by TMA straight into the
// A slots (mA0 / mA1: 2-D [rows][K * 2 bytes], 128-byte x 128-row boxes, 128-byte
// swizzle), no widening; the "routes" are the tokens in order (perm == nullptr).
template <bool kGateUp, bool kBf16A = false>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_dq_kernel(Args a, const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
                      const __grid_constant__ CUtensorMap mB) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  __shared__ __align__(8) uint64_t bfull[kBStages], bempty[kBStages];
  __shared__ __align__(8) uint64_t conv_full[kConvSlots], conv_empty[kConvSlots];
  __shared__ __align__(8) uint64_t acc_full, acc_empty, drain;
  __shared__ uint32_t tslot;
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  unsigned char* conv = base + kConvOff;
  const int* cs = a.chunk_start;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    for (int c = 0; c < kConvSlots; ++c) {
      mbar_init(&conv_full[c], kBf16A ? 1 : kGroupWarps);
      mbar_init(&conv_empty[c], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&acc_empty, kWorkWarps);
    mbar_init(&drain, 1);
    mbar_fence_init();
  }
  if (warp == kMmaWarp) umma::tmem_alloc(&tslot, 512);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = tslot;
  auto next_item = [&](int seq, Item& it) -> bool { return item_of(a, cs, blockIdx.x + seq * P, it); };

  // ------------------------------ B producer --------------------------------
  // Also requests the weight bytes of stage i + kPrefetch into L2 when it
  // issues the B rows of stage i.
  if (warp == kBProdWarp) {
    if (lane == 0) {
      bool ok = true;
      int it_k = 0;
      Item item, pitem;
      int pseq = 0, pks = 0;
      bool phave = next_item(0, pitem);
      auto pf_step = [&]() {
        if (kBf16A || !phave) return;
        prefetch_3d(&mA0, pks * 32, pitem.rb * a.rb_rows, pitem.e);
        prefetch_3d(&mA1, pks * 32, pitem.rb * a.rb_rows + a.acc1_rows, pitem.e);
        if (++pks == a.ks_count) {
          pks = 0;
          phave = next_item(++pseq, pitem);
        }
      };
      for (int q = 0; q < kPrefetch; ++q) pf_step();
      for (int seq = 0; ok && next_item(seq, item); ++seq) {
        const unsigned bytes = static_cast<unsigned>(item.n * 128);
        for (int ks = 0; ks < a.ks_count; ++ks, ++it_k) {
          const int s = it_k % kBStages;
          if (it_k >= kBStages) ok = dtc::wait1(&bempty[s], ((it_k / kBStages) - 1) & 1, a.status, kSiteBEmpty);
          if (!ok) break;
          unsigned char* bt = base + s * kBBytes;
          if (kBf16A) {  // the stage's A tiles into widened slot it_k % kConvSlots
            const int c = it_k % kConvSlots;
            if (it_k >= kConvSlots)
              ok = dtc::wait1(&conv_empty[c], ((it_k / kConvSlots) - 1) & 1, a.status, kSiteConvEmpty);
            if (!ok) break;
            unsigned char* at = conv + c * kConvBytes;
            const int y0 = item.rb * a.rb_rows;
            mbar_arrive_expect_tx(&conv_full[c], kConvBytes);
            dtc::tma_2d(at, &mA0, ks * 128, y0, &conv_full[c]);
            dtc::tma_2d(at + kConvBytes / 2, &mA1, ks * 128, y0 + a.acc1_rows, &conv_full[c]);
          }
          mbar_arrive_expect_tx(&bfull[s], bytes);
          for (int b = 0; b < item.n / kBoxRows; ++b)
            dtc::tma_2d(bt + b * (kBoxRows * 128), &mB, ks * 128, item.p0 + b * kBoxRows, &bfull[s]);
          pf_step();
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA leaves
        for (int q = (it_k > kBStages ? it_k - kBStages : 0); q < it_k; ++q)
          dtc::wait1(&bfull[q % kBStages], (q / kBStages) & 1, a.status, kSiteBFull);
        if (kBf16A)
          for (int q = (it_k > kConvSlots ? it_k - kConvSlots : 0); q < it_k; ++q)
            dtc::wait1(&conv_full[q % kConvSlots], (q / kConvSlots) & 1, a.status, kSiteConv);
      }
    }
    __syncwarp();
  }
  // ------------------------------ MMA issuer --------------------------------
  else if (warp == kMmaWarp) {
    if (lane == 0) {
      bool ok = true;
      int it_k = 0;
      Item item;
      const uint32_t acc0 = tbase, acc1 = tbase + kNMax;
      for (int seq = 0; ok && next_item(seq, item); ++seq) {
        if (seq >= 1) ok = dtc::wait1(&acc_empty, (seq - 1) & 1, a.status, kSiteAccEmpty);
        if (!ok) break;
        umma::fence_after_sync();
        const uint32_t idesc = umma::idesc_bf16(128, item.n);
        for (int ks = 0; ks < a.ks_count && ok; ++ks, ++it_k) {
          const int s = it_k % kBStages, c = it_k % kConvSlots;
          ok = dtc::wait1(&conv_full[c], (it_k / kConvSlots) & 1, a.status, kSiteConv) &&
               dtc::wait1(&bfull[s], (it_k / kBStages) & 1, a.status, kSiteBFull);
          if (!ok) break;
          umma::fence_after_sync();
          const uint64_t da0 = umma::desc_sw128(smem_u32(conv + c * kConvBytes));
          const uint64_t da1 = umma::desc_sw128(smem_u32(conv + c * kConvBytes + kConvBytes / 2));
          const uint64_t db = umma::desc_sw128(smem_u32(base + s * kBBytes));
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const bool accum = ks > 0 || m > 0;
            umma::mma_bf16(acc0, da0 + 2 * m, db + 2 * m, idesc, accum);
            umma::mma_bf16(acc1, da1 + 2 * m, db + 2 * m, idesc, accum);
          }
          umma::commit(&bempty[s]);
          umma::commit(&conv_empty[c]);
        }
        if (ok) umma::commit(&acc_full);
      }
      umma::commit(&drain);  // every MMA issued above has finished once this arrives
      dtc::wait1(&drain, 0, a.status, kSiteDrain);
    }
    __syncwarp();
  }
  // ------------------------------ workers -----------------------------------
  else {
    const int u = threadIdx.x - kWorkWarp0 * 32;  // 0..511
    const int grp = u >> 8;                        // stages ks % 2 == grp of every item
    const int row = u & 255;                       // A row: accumulator row / 128, row % 128 within it
    const int acc = row >> 7, r = row & 127;
    const int periods = a.ks_count / 8;           // 16 scale bytes (8 stages) per period
    auto row_of = [&](const Item it) { return it.rb * a.rb_rows + (acc ? a.acc1_rows : 0) + r; };
    auto scale_row = [&](const Item it) -> const uint8_t* {
      const uint8_t* bank = acc ? a.sc1 + it.e * a.sc1_stride : a.sc0 + it.e * a.sc0_stride;
      return bank + static_cast<size_t>(row_of(it)) * a.sc_row;
    };
    auto packed_row = [&](const Item it) -> const uint8_t* {
      const uint8_t* bank = acc ? a.pk1 + it.e * a.pk1_stride : a.pk0 + it.e * a.pk0_stride;
      return bank + static_cast<size_t>(row_of(it)) * a.pk_row;
    };
    // epilogue of one item: warp w reads tensor-memory lanes 32 (w & 3) ..,
    // quarter q = (w - kWorkWarp0) / 4 of the work.  Every worker calls it at
    // the same point with its own verdict; all leave together on a failure.
    const int sp = warp & 3, q = (warp - kWorkWarp0) >> 2;
    const uint32_t lanes = tbase + (static_cast<uint32_t>(sp * 32) << 16);
    const int er = sp * 32 + lane;
    auto epilogue = [&](const Item it, int seq, bool ok) -> bool {
      // down: the route slots of this warp's columns, loaded before the wait
      // (lane i holds the slots of columns c_lo + i, c_lo + 32 + i, ...)
      int slots[4] = {0, 0, 0, 0};
      const int dh = q >> 1, c_lo_d = (q & 1) * (it.n / 2);
      if (!kGateUp) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int c = c_lo_d + 32 * k + lane;
          if (32 * k < it.n / 2 && c < it.nt) slots[k] = kBf16A ? it.p0 + c : __ldg(a.perm + it.p0 + c);
        }
      }
      if (ok) ok = dtc::wait_warp1(&acc_full, seq & 1, a.status, kSiteAccFull);
      ok = named_and(kWorkBar, kWorkThreads, ok);
      if (!ok) return false;
      umma::fence_after_sync();
      if (kGateUp) {  // columns [q n/4, (q + 1) n/4) of both accumulators
        const int f = it.rb * 128 + er;
        const int c_lo = q * (it.n / 4), c_hi = c_lo + it.n / 4;
        for (int c0 = c_lo; c0 < c_hi; c0 += 8) {
          uint32_t vg[8], vu[8];
          umma::ld_32x32b_x8_nowait(lanes + c0, vg);
          umma::ld_32x32b_x8_nowait(lanes + kNMax + c0, vu);
          umma::wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (c0 + i < it.nt) {
              const float g = round_bf16(__uint_as_float(vg[i])), uu = round_bf16(__uint_as_float(vu[i]));
              a.act[static_cast<size_t>(it.p0 + c0 + i) * a.F + f] = swiglu_bf16_tab(g, uu, a.limit, a.silu);
            }
          }
        }
      } else {  // accumulator q / 2, columns [(q % 2) n/2, (q % 2 + 1) n/2)
        const int drow = it.rb * 256 + dh * 128 + er;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int cb = c_lo_d + 32 * k;
          if (32 * k >= it.n / 2) break;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t v[16];
            umma::ld_32x32b_x16_nowait(lanes + dh * kNMax + cb + 16 * hh, v);
            umma::wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int slot = __shfl_sync(0xffffffffu, slots[k], 16 * hh + i);
              if (cb + 16 * hh + i < it.nt)
                a.y[static_cast<size_t>(slot) * a.d + drow] = f32_to_bf16(__uint_as_float(v[i]));
            }
          }
        }
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty);
      return true;
    };
    if (kBf16A) {  // the A tiles come by TMA: the workers only run the epilogues
      Item it;
      for (int seq = 0; next_item(seq, it); ++seq)
        if (!epilogue(it, seq, true)) break;
    } else {
    // This group's stages: ks = grp, grp + 2, ... of every item.  Weight bytes
    // and scales are loaded ahead along that sequence, across items; the
    // iterators keep row pointers only (items are recomputed where needed).
    Item tmp;
    bool have = next_item(0, tmp);
    const uint8_t* ld_row = have ? packed_row(tmp) : nullptr;
    const uint8_t* sc_ptr = have ? scale_row(tmp) : nullptr;
    int ld_seq = 0, ld_ks = grp, sc_seq = 0, sc_per = 0;
    bool ld_have = have, sc_have = have;
    uint4 wq[2];  // packed bytes of this group's next stage
    auto ld_next = [&]() {
      if (ld_have) {
        const uint4* src = reinterpret_cast<const uint4*>(ld_row + ld_ks * 32);
        wq[0] = __ldg(src);
        wq[1] = __ldg(src + 1);
        ld_ks += 2;
        if (ld_ks >= a.ks_count) {
          ld_ks = grp;
          Item t;
          ld_have = next_item(++ld_seq, t);
          if (ld_have) ld_row = packed_row(t);
        }
      }
    };
    ld_next();
    uint4 sc_next = make_uint4(0, 0, 0, 0), sc_cur = sc_next;
    if (have) sc_next = __ldg(reinterpret_cast<const uint4*>(sc_ptr));
    const uint32_t conv_row = static_cast<uint32_t>(acc * (kConvBytes / 2) + (r >> 3) * 1024 + (r & 7) * 128);
    bool ok = true, done = false;
    int seq = 0;
    for (; have && !done; ++seq) {
      for (int ks = grp; ks < a.ks_count; ks += 2) {
        const int it_k = seq * a.ks_count + ks;
        if ((ks & 7) == grp) {  // this group's first stage of a period of 8
          sc_cur = sc_next;
          if (++sc_per == periods) {
            sc_per = 0;
            Item t;
            sc_have = next_item(++sc_seq, t);
            if (sc_have) sc_ptr = scale_row(t);
          }
          if (sc_have) sc_next = __ldg(reinterpret_cast<const uint4*>(sc_ptr) + sc_per);
        }
        // this stage's packed bytes, then the load of this group's next stage
        const uint4 w0 = wq[0], w1 = wq[1];
        ld_next();
        const int c = it_k % kConvSlots;
        if (ok && it_k >= kConvSlots)
          ok = dtc::wait_warp1(&conv_empty[c], ((it_k / kConvSlots) - 1) & 1, a.status, kSiteConvEmpty);
        if (ok) {
          const int j = ks & 7;
          const uint32_t wsc = j < 4 ? (j < 2 ? sc_cur.x : sc_cur.y) : (j < 6 ? sc_cur.z : sc_cur.w);
          unsigned char* cv = conv + c * kConvBytes + conv_row;
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // 32 values (one scale) per half
            const uint32_t S8 = (wsc >> ((j & 1) * 16 + 8 * h)) & 0xFFu;
            const uint4 qv = h ? w1 : w0;
            const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
            if (lut_exact(S8)) {
              const Lut lut = make_lut(S8);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4*>(cv + (((4 * h + k) ^ (r & 7)) << 4)) = widen8(qw[k], lut);
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4*>(cv + (((4 * h + k) ^ (r & 7)) << 4)) = widen8_slow(qw[k], S8);
            }
          }
          umma::fence_async_smem();  // the generic-proxy writes, seen by the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv_full[c]);
        }
        if (seq > 0 && ks == grp) {  // both groups have converted the item's first stage each
          Item pv;
          next_item(seq - 1, pv);
          if (!epilogue(pv, seq - 1, ok)) {
            done = true;
            break;
          }
        }
      }
      if (done) break;
      have = next_item(seq + 1, tmp);
    }
    if (!done && seq > 0) {
      Item pv;
      next_item(seq - 1, pv);
      epilogue(pv, seq - 1, ok);
    }
    }
  }
  __syncwarp();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) umma::tmem_dealloc(tbase, 512);
}

}  // namespace gdq
}  // namespace lg
