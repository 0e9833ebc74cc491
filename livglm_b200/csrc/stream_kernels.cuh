// Streaming expert kernels for decode shapes (M <= kDecodeMaxTokens), one CTA
// per SM: a producer warp moves contiguous weight chunks (~32 KB) into a ring
// of shared-memory stages with cp.async.bulk; two groups of 8 consumer warps
// take alternate stages and compute from shared memory.  With the ring in
// flight per SM, HBM latency is covered without tying up registers.
//
//   gate_up_stream_kernel  chunks: shared expert, 2 bf16 rows of gate and up
//                          (4 warps per row, one K-quarter each); routed
//                          experts, 8 MXFP4 rows of gate and up (warp per row)
//   down_stream_kernel     chunks: shared expert, 8 bf16 rows (warp per row);
//                          routed experts, 32 MXFP4 rows (LPR lanes per row)
//   combine_decode_kernel  f32 merge of routed rows and shared row
//
// The producer warp copies the routing tables into shared memory once per
// CTA and hands them to the consumers through an mbarrier.
//
// Chunk it of a CTA is chunk j = blockIdx.x + it * gridDim.x of the list
// [shared chunks..., routed chunks...]; consumer group it % 2 takes it.
// Shared chunks need no routing, so they run before griddepcontrol.wait;
// routed chunks are enumerated after it.  Each 32-column group is summed in
// four independent word chains to keep the FMA pipes busy.
//
// Error handling: all mbarrier waits are bounded (pipeline.cuh).  A warp whose
// wait gives up marks the status word and keeps walking the same chunk list
// without loading or computing, so every consumer still reaches every named
// barrier and the CTA exits.
#pragma once
#include "decode_kernels.cuh"
#include "pipeline.cuh"

namespace lg {

constexpr int kConsumerWarps = 8;  // warps of one consumer group
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGroups = 2;  // consumer groups take alternate stages
constexpr int kStreamThreads = kGroups * kConsumerThreads + 32;
constexpr int kProducerWarp = kGroups * kConsumerWarps;
constexpr int kMaxStages = 8;
constexpr int kGuRowsRouted = 8;
constexpr int kGuRowsShared = 2;
constexpr int kDnRowsRouted = 32;
constexpr int kDnRowsShared = 8;
// named barriers: 1 + group (one consumer group), 3 (all consumers)
constexpr int kBarAllConsumers = 3;

struct StreamCfg {
  int stages;
  int stage_bytes;
  int x_off;    // byte offset of staged activations
  int aux_off;  // byte offset of the reduction / scale scratch
  int rs;       // padded byte stride of a routed weight row in a stage
  int ss;       // byte stride of a routed scale row in a stage
  int ss_rows;  // 1: scale rows copied one by one (padded); 0: one contiguous block
};

// m16n8k16 tensor-core MMA, f16 x f16 -> f32 (fragment layout of the PTX ISA:
// a0/a2 rows g, a1/a3 rows g+8; a0/a1 k 2q..2q+1, a2/a3 k 2q+8..2q+9;
// b0 k 2q..2q+1, b1 k 2q+8..2q+9, column g; d0/d1 row g, d2/d3 row g+8,
// columns 2q, 2q+1; g = lane/4, q = lane%4)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}
// One 32-column group of a 16-row tile against up to 8 activation columns.
// Lane (g, q) holds the 4 bytes [4q, 4q+4) of the group's 16 bytes in rows g
// (wlo) and g+8 (whi): columns 8q..8q+7.  k-slots 2q+i <-> column 8q+i and
// 2q+8+i <-> column 8q+2+i (first MMA), then columns 8q+4..8q+7 (second), so
// the activation fragment is the 8 contiguous f16 at columns 8q..8q+7 of the
// lane's column g.  d += A * B for the group.
__device__ __forceinline__ void group_mma(float (&d)[4], uint32_t wlo, uint32_t whi, const uint4& xv) {
  uint32_t hl[4], hh[4];
  e2m1x8_to_f16x2(wlo, hl);
  e2m1x8_to_f16x2(whi, hh);
  mma16816(d, hl[0], hh[0], hl[1], hh[1], xv.x, xv.y);
  mma16816(d, hl[2], hh[2], hl[3], hh[3], xv.z, xv.w);
}

// Bulk-copy the routing tables (active list, offsets, perm) into shared
// memory; completion is signalled on `bar`.  Sizes are rounded up to 16 bytes
// (the workspace pads every region to 256 bytes, so the tail reads stay inside
// it).  Called by one thread.
__device__ __forceinline__ void copy_tables(const DecodeArgs& a, int* s_active, int* s_offsets, int* s_perm,
                                            uint64_t* bar) {
  const unsigned na = ((a.E + 1) * 4 + 15) & ~15u, no = na, np = ((a.M * a.k) * 4 + 15) & ~15u;
  mbar_arrive_expect_tx(bar, na + no + np);
  bulk_g2s(s_active, a.active, na, bar);
  bulk_g2s(s_offsets, a.offsets, no, bar);
  bulk_g2s(s_perm, a.perm, np, bar);
}

// sum of 32 E2M1 x f16 products of one group in four word chains
template <int TT>
__device__ __forceinline__ void group_dot_e2m1(const uint4& pw, const uint4* xv0, int xstride, int n,
                                               float (&gsum)[TT]) {
  const uint32_t w4[4] = {pw.x, pw.y, pw.z, pw.w};
  float c[4][TT];
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int q = 0; q < TT; ++q) c[w][q] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int q = 0; q < TT; ++q)
      if (q < n) c[w][q] = dot8_e2m1_f16(w4[w], xv0[q * xstride + w * 32], c[w][q]);
#pragma unroll
  for (int q = 0; q < TT; ++q) gsum[q] = __fadd_rn(__fadd_rn(c[0][q], c[1][q]), __fadd_rn(c[2][q], c[3][q]));
}

// Issue the bulk copies of `rows` weight rows (row_bytes each, global stride
// row_bytes) into padded shared rows (stride rs), and of their scale rows
// (g_bytes each) either row by row (stride ss) or as one block; lanes of the
// producer warp split the rows.  Returns the bytes the stage will receive.
__device__ __forceinline__ void issue_rows(unsigned char* dst, const uint8_t* src, int rows, int row_bytes,
                                           int rs, int lane, uint64_t* bar) {
  for (int r = lane; r < rows; r += 32)
    bulk_g2s(dst + static_cast<size_t>(r) * rs, src + static_cast<size_t>(r) * row_bytes, row_bytes, bar);
}
__device__ __forceinline__ void issue_scales(unsigned char* dst, const uint8_t* src, int rows, int g_bytes, int ss,
                                             int ss_rows, int lane, uint64_t* bar) {
  if (ss_rows) {
    for (int r = lane; r < rows; r += 32)
      bulk_g2s(dst + static_cast<size_t>(r) * ss, src + static_cast<size_t>(r) * g_bytes, g_bytes, bar);
  } else if (lane == 0) {
    bulk_g2s(dst, src, rows * g_bytes, bar);
  }
}

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(kStreamThreads, 1) gate_up_stream_kernel(DecodeArgs a, StreamCfg sc) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ __align__(8) uint64_t tbl;
  __shared__ unsigned amax_bits[TT];
  __shared__ float tok_mult[TT];
  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.d, G = K >> 5;
  const int M = a.M, F = a.F, Fs = a.Fs;
  const int S = sc.stages;
  const int KQ = K >> 2;               // shared-chunk quarter width
  const int WPL = (KQ / 8 + 31) / 32;  // 8-element words per lane per quarter
  uint16_t* xh = reinterpret_cast<uint16_t*>(smem + sc.x_off);  // f16 [t][K]
  uint4* xb = reinterpret_cast<uint4*>(xh + TT * K);              // bf16 [t][q][w4][lane]
  float* red = reinterpret_cast<float*>(smem + sc.aux_off);
  // red: shared-chunk partials [group][2][2 rows][4 q][TT][2], then routed
  // partials [group][2][8 warps][8 rows][TT][2]
  float* red_r = red + kGroups * 2 * kGuRowsShared * 4 * TT * 2;
  int* s_active = reinterpret_cast<int*>(red_r + kGroups * 2 * kConsumerWarps * 8 * TT * 2);
  int* s_offsets = s_active + (((a.E + 1) + 3) & ~3);
  int* s_perm = s_offsets + (((a.E + 1) + 3) & ~3);
  const int n_sh = Fs > 0 ? Fs / kGuRowsShared : 0;
  const int nrb = F / kGuRowsRouted;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kConsumerWarps); }
    mbar_init(&tbl, 1);
    mbar_fence_init();
  }
  if (threadIdx.x < TT) amax_bits[threadIdx.x] = 0u;
  __syncthreads();

  if (warp_id == kProducerWarp) {  // -------------- producer --------------
    bool ok = true;
    int it = 0;
    int j = blockIdx.x;
    const unsigned sh_bytes = kGuRowsShared * K * 2;
    for (; j < n_sh; j += gridDim.x, ++it) {
      const int s = it % S;
      const unsigned round = it / S;
      if (lane == 0) {
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteGuEmpty);
        if (ok) {
          unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
          mbar_arrive_expect_tx(&full[s], 2 * sh_bytes);
          bulk_g2s(st, a.sh_gate + static_cast<size_t>(j) * kGuRowsShared * K, sh_bytes, &full[s]);
          bulk_g2s(st + sh_bytes, a.sh_up + static_cast<size_t>(j) * kGuRowsShared * K, sh_bytes, &full[s]);
        }
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    pdl_wait();  // routing tables written by the router
    pdl_trigger();
    if (lane == 0) {
      copy_tables(a, s_active, s_offsets, s_perm, &tbl);
      if (ok) ok = mbar_wait(&tbl, 0, a.status, kSiteGuEmpty);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    const int n_r = ok ? s_active[0] * nrb : 0;
    const int rb = K >> 1;
    const unsigned bytes = 2u * kGuRowsRouted * rb + 2u * kGuRowsRouted * G;
    for (; j - n_sh < n_r; j += gridDim.x, ++it) {
      const int s = it % S;
      const unsigned round = it / S;
      if (lane == 0) {
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteGuEmpty);
        if (ok) mbar_arrive_expect_tx(&full[s], bytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) continue;
      const int jr = j - n_sh;
      const int e = s_active[1 + jr / nrb];
      const size_t f0 = static_cast<size_t>(jr % nrb) * kGuRowsRouted;
      unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
      // rows 0..7: gate rows f0..f0+7; rows 8..15: up rows; then 16 scale rows
      issue_rows(st, a.gate_p + e * a.gate_ps + f0 * rb, kGuRowsRouted, rb, sc.rs, lane, &full[s]);
      issue_rows(st + kGuRowsRouted * sc.rs, a.up_p + e * a.up_ps + f0 * rb, kGuRowsRouted, rb, sc.rs, lane,
                 &full[s]);
      unsigned char* sst = st + 2 * kGuRowsRouted * sc.rs;  // gate scales [8][G], then up scales [8][G]
      if (lane == 0) bulk_g2s(sst, a.gate_s + e * a.gate_ss + f0 * G, kGuRowsRouted * G, &full[s]);
      if (lane == 1) bulk_g2s(sst + kGuRowsRouted * G, a.up_s + e * a.up_ss + f0 * G, kGuRowsRouted * G, &full[s]);
    }
    if (!ok && lane == 0) {  // consumers stopped: let copies already issued land before leaving
      for (int q = (it > S ? it - S : 0); q < it; ++q)
        mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteGuDrain);
    }
    return;
  }

  // ------------------------------- consumers -------------------------------
  const int grp = warp_id / kConsumerWarps;   // consumer group
  const int warp = warp_id % kConsumerWarps;  // warp within the group
  const int ct = threadIdx.x;                 // 0 .. kGroups*kConsumerThreads-1
  const int gt = ct - grp * kConsumerThreads;
  constexpr int kAll = kGroups * kConsumerThreads;
  // stage bf16 rows for shared chunks: element qq*KQ + 8*(lane + 32*w4) + 0..7
  if (n_sh > 0) {
    const int per_row = 4 * WPL * 32;
    for (int i4 = ct; i4 < M * per_row; i4 += kAll) {
      const int t = i4 / per_row, rem = i4 - t * per_row;
      const int qq = rem / (WPL * 32), r2 = rem - qq * WPL * 32, w4 = r2 >> 5, ln = r2 & 31;
      const int el = 8 * (ln + 32 * w4);
      if (el < KQ)
        xb[(t * 4 + qq) * WPL * 32 + w4 * 32 + ln] =
            *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(t) * K + qq * KQ + el);
    }
  }
  // f16 rows for routed chunks with a per-token power-of-two prescale: one
  // load per element into registers, block max, then convert
  constexpr int kStageRegs = 4;  // M*K/8 <= kStageRegs*kAll
  uint4 xr[kStageRegs];
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * K / 8) xr[q] = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(i4) * 8);
  }
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * K / 8) {
      const uint4 u = xr[q];
      float m = fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y))));
      m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
      atomicMax(amax_bits + (i4 * 8) / K, __float_as_uint(m));
    }
  }
  named_sync(kBarAllConsumers, kAll);
  if (ct < M) tok_mult[ct] = pow2i(f16_shift_for(__uint_as_float(amax_bits[ct])));
  named_sync(kBarAllConsumers, kAll);
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * K / 8) {
      const uint4 u = xr[q];
      const float sc2 = __fdiv_rn(1.0f, tok_mult[(i4 * 8) / K]);
      reinterpret_cast<uint4*>(xh)[i4] =
          make_uint4(bf16x2_to_f16x2_scaled(u.x, sc2), bf16x2_to_f16x2_scaled(u.y, sc2),
                     bf16x2_to_f16x2_scaled(u.z, sc2), bf16x2_to_f16x2_scaled(u.w, sc2));
    }
  }
  named_sync(kBarAllConsumers, kAll);

  bool ok = true;
  int shi = 0, rti = 0;
  int it = grp;
  int j = blockIdx.x + it * gridDim.x;
  // shared-expert chunks: rows 2j, 2j+1; warp -> (row w/4, K quarter w%4)
  for (; j < n_sh; it += kGroups, j += kGroups * gridDim.x, ++shi) {
    const int s = it % S;
    if (ok) ok = mbar_wait(&full[s], (it / S) & 1, a.status, kSiteGuFull);
    const int rr = warp >> 2, qq = warp & 3;
    float ag[4][TT], au[4][TT];
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int t = 0; t < TT; ++t) { ag[w][t] = 0.f; au[w][t] = 0.f; }
    if (ok) {
      const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
      const unsigned char* gr = st + static_cast<size_t>(rr) * K * 2 + static_cast<size_t>(qq) * KQ * 2;
      const unsigned char* ur = gr + static_cast<size_t>(kGuRowsShared) * K * 2;
      for (int w0 = 0; w0 < WPL; w0 += 4) {
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int w4 = w0 + u4;
          const int el = 8 * (lane + 32 * w4);
          if (w4 < WPL && el < KQ) {
            const uint4 wg = *reinterpret_cast<const uint4*>(gr + 2 * el);
            const uint4 wu = *reinterpret_cast<const uint4*>(ur + 2 * el);
#pragma unroll
            for (int t = 0; t < TT; ++t)
              if (t < M) {
                const uint4 xv = xb[(t * 4 + qq) * WPL * 32 + w4 * 32 + lane];
                ag[u4][t] = dot8_bf16(wg, xv, ag[u4][t]);
                au[u4][t] = dot8_bf16(wu, xv, au[u4][t]);
              }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float g4[TT], u4s[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      g4[t] = __fadd_rn(__fadd_rn(ag[0][t], ag[1][t]), __fadd_rn(ag[2][t], ag[3][t]));
      u4s[t] = __fadd_rn(__fadd_rn(au[0][t], au[1][t]), __fadd_rn(au[2][t], au[3][t]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        g4[t] = __fadd_rn(g4[t], __shfl_xor_sync(0xffffffffu, g4[t], off));
        u4s[t] = __fadd_rn(u4s[t], __shfl_xor_sync(0xffffffffu, u4s[t], off));
      }
    float* rb = red + ((grp * 2 + (shi & 1)) * kGuRowsShared * 4 * TT * 2);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        rb[((rr * 4 + qq) * TT + t) * 2 + 0] = g4[t];
        rb[((rr * 4 + qq) * TT + t) * 2 + 1] = u4s[t];
      }
    }
    named_sync(1 + grp, kConsumerThreads);
    if (ok && warp < kGuRowsShared && lane < M) {
      float g = 0.f, u = 0.f;
      for (int q = 0; q < 4; ++q) {
        g = __fadd_rn(g, rb[((warp * 4 + q) * TT + lane) * 2 + 0]);
        u = __fadd_rn(u, rb[((warp * 4 + q) * TT + lane) * 2 + 1]);
      }
      a.act_s[static_cast<size_t>(lane) * Fs + j * kGuRowsShared + warp] =
          swiglu_bf16(round_bf16(g), round_bf16(u), a.limit);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (ok) ok = mbar_wait(&tbl, 0, a.status, kSiteGuFull);
  const int n_r = ok ? s_active[0] * nrb : 0;
  // routed chunks: 16-row tile = 8 gate rows over 8 up rows; the K groups are
  // split over the 8 warps of the group; columns = routes of the expert
  const int g8 = lane >> 2, q4 = lane & 3;
  const int gpw = (G + kConsumerWarps - 1) / kConsumerWarps;
  for (; j - n_sh < n_r; it += kGroups, j += kGroups * gridDim.x, ++rti) {
    const int s = it % S;
    if (ok) ok = mbar_wait(&full[s], (it / S) & 1, a.status, kSiteGuFull);
    const int jr = j - n_sh;
    const int e = s_active[1 + jr / nrb];
    const int f0 = (jr % nrb) * kGuRowsRouted;
    const int p0 = s_offsets[e];
    const int n = s_offsets[e + 1] - p0;
    const int col_tok = s_perm[p0 + (g8 < n ? g8 : 0)] / a.k;  // token of this lane's column
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
      const unsigned char* wlo = st + static_cast<size_t>(g8) * sc.rs + 4 * q4;                  // gate row g
      const unsigned char* whi = st + static_cast<size_t>(kGuRowsRouted + g8) * sc.rs + 4 * q4;  // up row g
      const unsigned char* sst = st + 2 * kGuRowsRouted * sc.rs;
      const unsigned char* slo = sst + g8 * G;
      const unsigned char* shi = sst + (kGuRowsRouted + g8) * G;
      const uint16_t* xrow = xh + static_cast<size_t>(col_tok) * K + 8 * q4;
      const int c0 = warp * gpw, c1 = min(G, c0 + gpw);
      if (gpw == 16 && (G & 15) == 0) {  // the warp's 16 scale bytes per row in one load
        const uint4 vl = *reinterpret_cast<const uint4*>(slo + c0);
        const uint4 vh = *reinterpret_cast<const uint4*>(shi + c0);
        const uint32_t sl4[4] = {vl.x, vl.y, vl.z, vl.w}, sh4[4] = {vh.x, vh.y, vh.z, vh.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = c0 + i;
          const uint32_t wl = *reinterpret_cast<const uint32_t*>(wlo + 16 * c);
          const uint32_t wh = *reinterpret_cast<const uint32_t*>(whi + 16 * c);
          const uint4 xv = *reinterpret_cast<const uint4*>(xrow + 32 * c);
          const float sl = e8m0_to_f32((sl4[i >> 2] >> (8 * (i & 3))) & 0xffu);
          const float sh = e8m0_to_f32((sh4[i >> 2] >> (8 * (i & 3))) & 0xffu);
          float t4[4] = {0.f, 0.f, 0.f, 0.f};
          group_mma(t4, wl, wh, xv);
          d[0] = __fmaf_rn(t4[0], sl, d[0]);
          d[1] = __fmaf_rn(t4[1], sl, d[1]);
          d[2] = __fmaf_rn(t4[2], sh, d[2]);
          d[3] = __fmaf_rn(t4[3], sh, d[3]);
        }
      } else {
        for (int c = c0; c < c1; ++c) {
          const uint32_t wl = *reinterpret_cast<const uint32_t*>(wlo + 16 * c);
          const uint32_t wh = *reinterpret_cast<const uint32_t*>(whi + 16 * c);
          const uint4 xv = *reinterpret_cast<const uint4*>(xrow + 32 * c);
          const float sl = e8m0_to_f32(slo[c]), sh = e8m0_to_f32(shi[c]);
          float t4[4] = {0.f, 0.f, 0.f, 0.f};
          group_mma(t4, wl, wh, xv);
          d[0] = __fmaf_rn(t4[0], sl, d[0]);
          d[1] = __fmaf_rn(t4[1], sl, d[1]);
          d[2] = __fmaf_rn(t4[2], sh, d[2]);
          d[3] = __fmaf_rn(t4[3], sh, d[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // cross-warp reduction of the K split: partials [warp][row][col][gate/up]
    float* rr2 = red_r + ((grp * 2 + (rti & 1)) * kConsumerWarps + warp) * 8 * TT * 2;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = 2 * q4 + h;
      if (col < n && col < TT) {
        rr2[(g8 * TT + col) * 2 + 0] = d[h];
        rr2[(g8 * TT + col) * 2 + 1] = d[2 + h];
      }
    }
    named_sync(1 + grp, kConsumerThreads);
    if (ok && gt < 8 * n) {
      const int row = gt / n, col = gt - row * n;
      const float* base = red_r + (grp * 2 + (rti & 1)) * kConsumerWarps * 8 * TT * 2;
      float g = 0.f, u = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) {
        g = __fadd_rn(g, base[(w * 8 * TT + row * TT + col) * 2 + 0]);
        u = __fadd_rn(u, base[(w * 8 * TT + row * TT + col) * 2 + 1]);
      }
      const int tj = s_perm[p0 + col] / a.k;
      const float m = tok_mult[tj];
      a.act[static_cast<size_t>(p0 + col) * F + f0 + row] =
          swiglu_bf16(round_bf16(__fmul_rn(g, m)), round_bf16(__fmul_rn(u, m)), a.limit);
    }
  }
}

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(kStreamThreads, 1) down_stream_kernel(DecodeArgs a, StreamCfg sc) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ __align__(8) uint64_t tbl;
  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.M, k = a.k, d = a.d, F = a.F, Fs = a.Fs;
  const int G = F >> 5;
  const int S = sc.stages;
  const int WS = (Fs / 8 + 31) / 32;  // 8-element words per lane of a shared row
  const int n_sh = Fs > 0 ? d / kDnRowsShared : 0;
  const int nrb = d / kDnRowsRouted;
  const int R = M * k;
  uint16_t* xr = reinterpret_cast<uint16_t*>(smem + sc.x_off);  // f16 [p][F]
  uint4* xsb = reinterpret_cast<uint4*>(xr + static_cast<size_t>(R) * F);  // bf16 [t][w4][lane]
  float* rscale = reinterpret_cast<float*>(smem + sc.aux_off);
  float* red_r = rscale + ((R + 3) & ~3);  // [group][2][8 warps][32 rows][TT]
  int* s_active = reinterpret_cast<int*>(red_r + kGroups * 2 * kConsumerWarps * kDnRowsRouted * TT);
  int* s_offsets = s_active + (((a.E + 1) + 3) & ~3);
  int* s_perm = s_offsets + (((a.E + 1) + 3) & ~3);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kConsumerWarps); }
    mbar_init(&tbl, 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp_id == kProducerWarp) {  // -------------- producer --------------
    // Weights depend on nothing earlier and the routing tables are complete
    // (the gate/up kernel waited on the router before letting this kernel
    // launch), so streaming starts before griddepcontrol.wait.
    bool ok = true;
    if (lane == 0) {
      copy_tables(a, s_active, s_offsets, s_perm, &tbl);
      ok = mbar_wait(&tbl, 0, a.status, kSiteDnEmpty);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    int it = 0;
    const int n_r = ok ? s_active[0] * nrb : 0;
    const unsigned shb = kDnRowsShared * Fs * 2;
    const int rb = F >> 1;
    const unsigned rbytes = kDnRowsRouted * (rb + G);
    for (int j = blockIdx.x; j < n_sh + n_r; j += gridDim.x, ++it) {
      const int s = it % S;
      const unsigned round = it / S;
      if (lane == 0) {
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteDnEmpty);
        if (ok) mbar_arrive_expect_tx(&full[s], j < n_sh ? shb : rbytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) continue;
      unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
      if (j < n_sh) {
        if (lane == 0) bulk_g2s(st, a.sh_down + static_cast<size_t>(j) * kDnRowsShared * Fs, shb, &full[s]);
      } else {
        const int jr = j - n_sh;
        const int e = s_active[1 + jr / nrb];
        const size_t r0 = static_cast<size_t>(jr % nrb) * kDnRowsRouted;
        // 8 blocks of 4 consecutive rows at padded stride sc.rs, then the
        // chunk's scale rows as one block [32][G]
        issue_rows(st, a.down_p + e * a.down_ps + r0 * rb, kDnRowsRouted / 4, 4 * rb, sc.rs, lane, &full[s]);
        if (lane == 31)
          bulk_g2s(st + (kDnRowsRouted / 4) * sc.rs, a.down_s + e * a.down_ss + r0 * G, kDnRowsRouted * G, &full[s]);
      }
    }
    if (!ok && lane == 0) {
      for (int q = (it > S ? it - S : 0); q < it; ++q)
        mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteDnDrain);
    }
    pdl_wait();
    pdl_trigger();
    return;
  }

  // ------------------------------- consumers -------------------------------
  const int grp = warp_id / kConsumerWarps;
  const int warp = warp_id % kConsumerWarps;
  const int ct = threadIdx.x;
  const int gt = ct - grp * kConsumerThreads;
  constexpr int kAll = kGroups * kConsumerThreads;
  pdl_wait();  // activations from the gate/up kernel
  pdl_trigger();
  bool ok = mbar_wait(&tbl, 0, a.status, kSiteDnFull);
  const int n_active = ok ? s_active[0] : 0;
  const int n_r = n_active * nrb;
  // routed activations as f16 with a per-route power-of-two prescale; a warp
  // holds its row in registers (F/8 <= 32*kRowRegs uint4) across the max
  constexpr int kRowRegs = 8;
  for (int r = warp_id; r < R; r += kGroups * kConsumerWarps) {
    const uint16_t* src = a.act + static_cast<size_t>(r) * F;
    uint4 v8[kRowRegs];
    float m = 0.f;
#pragma unroll
    for (int q = 0; q < kRowRegs; ++q) {
      const int v = lane + 32 * q;
      if (v < F / 8) v8[q] = __ldcg(reinterpret_cast<const uint4*>(src + 8 * v));
    }
#pragma unroll
    for (int q = 0; q < kRowRegs; ++q) {
      const int v = lane + 32 * q;
      if (v < F / 8) {
        const uint4 u = v8[q];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y)))));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const int sh = f16_shift_for(m);
    const float sc2 = pow2i(-sh);
    if (lane == 0) rscale[r] = pow2i(sh);
#pragma unroll
    for (int q = 0; q < kRowRegs; ++q) {
      const int v = lane + 32 * q;
      if (v < F / 8) {
        const uint4 u = v8[q];
        reinterpret_cast<uint4*>(xr + static_cast<size_t>(r) * F)[v] =
            make_uint4(bf16x2_to_f16x2_scaled(u.x, sc2), bf16x2_to_f16x2_scaled(u.y, sc2),
                       bf16x2_to_f16x2_scaled(u.z, sc2), bf16x2_to_f16x2_scaled(u.w, sc2));
      }
    }
  }
  // shared activations (bf16) as [t][w4][lane], element 8*(lane + 32*w4)
  if (Fs > 0) {
    for (int i4 = ct; i4 < M * WS * 32; i4 += kAll) {
      const int t = i4 / (WS * 32), rem = i4 - t * WS * 32;
      const int el = 8 * rem;
      if (el < Fs) xsb[i4] = __ldcg(reinterpret_cast<const uint4*>(a.act_s + static_cast<size_t>(t) * Fs + el));
    }
  }
  named_sync(kBarAllConsumers, kAll);

  const int g8 = lane >> 2, q4 = lane & 3;
  const int gpw = (G + kConsumerWarps - 1) / kConsumerWarps;
  int rti = 0;
  for (int it = grp, j = blockIdx.x + grp * gridDim.x; j < n_sh + n_r; it += kGroups, j += kGroups * gridDim.x) {
    const int s = it % S;
    if (ok) ok = mbar_wait(&full[s], (it / S) & 1, a.status, kSiteDnFull);
    const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
    if (j < n_sh) {  // shared: warp -> row j*8 + warp, whole Fs
      const int row = j * kDnRowsShared + warp;
      float acc[4][TT];
#pragma unroll
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[w][t] = 0.f;
      if (ok) {
        const unsigned char* wr = st + static_cast<size_t>(warp) * Fs * 2;
        for (int w0 = 0; w0 < WS; w0 += 4) {
#pragma unroll
          for (int u4 = 0; u4 < 4; ++u4) {
            const int w4 = w0 + u4;
            const int el = 8 * (lane + 32 * w4);
            if (w4 < WS && el < Fs) {
              const uint4 wv = *reinterpret_cast<const uint4*>(wr + 2 * el);
#pragma unroll
              for (int t = 0; t < TT; ++t)
                if (t < M) acc[u4][t] = dot8_bf16(wv, xsb[t * WS * 32 + w4 * 32 + lane], acc[u4][t]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float v[TT];
#pragma unroll
      for (int t = 0; t < TT; ++t) v[t] = __fadd_rn(__fadd_rn(acc[0][t], acc[1][t]), __fadd_rn(acc[2][t], acc[3][t]));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int t = 0; t < TT; ++t) v[t] = __fadd_rn(v[t], __shfl_xor_sync(0xffffffffu, v[t], off));
      if (ok && lane < M) {
        float o = v[0];
#pragma unroll
        for (int t = 1; t < TT; ++t)
          if (lane == t) o = v[t];
        a.ys[static_cast<size_t>(lane) * d + row] = f32_to_bf16(o);
      }
    } else {  // routed: rows r0 .. r0+31 (two 16-row tiles) of expert e, K split over warps
      const int jr = j - n_sh;
      const int e = s_active[1 + jr / nrb];
      const int r0 = (jr % nrb) * kDnRowsRouted;
      const int p0 = s_offsets[e];
      const int n = s_offsets[e + 1] - p0;
      // tile t (0, 1): MMA row m < 8 is row 4m + 2t, row m + 8 is row 4m + 2t + 1;
      // the 8 rows of one fragment load sit in 8 differently padded blocks
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok) {
        const uint16_t* xrow = xr + static_cast<size_t>(p0 + (g8 < n ? g8 : 0)) * F + 8 * q4;
        const int rb = F >> 1;
        const unsigned char* blkp = st + static_cast<size_t>(g8) * sc.rs + 4 * q4;
        const unsigned char* w0r = blkp;           // row 4g
        const unsigned char* w1r = blkp + rb;      // row 4g + 1
        const unsigned char* w2r = blkp + 2 * rb;  // row 4g + 2
        const unsigned char* w3r = blkp + 3 * rb;  // row 4g + 3
        const unsigned char* s0 = st + (kDnRowsRouted / 4) * sc.rs + (4 * g8) * G;
        const int c0 = warp * gpw, c1 = min(G, c0 + gpw);
#pragma unroll 2
        for (int c = c0; c < c1; ++c) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xrow + 32 * c);
          const uint32_t wa = *reinterpret_cast<const uint32_t*>(w0r + 16 * c);
          const uint32_t wb = *reinterpret_cast<const uint32_t*>(w1r + 16 * c);
          const uint32_t wc = *reinterpret_cast<const uint32_t*>(w2r + 16 * c);
          const uint32_t wd = *reinterpret_cast<const uint32_t*>(w3r + 16 * c);
          const float sa = e8m0_to_f32(s0[c]), sb = e8m0_to_f32(s0[G + c]);
          const float sc_ = e8m0_to_f32(s0[2 * G + c]), sd = e8m0_to_f32(s0[3 * G + c]);
          float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
          group_mma(t0, wa, wb, xv);  // rows 4g (m = g) and 4g+1 (m = g+8)
          group_mma(t1, wc, wd, xv);  // rows 4g+2 and 4g+3
          d0[0] = __fmaf_rn(t0[0], sa, d0[0]);
          d0[1] = __fmaf_rn(t0[1], sa, d0[1]);
          d0[2] = __fmaf_rn(t0[2], sb, d0[2]);
          d0[3] = __fmaf_rn(t0[3], sb, d0[3]);
          d1[0] = __fmaf_rn(t1[0], sc_, d1[0]);
          d1[1] = __fmaf_rn(t1[1], sc_, d1[1]);
          d1[2] = __fmaf_rn(t1[2], sd, d1[2]);
          d1[3] = __fmaf_rn(t1[3], sd, d1[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float* rr2 = red_r + ((grp * 2 + (rti & 1)) * kConsumerWarps + warp) * kDnRowsRouted * TT;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = 2 * q4 + h;
        if (col < n && col < TT) {
          rr2[(4 * g8 + 0) * TT + col] = d0[h];
          rr2[(4 * g8 + 1) * TT + col] = d0[2 + h];
          rr2[(4 * g8 + 2) * TT + col] = d1[h];
          rr2[(4 * g8 + 3) * TT + col] = d1[2 + h];
        }
      }
      named_sync(1 + grp, kConsumerThreads);
      if (ok) {
        const float* base = red_r + (grp * 2 + (rti & 1)) * kConsumerWarps * kDnRowsRouted * TT;
        for (int o = gt; o < kDnRowsRouted * n; o += kConsumerThreads) {
          const int row = o / n, col = o - row * n;
          float v = 0.f;
          for (int w = 0; w < kConsumerWarps; ++w) v = __fadd_rn(v, base[(w * kDnRowsRouted + row) * TT + col]);
          a.y[static_cast<size_t>(s_perm[p0 + col]) * d + r0 + row] = f32_to_bf16(__fmul_rn(v, rscale[p0 + col]));
        }
      }
      ++rti;
    }
  }
}

// ---------------------------------------------------------------------------
// f32 merge of the routed rows (route order) and the shared row, moe.py:199-201.
__global__ void __launch_bounds__(256) combine_decode_kernel(DecodeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int d = a.d, k = a.k;
  for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < a.M * (d >> 2); o += gridDim.x * blockDim.x) {
    const int t = o / (d >> 2), c = o - t * (d >> 2);
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    for (int q = 0; q < k; ++q) {
      const float wq = __ldcg(a.weights + static_cast<size_t>(t) * k + q);
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(a.y + (static_cast<size_t>(t) * k + q) * d + 4 * c));
      s0 = __fadd_rn(s0, __fmul_rn(bf16lo(u.x), wq));
      s1 = __fadd_rn(s1, __fmul_rn(bf16hi(u.x), wq));
      s2 = __fadd_rn(s2, __fmul_rn(bf16lo(u.y), wq));
      s3 = __fadd_rn(s3, __fmul_rn(bf16hi(u.y), wq));
    }
    if (a.Fs > 0) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(a.ys + static_cast<size_t>(t) * d + 4 * c));
      s0 = __fadd_rn(s0, bf16lo(u.x));
      s1 = __fadd_rn(s1, bf16hi(u.x));
      s2 = __fadd_rn(s2, bf16lo(u.y));
      s3 = __fadd_rn(s3, bf16hi(u.y));
    }
    reinterpret_cast<float4*>(a.out)[o] = make_float4(s0, s1, s2, s3);
  }
}

}  // namespace lg
