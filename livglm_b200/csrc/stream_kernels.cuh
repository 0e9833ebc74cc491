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
};

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

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(kStreamThreads, 1) gate_up_stream_kernel(DecodeArgs a, StreamCfg sc) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ unsigned amax_bits[TT];
  __shared__ float tok_mult[TT];
  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.d, G = K >> 5, KI = (G + 31) >> 5;
  const int M = a.M, F = a.F, Fs = a.Fs;
  const int S = sc.stages;
  const int KQ = K >> 2;               // shared-chunk quarter width
  const int WPL = (KQ / 8 + 31) / 32;  // 8-element words per lane per quarter
  uint4* xh = reinterpret_cast<uint4*>(smem + sc.x_off);  // f16 [t][i][w][lane]
  uint4* xb = xh + TT * KI * 128;                         // bf16 [t][q][w4][lane]
  float* red = reinterpret_cast<float*>(smem + sc.aux_off);  // [group][2][2 rows][4 q][TT][2]
  int* s_active = reinterpret_cast<int*>(red + kGroups * 2 * kGuRowsShared * 4 * TT * 2);
  int* s_offsets = s_active + (((a.E + 1) + 3) & ~3);
  int* s_perm = s_offsets + (((a.E + 1) + 3) & ~3);
  __shared__ __align__(8) uint64_t tbl;
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
    if (lane == 0) {
      const unsigned sh_bytes = kGuRowsShared * K * 2;
      for (; j < n_sh; j += gridDim.x, ++it) {
        const int s = it % S;
        const unsigned round = it / S;
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteGuEmpty);
        if (!ok) continue;
        unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
        mbar_arrive_expect_tx(&full[s], 2 * sh_bytes);
        bulk_g2s(st, a.sh_gate + static_cast<size_t>(j) * kGuRowsShared * K, sh_bytes, &full[s]);
        bulk_g2s(st + sh_bytes, a.sh_up + static_cast<size_t>(j) * kGuRowsShared * K, sh_bytes, &full[s]);
      }
    }
    __syncwarp();
    pdl_wait();  // routing tables written by the router
    pdl_trigger();
    if (lane == 0) {
      copy_tables(a, s_active, s_offsets, s_perm, &tbl);
      if (ok) ok = mbar_wait(&tbl, 0, a.status, kSiteGuEmpty);
      const int n_r = ok ? s_active[0] * nrb : 0;
      const unsigned pk = kGuRowsRouted * (K >> 1), sk = kGuRowsRouted * G;
      for (; j - n_sh < n_r; j += gridDim.x, ++it) {
        const int s = it % S;
        const unsigned round = it / S;
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteGuEmpty);
        if (!ok) continue;
        const int jr = j - n_sh;
        const int e = s_active[1 + jr / nrb];
        const size_t f0 = static_cast<size_t>(jr % nrb) * kGuRowsRouted;
        unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
        mbar_arrive_expect_tx(&full[s], 2 * pk + 2 * sk);
        bulk_g2s(st, a.gate_p + e * a.gate_ps + f0 * (K >> 1), pk, &full[s]);
        bulk_g2s(st + pk, a.up_p + e * a.up_ps + f0 * (K >> 1), pk, &full[s]);
        bulk_g2s(st + 2 * pk, a.gate_s + e * a.gate_ss + f0 * G, sk, &full[s]);
        bulk_g2s(st + 2 * pk + sk, a.up_s + e * a.up_ss + f0 * G, sk, &full[s]);
      }
      if (!ok) {  // consumers stopped: let copies already issued land before leaving
        for (int q = (it > S ? it - S : 0); q < it; ++q)
          mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteGuDrain);
      }
    }
    return;
  }

  // ------------------------------- consumers -------------------------------
  const int grp = warp_id / kConsumerWarps;  // consumer group
  const int warp = warp_id % kConsumerWarps;  // warp within the group
  const int ct = threadIdx.x;                 // 0 .. kGroups*kConsumerThreads-1
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
  // f16 rows for routed chunks, with a per-token power-of-two prescale:
  // one load per element into registers, block max, then convert
  constexpr int kStageRegs = 4;  // uint4 per thread held across the max (M*G*4 <= 4*kAll)
  uint4 xr[kStageRegs];
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * G * 4) {
      const int t = i4 / (G * 4), rem = i4 - t * G * 4;
      xr[q] = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(t) * K + 8 * rem);
    }
  }
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * G * 4) {
      const uint4 u = xr[q];
      float m = fmaxf(fmaxf(fabsf(bf16lo(u.x)), fabsf(bf16hi(u.x))), fmaxf(fabsf(bf16lo(u.y)), fabsf(bf16hi(u.y))));
      m = fmaxf(m, fmaxf(fmaxf(fabsf(bf16lo(u.z)), fabsf(bf16hi(u.z))), fmaxf(fabsf(bf16lo(u.w)), fabsf(bf16hi(u.w)))));
      atomicMax(amax_bits + i4 / (G * 4), __float_as_uint(m));
    }
  }
  named_sync(kBarAllConsumers, kAll);
  if (ct < M) tok_mult[ct] = pow2i(f16_shift_for(__uint_as_float(amax_bits[ct])));
  named_sync(kBarAllConsumers, kAll);
#pragma unroll
  for (int q = 0; q < kStageRegs; ++q) {
    const int i4 = ct + q * kAll;
    if (i4 < M * G * 4) {
      const int t = i4 / (G * 4), rem = i4 - t * G * 4, c = rem >> 2, w = rem & 3;
      const uint4 u = xr[q];
      const float sc2 = __fdiv_rn(1.0f, tok_mult[t]);
      xh[((t * KI + (c >> 5)) * 4 + w) * 32 + (c & 31)] =
          make_uint4(bf16x2_to_f16x2_scaled(u.x, sc2), bf16x2_to_f16x2_scaled(u.y, sc2),
                     bf16x2_to_f16x2_scaled(u.z, sc2), bf16x2_to_f16x2_scaled(u.w, sc2));
    }
  }
  named_sync(kBarAllConsumers, kAll);

  bool ok = true;
  int shi = 0;
  int it = grp;
  int j = blockIdx.x + it * gridDim.x;
  // shared-expert chunks: rows 2j, 2j+1; warp -> (row w/4, K quarter w%4)
  for (; j < n_sh; it += kGroups, j += kGroups * gridDim.x, ++shi) {
    const int s = it % S;
    if (ok) ok = mbar_wait_warp(&full[s], (it / S) & 1, a.status, kSiteGuFull);
    const int rr = warp >> 2, qq = warp & 3;
    float ag[4][TT], au[4][TT];
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int t = 0; t < TT; ++t) { ag[w][t] = 0.f; au[w][t] = 0.f; }
    const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
    const unsigned char* gr = st + static_cast<size_t>(rr) * K * 2 + static_cast<size_t>(qq) * KQ * 2;
    const unsigned char* ur = gr + static_cast<size_t>(kGuRowsShared) * K * 2;
    const bool regs = WPL <= 4;  // copy this lane's slice out and release the stage first
    uint4 wgr[4], wur[4];
    if (ok && regs) {
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        const int el = 8 * (lane + 32 * u4);
        if (u4 < WPL && el < KQ) {
          wgr[u4] = *reinterpret_cast<const uint4*>(gr + 2 * el);
          wur[u4] = *reinterpret_cast<const uint4*>(ur + 2 * el);
        }
      }
    }
    __syncwarp();
    const bool early = regs || !ok;
    if (early && lane == 0) mbar_arrive(&empty[s]);
    if (ok) {
      for (int w0 = 0; w0 < WPL; w0 += 4) {
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int w4 = w0 + u4;
          const int el = 8 * (lane + 32 * w4);
          if (w4 < WPL && el < KQ) {
            const uint4 wg = regs ? wgr[u4] : *reinterpret_cast<const uint4*>(gr + 2 * el);
            const uint4 wu = regs ? wur[u4] : *reinterpret_cast<const uint4*>(ur + 2 * el);
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
    if (!early) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    float gt[TT], ut[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      gt[t] = __fadd_rn(__fadd_rn(ag[0][t], ag[1][t]), __fadd_rn(ag[2][t], ag[3][t]));
      ut[t] = __fadd_rn(__fadd_rn(au[0][t], au[1][t]), __fadd_rn(au[2][t], au[3][t]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        gt[t] = __fadd_rn(gt[t], __shfl_xor_sync(0xffffffffu, gt[t], off));
        ut[t] = __fadd_rn(ut[t], __shfl_xor_sync(0xffffffffu, ut[t], off));
      }
    float* rb = red + ((grp * 2 + (shi & 1)) * kGuRowsShared * 4 * TT * 2);
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        rb[((rr * 4 + qq) * TT + t) * 2 + 0] = gt[t];
        rb[((rr * 4 + qq) * TT + t) * 2 + 1] = ut[t];
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
  if (ok) ok = mbar_wait_warp(&tbl, 0, a.status, kSiteGuFull);
  const int n_r = ok ? s_active[0] * nrb : 0;
  for (; j - n_sh < n_r; it += kGroups, j += kGroups * gridDim.x) {
    const int s = it % S;
    if (ok) ok = mbar_wait_warp(&full[s], (it / S) & 1, a.status, kSiteGuFull);
    const int jr = j - n_sh;
    const int e = s_active[1 + jr / nrb];
    const int f = (jr % nrb) * kGuRowsRouted + warp;
    const int p0 = s_offsets[e];
    const int n = s_offsets[e + 1] - p0;
    int tok[TT];
#pragma unroll
    for (int q = 0; q < TT; ++q) tok[q] = q < n ? s_perm[p0 + q] / a.k : 0;
    float ag[TT], au[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) { ag[t] = 0.f; au[t] = 0.f; }
    // This lane's slice of the stage (16 packed bytes of gate and of up and a
    // scale byte each, per group) goes to registers first and the stage is
    // released before the arithmetic, so the ring refills during compute.
    constexpr int kRegGroups = 4;
    const bool regs = KI <= kRegGroups;
    const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
    const size_t pk = static_cast<size_t>(kGuRowsRouted) * (K >> 1);
    const unsigned char* gp = st + static_cast<size_t>(warp) * (K >> 1);
    const unsigned char* up = gp + pk;
    const unsigned char* gs = st + 2 * pk + warp * G;
    const unsigned char* us = gs + kGuRowsRouted * G;
    uint4 pgr[kRegGroups], pur[kRegGroups];
    uint32_t sgr[kRegGroups], sur[kRegGroups];
    if (ok && regs) {
#pragma unroll
      for (int i = 0; i < kRegGroups; ++i) {
        const int c = lane + 32 * i;
        if (i < KI && c < G) {
          pgr[i] = *reinterpret_cast<const uint4*>(gp + 16 * c);
          pur[i] = *reinterpret_cast<const uint4*>(up + 16 * c);
          sgr[i] = gs[c];
          sur[i] = us[c];
        }
      }
    }
    __syncwarp();
    const bool early = regs || !ok;
    if (early && lane == 0) mbar_arrive(&empty[s]);
    // one 32-column group: 4-chain dot products for every routed token
    auto group = [&](const uint4& pg, const uint4& pu, uint32_t sgb, uint32_t sub_, int i) {
      const float s_g = e8m0_to_f32(sgb), s_u = e8m0_to_f32(sub_);
      const uint4* xv0 = xh + i * 128 + lane;  // token t: + t*KI*128, word w: + w*32
      float gg[TT], gu[TT];
      if (n == 1 || TT == 1) {
        group_dot_e2m1<TT>(pg, xv0 + tok[0] * KI * 128, 0, n, gg);
        group_dot_e2m1<TT>(pu, xv0 + tok[0] * KI * 128, 0, n, gu);
      } else {
#pragma unroll
        for (int q = 0; q < TT; ++q) {
          float g1[1], u1[1];
          if (q < n) {
            group_dot_e2m1<1>(pg, xv0 + tok[q] * KI * 128, 0, 1, g1);
            group_dot_e2m1<1>(pu, xv0 + tok[q] * KI * 128, 0, 1, u1);
          } else {
            g1[0] = 0.f; u1[0] = 0.f;
          }
          gg[q] = g1[0];
          gu[q] = u1[0];
        }
      }
#pragma unroll
      for (int q = 0; q < TT; ++q) {
        ag[q] = __fmaf_rn(gg[q], s_g, ag[q]);
        au[q] = __fmaf_rn(gu[q], s_u, au[q]);
      }
    };
    if (ok && regs) {
#pragma unroll
      for (int i = 0; i < kRegGroups; ++i)
        if (i < KI && lane + 32 * i < G) group(pgr[i], pur[i], sgr[i], sur[i], i);
    } else if (ok) {
#pragma unroll 2
      for (int i = 0; i < KI; ++i) {
        const int c = lane + 32 * i;
        if (c < G)
          group(*reinterpret_cast<const uint4*>(gp + 16 * c), *reinterpret_cast<const uint4*>(up + 16 * c), gs[c],
                us[c], i);
      }
    }
    if (!early) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int q = 0; q < TT; ++q) {
        ag[q] = __fadd_rn(ag[q], __shfl_xor_sync(0xffffffffu, ag[q], off));
        au[q] = __fadd_rn(au[q], __shfl_xor_sync(0xffffffffu, au[q], off));
      }
    if (ok && lane < TT && lane < n) {
      float g = ag[0], uu = au[0];
      int tj = tok[0];
#pragma unroll
      for (int q = 1; q < TT; ++q)
        if (lane == q) { g = ag[q]; uu = au[q]; tj = tok[q]; }
      const float m = tok_mult[tj];
      a.act[static_cast<size_t>(p0 + lane) * F + f] =
          swiglu_bf16(round_bf16(__fmul_rn(g, m)), round_bf16(__fmul_rn(uu, m)), a.limit);
    }
  }
}

// One 32-column MXFP4 group of a down row against the staged activations of
// the expert's routes: acc[q] += scale * sum of 32 products for route q.
template <int TT>
__device__ __forceinline__ void down_group(const uint4& pkv, uint32_t sbyte, const uint4* xv0, int G, int n,
                                           float (&acc)[TT]) {
  const float scl = e8m0_to_f32(sbyte);
  const uint32_t w4v[4] = {pkv.x, pkv.y, pkv.z, pkv.w};
  float c[4][TT];
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int q = 0; q < TT; ++q) c[w][q] = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int q = 0; q < TT; ++q)
      if (q < n) c[w][q] = dot8_e2m1_f16(w4v[w], xv0[(q * 4 + w) * G], c[w][q]);
#pragma unroll
  for (int q = 0; q < TT; ++q)
    acc[q] = __fmaf_rn(__fadd_rn(__fadd_rn(c[0][q], c[1][q]), __fadd_rn(c[2][q], c[3][q])), scl, acc[q]);
}

// What a routed down consumer lane works on within one stage.
template <int TT>
struct DnRouted {
  const unsigned char* st;  // stage: packed rows then scale rows
  size_t pk;                // bytes of packed rows
  int F, G, d, LPR, slots, slot, sub, per_lane, warp, p0, n, r0;
  const uint4* xv;          // staged activations of route p0 (word w of route q: + (q*4+w)*G)
  const float* rscale;      // per-route activation scale, from route p0
  uint16_t* y;
  int slot_of[TT];          // route slot of route p0+q

  // reduce a row's partial sums over its LPR lanes and write the routes' outputs
  __device__ __forceinline__ void finish_row(float (&acc)[TT], int rl) const {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
      if (off < LPR)
#pragma unroll
        for (int q = 0; q < TT; ++q) acc[q] = __fadd_rn(acc[q], __shfl_xor_sync(0xffffffffu, acc[q], off));
    if (rl < kDnRowsRouted && sub < TT && sub < n) {
      float v = acc[0];
      int sl = slot_of[0];
#pragma unroll
      for (int q = 1; q < TT; ++q)
        if (sub == q) { v = acc[q]; sl = slot_of[q]; }
      y[static_cast<size_t>(sl) * d + r0 + rl] = f32_to_bf16(__fmul_rn(v, rscale[sub]));
    }
  }
};

// ---------------------------------------------------------------------------
template <int TT>
__global__ void __launch_bounds__(kStreamThreads, 1) down_stream_kernel(DecodeArgs a, StreamCfg sc) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.M, k = a.k, d = a.d, F = a.F, Fs = a.Fs;
  const int G = F >> 5;
  const int S = sc.stages;
  const int LPR = a.lpr_down;
  const int slots = 32 / LPR;
  const int sub = lane & (LPR - 1), slot = lane / LPR;
  const int per_lane = (G + LPR - 1) / LPR;
  const int WS = (Fs / 8 + 31) / 32;  // 8-element words per lane of a shared row
  const int n_sh = Fs > 0 ? d / kDnRowsShared : 0;
  const int nrb = d / kDnRowsRouted;
  const int R = M * k;
  uint4* xr = reinterpret_cast<uint4*>(smem + sc.x_off);  // f16 [p][q4][grp]
  uint4* xsb = xr + R * G * 4;                            // bf16 [t][w4][lane]
  float* rscale = reinterpret_cast<float*>(smem + sc.aux_off);
  int* s_active = reinterpret_cast<int*>(rscale + ((R + 3) & ~3));
  int* s_offsets = s_active + (((a.E + 1) + 3) & ~3);
  int* s_perm = s_offsets + (((a.E + 1) + 3) & ~3);
  __shared__ __align__(8) uint64_t tbl;
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
    if (lane == 0) {
      copy_tables(a, s_active, s_offsets, s_perm, &tbl);
      bool ok = mbar_wait(&tbl, 0, a.status, kSiteDnEmpty);
      int it = 0;
      const int n_r = ok ? s_active[0] * nrb : 0;
      const unsigned shb = kDnRowsShared * Fs * 2;
      const unsigned pk = kDnRowsRouted * (F >> 1), sk = kDnRowsRouted * G;
      for (int j = blockIdx.x; j < n_sh + n_r; j += gridDim.x, ++it) {
        const int s = it % S;
        const unsigned round = it / S;
        if (ok && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, a.status, kSiteDnEmpty);
        if (!ok) continue;
        unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
        if (j < n_sh) {
          mbar_arrive_expect_tx(&full[s], shb);
          bulk_g2s(st, a.sh_down + static_cast<size_t>(j) * kDnRowsShared * Fs, shb, &full[s]);
        } else {
          const int jr = j - n_sh;
          const int e = s_active[1 + jr / nrb];
          const size_t r0 = static_cast<size_t>(jr % nrb) * kDnRowsRouted;
          mbar_arrive_expect_tx(&full[s], pk + sk);
          bulk_g2s(st, a.down_p + e * a.down_ps + r0 * (F >> 1), pk, &full[s]);
          bulk_g2s(st + pk, a.down_s + e * a.down_ss + r0 * G, sk, &full[s]);
        }
      }
      if (!ok) {
        for (int q = (it > S ? it - S : 0); q < it; ++q)
          mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteDnDrain);
      }
    }
    pdl_wait();
    pdl_trigger();
    return;
  }

  // ------------------------------- consumers -------------------------------
  const int grp = warp_id / kConsumerWarps;
  const int warp = warp_id % kConsumerWarps;
  const int ct = threadIdx.x;
  constexpr int kAll = kGroups * kConsumerThreads;
  pdl_wait();  // activations from the gate/up kernel
  pdl_trigger();
  bool ok = mbar_wait_warp(&tbl, 0, a.status, kSiteDnFull);
  const int n_active = ok ? s_active[0] : 0;
  const int n_r = n_active * nrb;
  // routed activations as f16 with a per-route power-of-two prescale; a warp
  // holds its row in registers (G*4 <= 32*kRowRegs uint4) across the max
  constexpr int kRowRegs = 8;
  for (int r = warp_id; r < R; r += kGroups * kConsumerWarps) {
    const uint16_t* src = a.act + static_cast<size_t>(r) * F;
    uint4 v8[kRowRegs];
    float m = 0.f;
#pragma unroll
    for (int q = 0; q < kRowRegs; ++q) {
      const int v = lane + 32 * q;
      if (v < G * 4) v8[q] = __ldcg(reinterpret_cast<const uint4*>(src + 8 * v));
    }
#pragma unroll
    for (int q = 0; q < kRowRegs; ++q) {
      const int v = lane + 32 * q;
      if (v < G * 4) {
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
      if (v < G * 4) {
        const uint4 u = v8[q];
        xr[(r * 4 + (v & 3)) * G + (v >> 2)] =
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

  for (int it = grp, j = blockIdx.x + grp * gridDim.x; j < n_sh + n_r;
       it += kGroups, j += kGroups * gridDim.x) {
    const int s = it % S;
    if (ok) ok = mbar_wait_warp(&full[s], (it / S) & 1, a.status, kSiteDnFull);
    const unsigned char* st = smem + static_cast<size_t>(s) * sc.stage_bytes;
    if (j < n_sh) {  // shared: warp -> row j*8 + warp, whole Fs
      const int row = j * kDnRowsShared + warp;
      float acc[4][TT];
#pragma unroll
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[w][t] = 0.f;
      const unsigned char* wr = st + static_cast<size_t>(warp) * Fs * 2;
      const bool regs = WS <= 8;  // copy this lane's slice out and release the stage first
      uint4 wrg[8];
      if (ok && regs) {
#pragma unroll
        for (int w4 = 0; w4 < 8; ++w4) {
          const int el = 8 * (lane + 32 * w4);
          if (w4 < WS && el < Fs) wrg[w4] = *reinterpret_cast<const uint4*>(wr + 2 * el);
        }
      }
      __syncwarp();
      const bool early = regs || !ok;
      if (early && lane == 0) mbar_arrive(&empty[s]);
      if (ok && regs) {
#pragma unroll
        for (int w4 = 0; w4 < 8; ++w4) {
          const int el = 8 * (lane + 32 * w4);
          if (w4 < WS && el < Fs) {
#pragma unroll
            for (int t = 0; t < TT; ++t)
              if (t < M) acc[w4 & 3][t] = dot8_bf16(wrg[w4], xsb[t * WS * 32 + w4 * 32 + lane], acc[w4 & 3][t]);
          }
        }
      } else if (ok) {
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
      if (!early) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
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
    } else {  // routed: rows r0 .. r0+31 of expert e; a warp iteration covers `slots` rows
      const int jr = j - n_sh;
      const int e = s_active[1 + jr / nrb];
      const int r0 = (jr % nrb) * kDnRowsRouted;
      const int p0 = s_offsets[e];
      const int n = s_offsets[e + 1] - p0;
      int slot_of[TT];
#pragma unroll
      for (int q = 0; q < TT; ++q) slot_of[q] = q < n ? s_perm[p0 + q] : 0;
      const size_t pk = static_cast<size_t>(kDnRowsRouted) * (F >> 1);
      DnRouted<TT> dr{st, pk, F, G, d, LPR, slots, slot, sub, per_lane, warp, p0, n, r0,
                      xr + p0 * 4 * G, rscale + p0, a.y};
#pragma unroll
      for (int q = 0; q < TT; ++q) dr.slot_of[q] = slot_of[q];
      // A lane's rows are rl = warp*slots + slot + it*8*slots and its groups
      // gi = sub + LPR*qg.  The warp computes from the stage and releases it
      // afterwards: a register copy of the slice spills at this CTA size.
      const int row_iters = (kDnRowsRouted + kConsumerWarps * slots - 1) / (kConsumerWarps * slots);
      if (ok) {
        for (int it2 = 0; it2 < row_iters; ++it2) {
          float acc[TT];
#pragma unroll
          for (int q = 0; q < TT; ++q) acc[q] = 0.f;
          const int rl = warp * slots + slot + it2 * kConsumerWarps * slots;
          if (rl < kDnRowsRouted) {
            const unsigned char* wp = st + static_cast<size_t>(rl) * (F >> 1);
            const unsigned char* ws = st + pk + rl * G;
            for (int qg = 0; qg < per_lane; ++qg) {
              const int gi = sub + LPR * qg;
              if (gi < G) down_group<TT>(*reinterpret_cast<const uint4*>(wp + 16 * gi), ws[gi], dr.xv + gi, G, n, acc);
            }
          }
          dr.finish_row(acc, rl);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
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
