// One-token down projection of the decode chain (sm_100a).
//
// Restates the per-route down product of ExpertSSD.__call__
// (expert_ssd.py:188; native masked QMV, native_expert_ssd.py:707-712) and
// the shared expert's down projection (layers.py:160-171) for one token:
//   y[slot, r]  = bf16( act[p] . deq(Wd[e_p])[r] )     (routed, route p -> slot)
//   ys[r]       = bf16( act_s . Wsd[r] )               (shared, bf16 weights)
// The merge stays in combine_decode_kernel.
//
// Work split: CTA b owns shared rows [b*d/P, (b+1)*d/P) and an even slice of
// the routed rows, routes concatenated (route p owns rows [p*d, (p+1)*d)).
// One producer lane streams the weights (bulk copies into an mbarrier ring,
// no multicast) from the start, before the dependency wait; eight consumer
// warps wait for the gate/up kernel, copy this CTA's activation rows from L2
// into shared memory once, then:
//  - shared chunk (8 rows): warp w owns row w, lanes over 8-column words,
//    act_s in registers;
//  - routed chunk (up to 32 rows of one route): half-warp h of warp w owns
//    rows 4w+2h and 4w+2h+1, lane l (of 16) the 32-column groups l + 16*c, with the route's
//    activations in registers as f16 scaled by a power of two (max |v| <
//    2^8); a lane's three scale bytes of a row come from three 32-bit loads,
//    no byte loads.
// The next chunk's loads are issued while the current sums are reduced.
#pragma once
#include "decode_helpers.cuh"

namespace lg {
namespace down1 {

using dh::bf16x8_to_f16x8_scaled;
using dh::absmax8_bf16;
using dh::act_shift;
using dh::fold4;
using dh::lds128;
using dh::lds32;
using dh::mx_dot_reg;
using dh::reduce_scatter;
using dh::wait_all;

constexpr int kWarps = 8;
constexpr int kConsumers = kWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kRows = 32;                  // routed rows per chunk
constexpr int kShRows = 8;                 // shared rows per chunk
constexpr int kDcg = 3;                    // routed column groups per half-warp lane (F <= 1536)
constexpr int kScg = 6;                    // shared 8-column words per lane (Fs <= 1536)
constexpr int kMaxStages = 8;
static_assert(kShRows == kWarps && kRows == 4 * kWarps, "row ownership of the consumer warps");
constexpr int kSiteFull = 17 << 8, kSiteEmpty = 18 << 8, kSiteDrain = 19 << 8, kSiteRoute = 20 << 8;

struct Cfg {
  int stages, stage_bytes, unit;
  int act_off;  // this CTA's routed activation rows, bf16 [routes][F]
  int yb_off;   // this CTA's finished rows, bf16: routed slice, then shared block
  int yb_rows;  // most routed rows of one CTA
};

// CTA b's rows: shared [sr_lo, sr_hi), routed [u_lo, u_hi) in units of `unit`
struct Split {
  int sr_lo, sr_hi, u_lo, u_hi;
  __device__ __forceinline__ Split(const DecodeArgs& a, const Cfg& c, int b, int P) {
    const unsigned d = a.d, p = P, nu = static_cast<unsigned>(a.M * a.k) * d / c.unit;
    sr_lo = static_cast<int>(b * d / p);
    sr_hi = static_cast<int>((b + 1) * d / p);
    u_lo = c.unit * static_cast<int>(b * nu / p);
    u_hi = c.unit * static_cast<int>((b + 1) * nu / p);
  }
};

__global__ void __launch_bounds__(kThreads, 1) down1_stream_kernel(DecodeArgs a, Cfg c) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ volatile unsigned rel_sink[kConsumers];
  const int warp_id = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.d, F = a.F, Fs = a.Fs, G2 = F >> 5, E = a.E;
  const int P = gridDim.x, b = blockIdx.x, S = c.stages;
  const Split sp(a, c, b, P);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  // ------------------------------ producer ------------------------------
  if (warp_id == kWarps) {
    if (lane == 0) {
      bool ok = true;
      int it = 0;
      auto stage_free = [&]() -> bool {
        if (!ok) return false;
        if (it >= S) ok = mbar_wait(&empty[it % S], ((it / S) - 1) & 1, a.status, kSiteEmpty);
        return ok;
      };
      // experts of this CTA's routes, loaded once (a global round trip per
      // chunk would pace the whole ring)
      constexpr int kMaxSpan = 4;
      const int p_lo = sp.u_lo / d;
      int ex[kMaxSpan];
#pragma unroll
      for (int q = 0; q < kMaxSpan; ++q) ex[q] = p_lo + q < a.M * a.k ? __ldcg(a.active + 1 + p_lo + q) : -1;
      if (Fs > 0) {
        for (int r0 = sp.sr_lo; r0 < sp.sr_hi; r0 += kShRows, ++it) {
          if (!stage_free()) continue;
          const unsigned bytes = static_cast<unsigned>(min(kShRows, sp.sr_hi - r0)) * Fs * 2u;
          unsigned char* st = smem + static_cast<size_t>(it % S) * c.stage_bytes;
          mbar_arrive_expect_tx(&full[it % S], bytes);
          bulk_g2s(st, a.sh_down + static_cast<size_t>(r0) * Fs, bytes, &full[it % S]);
        }
      }
      // route p is the p-th active expert (one route per expert for one token;
      // the router kernel finished before this kernel was launched)
      for (int u = sp.u_lo; u < sp.u_hi; ++it) {
        const int p = u / d, r0 = u - p * d, nr = min(kRows, min(sp.u_hi, (p + 1) * d) - u);
        u += nr;
        if (!stage_free()) continue;
        int e = -1;
#pragma unroll
        for (int q = 0; q < kMaxSpan; ++q)
          if (p - p_lo == q) e = ex[q];
        if (e < 0 || e >= E) {
          atomicExch(a.status, 1 | kSiteRoute);
          ok = false;
          continue;
        }
        const unsigned pb = static_cast<unsigned>(nr) * (F / 2), sb = static_cast<unsigned>(nr) * G2;
        unsigned char* st = smem + static_cast<size_t>(it % S) * c.stage_bytes;
        uint64_t* fb = &full[it % S];
        mbar_arrive_expect_tx(fb, pb + sb);
        bulk_g2s(st, a.down_p + e * a.down_ps + static_cast<size_t>(r0) * (F / 2), pb, fb);
        bulk_g2s(st + pb, a.down_s + e * a.down_ss + static_cast<size_t>(r0) * G2, sb, fb);
      }
      if (!ok) {  // copies already issued land before the CTA leaves
        for (int q = (it > S ? it - S : 0); q < it; ++q)
          mbar_wait(&full[q % S], (q / S) & 1, a.status, kSiteDrain);
      }
    }
    pdl_wait();
    pdl_trigger();
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int wg = warp_id, ct = threadIdx.x;
  pdl_wait();  // act and act_s from the gate/up kernel
  pdl_trigger();
  bool ok = true;
  int it = 0;
  auto release_after = [&](int s, unsigned dep) {
    // every copied word is in registers before the stage goes back
    rel_sink[ct] = dep;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  };

  // this CTA's routed activation rows (at most a few routes), one pass from L2
  const int p_lo = sp.u_lo / d, np = sp.u_hi > sp.u_lo ? (sp.u_hi - 1) / d - p_lo + 1 : 0;
  uint4* sact = reinterpret_cast<uint4*>(smem + c.act_off);
  // finished rows wait in shared memory until the end: a global store ahead
  // of a stage release held the release up
  uint16_t* yb = reinterpret_cast<uint16_t*>(smem + c.yb_off);
  uint16_t* ysb = yb + c.yb_rows;
  for (int i = ct; i < np * (F >> 3); i += kConsumers)
    sact[i] = __ldcg(reinterpret_cast<const uint4*>(a.act) + static_cast<size_t>(p_lo) * (F >> 3) + i);
  named_sync(1, kConsumers);

  // shared down: warp wg owns row r0 + wg of each chunk, act_s in registers
  if (Fs > 0 && sp.sr_hi > sp.sr_lo) {
    const int fs8 = Fs >> 3;
    uint4 xs[kScg];
#pragma unroll
    for (int i = 0; i < kScg; ++i)
      xs[i] = lane + 32 * i < fs8 ? __ldcg(reinterpret_cast<const uint4*>(a.act_s) + lane + 32 * i)
                                  : make_uint4(0u, 0u, 0u, 0u);
    for (int r0 = sp.sr_lo; r0 < sp.sr_hi; r0 += kShRows, ++it) {
      const int s = it % S;
      if (ok) ok = wait_all(&full[s], (it / S) & 1, a.status, kSiteFull, lane);
      const int nr = min(kShRows, sp.sr_hi - r0);
      const unsigned char* st = smem + static_cast<size_t>(s) * c.stage_bytes + static_cast<size_t>(wg) * Fs * 2;
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
      if (lane == 0 && wg < nr) ysb[r0 - sp.sr_lo + wg] = f32_to_bf16(acc);
    }
  }

  // routed down
  if (sp.u_hi > sp.u_lo) {
    const int hl = lane & 15, hh = lane >> 4, f8 = F >> 3;
    int cgd[kDcg];
#pragma unroll
    for (int cc = 0; cc < kDcg; ++cc) cgd[cc] = hl + 16 * cc;
    uint4 xr[kDcg][4];
    float rsc = 1.f;
    // the route's act row: power-of-two scale from its max, f16 copy of this
    // lane's column groups (both half-warps hold the same row)
    auto load_route = [&](int p) {
      const uint4* row = sact + static_cast<size_t>(p - p_lo) * f8;
      unsigned m = 0u;  // two passes over shared memory: max, then convert
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
      const unsigned char* st = smem + static_cast<size_t>(s) * c.stage_bytes;
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
    int u = sp.u_lo;
    int p = u / d, nr = min(kRows, min(sp.u_hi, (p + 1) * d) - u);
    fetch(nr);
    release_after(s, loaded());
    int pcur = -1;
    while (u < sp.u_hi) {
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
      const int cu = u - sp.u_lo, cnr = nr;
      const float crs = rsc;
      u += nr;
      ++it;
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
      const bool more = u < sp.u_hi;
      if (more) {
        p = u / d;
        nr = min(kRows, min(sp.u_hi, (p + 1) * d) - u);
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
  // write this CTA's rows: routed rows to their route slots, shared rows
  named_sync(1, kConsumers);
  if (ok) {
    for (int i = ct; i < sp.u_hi - sp.u_lo; i += kConsumers) {
      const int u = sp.u_lo + i, pp = u / d;
      a.y[static_cast<size_t>(__ldcg(a.perm + pp)) * d + (u - pp * d)] = yb[i];
    }
    if (Fs > 0)
      for (int i = ct; i < sp.sr_hi - sp.sr_lo; i += kConsumers) a.ys[sp.sr_lo + i] = ysb[i];
  }
}

}  // namespace down1
}  // namespace lg
