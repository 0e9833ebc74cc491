// One-token down projection on the fifth-generation tensor core (sm_100a).
//
// Same products as down1_kernel.cuh (expert_ssd.py:188, layers.py:160-171):
//   y[slot(p), r] = bf16( act[p] . deq(Wd[e_p])[r] )   routed, route p
//   ys[r]         = bf16( act_s . Wsd[r] )             shared, bf16 weights
// computed as 128-row tiles with tcgen05 MMAs:
//  - routed tile: A = 128 rows of the expert's MXFP4 down weights (E2M1 +
//    UE8M0), B = the route's activations split into kTerms E2M1 terms by
//    split_act_kernel (B rows 0..kTerms-1 of a 32-row operand, umma.cuh),
//    kind::mxf4 block-scaled MMAs over K = F, y = sum of the accumulator's
//    kTerms columns;
//  - shared tile: A = 128 bf16 rows, B = act_s as row 0 of a 16-row operand,
//    kind::f16 MMAs.
// Work split: CTA b < n_sh owns shared tile b; the other CTAs own contiguous
// ranges of the routed tiles (route-major), at most kMaxUnits tiles and two
// routes each (checked on the host).
//
// Warps: 0-3 copy the split route activations, stage scale factors into tensor
// memory and read the accumulators; warps 4 and 6 issue the MMAs of the even
// and odd atom columns (one lane each, into their own accumulators), with
// warps 7 and 8 joining for the 24-column shared tile (columns mod 4); warp 5
// issues the TMA loads (one lane; 128-byte-swizzled 128 B x 128-row boxes
// into a stage ring, no multicast) from the start, before the dependency
// wait, since weights and routes are ready when this kernel launches.
// Accumulators and scale-factor columns are double buffered (two route
// operands per CTA) so the MMAs of one tile overlap the epilogue of the
// previous one.  One thread issues at most one tcgen05.mma per ~47 ns
// (measured), so a tile's MMAs are spread over two issuing warps (four for
// the shared tile), each into its own accumulators, which the epilogue adds.
// Every wait is bounded; a timeout records a status word and ends the CTA.
#pragma once
#include <cuda.h>

#include "decode_kernels.cuh"
#include "pipeline.cuh"
#include "umma.cuh"

namespace lg {
namespace dtc {

constexpr int kTerms = 8;          // activation terms (B rows) per route
constexpr int kBRows = 32;         // routed B operand rows (N of the MMA)
constexpr int kShBRows = 16;       // shared B operand rows
constexpr int kTile = 128;         // output rows per tile (M of the MMA)
constexpr int kBox = 16384;        // one 128 B x 128-row weight box
constexpr int kMaxUnits = 3;       // routed tiles per CTA
constexpr int kMaxStages = 10;
constexpr int kThreads = 288;
constexpr int kCompute = 128;      // threads of warps 0-3
// MMA issuers: warps 4, 6 (and 7, 8 for the shared tile); one issuing thread
// keeps at most one MMA per ~47 ns
constexpr int kMmaWarp = 4, kTmaWarp = 5, kMmaWarp1 = 6;
// tensor memory columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD = 0;      // routed: 2 buffers x 2 accumulators x 32; shared: 8 x 16
constexpr uint32_t kColSfa = 128;  // 2 x 96 (24 MMAs x 4 row quarters)
constexpr uint32_t kColSfb = 320;  // 2 routes x 96 (24 MMAs, 4-column aligned)
constexpr int kSiteFull = 21 << 8, kSiteEmpty = 22 << 8, kSiteScale = 23 << 8, kSiteSf = 24 << 8,
              kSiteD = 25 << 8, kSiteRoute = 26 << 8;

struct Cfg {
  int stages;
  int n_sh;        // CTAs [0, n_sh) own one shared tile each
  int n_units;     // routed tiles = k * d / 128
  int cols;        // MXFP4 atom columns per routed row (F / 256)
  int sh_cols;     // bf16 atom columns per shared row (Fs / 64)
  int sc_bytes;    // scale bytes per routed row (F / 32)
  int ring_off, scale_off, b_off;  // shared-memory regions (from the 1024-aligned base)
  uint8_t* bimg;   // split route activations: [route][col] 1 KB = term rows 0-7 of the swizzled B tile
  uint8_t* bsc;    // their scales: [route][term][F / 32]
};

// Activation split of every route, once per call: half-warp h of the grid
// takes 32-value block j of route p (h = p * blocks + j) and writes its
// kTerms term bytes into the swizzled B image and the term scales.  Runs
// between the gate/up kernel (act) and down_tc_kernel, chained by PDL.
__global__ void __launch_bounds__(64) split_act_kernel(DecodeArgs a, Cfg c) {
  // let down_tc_kernel launch (and start its weight loads) at once: its own
  // dependency wait covers this kernel's completion, which follows the
  // gate/up kernel's
  pdl_trigger();
  pdl_wait();  // act from the gate/up kernel
  const int nblk = c.cols * 8, routes = a.M * a.k;
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) >> 4, hl = threadIdx.x & 15;
  if (h >= routes * nblk) return;  // whole half-warps leave together (nblk * routes % 2 == 0)
  const int p = h / nblk, j = h - p * nblk, col = j >> 3, jb = j & 7;
  const uint32_t pair = __ldcg(reinterpret_cast<const uint32_t*>(a.act + static_cast<size_t>(p) * a.F + j * 32) + hl);
  float r0 = __uint_as_float(pair << 16), r1 = __uint_as_float(pair & 0xFFFF0000u);
  bool live;
  const int s0 = umma::split_base(r0, r1, &live);
  uint8_t* img = c.bimg + (static_cast<size_t>(p) * c.cols + col) * 1024;
#pragma unroll
  for (int t = 0; t < kTerms; ++t) {
    const int e = umma::term_scale(s0, t);
    img[umma::sw128_offset(t, jb * 16 + hl)] = static_cast<uint8_t>(live ? umma::split_step(r0, r1, e) : 0u);
    if (hl == 0) c.bsc[(static_cast<size_t>(p) * kTerms + t) * c.sc_bytes + j] = static_cast<uint8_t>(live ? 127 + e : 127);
  }
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Bounded wait with a short suspend hint: a waiter parked in try_wait without
// one (or with a long one) was seen to resume microseconds after the phase
// completed, which every stage handoff of this kernel would pay.
constexpr unsigned kHintNs = 100;
__device__ __forceinline__ bool wait1(uint64_t* b, unsigned parity, int* status, int site,
                                      unsigned long long limit_ns = kWaitLimitNs) {
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(b)), "r"(parity), "r"(kHintNs)
        : "memory");
    if (done) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      if (status) atomicExch(status, 6 | site);
      return false;
    }
  }
}
// the same by every lane of a warp, with one verdict for the warp
__device__ __forceinline__ bool wait_warp1(uint64_t* b, unsigned parity, int* status, int site) {
  return __all_sync(0xffffffffu, wait1(b, parity, status, site));
}

// routed tiles [lo, hi) of CTA b (b >= n_sh)
__device__ __forceinline__ void unit_range(const Cfg& c, int b, int P, int& lo, int& hi) {
  const int q = P - c.n_sh, i = b - c.n_sh;
  lo = static_cast<int>(static_cast<long long>(i) * c.n_units / q);
  hi = static_cast<int>(static_cast<long long>(i + 1) * c.n_units / q);
}

__global__ void __launch_bounds__(kThreads, 1)
    down_tc_kernel(DecodeArgs a, Cfg c, const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                   const __grid_constant__ CUtensorMap tm_sh) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ __align__(8) uint64_t sfull[2], sfree[2], sf_ready[2], dfull[2];
  __shared__ uint32_t tslot;
  __shared__ uint8_t sfb_s[2][kBRows][48];  // term scales of up to two routes (F <= 1536)
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = base + c.ring_off;
  unsigned char* sslot = base + c.scale_off;  // 2 x (128 rows x sc_bytes)
  unsigned char* bop = base + c.b_off;        // B operands
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, b = blockIdx.x, S = c.stages, d = a.d;
  const bool shared_cta = b < c.n_sh;
  int u_lo = 0, u_hi = 0;
  if (!shared_cta) unit_range(c, b, P, u_lo, u_hi);
  const int nu = shared_cta ? 1 : u_hi - u_lo;
  const int blocks = d / kTile;
  const int p_first = shared_cta ? 0 : u_lo / blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], kCompute / 32);
      mbar_init(&sf_ready[i], kCompute / 32);
      mbar_init(&dfull[i], shared_cta ? 4 : 2);  // one commit per MMA issuer
    }
    mbar_fence_init();
  }
  if (warp == 0) umma::tmem_alloc(&tslot, kTmemCols);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = tslot;

  // ------------------------------- TMA producer -------------------------------
  if (warp == kTmaWarp) {
    if (lane == 0 && nu > 0) {
      bool ok = true;
      int it = 0;
      for (int li = 0; li < nu && ok; ++li) {
        int row0, ncols;
        const CUtensorMap* map;
        if (shared_cta) {
          row0 = b * kTile;
          ncols = c.sh_cols;
          map = &tm_sh;
        } else {
          const int u = u_lo + li, p = u / blocks, rb = u - p * blocks;
          const int e = __ldcg(a.active + 1 + p);
          if (e < 0 || e >= a.E) {
            atomicExch(a.status, 1 | kSiteRoute);
            ok = false;
            break;
          }
          row0 = e * d + rb * kTile;
          ncols = c.cols;
          map = &tm_w;
          const int sb = li & 1;
          if (li >= 2) ok = wait1(&sfree[sb], ((li >> 1) - 1) & 1, a.status, kSiteScale);
          if (!ok) break;
          mbar_arrive_expect_tx(&sfull[sb], static_cast<unsigned>(kTile * c.sc_bytes));
          tma_2d(sslot + sb * kTile * c.sc_bytes, &tm_s, 0, row0, &sfull[sb]);
        }
        for (int col = 0; col < ncols; ++col, ++it) {
          const int s = it % S;
          if (it >= S) ok = wait1(&empty[s], ((it / S) - 1) & 1, a.status, kSiteEmpty);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], kBox);
          tma_2d(ring + s * kBox, map, col * 128, row0, &full[s]);
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA leaves
        for (int q = (it > S ? it - S : 0); q < it; ++q) wait1(&full[q % S], (q / S) & 1, a.status, kSiteFull);
      }
    }
    pdl_wait();
    pdl_trigger();
  }
  // ------------------------------- MMA issuer ---------------------------------
  else if (warp == kMmaWarp || warp >= kMmaWarp1) {
    pdl_wait();
    pdl_trigger();
    const int n_iss = shared_cta ? 4 : 2;
    const int w = warp == kMmaWarp ? 0 : warp - kMmaWarp1 + 1;  // this issuer's atom columns: w, w + n_iss, ...
    if (lane == 0 && nu > 0 && w < n_iss) {
      bool ok = true;
      const uint32_t id_mx = umma::idesc_mxf4(kTile, kBRows), id_bf = umma::idesc_bf16(kTile, kShBRows);
      for (int li = 0; li < nu && ok; ++li) {
        const int db = li & 1;
        ok = wait1(&sf_ready[db], (li >> 1) & 1, a.status, kSiteSf);
        if (!ok) break;
        umma::fence_after_sync();
        const uint32_t dcol = tbase + kColD + 64u * db;
        const int ncols = shared_cta ? c.sh_cols : c.cols;
        const int rbuf = shared_cta ? 0 : (u_lo + li) / blocks - p_first;
        for (int col = w; col < ncols; col += n_iss) {
          const int it = li * ncols + col, s = it % S;  // the producer's stage count
          ok = wait1(&full[s], (it / S) & 1, a.status, kSiteFull);
          if (!ok) break;
          umma::fence_after_sync();
          const uint64_t da = umma::desc_sw128(smem_u32(ring + s * kBox));
          if (shared_cta) {
            const uint64_t dbd = umma::desc_sw128(smem_u32(bop + col * (kShBRows * 128)));
#pragma unroll
            for (int i = 0; i < 4; ++i)  // accumulator 2 w + (i & 1), first written at column w
              umma::mma_bf16(tbase + kColD + 16u * (2 * w + (i & 1)), da + 2 * i, dbd + 2 * i, id_bf, col >= 4 || i >= 2);
          } else {
            const uint64_t dbd = umma::desc_sw128(smem_u32(bop + (rbuf * c.cols + col) * (kBRows * 128)));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int m = 4 * col + i;
              umma::mma_mxf4(dcol + 32u * w, da + 2 * i, dbd + 2 * i, id_mx, tbase + kColSfa + 96u * db + 4u * m,
                             tbase + kColSfb + 96u * rbuf + 4u * m, col >= 2 || i > 0);
            }
          }
          umma::commit(&empty[s]);
        }
        if (ok) umma::commit(&dfull[db]);
      }
    }
  }
  // ---------------------- activations, scale factors, epilogue ----------------
  else {
    const int ct = threadIdx.x;  // 0..127
    const uint32_t lanes = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    bool ok = nu > 0;
    const int nr = shared_cta || !ok ? 0 : (u_hi - 1) / blocks - p_first + 1;  // routes of this CTA
    // zero B rows and the constant scales of the zero term rows: no dependence
    // on the gate/up kernel, so before the dependency wait
    if (ok) {
      const int n16 = shared_cta ? c.sh_cols * kShBRows * 128 / 16 : nr * c.cols * kBRows * 128 / 16;
      for (int i = ct; i < n16; i += kCompute) reinterpret_cast<uint4*>(bop)[i] = make_uint4(0u, 0u, 0u, 0u);
      for (int i = ct; i < nr * (kBRows - kTerms) * c.sc_bytes; i += kCompute) {
        const int r = i / ((kBRows - kTerms) * c.sc_bytes), rem = i - r * ((kBRows - kTerms) * c.sc_bytes);
        sfb_s[r][kTerms + rem / c.sc_bytes][rem % c.sc_bytes] = 127;
      }
    }
    named_sync(1, kCompute);
    pdl_wait();  // act / act_s from the gate/up kernel, the split from split_act_kernel
    pdl_trigger();
    if (shared_cta && ok) {
      // B: act_s as row 0 of each 16-row column tile
      for (int i = ct; i < c.sh_cols * 8; i += kCompute) {
        const int col = i >> 3, ch = i & 7;
        *reinterpret_cast<uint4*>(bop + col * (kShBRows * 128) + umma::sw128_offset(0, ch * 16)) =
            __ldcg(reinterpret_cast<const uint4*>(a.act_s) + i);
      }
    } else if (ok) {
      // B: the routes' split activations (split_act_kernel), term rows 0-7 of each column tile
      for (int i = ct; i < nr * c.cols * 64; i += kCompute) {
        const int rc = i >> 6, w16 = i & 63;  // (route, column) image, 16-byte word
        *reinterpret_cast<uint4*>(bop + rc * (kBRows * 128) + w16 * 16) =
            __ldcg(reinterpret_cast<const uint4*>(c.bimg + (static_cast<size_t>(p_first) * c.cols + rc) * 1024) + w16);
      }
      for (int i = ct; i < nr * kTerms * c.sc_bytes; i += kCompute) {
        const int r = i / (kTerms * c.sc_bytes), rem = i - r * (kTerms * c.sc_bytes);
        sfb_s[r][rem / c.sc_bytes][rem % c.sc_bytes] =
            __ldcg(c.bsc + (static_cast<size_t>(p_first + r) * kTerms) * c.sc_bytes + rem);
      }
      named_sync(1, kCompute);
      // term scales into tensor memory: lane l = B row l, byte s = block 2m + s
      for (int r = 0; r < nr; ++r)
        for (int m = 0; m < c.cols * 4; ++m)
          umma::st_32x32b_x1(lanes + kColSfb + 96u * r + 4u * m,
                             static_cast<uint32_t>(sfb_s[r][lane][2 * m]) |
                                 (static_cast<uint32_t>(sfb_s[r][lane][2 * m + 1]) << 8));
    }
    umma::fence_async_smem();

    auto stage_scales = [&](int li) -> bool {  // routed tile li: SFA into tensor memory
      const int sb = li & 1;
      if (!wait_warp1(&sfull[sb], (li >> 1) & 1, a.status, kSiteScale)) return false;
      // MMA m's scales sit in columns 4m + q (q = row quarter), so a chunk of
      // eight MMAs is 32 consecutive columns: bytes 16g..16g+15 of this
      // lane's row in each quarter, one 16-byte load per quarter
      const unsigned char* sc = sslot + sb * kTile * c.sc_bytes;
      for (int g = 0; g < c.cols / 2; ++g) {
        uint4 rq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) rq[q] = *reinterpret_cast<const uint4*>(sc + (32 * q + lane) * c.sc_bytes + 16 * g);
        uint32_t v[32];
#pragma unroll
        for (int m = 0; m < 8; ++m)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t word = m < 2 ? rq[q].x : (m < 4 ? rq[q].y : (m < 6 ? rq[q].z : rq[q].w));
            v[4 * m + q] = (word >> (16 * (m & 1))) & 0xFFFFu;
          }
        umma::st_32x32b_x32(lanes + kColSfa + 96u * (li & 1) + 32u * g, v);
      }
      umma::wait_st();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[sb]);
      return true;
    };
    auto epilogue = [&](int li) -> bool {
      const int db = li & 1;
      if (!wait_warp1(&dfull[db], (li >> 1) & 1, a.status, kSiteD)) return false;
      umma::fence_after_sync();
      uint32_t dv[32];
      const int row = warp * 32 + lane;
      float s = 0.f;
      if (shared_cta) {  // accumulator j in columns 16 j, its value in column 0
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          umma::ld_32x32b_x32(lanes + kColD + 32u * h, dv);
          s = __fadd_rn(s, __fadd_rn(__uint_as_float(dv[0]), __uint_as_float(dv[16])));
        }
        a.ys[b * kTile + row] = f32_to_bf16(s);
      } else {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          umma::ld_32x32b_x32(lanes + kColD + 64u * db + 32u * j, dv);
#pragma unroll
          for (int t = 0; t < kTerms; ++t) s = __fadd_rn(s, __uint_as_float(dv[t]));
        }
        const int u = u_lo + li, p = u / blocks, rb = u - p * blocks;
        a.y[static_cast<size_t>(__ldcg(a.perm + p)) * d + rb * kTile + row] = f32_to_bf16(s);
      }
      return true;
    };
    for (int li = 0; li < nu && ok; ++li) {
      if (!shared_cta) ok = stage_scales(li);
      if (!ok) break;
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_ready[li & 1]);
      if (li >= 1) ok = epilogue(li - 1);
    }
    if (ok && nu > 0) ok = epilogue(nu - 1);
  }
  __syncwarp();  // warps 4 and 5 ran one lane alone
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tbase, kTmemCols);
}

}  // namespace dtc
}  // namespace lg
