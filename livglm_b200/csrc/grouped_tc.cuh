// Batched MoE expert products on the fifth-generation tensor core (sm_100a).
//
// Restates, for many tokens per call, the routed expert chain of
// ExpertSSD.__call__ (kg36/livglm src/glm53flash/expert_ssd.py:159-188: MXFP4
// gather_qmm gate/up, limited SwiGLU, down) and the shared DenseMLP
// (layers.py:160-171) as grouped GEMMs:
//
//   routed gate/up   act[p]   = swiglu(bf16(Wg_e x_t), bf16(Wu_e x_t))  kind::mxf4
//   routed down      y[s(p)]  = bf16(Wd_e act[p])                       kind::mxf4
//   shared gate/up   act_s[t] = swiglu(bf16(Wsg x_t), bf16(Wsu x_t))    kind::f16
//   shared down      ys[t]    = bf16(Wsd act_s[t])                      kind::f16
//
// for every route p = (token t, slot j) of expert e, in the stable
// expert-sorted order of the dispatch (perm).  The weights are read straight
// from the checkpoint's MXFP4 bytes (E2M1 nibbles + UE8M0 group-32 scales);
// kind::mxf4 needs E2M1 on both sides, so the bf16 activations enter as kTerms
// E2M1 terms with their own UE8M0 block scales (umma.cuh): split_routes_kernel
// splits every token once and writes its terms to each dispatch position
// that routes it, the routed gate/up epilogue writes the terms of act.
//
// Operands in HBM (row-major, K contiguous, bytes), route-major so that the B
// rows of one (expert, route tile) pair are one contiguous block:
//   x terms     [R][T][d/2]  + scales [R][T][d/32]    row p*T + t (dispatch order)
//   act terms   [R][T][F/2]  + scales [R][T][F/32]
// A tile: 128 weight rows x 128 bytes (256 E2M1 or 64 bf16 values), loaded by
// TMA with the 128-byte swizzle (no multicast).  Routed gate/up: rows 0-63 are
// gate rows f0..f0+63, rows 64-127 the up rows with the same indices, so one
// accumulator holds both halves of 64 SwiGLU columns.  B tile: the ntp routes
// (16 or 32: the tile's route count rounded up) x T terms, row i*T + t, so
// N = T * ntp and one TMA box per k-block brings it (the TMA front end, not
// HBM, bounded an earlier version that gathered four rows per instruction).
// Scale tiles (per item, all k-blocks) land row-major, with the 128-byte
// swizzle where a scale row is 128 bytes, so that the scale-factor warps'
// lanes (one row each, same column) spread over the banks.
//
// Work items: (expert, row block, route tile) with the route tile fastest, so
// the CTAs working at the same time share one weight row block (read from HBM
// once, then from L2); the shared expert's items are (row block, token tile).
// One persistent CTA per SM walks items b, b + P, b + 2P, ...
//
// Warps: 0 TMA producer, 1 MMA issuer (one lane), 2-5 scale-factor staging
// (routed: per k-block, A and B scale words from shared memory into a ring of
// tensor-memory slots with tcgen05.st), 6-9 epilogue (tcgen05.ld of the
// double-buffered accumulator), 10-13 help 6-9 with the gate/up epilogue's
// SwiGLU and activation split, the longest per-item work.  Every wait is bounded: a timeout records
// 6 | site in the status word and the CTA leaves after its copies and MMAs in
// flight have landed.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "pipeline.cuh"
#include "umma.cuh"
#include "down_tc.cuh"

namespace lg {
namespace gtc {

constexpr int kThreads = 448;
constexpr int kProdWarp = 0, kMmaWarp = 1, kSfWarp0 = 2, kEpiWarp0 = 6, kMathWarp0 = 10;
constexpr int kMathWarps = 8;     // gate/up epilogue: warps 6-13 share the SwiGLU and split
constexpr int kTerms = 6;         // E2M1 terms per bf16 activation
constexpr int kNtMax = 32;        // routes per routed tile
constexpr int kNtShared = 128;    // tokens per shared tile
constexpr int kMaxStages = 8;
constexpr int kSfSlots = kMaxStages;
constexpr int kSfaCols = 8;       // A: 2 MMA pairs x 4 row quarters
constexpr int kSfbCols = 16;      // B: 2 MMA pairs x 8 row groups (N <= 256)
constexpr int kSfSlotCols = kSfaCols + kSfbCols;
constexpr int kABytes = 16384;    // 128 rows x 128 bytes
// Routed kernels hold two accumulators of kTerms * kNtMax columns and one
// scale-factor slot per ring stage in the 512 tensor-memory columns: 2 * 192 +
// 5 * 24 = 504, so their ring has at most kRoutedStages stages.
constexpr int kRoutedStages = (512 - 2 * kTerms * kNtMax) / kSfSlotCols;
static_assert(kRoutedStages >= 2 && kRoutedStages <= kSfSlots, "tensor-memory plan of the routed kernels");
constexpr int kEpiBar = 2;        // named barrier of the epilogue warps
constexpr int kSiteFull = 40 << 8, kSiteEmpty = 41 << 8, kSiteSfFull = 42 << 8, kSiteSfEmpty = 43 << 8,
              kSiteScFull = 44 << 8, kSiteScFree = 45 << 8, kSiteAccFull = 46 << 8, kSiteAccEmpty = 47 << 8,
              kSiteDrain = 48 << 8;

struct Args {
  int M, d, F, Fs, E, k, R;  // R = M * k route slots
  int kb_count;              // K atoms per item
  int rb_count;              // row blocks per route tile (routed) / per token tile (shared)
  int sc_bytes;              // scale bytes per row (routed: K / 32)
  int sc_swz;                // scale tiles carry the 128-byte swizzle (sc_bytes == 128)
  int n_tok_tiles;           // shared: token tiles
  int stages, stage_bytes, b_off;       // ring: stage s at ring + s * stage_bytes, B at + b_off
  int ring_off, sfa_off, sfb_off, xch_off, tab_off;  // shared-memory regions (1024-aligned base)
  int sfa_bytes, sfb_bytes;             // one item's scale tiles (routed; two buffers each)
  float limit;
  const int* offsets;     // [E + 1] dispatch offsets
  const int* perm;        // [R] route slot of dispatch position p
  const int* tile_start;  // [E + 1] route tiles before expert e (routed)
  uint8_t* act_terms;     // [R][T][F/2]   routed gate/up output
  uint8_t* act_tsc;       // [R][T][F/32]
  uint16_t* act_s;        // [M][Fs]       shared gate/up output
  uint16_t* y;            // [R][d]        routed down output, slot order
  uint16_t* ys;           // [M][d]        shared down output
  int* status;
};

// ---- TMA ----------------------------------------------------------------------
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ---- route terms -----------------------------------------------------------------
// inv[s] = dispatch position of route slot s (-1: the slot's expert id was
// out of range and the dispatch skipped it).  inv must be preset to -1.
__global__ void __launch_bounds__(256) inverse_perm_kernel(const int* __restrict__ perm, const int* __restrict__ offsets,
                                                           int E, int* __restrict__ inv) {
  const int n = offsets[E];
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) inv[perm[p]] = p;
}

// Split every token row into kTerms E2M1 terms (umma.cuh) once and write them
// to each of its k dispatch positions.  Thread q of a 4-thread group holds
// values 8q .. 8q + 7 of one 32-value block (16 bytes of x); a warp covers 8
// consecutive blocks (one 256-value k-block) of one token, so each term row
// is written as one 128-byte line per store instruction.  d % 256 == 0.
__global__ void __launch_bounds__(256) split_routes_kernel(const uint16_t* __restrict__ x, int M, int d, int k,
                                                           const int* __restrict__ inv, uint8_t* __restrict__ terms,
                                                           uint8_t* __restrict__ tsc) {
  const int nkb = d / 256;  // warps per token
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(M) * nkb) return;  // whole warps leave together
  const int t = static_cast<int>(w / nkb), kb = static_cast<int>(w - static_cast<long long>(t) * nkb);
  const int col = kb * 256 + 8 * lane;  // first of this thread's 8 values
  const uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * d + col);
  float r[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y), bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) a = fmaxf(a, fabsf(r[i]));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
  a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));  // the 32-value block's largest magnitude
  const bool live = a >= 0x1p-100f;
  const int s0 = live ? umma::term_exponent(a) : 0;
  uint32_t word[kTerms];
  uint8_t scale[kTerms];
#pragma unroll
  for (int q = 0; q < kTerms; ++q) {
    const int e = umma::term_scale(s0, q);
    uint32_t v = 0u;
    if (live) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v |= umma::split_step(r[2 * i], r[2 * i + 1], e) << (8 * i);
    }
    word[q] = v;
    scale[q] = static_cast<uint8_t>(live ? 127 + e : 127);
  }
  // the token's dispatch positions (k <= 32), loaded once per warp
  const int pl = lane < k ? __ldg(inv + static_cast<size_t>(t) * k + lane) : -1;
  for (int jj = 0; jj < k; ++jj) {
    const int p = __shfl_sync(0xffffffffu, pl, jj);
    if (p < 0) continue;
#pragma unroll
    for (int q = 0; q < kTerms; ++q) {
      const size_t row = static_cast<size_t>(p) * kTerms + q;
      reinterpret_cast<uint32_t*>(terms + row * (d / 2))[col / 8] = word[q];
      if ((lane & 3) == 0) tsc[row * (d / 32) + col / 32] = scale[q];
    }
  }
}

// ---- route tiles ---------------------------------------------------------------
// tile_start[e] = route tiles (of kNtMax routes) of experts before e; one CTA.
__global__ void __launch_bounds__(1024) tile_table_kernel(const int* __restrict__ offsets, int E,
                                                          int* __restrict__ tile_start) {
  __shared__ int part[32];
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  const int n = e < E ? (offsets[e + 1] - offsets[e] + kNtMax - 1) / kNtMax : 0;
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
    part[lane] = w;  // inclusive prefix over warps
  }
  __syncthreads();
  const int incl = v + (warp > 0 ? part[warp - 1] : 0);
  if (e < E) tile_start[e + 1] = incl;
  if (e == 0) tile_start[0] = 0;
}

// ---- work items ------------------------------------------------------------------
struct Item {
  int e;     // expert (routed)
  int rb;    // row block
  int p0;    // first dispatch position (routed) / first token (shared)
  int nt;    // routes / tokens in the tile
  int ntp;   // routed: 16 or 32 (nt rounded up); shared: nt rounded up to 16
};

// routed item i: expert e owns items [rb_count * ts[e], rb_count * ts[e + 1]),
// ordered (row block, route tile) with the tile fastest; ts is the CTA's copy
// of tile_start in shared memory
__device__ __forceinline__ bool routed_item(const Args& a, const int* ts, int i, Item& it) {
  const int RB = a.rb_count;
  if (i >= RB * ts[a.E]) return false;
  int lo = 0, hi = a.E;  // RB * ts[lo] <= i < RB * ts[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (RB * ts[mid] <= i) lo = mid;
    else hi = mid;
  }
  const int n_e = ts[lo + 1] - ts[lo];
  const int local = i - RB * ts[lo];
  const int rb = local / n_e, j = local - rb * n_e;
  const int cnt = a.offsets[lo + 1] - a.offsets[lo];
  it.e = lo;
  it.rb = rb;
  it.p0 = a.offsets[lo] + j * kNtMax;
  it.nt = min(kNtMax, cnt - j * kNtMax);
  it.ntp = it.nt <= 16 ? 16 : 32;
  return true;
}
__device__ __forceinline__ bool shared_item(const Args& a, int i, Item& it) {
  if (i >= a.rb_count * a.n_tok_tiles) return false;
  const int rb = i / a.n_tok_tiles, j = i - rb * a.n_tok_tiles;
  it.e = 0;
  it.rb = rb;
  it.p0 = j * kNtShared;
  it.nt = min(kNtShared, a.M - it.p0);
  it.ntp = (it.nt + 15) & ~15;
  return true;
}

// byte offset of (row, byte) in a scale tile of sc-byte rows, with the TMA's
// 128-byte swizzle (16-byte chunk index XOR address bits 7-9) when swz
__device__ __forceinline__ uint32_t sc_off(int row, int byte, int sc, int swz) {
  const uint32_t o = static_cast<uint32_t>(row * sc + byte);
  return swz ? (o ^ (((o >> 7) & 7u) << 4)) : o;
}

// ---- the SwiGLU output split of one route: 32 values, one per lane ---------------
// Same terms as umma.cuh's split (first scale maps the block max into [0, 6],
// term t at s0 - 2t, round-to-nearest E2M1 of the residual), with the block
// held by a whole warp: the pair (2i, 2i+1) of a byte is formed by a shuffle.
__device__ __forceinline__ void split_warp_write(float v, int lane, int T, uint8_t* img, size_t term_stride,
                                                 uint8_t* sc, size_t sc_stride) {
  float a = fabsf(v);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
  const bool live = a >= 0x1p-100f;
  const int s0 = live ? umma::term_exponent(a) : 0;
  const bool odd = lane & 1;
  float r = v;
  for (int t = 0; t < T; ++t) {
    const int e = umma::term_scale(s0, t);
    const float inv = __int_as_float((127 - e) << 23), scl = __int_as_float((127 + e) << 23);
    const float other = __shfl_xor_sync(0xffffffffu, r, 1);
    const float lo = odd ? other : r, hi = odd ? r : other;
    const uint32_t byte = live ? umma::e2m1x2_rn(lo * inv, hi * inv) : 0u;
    float q0, q1;
    umma::e2m1x2_to_f32(byte, q0, q1);
    r = __fsub_rn(r, (odd ? q1 : q0) * scl);
    if (!odd) img[t * term_stride + (lane >> 1)] = static_cast<uint8_t>(byte);
    if (lane == 0) sc[t * sc_stride] = static_cast<uint8_t>(live ? 127 + e : 127);
  }
}

// ---- the kernel ------------------------------------------------------------------
// kRouted: MXFP4 experts (else the bf16 shared expert); kGateUp: gate/up with
// the SwiGLU epilogue (else down).
// Tensor maps: mA0 / mA1 A boxes (routed: 3-D [E][rows][bytes] banks; shared:
// 2-D); mB / mB80 B rows (routed: term rows, boxes of 160 / 80 rows for tiles
// of 32 / 16 routes; shared: tokens or act_s, 128-row box); mSA0 / mSA1 A
// scale tiles (3-D banks); mSB / mSB80 B scale rows (160 / 80-row boxes).
template <bool kRouted, bool kGateUp>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_kernel(Args a, const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
                   const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mB80,
                   const __grid_constant__ CUtensorMap mSA0, const __grid_constant__ CUtensorMap mSA1,
                   const __grid_constant__ CUtensorMap mSB, const __grid_constant__ CUtensorMap mSB80) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ __align__(8) uint64_t sf_full[kSfSlots];
  __shared__ __align__(8) uint64_t sc_full[2], sc_free[2], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tslot;
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  unsigned char* ring = base + a.ring_off;
  int* ts = reinterpret_cast<int*>(base + a.tab_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, S = a.stages;
  constexpr int T = kRouted ? kTerms : 1;
  constexpr uint32_t kAccStride = kRouted ? kTerms * kNtMax : kNtShared;  // columns per accumulator buffer
  constexpr uint32_t kColSf = 2 * kAccStride;                             // scale-factor ring

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < S; ++s) mbar_init(&sf_full[s], 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sc_full[i], 1);
      mbar_init(&sc_free[i], 4);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(&drain, 1);
    mbar_fence_init();
  }
  if (kRouted)
    for (int e = threadIdx.x; e <= a.E; e += kThreads) ts[e] = a.tile_start[e];
  if (warp == kMmaWarp) umma::tmem_alloc(&tslot, 512);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tbase = tslot;
  auto next_item = [&](int seq, Item& it) -> bool {
    const int i = blockIdx.x + seq * P;
    return kRouted ? routed_item(a, ts, i, it) : shared_item(a, i, it);
  };

  // ------------------------------ TMA producer ------------------------------
  if (warp == kProdWarp) {
    if (lane == 0) {
      bool ok = true;
      int it_k = 0;  // stages issued
      // the scale tiles of item q (routed), one item ahead of its k-blocks so
      // that their latency hides behind the previous item's MMAs
      auto load_scales = [&](int q, const Item& it) -> bool {
        const int sb = q & 1, n_rows = T * it.ntp;
        if (q >= 2 && !dtc::wait1(&sc_free[sb], ((q >> 1) - 1) & 1, a.status, kSiteScFree)) return false;
        unsigned char* sfa = base + a.sfa_off + sb * a.sfa_bytes;
        unsigned char* sfb = base + a.sfb_off + sb * a.sfb_bytes;
        mbar_arrive_expect_tx(&sc_full[sb], static_cast<unsigned>((128 + n_rows) * a.sc_bytes));
        if (kGateUp) {
          tma_3d(sfa, &mSA0, 0, it.rb * 64, it.e, &sc_full[sb]);
          tma_3d(sfa + 64 * a.sc_bytes, &mSA1, 0, it.rb * 64, it.e, &sc_full[sb]);
        } else {
          tma_3d(sfa, &mSA0, 0, it.rb * 128, it.e, &sc_full[sb]);
        }
        dtc::tma_2d(sfb, it.ntp > 16 ? &mSB : &mSB80, 0, it.p0 * T, &sc_full[sb]);
        return true;
      };
      Item item, nitem;
      bool have = next_item(0, item);
      if (kRouted && have) ok = load_scales(0, item);
      for (int seq = 0; ok && have; ++seq) {
        const bool have_next = next_item(seq + 1, nitem);
        const int n_rows = T * item.ntp;  // B rows (MMA N)
        const bool wide = item.ntp > 16;  // routed: 160-row boxes, else 80
        // bytes of B: the routed rows, or the shared expert's whole 128-row box
        // (rows past the last token are zero-filled and still counted)
        const unsigned bytes = static_cast<unsigned>(kABytes + (kRouted ? n_rows : kNtShared) * 128);
        for (int kb = 0; kb < a.kb_count; ++kb, ++it_k) {
          const int s = it_k % S;
          if (it_k >= S) ok = dtc::wait1(&empty[s], ((it_k / S) - 1) & 1, a.status, kSiteEmpty);
          if (!ok) break;
          unsigned char* st = ring + s * a.stage_bytes;
          unsigned char* bt = st + a.b_off;
          mbar_arrive_expect_tx(&full[s], bytes);
          const int x = kb * 128;
          if (kRouted && kGateUp) {
            tma_3d(st, &mA0, x, item.rb * 64, item.e, &full[s]);
            tma_3d(st + 8192, &mA1, x, item.rb * 64, item.e, &full[s]);
          } else if (kRouted) {
            tma_3d(st, &mA0, x, item.rb * 128, item.e, &full[s]);
          } else if (kGateUp) {
            dtc::tma_2d(st, &mA0, x, item.rb * 64, &full[s]);
            dtc::tma_2d(st + 8192, &mA1, x, item.rb * 64, &full[s]);
          } else {
            dtc::tma_2d(st, &mA0, x, item.rb * 128, &full[s]);
          }
          if (kRouted) dtc::tma_2d(bt, wide ? &mB : &mB80, x, item.p0 * T, &full[s]);
          else dtc::tma_2d(bt, &mB, x, item.p0, &full[s]);
          if (kRouted && have_next && kb == min(1, a.kb_count - 1)) ok = load_scales(seq + 1, nitem);
          if (!ok) break;
        }
        item = nitem;
        have = have_next;
      }
      if (!ok) {  // let the copies in flight land before the CTA leaves
        for (int q = (it_k > S ? it_k - S : 0); q < it_k; ++q)
          dtc::wait1(&full[q % S], (q / S) & 1, a.status, kSiteFull);
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
      for (int seq = 0; ok && next_item(seq, item); ++seq) {
        const int ab = seq & 1;
        if (seq >= 2) ok = dtc::wait1(&acc_empty[ab], ((seq >> 1) - 1) & 1, a.status, kSiteAccEmpty);
        if (!ok) break;
        umma::fence_after_sync();
        const int n = T * item.ntp;
        const uint32_t acc = tbase + ab * kAccStride;
        const uint32_t idesc = kRouted ? umma::idesc_mxf4(128, n) : umma::idesc_bf16(128, n);
        for (int kb = 0; kb < a.kb_count && ok; ++kb, ++it_k) {
          const int s = it_k % S;
          ok = dtc::wait1(&full[s], (it_k / S) & 1, a.status, kSiteFull);
          if (!ok) break;
          const int sl = s;  // the scale-factor slot of a k-block is its ring stage
          if (kRouted) {
            ok = dtc::wait1(&sf_full[sl], (it_k / S) & 1, a.status, kSiteSfFull);
            if (!ok) break;
          }
          umma::fence_after_sync();
          unsigned char* st = ring + s * a.stage_bytes;
          const uint64_t da = umma::desc_sw128(smem_u32(st)), db = umma::desc_sw128(smem_u32(st + a.b_off));
          const uint32_t sfa = tbase + kColSf + sl * kSfSlotCols, sfb = sfa + kSfaCols;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const bool accum = kb > 0 || m > 0;
            if (kRouted)
              umma::mma_mxf4(acc, da + 2 * m, db + 2 * m, idesc | umma::idesc_sf_ids(2 * (m & 1)), sfa + 4 * (m >> 1),
                             sfb + 8 * (m >> 1), accum);
            else
              umma::mma_bf16(acc, da + 2 * m, db + 2 * m, idesc, accum);
          }
          // one commit frees the stage and (for the scale-factor warps, who
          // wait on the same barrier) the scale-factor slot of this k-block
          umma::commit(&empty[s]);
        }
        if (ok) umma::commit(&acc_full[ab]);
      }
      umma::commit(&drain);  // every MMA issued above has finished once this arrives
      dtc::wait1(&drain, 0, a.status, kSiteDrain);
    }
    __syncwarp();
  }
  // ------------------------------ scale factors -----------------------------
  else if (warp < kEpiWarp0) {
    if (kRouted) {
      const uint32_t lanes = tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      bool ok = true;
      int it_sf = 0;
      Item item;
      for (int seq = 0; ok && next_item(seq, item); ++seq) {
        const int sb = seq & 1;
        ok = dtc::wait_warp1(&sc_full[sb], (seq >> 1) & 1, a.status, kSiteScFull);
        if (!ok) break;
        const int n_rows = T * item.ntp;
        const unsigned char* sfa = base + a.sfa_off + sb * a.sfa_bytes;
        const unsigned char* sfb = base + a.sfb_off + sb * a.sfb_bytes;
        for (int kb = 0; kb < a.kb_count; ++kb, ++it_sf) {
          const int sl = it_sf % S;  // slot = ring stage of this k-block
          // MMA pair j (MMAs 2j, 2j+1 of this k-block) reads scale word j of each
          // row: A row 32q + lane in column 4j + q, B row 32q + lane in column 8j + q.
          // The words are read from shared memory before waiting for the slot.
          uint32_t va[8], vb[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint2 w = *reinterpret_cast<const uint2*>(sfa + sc_off(32 * q + lane, kb * 8, a.sc_bytes, a.sc_swz));
            va[q] = w.x;
            va[4 + q] = w.y;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int row = 32 * q + lane;
            uint2 w = make_uint2(0x7F7F7F7Fu, 0x7F7F7F7Fu);
            if (row < n_rows) w = *reinterpret_cast<const uint2*>(sfb + sc_off(row, kb * 8, a.sc_bytes, a.sc_swz));
            vb[q] = w.x;
            vb[8 + q] = w.y;
          }
          // slot sl was last used by k-block it_sf - S, whose MMAs' completion
          // frees the ring stage too (empty[sl], the producer's wait); the
          // barrier cannot pass that phase twice before this slot is refilled,
          // since k-block it_sf needs this slot
          if (it_sf >= S) ok = dtc::wait_warp1(&empty[sl], ((it_sf / S) - 1) & 1, a.status, kSiteSfEmpty);
          if (!ok) break;
          const uint32_t col = kColSf + sl * kSfSlotCols;
          umma::st_32x32b_x8(lanes + col, va);
          umma::st_32x32b_x16(lanes + col + kSfaCols, vb);
          umma::wait_st();
          umma::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sf_full[sl]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sc_free[sb]);
      }
    }
  }
  // ------------------------------ epilogue ----------------------------------
  else if (warp < kMathWarp0 || kGateUp) {
    const bool tm = warp < kMathWarp0;  // reads the accumulator (else: SwiGLU / split helper)
    const int sp = warp & 3;            // tensor-memory lanes 32 sp .. 32 sp + 31
    const int mw = warp - kEpiWarp0;    // 0..7 among the gate/up epilogue warps
    const int nbar = kGateUp ? 32 * kMathWarps : 128;
    const uint32_t lanes = tbase + (static_cast<uint32_t>(sp * 32) << 16);
    uint16_t* xch = reinterpret_cast<uint16_t*>(base + a.xch_off);  // [4][ntp max][32]
    const int xrows = kRouted ? kNtMax : kNtShared;
    bool ok = true;
    Item item;
    for (int seq = 0; ok && next_item(seq, item); ++seq) {
      const int ab = seq & 1;
      if (tm) ok = dtc::wait_warp1(&acc_full[ab], (seq >> 1) & 1, a.status, kSiteAccFull);
      ok = named_and(kEpiBar, nbar, ok);  // the epilogue warps leave together
      if (!ok) break;
      if (tm) {
        umma::fence_after_sync();
        const uint32_t acc = lanes + ab * kAccStride;
        // accumulator column of (route i, term t) = i * T + t: 16 routes are 16 T
        // consecutive columns, read as T loads of 16 columns
        for (int c0 = 0; c0 < item.ntp; c0 += 16) {
          float s[16];
          {
            uint32_t v[16 * T];
  #pragma unroll
            for (int q = 0; q < T; ++q) {
              uint32_t (&vq)[16] = *reinterpret_cast<uint32_t(*)[16]>(v + 16 * q);
              umma::ld_32x32b_x16_nowait(acc + c0 * T + 16 * q, vq);
            }
            umma::wait_ld();
  #pragma unroll
            for (int i = 0; i < 16; ++i) {
              float t0 = __uint_as_float(v[i * T]);
  #pragma unroll
              for (int t = 1; t < T; ++t) t0 = __fadd_rn(t0, __uint_as_float(v[i * T + t]));
              s[i] = t0;
            }
          }
          if (kGateUp) {
  #pragma unroll
            for (int i = 0; i < 16; ++i) xch[(sp * xrows + c0 + i) * 32 + lane] = f32_to_bf16(s[i]);
          } else {
            // down: output rows d0 + 32 sp + lane of routes / tokens c0 .. c0 + 15
            const int row = item.rb * 128 + sp * 32 + lane;
            int my_slot = 0;  // lane i < 16: the route slot of route c0 + i
            if (kRouted && lane < 16 && c0 + lane < item.nt) my_slot = __ldg(a.perm + item.p0 + c0 + lane);
  #pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int slot = __shfl_sync(0xffffffffu, my_slot, i);
              if (c0 + i < item.nt) {
                if (kRouted) {
                  a.y[static_cast<size_t>(slot) * a.d + row] = f32_to_bf16(s[i]);
                } else {
                  a.ys[static_cast<size_t>(item.p0 + c0 + i) * a.d + row] = f32_to_bf16(s[i]);
                }
              }
            }
          }
        }
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
      }  // tm
      if (kGateUp) {
        named_sync(kEpiBar, nbar);
        // warp mw: columns f0 + 32 h + lane (h = mw & 1), routes / tokens i with
        // i % 4 == mw >> 1
        const int h = mw & 1, f = item.rb * 64 + 32 * h + lane;
        for (int i = mw >> 1; i < item.nt; i += kMathWarps / 2) {
          const float g = bf16_to_f32(xch[(h * xrows + i) * 32 + lane]);
          const float u = bf16_to_f32(xch[((2 + h) * xrows + i) * 32 + lane]);
          const uint16_t act = swiglu_bf16(g, u, a.limit);
          if (kRouted) {
            const size_t row0 = static_cast<size_t>(item.p0 + i) * kTerms;  // term rows of this route
            uint8_t* img = a.act_terms + row0 * (a.F / 2) + (item.rb * 64 + 32 * h) / 2;
            uint8_t* sc = a.act_tsc + row0 * (a.F / 32) + item.rb * 2 + h;
            split_warp_write(bf16_to_f32(act), lane, kTerms, img, a.F / 2, sc, a.F / 32);
          } else {
            a.act_s[static_cast<size_t>(item.p0 + i) * a.Fs + f] = act;
          }
        }
        named_sync(kEpiBar, nbar);  // xch is rewritten by the next item
      }
    }
  }
  __syncwarp();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) umma::tmem_dealloc(tbase, 512);
}

}  // namespace gtc
}  // namespace lg
