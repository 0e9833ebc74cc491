// Kernels of the GLM MoE block for sm_100a.
//
//   router_logits_kernel   x @ W_r^T in the canonical fp32 order     moe.py:37-38
//   router_select_kernel   sigmoid, bias, group top-2, top-k, norm   moe.py:39-62
//   dispatch_kernel        counts / offsets / stable permutation     (build contract)
//   grouped_gemv_kernel    MXFP4 or bf16 expert rows x routed tokens expert_ssd.py:172-188
//   combine_kernel         weighted top-k sum + shared add           moe.py:199-201
#pragma once
#include "common.cuh"
#include "umma.cuh"

namespace lg {

// --------------------------------------------------------------------------
// Router logits: one warp owns TEW experts x TM tokens.  Lane l accumulates
// the 8-element chunks c = l, l+32, ... in increasing element order with
// fma, then a 16/8/4/2/1 xor butterfly adds the 32 partials.  This is the
// summation order the CPU checker restates.
template <int TM, int TEW>
__global__ void __launch_bounds__(256)
router_logits_kernel(const uint16_t* __restrict__ x, const float* __restrict__ W,
                     int M, int d, int E, float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * TM;
  const int e0 = (blockIdx.y * 8 + warp) * TEW;
  if (e0 >= E) return;
  float acc[TM][TEW];
#pragma unroll
  for (int a = 0; a < TM; ++a)
#pragma unroll
    for (int b = 0; b < TEW; ++b) acc[a][b] = 0.0f;
  const int chunks = d >> 3;
  for (int c = lane; c < chunks; c += 32) {
    float xv[TM][8];
#pragma unroll
    for (int a = 0; a < TM; ++a) {
      const int t = t0 + a;
      if (t < M) {
        uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * d + 8 * c);
        xv[a][0] = bf16lo(u.x); xv[a][1] = bf16hi(u.x);
        xv[a][2] = bf16lo(u.y); xv[a][3] = bf16hi(u.y);
        xv[a][4] = bf16lo(u.z); xv[a][5] = bf16hi(u.z);
        xv[a][6] = bf16lo(u.w); xv[a][7] = bf16hi(u.w);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) xv[a][q] = 0.0f;
      }
    }
#pragma unroll
    for (int b = 0; b < TEW; ++b) {
      const int e = e0 + b;
      if (e < E) {
        const float4* wp = reinterpret_cast<const float4*>(W + static_cast<size_t>(e) * d + 8 * c);
        float4 w0 = wp[0], w1 = wp[1];
        float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int a = 0; a < TM; ++a)
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[a][b] = __fmaf_rn(xv[a][q], wv[q], acc[a][b]);
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TEW; ++b)
        acc[a][b] = __fadd_rn(acc[a][b], __shfl_xor_sync(0xffffffffu, acc[a][b], off));
  if (lane == 0) {
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TEW; ++b) {
        const int t = t0 + a, e = e0 + b;
        if (t < M && e < E) logits[static_cast<size_t>(t) * E + e] = acc[a][b];
      }
  }
}

// --------------------------------------------------------------------------
// Router logits for many tokens, same arithmetic as router_logits_kernel
// (lane l sums the 8-element chunks c = l, l + 32, ... in increasing order with
// fma, then the 16/8/4/2/1 xor butterfly), with the operands staged through
// shared memory: a block owns 8 * TW tokens x EW experts and walks d in
// k-blocks of 256 elements (32 chunks, one per lane), so every staged x and
// W_r element serves all the block's pairs instead of being re-read from L2
// per warp.  Warp w owns tokens t0 + TW w .. + TW - 1 and all EW experts.
// W_r is staged as [expert][half][lane] float4 (lane l's chunk in two
// consecutive-lane rows), so a warp's reads touch 32 consecutive 16-byte words.
// d must be a multiple of 256.
constexpr int kRlExperts = 16;
template <int TW, int EW = kRlExperts>
__global__ void __launch_bounds__(256)
router_logits_tiled_kernel(const uint16_t* __restrict__ x, const float* __restrict__ W,
                           int M, int d, int E, float* __restrict__ logits) {
  constexpr int TB = 8 * TW;  // tokens per block
  __shared__ __align__(16) uint16_t xs[TB * 256];
  __shared__ __align__(16) float4 ws[EW * 64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * TB, e0 = blockIdx.y * EW;
  float acc[TW][EW];
#pragma unroll
  for (int a = 0; a < TW; ++a)
#pragma unroll
    for (int b = 0; b < EW; ++b) acc[a][b] = 0.0f;
  // the next k-block's share of this thread, loaded while the current one is
  // multiplied: TB * 32 uint4 of x and EW * 64 float4 of W_r over 256 threads
  constexpr int XV = (TB * 32 + 255) / 256, WV = (EW * 64 + 255) / 256;
  uint4 xr[XV];
  float4 wr[WV];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = threadIdx.x + 256 * u, r = i >> 5, c = i & 31, t = t0 + r;
      xr[u] = (i < TB * 32 && t < M) ? *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * d + k0 + 8 * c)
                                     : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < WV; ++u) {
      const int i = threadIdx.x + 256 * u, r = i >> 6, c = i & 63, e = e0 + r;
      wr[u] = (i < EW * 64 && e < E) ? *reinterpret_cast<const float4*>(W + static_cast<size_t>(e) * d + k0 + 4 * c)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  fetch(0);
  for (int k0 = 0; k0 < d; k0 += 256) {
    __syncthreads();  // the previous k-block's operands are consumed
#pragma unroll
    for (int u = 0; u < XV; ++u) {
      const int i = threadIdx.x + 256 * u;
      if (i < TB * 32) reinterpret_cast<uint4*>(xs)[i] = xr[u];
    }
#pragma unroll
    for (int u = 0; u < WV; ++u) {
      const int i = threadIdx.x + 256 * u;  // expert i / 64, float4 c = i % 64 = lane c / 2, half c % 2
      if (i < EW * 64) ws[(i >> 6) * 64 + (i & 1) * 32 + ((i & 63) >> 1)] = wr[u];
    }
    __syncthreads();
    if (k0 + 256 < d) fetch(k0 + 256);
    // lane l: chunk c = k0 / 8 + l (elements 8 l .. 8 l + 7 of this k-block)
    float xv[TW][8];
#pragma unroll
    for (int a = 0; a < TW; ++a) {
      const uint4 u = reinterpret_cast<const uint4*>(xs)[(warp * TW + a) * 32 + lane];
      xv[a][0] = bf16lo(u.x); xv[a][1] = bf16hi(u.x);
      xv[a][2] = bf16lo(u.y); xv[a][3] = bf16hi(u.y);
      xv[a][4] = bf16lo(u.z); xv[a][5] = bf16hi(u.z);
      xv[a][6] = bf16lo(u.w); xv[a][7] = bf16hi(u.w);
    }
#pragma unroll
    for (int b = 0; b < EW; ++b) {
      const float4 w0 = ws[b * 64 + lane];
      const float4 w1 = ws[b * 64 + 32 + lane];
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int a = 0; a < TW; ++a)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[a][b] = __fmaf_rn(xv[a][q], wv[q], acc[a][b]);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
    for (int a = 0; a < TW; ++a)
#pragma unroll
      for (int b = 0; b < EW; ++b)
        acc[a][b] = __fadd_rn(acc[a][b], __shfl_xor_sync(0xffffffffu, acc[a][b], off));
  // lane b < EW writes expert e0 + b of the warp's tokens
#pragma unroll
  for (int a = 0; a < TW; ++a) {
    const int t = t0 + warp * TW + a;
    float v = 0.f;
#pragma unroll
    for (int b = 0; b < EW; ++b) v = lane == b ? acc[a][b] : v;
    if (t < M && lane < EW && e0 + lane < E) logits[static_cast<size_t>(t) * E + e0 + lane] = v;
  }
}

// --------------------------------------------------------------------------
// router_logits_tiled_kernel's arithmetic (same lanes, chunks, fma order and
// butterfly, so the logits are bit-identical) with the operands streamed into
// an ST-stage shared-memory ring by cp.async instead of through registers:
// no prefetch registers and no load latency between the k-block barriers, so
// two CTAs fit per SM.  Stage layout: x [TB][32] uint4, then W_r as
// [expert][half][lane] float4.  d must be a multiple of 256; x and W_r 16-byte
// aligned.
template <int TW, int EW, int ST>
__global__ void __launch_bounds__(256, 2)
router_logits_pipe_kernel(const uint16_t* __restrict__ x, const float* __restrict__ W,
                          int M, int d, int E, float* __restrict__ logits) {
  constexpr int TB = 8 * TW;
  constexpr int XB = TB * 512;           // x bytes per stage
  constexpr int SB = XB + EW * 1024;     // stage bytes
  extern __shared__ __align__(16) unsigned char rl_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * TB, e0 = blockIdx.y * EW;
  const int nk = d / 256;
  auto issue = [&](int kb, int st) {
    const int k0 = kb * 256;
    unsigned char* base = rl_smem + st * SB;
#pragma unroll
    for (int u = 0; u < (TB * 32 + 255) / 256; ++u) {
      const int i = threadIdx.x + 256 * u;
      if (i < TB * 32) {
        const int r = i >> 5, c = i & 31, t = t0 + r;
        const uint16_t* src = x + static_cast<size_t>(t < M ? t : 0) * d + k0 + 8 * c;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(base + 16 * i)), "l"(src),
                     "r"(t < M ? 16 : 0)
                     : "memory");
      }
    }
#pragma unroll
    for (int u = 0; u < (EW * 64 + 255) / 256; ++u) {
      const int i = threadIdx.x + 256 * u;
      if (i < EW * 64) {
        const int r = i >> 6, c = i & 63, e = e0 + r;
        const float* src = W + static_cast<size_t>(e < E ? e : 0) * d + k0 + 4 * c;
        const int slot = r * 64 + (i & 1) * 32 + ((i & 63) >> 1);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(base + XB + 16 * slot)),
                     "l"(src), "r"(e < E ? 16 : 0)
                     : "memory");
      }
    }
  };
  float acc[TW][EW];
#pragma unroll
  for (int a = 0; a < TW; ++a)
#pragma unroll
    for (int b = 0; b < EW; ++b) acc[a][b] = 0.0f;
#pragma unroll
  for (int st = 0; st < ST - 1; ++st) {
    if (st < nk) issue(st, st);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int kb = 0; kb < nk; ++kb) {
    asm volatile("cp.async.wait_group %0;" ::"n"(ST - 2) : "memory");
    __syncthreads();  // k-block kb is in place; every warp is done with kb - 1
    if (kb + ST - 1 < nk) issue(kb + ST - 1, (kb + ST - 1) % ST);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const unsigned char* base = rl_smem + (kb % ST) * SB;
    const uint4* xs = reinterpret_cast<const uint4*>(base);
    const float4* ws = reinterpret_cast<const float4*>(base + XB);
    // lane l: chunk c = kb * 32 + l (elements 8 l .. 8 l + 7 of this k-block)
    float xv[TW][8];
#pragma unroll
    for (int a = 0; a < TW; ++a) {
      const uint4 u = xs[(warp * TW + a) * 32 + lane];
      xv[a][0] = bf16lo(u.x); xv[a][1] = bf16hi(u.x);
      xv[a][2] = bf16lo(u.y); xv[a][3] = bf16hi(u.y);
      xv[a][4] = bf16lo(u.z); xv[a][5] = bf16hi(u.z);
      xv[a][6] = bf16lo(u.w); xv[a][7] = bf16hi(u.w);
    }
#pragma unroll
    for (int b = 0; b < EW; ++b) {
      const float4 w0 = ws[b * 64 + lane];
      const float4 w1 = ws[b * 64 + 32 + lane];
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int a = 0; a < TW; ++a)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[a][b] = __fmaf_rn(xv[a][q], wv[q], acc[a][b]);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
    for (int a = 0; a < TW; ++a)
#pragma unroll
      for (int b = 0; b < EW; ++b)
        acc[a][b] = __fadd_rn(acc[a][b], __shfl_xor_sync(0xffffffffu, acc[a][b], off));
#pragma unroll
  for (int a = 0; a < TW; ++a) {
    const int t = t0 + warp * TW + a;
    float v = 0.f;
#pragma unroll
    for (int b = 0; b < EW; ++b) v = lane == b ? acc[a][b] : v;
    if (t < M && lane < EW && e0 + lane < E) logits[static_cast<size_t>(t) * E + e0 + lane] = v;
  }
}

// --------------------------------------------------------------------------
// Router selection: one warp per token.  E <= 1024 (32 experts per lane).
// Shared memory per warp: scores[E], choice[E], gscore[G].
constexpr int kSelectWarps = 4;
__global__ void __launch_bounds__(kSelectWarps * 32)
router_select_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                     int M, int E, int G, int g, int k, int norm, float scale,
                     float* __restrict__ weights, uint32_t* __restrict__ indices,
                     int* __restrict__ counts) {
  extern __shared__ float sm[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = blockIdx.x * kSelectWarps + warp;
  if (t >= M) return;
  float* sc = sm + warp * (2 * E + G);
  float* ch = sc + E;
  float* gs = ch + E;
  for (int e = lane; e < E; e += 32) {
    float s = own_sigmoidf(logits[static_cast<size_t>(t) * E + e]);
    sc[e] = s;
    ch[e] = __fadd_rn(s, bias[e]);
  }
  __syncwarp();
  const int per = E / G;
  for (int gi = lane; gi < G; gi += 32) {
    int b1 = -1, b2 = -1;
    float v1 = 0.f, v2 = 0.f;
    for (int j = 0; j < per; ++j) {
      const int e = gi * per + j;
      const float v = ch[e];
      if (after(v, e, v1, b1)) { b2 = b1; v2 = v1; b1 = e; v1 = v; }
      else if (after(v, e, v2, b2)) { b2 = e; v2 = v; }
    }
    gs[gi] = __fadd_rn(v2, v1);
  }
  __syncwarp();
  // topk_group best groups; lane owns groups lane + 32u (G <= 1024)
  uint32_t gtaken = 0u;
  for (int s = 0; s < g; ++s) {
    float bv = 0.f; int bi = -1;
    for (int u = 0; lane + 32 * u < G; ++u) {
      const int gi = lane + 32 * u;
      if (!((gtaken >> u) & 1u) && after(gs[gi], gi, bv, bi)) { bv = gs[gi]; bi = gi; }
    }
    warp_best(bv, bi);
    if ((bi & 31) == lane) gtaken |= 1u << (bi >> 5);
  }
  // broadcast the group mask through shared memory (reuse gs as flags)
  __syncwarp();
  for (int u = 0; lane + 32 * u < G; ++u) gs[lane + 32 * u] = ((gtaken >> u) & 1u) ? 1.f : 0.f;
  __syncwarp();
  const float ninf = __uint_as_float(0xff800000u);
  for (int e = lane; e < E; e += 32)
    if (gs[e / per] == 0.f) ch[e] = ninf;
  __syncwarp();
  uint32_t taken = 0u;
  int mine = -1;  // lane j < k keeps the expert of output slot j
  for (int s = 0; s < k; ++s) {
    float bv = 0.f; int bi = -1;
    for (int u = 0; lane + 32 * u < E; ++u) {
      const int e = lane + 32 * u;
      if (!((taken >> u) & 1u) && after(ch[e], e, bv, bi)) { bv = ch[e]; bi = e; }
    }
    warp_best(bv, bi);
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == k - 1 - s) mine = bi;
  }
  // weights: sequential sum in output order (lane 0), then each lane j < k
  float wj = (lane < k) ? sc[mine] : 0.f;
  float denom = 0.f;
  if (norm) {
    float sum = __shfl_sync(0xffffffffu, wj, 0);
    for (int j = 1; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wj, j));
    denom = __fadd_rn(sum, 0x1.79ca1p-67f);  // float32(1e-20)
  }
  if (lane < k) {
    float w = norm ? __fdiv_rn(wj, denom) : wj;
    w = __fmul_rn(w, scale);
    weights[static_cast<size_t>(t) * k + lane] = w;
    indices[static_cast<size_t>(t) * k + lane] = static_cast<uint32_t>(mine);
    if (counts) atomicAdd(counts + mine, 1);
  }
}

// --------------------------------------------------------------------------
// Dispatch: block e scans all route slots and writes, in slot order, the
// slots routed to expert e (stable counting sort).  It also writes offsets[e]
// and the compact list of active experts: active[0] = #experts with routes,
// active[1 + r] = r-th such expert in increasing id.
__global__ void __launch_bounds__(256)
dispatch_kernel(const uint32_t* __restrict__ idx, int S, int E,
                const int* __restrict__ counts, int* __restrict__ offsets,
                int* __restrict__ perm, int* __restrict__ active) {
  __shared__ int red[2][8];
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int start = 0, nz = 0;
  for (int j = threadIdx.x; j < e; j += 256) {
    const int c = counts[j];
    start += c;
    nz += c > 0;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    start += __shfl_xor_sync(0xffffffffu, start, off);
    nz += __shfl_xor_sync(0xffffffffu, nz, off);
  }
  if (lane == 0) { red[0][warp] = start; red[1][warp] = nz; }
  __syncthreads();
  start = 0; nz = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) { start += red[0][w]; nz += red[1][w]; }
  const int cnt = counts[e];
  if (threadIdx.x == 0) {
    offsets[e] = start;
    if (e == E - 1) { offsets[E] = start + cnt; active[0] = nz + (cnt > 0); }
    if (cnt > 0) active[1 + nz] = e;
  }
  if (cnt == 0) return;
  // slots in blocks of 1024 (four 256-slot rows, thread t holds slot 256 j + t
  // of row j): one ballot per row and warp, one barrier pair per block
  __shared__ int rsum[2][4][8];
  int base = start, par = 0;
  for (int s0 = 0; s0 < S; s0 += 1024, par ^= 1) {
    bool f[4];
    unsigned b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + 256 * j + threadIdx.x;
      f[j] = s < S && __ldg(idx + s) == static_cast<uint32_t>(e);
      b[j] = __ballot_sync(0xffffffffu, f[j]);
      if (lane == 0) rsum[par][j][warp] = __popc(b[j]);
    }
    __syncthreads();  // rsum[par] complete; rsum[par ^ 1] was read before the previous barrier
    int tot = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int rpre = 0, rtot = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const int v = rsum[par][j][w];
        rpre += (w < warp) ? v : 0;
        rtot += v;
      }
      if (f[j]) perm[base + tot + rpre + __popc(b[j] & ((1u << lane) - 1u))] = s0 + 256 * j + threadIdx.x;
      tot += rtot;
    }
    base += tot;
    if (base - start >= cnt) break;  // every thread sees the same tot
  }
}

// --------------------------------------------------------------------------
// Grouped GEMV over (expert, row block) work items.
//
// Work items 0 .. n_active*nrb-1 are routed: expert e = active[1 + item/nrb],
// rows rb*ROWS .. +ROWS of its weight matrix, against the rows of the
// routes offsets[e] .. offsets[e+1]-1 (in permuted order).  The remaining
// nrb_s items are shared-expert row blocks against all M tokens.
//
// A "slot" of LPR lanes owns one weight row; lane `sub` of the slot owns
// the 32-column groups c = sub, sub + LPR, ...: one 16-byte load of packed
// E2M1 nibbles plus one E8M0 scale byte per group (64 bytes for bf16 rows).
// Token rows are staged in shared memory as f32 in a lane-interleaved
// layout so that the LPR lanes read consecutive float4s.
struct GemvArgs {
  int K, N;          // routed: reduction length, rows per expert
  int Ks, Ns;        // shared: reduction length, rows (Ns = 0: no shared)
  int k;             // routes per token
  int M;             // tokens
  int pair;          // 1: gate+up with SwiGLU epilogue; 0: single matrix
  float limit;
  const uint8_t *a_packed, *a_scale, *b_packed, *b_scale;
  long long a_pstride, a_sstride, b_pstride, b_sstride;
  const uint16_t *sa, *sb;  // shared weights bf16 [Ns, Ks]
  const uint16_t* xin;      // routed input rows
  int xin_by_token;         // 1: row = perm[p] / k (token rows); 0: row = p
  const uint16_t* xin_s;    // shared input rows [M, Ks]
  const int *offsets, *perm, *active;
  uint16_t* out;            // routed output [*, N]
  int out_by_slot;          // 1: row = perm[p]; 0: row = p
  uint16_t* out_s;          // shared output [M, Ns]
};

template <int LPR, int TT>
__global__ void __launch_bounds__(256)
grouped_gemv_kernel(GemvArgs a) {
  extern __shared__ float4 xs[];
  constexpr int SLOTS = 32 / LPR;
  constexpr int ROWS = 8 * SLOTS;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = lane & (LPR - 1);
  const int slot = lane / LPR;
  const int n_active = a.active[0];
  const int nrb = (a.N + ROWS - 1) / ROWS;
  const int nrb_s = (a.Ns + ROWS - 1) / ROWS;
  const long long n_routed = static_cast<long long>(n_active) * nrb;
  const long long total = n_routed + nrb_s;
  for (long long w = blockIdx.x; w < total; w += gridDim.x) {
    const bool sh = w >= n_routed;
    int e = 0, rb, r0, nr, K, N;
    if (!sh) {
      const int u = static_cast<int>(w / nrb);
      rb = static_cast<int>(w - static_cast<long long>(u) * nrb);
      e = a.active[1 + u];
      r0 = a.offsets[e];
      nr = a.offsets[e + 1] - r0;
      K = a.K; N = a.N;
    } else {
      rb = static_cast<int>(w - n_routed);
      r0 = 0; nr = a.M;
      K = a.Ks; N = a.Ns;
    }
    const int G = K >> 5;
    const int KI = (G + LPR - 1) / LPR;
    const int row = rb * ROWS + warp * SLOTS + slot;
    const bool valid = row < N;
    const int rr = valid ? row : 0;
    for (int c0 = 0; c0 < nr; c0 += TT) {
      const int nt = min(TT, nr - c0);
      __syncthreads();
      for (int i4 = threadIdx.x; i4 < nt * G * 8; i4 += blockDim.x) {
        const int t = i4 / (G * 8);
        const int rem = i4 - t * G * 8;
        const int c = rem >> 3, q4 = rem & 7;
        const uint16_t* src;
        if (!sh) {
          const int p = r0 + c0 + t;
          const int srow = a.xin_by_token ? a.perm[p] / a.k : p;
          src = a.xin + static_cast<size_t>(srow) * K;
        } else {
          src = a.xin_s + static_cast<size_t>(c0 + t) * K;
        }
        const uint2 u = *reinterpret_cast<const uint2*>(src + 32 * c + 4 * q4);
        xs[((t * KI + c / LPR) * 8 + q4) * LPR + (c & (LPR - 1))] =
            make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
      }
      __syncthreads();
      float acc_a[TT], acc_b[TT];
#pragma unroll
      for (int t = 0; t < TT; ++t) { acc_a[t] = 0.f; acc_b[t] = 0.f; }
      for (int i = 0; i < KI; ++i) {
        const int c = sub + LPR * i;
        if (c >= G) break;
        if (!sh) {
          const size_t poff = static_cast<size_t>(rr) * (K >> 1) + 16 * c;
          const size_t soff = static_cast<size_t>(rr) * G + c;
          const uint4 pa = ldg_nc_v4(a.a_packed + e * a.a_pstride + poff);
          const float sa = e8m0_to_f32(a.a_scale[e * a.a_sstride + soff]);
          uint4 pb = make_uint4(0, 0, 0, 0);
          float sb = 0.f;
          if (a.pair) {
            pb = ldg_nc_v4(a.b_packed + e * a.b_pstride + poff);
            sb = e8m0_to_f32(a.b_scale[e * a.b_sstride + soff]);
          }
          float ga[TT], gb[TT];
#pragma unroll
          for (int t = 0; t < TT; ++t) { ga[t] = 0.f; gb[t] = 0.f; }
          const uint32_t wa4[4] = {pa.x, pa.y, pa.z, pa.w};
          const uint32_t wb4[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            float va[8], vb[8];
            e2m1x8_to_f32(wa4[wd], va);
            if (a.pair) e2m1x8_to_f32(wb4[wd], vb);
#pragma unroll
            for (int t = 0; t < TT; ++t) {
              if (t < nt) {
                const float4 x0 = xs[((t * KI + i) * 8 + 2 * wd) * LPR + sub];
                const float4 x1 = xs[((t * KI + i) * 8 + 2 * wd + 1) * LPR + sub];
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int q = 0; q < 8; ++q) ga[t] = __fmaf_rn(xv[q], va[q], ga[t]);
                if (a.pair) {
#pragma unroll
                  for (int q = 0; q < 8; ++q) gb[t] = __fmaf_rn(xv[q], vb[q], gb[t]);
                }
              }
            }
          }
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            acc_a[t] = __fmaf_rn(ga[t], sa, acc_a[t]);
            acc_b[t] = __fmaf_rn(gb[t], sb, acc_b[t]);
          }
        } else {
          const uint16_t* wa = a.sa + static_cast<size_t>(rr) * K + 32 * c;
          const uint16_t* wb = a.pair ? a.sb + static_cast<size_t>(rr) * K + 32 * c : nullptr;
#pragma unroll
          for (int wd = 0; wd < 4; ++wd) {
            const uint4 ua = ldg_nc_v4(wa + 8 * wd);
            const float va[8] = {bf16lo(ua.x), bf16hi(ua.x), bf16lo(ua.y), bf16hi(ua.y),
                                 bf16lo(ua.z), bf16hi(ua.z), bf16lo(ua.w), bf16hi(ua.w)};
            float vb[8];
            if (a.pair) {
              const uint4 ub = ldg_nc_v4(wb + 8 * wd);
              vb[0] = bf16lo(ub.x); vb[1] = bf16hi(ub.x); vb[2] = bf16lo(ub.y); vb[3] = bf16hi(ub.y);
              vb[4] = bf16lo(ub.z); vb[5] = bf16hi(ub.z); vb[6] = bf16lo(ub.w); vb[7] = bf16hi(ub.w);
            }
#pragma unroll
            for (int t = 0; t < TT; ++t) {
              if (t < nt) {
                const float4 x0 = xs[((t * KI + i) * 8 + 2 * wd) * LPR + sub];
                const float4 x1 = xs[((t * KI + i) * 8 + 2 * wd + 1) * LPR + sub];
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int q = 0; q < 8; ++q) acc_a[t] = __fmaf_rn(xv[q], va[q], acc_a[t]);
                if (a.pair) {
#pragma unroll
                  for (int q = 0; q < 8; ++q) acc_b[t] = __fmaf_rn(xv[q], vb[q], acc_b[t]);
                }
              }
            }
          }
        }
      }
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1)
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          acc_a[t] = __fadd_rn(acc_a[t], __shfl_xor_sync(0xffffffffu, acc_a[t], off));
          acc_b[t] = __fadd_rn(acc_b[t], __shfl_xor_sync(0xffffffffu, acc_b[t], off));
        }
      if (valid && sub == 0) {
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          if (t < nt) {
            uint16_t v;
            if (a.pair) v = swiglu_bf16(round_bf16(acc_a[t]), round_bf16(acc_b[t]), a.limit);
            else v = f32_to_bf16(acc_a[t]);
            if (!sh) {
              const int p = r0 + c0 + t;
              const int orow = a.out_by_slot ? a.perm[p] : p;
              a.out[static_cast<size_t>(orow) * N + row] = v;
            } else {
              a.out_s[static_cast<size_t>(c0 + t) * N + row] = v;
            }
          }
        }
      }
    }
  }
}

// --------------------------------------------------------------------------
// Combine: out[t, i] = ((0 + y0*w0) + y1*w1) + ... (+ shared), products and
// sums each rounded to f32 as in the MLX graph (bf16 * f32 -> f32).  A thread
// owns 8 consecutive outputs of a token (16-byte loads of each route's row).
// rowmap (optional): y row of route slot t*k + j is rowmap[t*k + j] (rows in
// dispatch order), else the slot itself.  d % 8 == 0.
__global__ void __launch_bounds__(256)
combine_kernel(const uint16_t* __restrict__ y, const float* __restrict__ w,
               const uint16_t* __restrict__ ys, int M, int k, int d, float* __restrict__ out,
               const int* __restrict__ rowmap = nullptr) {
  const int d8 = d >> 3;
  const long long n = static_cast<long long>(M) * d8;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
    const int t = static_cast<int>(i / d8);
    const int c = static_cast<int>(i - static_cast<long long>(t) * d8);
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const float wj = __ldg(w + static_cast<size_t>(t) * k + j);
      const size_t slot = static_cast<size_t>(t) * k + j;
      const size_t row = rowmap ? static_cast<size_t>(__ldg(rowmap + slot)) : slot;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + row * d) + c);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        s[2 * q] = __fadd_rn(s[2 * q], __fmul_rn(bf16lo(uw[q]), wj));
        s[2 * q + 1] = __fadd_rn(s[2 * q + 1], __fmul_rn(bf16hi(uw[q]), wj));
      }
    }
    if (ys) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(ys + static_cast<size_t>(t) * d) + c);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        s[2 * q] = __fadd_rn(s[2 * q], bf16lo(uw[q]));
        s[2 * q + 1] = __fadd_rn(s[2 * q + 1], bf16hi(uw[q]));
      }
    }
    float4* o = reinterpret_cast<float4*>(out) + 2 * i;
    o[0] = make_float4(s[0], s[1], s[2], s[3]);
    o[1] = make_float4(s[4], s[5], s[6], s[7]);
  }
}

// --------------------------------------------------------------------------
// Expert-parallel send buffers: for dispatch position p (route slot
// perm[p] = t*k + j, slots sorted by expert id, hence by owning rank)
// x_send[p] = x[t], e_send[p] = expert id mod per_rank (local to the owner),
// inv[perm[p]] = p.  One thread per 16-byte chunk of a row; d % 8 == 0.
__global__ void __launch_bounds__(256)
ep_pack_kernel(const uint16_t* __restrict__ x, const uint32_t* __restrict__ indices, const int* __restrict__ perm,
               int R, int k, int d, int per_rank, uint16_t* __restrict__ x_send, int* __restrict__ e_send,
               int* __restrict__ inv) {
  const int per_row = d >> 3;
  const long long n = static_cast<long long>(R) * per_row;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
    const int p = static_cast<int>(i / per_row);
    const int c = static_cast<int>(i - static_cast<long long>(p) * per_row);
    const int slot = __ldg(perm + p);
    reinterpret_cast<uint4*>(x_send + static_cast<size_t>(p) * d)[c] =
        __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(slot / k) * d) + c);
    if (c == 0) {
      e_send[p] = static_cast<int>(__ldg(indices + slot) % static_cast<uint32_t>(per_rank));
      inv[slot] = p;
    }
  }
}

// --------------------------------------------------------------------------
// Block-FP8 -> bf16 (checkpoint loading of the shared expert, the resident
// plan's block_fp8_to_bf16 transform: kg36/livglm src/glm53flash/fp8.py:43-78,
// resident_plan.py:177-220).  E4M3FN: sign, 4-bit exponent (bias 7), 3-bit
// mantissa; exponent 0 is subnormal (m/8 * 2^-6); exponent 15 with mantissa 7
// is NaN; there are no infinities.
__device__ __forceinline__ float e4m3fn_to_f32(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 0u) v = static_cast<float>(m) * 0x1p-9f;
  else if (e == 15u && m == 7u) v = __uint_as_float(0x7FC00000u);
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return (b & 0x80u) ? -v : v;
}
// out[r][c] = bf16(e4m3fn(w[r][c]) * scale[r / B][c / B]) with the product in
// f32; *nonfinite counts the products that are not finite.  Thread per 8
// consecutive values of a row; cols % 8 == 0.
__global__ void __launch_bounds__(256)
fp8_block_dequant_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale, long long rows,
                         long long cols, int B, uint16_t* __restrict__ out, int* __restrict__ nonfinite) {
  const long long per_row = cols / 8, n = rows * per_row;
  const long long scols = cols / B;
  int bad = 0;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
    const long long r = i / per_row, c0 = (i - r * per_row) * 8;
    const uint2 q = *reinterpret_cast<const uint2*>(w + r * cols + c0);
    const float s = scale[(r / B) * scols + c0 / B];
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? q.x : q.y;
      const float v0 = __fmul_rn(e4m3fn_to_f32((word >> (16 * (j & 1))) & 0xFFu), s);
      const float v1 = __fmul_rn(e4m3fn_to_f32((word >> (16 * (j & 1) + 8)) & 0xFFu), s);
      bad += !isfinite(v0) + !isfinite(v1);
      o[j] = static_cast<uint32_t>(f32_to_bf16(v0)) | (static_cast<uint32_t>(f32_to_bf16(v1)) << 16);
    }
    *reinterpret_cast<uint4*>(out + r * cols + c0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (bad) atomicAdd(nonfinite, bad);
}

// --------------------------------------------------------------------------
// MX requantisation of a bf16 weight matrix: the resident-linear
// quantisation of kg36/livglm layers.py:67-104 (mx.quantize, group_size 32,
// mode "mxfp8" / "mxfp4") as the OCP MX rule: per 32-value group of a row the
// shared exponent X = clamp(floor(log2(amax)) - emax, -127, 127) (emax 8 for
// E4M3, 2 for E2M1; X = -127 for an all-zero group), each element the
// round-to-nearest-even of v * 2^-X in the element format, saturated to its
// largest finite value.  The output holds element * 2^X as bf16 -- exact, so
// bf16 kernels compute the quantised products.  One thread per group.
__device__ __forceinline__ float pow2_mx(int e) {  // 2^e, -127 <= e <= 127 (2^-127 is subnormal)
  return e >= -126 ? pow2i(e) : __uint_as_float(0x00400000u);
}
__device__ __forceinline__ void e4m3x2_roundtrip(float& lo, float& hi) {
  uint32_t h;
  asm("{\n\t.reg .b16 b;\n\tcvt.rn.satfinite.e4m3x2.f32 b, %1, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, b;\n\t}"
      : "=r"(h)
      : "f"(hi), "f"(lo));
  lo = __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
  hi = __half2float(__ushort_as_half(static_cast<unsigned short>(h >> 16)));
}
template <int kBits>
__global__ void __launch_bounds__(256)
mx_requantize_kernel(const uint16_t* __restrict__ w, long long groups, uint16_t* __restrict__ out) {
  constexpr int kEmax = kBits == 8 ? 8 : 2;
  for (long long g = blockIdx.x * 256LL + threadIdx.x; g < groups; g += 256LL * gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(w + g * 32);
    uint32_t u[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 q = src[i];
      u[4 * i] = q.x; u[4 * i + 1] = q.y; u[4 * i + 2] = q.z; u[4 * i + 3] = q.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16lo(u[i])), fabsf(bf16hi(u[i]))));
    int X = amax > 0.f ? ilogbf(amax) - kEmax : -127;
    X = X < -127 ? -127 : (X > 127 ? 127 : X);
    const float down = pow2_mx(-X), up = pow2_mx(X);
    uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float lo = __fmul_rn(bf16lo(u[i]), down), hi = __fmul_rn(bf16hi(u[i]), down);
      if (kBits == 8) {
        e4m3x2_roundtrip(lo, hi);
      } else {
        umma::e2m1x2_to_f32(umma::e2m1x2_rn(lo, hi), lo, hi);
      }
      o[i] = static_cast<uint32_t>(f32_to_bf16(__fmul_rn(lo, up))) |
             (static_cast<uint32_t>(f32_to_bf16(__fmul_rn(hi, up))) << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + g * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }
}

}  // namespace lg
