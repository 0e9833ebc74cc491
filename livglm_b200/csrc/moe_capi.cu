// C ABI of the GLM MoE block (see include/livglm_moe.h).
//
// Host-side argument validation mirrors the reference's ContractError checks
// (kg36/livglm src/glm53flash/model_config.py:142-176) plus the kernels' own
// layout requirements; nothing is launched when validation fails.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <cstdlib>
#include <utility>

#include "livglm_moe.h"
#include "decode_kernels.cuh"
#include "stream_kernels.cuh"
#include "moe_kernels.cuh"
#include "down1_kernel.cuh"
#include "down_tc.cuh"
#include "grouped_tc.cuh"
#include "grouped_dq.cuh"

#include <cudaTypedefs.h>

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(LG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return LG_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The address kernels on the current device use for a caller pointer: device
// memory of this device and managed memory as given, page-locked host memory
// (cudaHostAlloc / cudaHostRegister) through its device mapping, with *host
// set.  Pageable host memory and another device's memory are refused here
// rather than faulting in a kernel.
int resolve(const void* p, const char* what, const void** dp, bool* host) {
  cudaPointerAttributes at{};
  const cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LG_ERR_INVALID_ARG, "%s: pointer attributes: %s", what, cudaGetErrorString(e));
  }
  *host = false;
  *dp = p;
  switch (at.type) {
    case cudaMemoryTypeDevice: {
      int dev = -1;
      cudaGetDevice(&dev);
      if (at.device != dev)
        return fail(LG_ERR_INVALID_ARG, "%s: memory of device %d, but the current device is %d", what, at.device, dev);
      return LG_OK;
    }
    case cudaMemoryTypeManaged:
      return LG_OK;
    case cudaMemoryTypeHost:
      if (!at.devicePointer)
        return fail(LG_ERR_INVALID_ARG, "%s: page-locked host memory not mapped for the current device", what);
      *dp = at.devicePointer;
      *host = true;
      return LG_OK;
    default:
      return fail(LG_ERR_INVALID_ARG, "%s: pageable host memory; pass device or page-locked host memory", what);
  }
}

constexpr size_t kAlign = 256;
size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int validate_cfg(const lg_moe_config* c) {
  if (!c) return fail(LG_ERR_INVALID_ARG, "config is NULL");
  const int d = c->hidden_size, F = c->moe_intermediate_size, E = c->n_routed_experts;
  const int k = c->num_experts_per_tok, G = c->n_group, g = c->topk_group;
  if (d < 32 || d % 32) return fail(LG_ERR_INVALID_ARG, "hidden_size %d must be a positive multiple of 32", d);
  if (F < 32 || F % 32) return fail(LG_ERR_INVALID_ARG, "moe_intermediate_size %d must be a positive multiple of 32", F);
  if (E < 2 || E > 1024) return fail(LG_ERR_UNSUPPORTED, "n_routed_experts %d outside 2..1024", E);
  if (k < 1 || k > E) return fail(LG_ERR_INVALID_ARG, "invalid routed top-k geometry: k=%d E=%d", k, E);
  if (k > 32) return fail(LG_ERR_UNSUPPORTED, "num_experts_per_tok %d > 32", k);
  if (G < 1 || E % G) return fail(LG_ERR_INVALID_ARG, "expert count must be divisible by n_group (%d %% %d)", E, G);
  if (g < 1 || g > G) return fail(LG_ERR_INVALID_ARG, "invalid topk_group %d for n_group %d", g, G);
  if (E / G < 2) return fail(LG_ERR_INVALID_ARG, "router groups must contain at least two experts");
  if (c->n_shared_experts < 0) return fail(LG_ERR_INVALID_ARG, "n_shared_experts < 0");
  if (static_cast<long long>(F) * c->n_shared_experts > (1 << 20))
    return fail(LG_ERR_UNSUPPORTED, "shared expert width too large");
  return LG_OK;
}

int validate_tokens(int64_t M, const lg_moe_config* c) {
  if (M < 0) return fail(LG_ERR_INVALID_ARG, "token count %lld < 0", static_cast<long long>(M));
  const long long big = static_cast<long long>(M) *
                        (c->hidden_size > c->n_routed_experts ? c->hidden_size : c->n_routed_experts) *
                        c->num_experts_per_tok;
  if (big >= (1LL << 40)) return fail(LG_ERR_UNSUPPORTED, "token count %lld too large", static_cast<long long>(M));
  if (static_cast<long long>(M) * c->num_experts_per_tok >= (1LL << 31))
    return fail(LG_ERR_UNSUPPORTED, "route count overflows int32");
  return LG_OK;
}

struct Layout {
  size_t status, logits, weights, indices, counts, offsets, perm, active, act, act_s, y, ys, tickets, xs, bimg, bsc,
      xterm, xtsc, aterm, atsc, tiles, inv, silu, shtab, total;
  bool tc;  // batched tensor-core buffers reserved
};

// Batched calls of at least this many tokens run the tensor-core grouped GEMMs
// (grouped_tc.cuh) when the geometry allows; smaller ones the CUDA-core
// grouped GEMV.  kTcTerms E2M1 terms carry each bf16 activation.
constexpr int kTcMinTokens = 64;
constexpr int kTcTerms = lg::gtc::kTerms;

// Geometry the batched tensor-core kernels take: whole 256-value atoms and
// 16-byte scale rows along F (F a multiple of 512), scale rows of at most 256
// bytes (d, F <= 8192), shared width in 64-value atoms, and d a multiple of
// 1024: the gate/up kernel gathers the token-term scale rows (d/32 bytes) four
// at a time, and a tensor copy's shared-memory destination must sit on 128
// bytes, so 4 * d/32 must be a multiple of 128.
bool tc_geometry(const lg_moe_config* c) {
  const int d = c->hidden_size, F = c->moe_intermediate_size, Fs = F * c->n_shared_experts;
  return d % 1024 == 0 && d <= 8192 && F % 512 == 0 && F <= 8192 && Fs % 64 == 0 && c->n_routed_experts <= 1024;
}
bool tc_batched_env() {
  static const bool on = [] {
    const char* v = std::getenv("LIVGLM_BATCHED_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}
// LIVGLM_ROUTER_PIPE=0: large batches use the register-prefetch router kernel
bool router_pipe_env() {
  static const bool on = [] {
    const char* v = std::getenv("LIVGLM_ROUTER_PIPE");
    return !(v && v[0] == '0');
  }();
  return on;
}

Layout layout(const lg_moe_config* c, int64_t M) {
  const size_t E = c->n_routed_experts, k = c->num_experts_per_tok, d = c->hidden_size;
  const size_t F = c->moe_intermediate_size, Fs = F * c->n_shared_experts;
  const size_t m = static_cast<size_t>(M);
  Layout L{};
  size_t o = 0;
  L.status = o;  o += up(4);
  L.logits = o;  o += up(m * E * 4);
  L.weights = o; o += up(m * k * 4);
  L.indices = o; o += up(m * k * 4);
  L.counts = o;  o += up(E * 4);
  L.offsets = o; o += up((E + 1) * 4);
  L.perm = o;    o += up(m * k * 4);
  L.active = o;  o += up((E + 1) * 4);
  // the batched tensor-core path writes act as T E2M1 terms + scales into the
  // same region (route-major [M*k][T][F/2], then [M*k][T][F/32])
  L.tc = M >= kTcMinTokens && tc_geometry(c);
  const size_t aterm = kTcTerms * m * k * (F / 2), atsc = kTcTerms * m * k * (F / 32);
  L.act = o;     o += up(std::max(m * k * F * 2, L.tc ? up(aterm) + atsc : size_t(0)));
  L.aterm = L.act;
  L.atsc = L.act + up(aterm);
  L.act_s = o;   o += up(m * Fs * 2);
  L.y = o;       o += up(m * k * d * 2);
  L.ys = o;      o += up(m * d * 2);
  L.tickets = o; o += up(d * 4);
  L.xs = o;      o += up(m * d * 2);  // tokens staged from page-locked host memory
  // one-token tensor-core down: split route activations (a swizzled 1 KB image
  // per 256-value column and route) and their scales
  L.bimg = o;    o += m == 1 ? up(k * (F / 256) * 1024) : 0;
  L.bsc = o;     o += m == 1 ? up(k * lg::dtc::kTerms * (F / 32)) : 0;
  // batched tensor core: token terms at every dispatch position [M*k][T][d/2]
  // + scales [M*k][T][d/32], route tiles, inverse dispatch permutation
  L.xterm = o;   o += L.tc ? up(kTcTerms * m * k * (d / 2)) : 0;
  L.xtsc = o;    o += L.tc ? up(kTcTerms * m * k * (d / 32)) : 0;
  L.tiles = o;   o += L.tc ? up((E + 1) * 4) : 0;
  L.inv = o;     o += L.tc ? up(m * k * 4) : 0;
  L.silu = o;    o += L.tc ? up(65536 * 2) : 0;  // SwiGLU factor table of the bf16 grouped GEMMs
  L.shtab = o;   o += L.tc ? up(16) : 0;         // the shared expert's offsets and chunk table
  L.total = o;
  return L;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

int check_ws(const lg_moe_config* c, int64_t M, void* ws, size_t bytes) {
  const size_t need = layout(c, M).total;
  if (!ws) return fail(LG_ERR_WORKSPACE, "workspace is NULL (need %zu bytes)", need);
  if (!aligned(ws, kAlign)) return fail(LG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (bytes < need) return fail(LG_ERR_WORKSPACE, "workspace has %zu bytes, need %zu", bytes, need);
  return LG_OK;
}

int validate_weights(const lg_moe_config* c, const lg_moe_weights* w, bool routed, bool shared) {
  if (!w) return fail(LG_ERR_INVALID_ARG, "weights is NULL");
  if (routed) {
    const void* ps[6] = {w->gate_packed, w->gate_scale, w->up_packed, w->up_scale, w->down_packed, w->down_scale};
    for (const void* p : ps)
      if (!p) return fail(LG_ERR_INVALID_ARG, "routed expert tensor pointer is NULL");
    if (!aligned(w->gate_packed, 16) || !aligned(w->up_packed, 16) || !aligned(w->down_packed, 16))
      return fail(LG_ERR_INVALID_ARG, "weight_packed banks must be 16-byte aligned");
    const long long d = c->hidden_size, F = c->moe_intermediate_size;
    const long long gp = F * d / 2, gs = F * d / 32, dp = d * F / 2, ds = d * F / 32;
    if (w->gate_packed_stride % 16 || w->up_packed_stride % 16 || w->down_packed_stride % 16)
      return fail(LG_ERR_INVALID_ARG, "weight_packed expert strides must be multiples of 16 bytes");
    if (w->gate_packed_stride < gp || w->up_packed_stride < gp || w->down_packed_stride < dp ||
        w->gate_scale_stride < gs || w->up_scale_stride < gs || w->down_scale_stride < ds)
      return fail(LG_ERR_INVALID_ARG, "expert strides smaller than one expert's tensor");
  }
  if (shared && c->n_shared_experts > 0) {
    if (!w->shared_gate || !w->shared_up || !w->shared_down)
      return fail(LG_ERR_INVALID_ARG, "shared expert weight pointer is NULL");
    if (!aligned(w->shared_gate, 16) || !aligned(w->shared_up, 16) || !aligned(w->shared_down, 16))
      return fail(LG_ERR_INVALID_ARG, "shared expert weights must be 16-byte aligned");
  }
  return LG_OK;
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// ---- launches --------------------------------------------------------------

int launch_router(const lg_moe_config* c, const uint16_t* x, int M, const float* Wr,
                  const float* bias, float* logits, float* weights, uint32_t* indices,
                  int* counts, cudaStream_t s) {
  using namespace lg;
  const int d = c->hidden_size, E = c->n_routed_experts;
  if (M <= 4) {
    dim3 grid((M + 0) / 1, (E + 7) / 8);
    router_logits_kernel<1, 1><<<grid, 256, 0, s>>>(x, Wr, M, d, E, logits);
  } else if (d % 256 == 0 && M >= 1024 && router_pipe_env()) {
    // 32 tokens x 16 experts per block, operands through a 3-stage cp.async ring
    constexpr int kTW = 4, kST = 3;
    const size_t smem = static_cast<size_t>(kST) * (8 * kTW * 512 + kRlExperts * 1024);
    auto kern = router_logits_pipe_kernel<kTW, kRlExperts, kST>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_check(e, "router smem attribute");
    dim3 grid((M + 8 * kTW - 1) / (8 * kTW), (E + kRlExperts - 1) / kRlExperts);
    kern<<<grid, 256, smem, s>>>(x, Wr, M, d, E, logits);
  } else if (d % 256 == 0 && M >= 8192) {  // 64 tokens x 16 experts per block: fewer re-reads of W_r
    dim3 grid((M + 63) / 64, (E + kRlExperts - 1) / kRlExperts);
    router_logits_tiled_kernel<8><<<grid, 256, 0, s>>>(x, Wr, M, d, E, logits);
  } else if (d % 256 == 0 && M >= 1024) {
    dim3 grid((M + 31) / 32, (E + kRlExperts - 1) / kRlExperts);
    router_logits_tiled_kernel<4><<<grid, 256, 0, s>>>(x, Wr, M, d, E, logits);
  } else if (d % 256 == 0 && M >= 64) {
    dim3 grid((M + 15) / 16, (E + kRlExperts - 1) / kRlExperts);
    router_logits_tiled_kernel<2><<<grid, 256, 0, s>>>(x, Wr, M, d, E, logits);
  } else {
    dim3 grid((M + 3) / 4, (E + 31) / 32);
    router_logits_kernel<4, 4><<<grid, 256, 0, s>>>(x, Wr, M, d, E, logits);
  }
  const size_t smem = static_cast<size_t>(kSelectWarps) * (2 * E + c->n_group) * sizeof(float);
  router_select_kernel<<<(M + kSelectWarps - 1) / kSelectWarps, kSelectWarps * 32, smem, s>>>(
      logits, bias, M, E, c->n_group, c->topk_group, c->num_experts_per_tok, c->norm_topk_prob,
      c->routed_scaling_factor, weights, indices, counts);
  return cuda_check(cudaGetLastError(), "router launch");
}

// Routes whose expert id is >= E are skipped (never counted, never placed in
// perm); their slots' outputs are left unwritten.
__global__ void histogram_kernel(const uint32_t* __restrict__ idx, int S, int E, int* __restrict__ counts) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S; s += gridDim.x * blockDim.x) {
    const uint32_t e = idx[s];
    if (e < static_cast<uint32_t>(E)) atomicAdd(counts + e, 1);
  }
}

int launch_dispatch(const lg_moe_config* c, const uint32_t* idx, int M, int* counts,
                    int* offsets, int* perm, int* active, bool need_hist, cudaStream_t s) {
  const int E = c->n_routed_experts, S = M * c->num_experts_per_tok;
  if (need_hist) {
    cudaMemsetAsync(counts, 0, E * sizeof(int), s);
    histogram_kernel<<<(S + 255) / 256 < 1024 ? (S + 255) / 256 : 1024, 256, 0, s>>>(idx, S, E, counts);
  }
  lg::dispatch_kernel<<<E, 256, 0, s>>>(idx, S, E, counts, offsets, perm, active);
  return cuda_check(cudaGetLastError(), "dispatch launch");
}

template <int LPR, int TT>
int launch_gemv_t(const lg::GemvArgs& a, int max_items, cudaStream_t s) {
  const int G = (a.K > a.Ks ? a.K : a.Ks) / 32;
  const int KI = (G + LPR - 1) / LPR;
  const size_t smem = static_cast<size_t>(TT) * KI * 8 * LPR * sizeof(float4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(lg::grouped_gemv_kernel<LPR, TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr = true;
  }
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, lg::grouped_gemv_kernel<LPR, TT>, 256, smem);
  if (occ < 1) occ = 1;
  int grid = num_sms() * occ;
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  lg::grouped_gemv_kernel<LPR, TT><<<grid, 256, smem, s>>>(a);
  return cuda_check(cudaGetLastError(), "grouped gemv launch");
}

template <int LPR>
int launch_gemv_tt(const lg::GemvArgs& a, int tt, int max_items, cudaStream_t s) {
  switch (tt) {
    case 1: return launch_gemv_t<LPR, 1>(a, max_items, s);
    case 2: return launch_gemv_t<LPR, 2>(a, max_items, s);
    default: return launch_gemv_t<LPR, 4>(a, max_items, s);
  }
}

int pick_lpr(int K) {
  const int G = K / 32;
  for (int l = 32; l >= 4; l >>= 1)
    if (G % l == 0) return l;
  return 4;
}

int launch_gemv(const lg::GemvArgs& a, int M, int max_routes_per_expert, int E, cudaStream_t s) {
  const int K = a.K > 0 ? a.K : a.Ks;
  const int lpr = pick_lpr(K);
  const int rows = 8 * (32 / lpr);
  int tt = 4;
  const int need = max_routes_per_expert > M ? max_routes_per_expert : M;
  if (need <= 1) tt = 1;
  else if (need <= 2) tt = 2;
  const int G = (a.K > a.Ks ? a.K : a.Ks) / 32;
  while (tt > 1 && static_cast<size_t>(tt) * ((G + lpr - 1) / lpr) * 8 * lpr * 16 > 200 * 1024) tt >>= 1;
  if (static_cast<size_t>(tt) * ((G + lpr - 1) / lpr) * 8 * lpr * 16 > 200 * 1024)
    return fail(LG_ERR_UNSUPPORTED, "reduction length %d too large for the staged GEMV", K);
  const long long items = static_cast<long long>(E) * ((a.N + rows - 1) / rows) + (a.Ns + rows - 1) / rows;
  const int max_items = items > (1 << 30) ? (1 << 30) : static_cast<int>(items);
  switch (lpr) {
    case 32: return launch_gemv_tt<32>(a, tt, max_items, s);
    case 16: return launch_gemv_tt<16>(a, tt, max_items, s);
    case 8: return launch_gemv_tt<8>(a, tt, max_items, s);
    default: return launch_gemv_tt<4>(a, tt, max_items, s);
  }
}

// ---- batched tensor-core path (grouped_tc.cuh) ----------------------------------
void trace_mark(int slot, int i, cudaStream_t s);
bool map_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
            bool sw128);
bool map_3d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t n, uint64_t n_stride,
            uint32_t box_inner, uint32_t box_rows, bool sw128);
// Weight banks and scale tensors the TMA reads: 16-byte aligned bases and
// expert strides (checked for the packed banks by validate_weights).
bool tc_weights_fit(const lg_moe_config* c, const lg_moe_weights* w, bool routed, bool shared) {
  if (routed) {
    if (!aligned(w->gate_scale, 16) || !aligned(w->up_scale, 16) || !aligned(w->down_scale, 16)) return false;
    if (w->gate_scale_stride % 16 || w->up_scale_stride % 16 || w->down_scale_stride % 16) return false;
  }
  (void)c;
  (void)shared;
  return true;
}

struct GgMaps {
  CUtensorMap A0, A1, B, B80, SA0, SA1, SB, SB80;
};

template <bool kRouted, bool kGateUp>
int launch_grouped(const lg::gtc::Args& a0, int items_max, const GgMaps& m, cudaStream_t s) {
  using namespace lg::gtc;
  Args a = a0;
  const int b_rows = kRouted ? kTerms * kNtMax : kNtShared;
  a.stage_bytes = kABytes + b_rows * 128;
  a.b_off = kABytes;
  size_t fixed = 0;
  size_t sfa = 0, sfb = 0, xch = 0, tab = 0;
  if (kRouted) {
    sfa = static_cast<size_t>(128) * a.sc_bytes;
    sfb = static_cast<size_t>(b_rows) * a.sc_bytes;
    tab = (static_cast<size_t>(a.E) + 1) * 4;
  }
  if (kGateUp) xch = static_cast<size_t>(4) * (kRouted ? kNtMax : kNtShared) * 32 * 2;
  auto r1k = [](size_t v) { return (v + 1023) / 1024 * 1024; };
  fixed = r1k(2 * sfa) + r1k(2 * sfb) + r1k(xch) + r1k(tab);
  const size_t budget = 227 * 1024 - 1024 - 1024;  // dynamic limit less alignment slack and static barriers
  if (fixed + 2 * static_cast<size_t>(a.stage_bytes) > budget)
    return fail(LG_ERR_UNSUPPORTED, "batched tensor-core plan does not fit in shared memory");
  a.stages = static_cast<int>(std::min<size_t>(kRouted ? kRoutedStages : kMaxStages, (budget - fixed) / a.stage_bytes));

  a.ring_off = 0;
  a.sfa_off = a.stages * a.stage_bytes;
  a.sfa_bytes = static_cast<int>(sfa);
  a.sfb_off = a.sfa_off + static_cast<int>(r1k(2 * sfa));
  a.sfb_bytes = static_cast<int>(sfb);
  a.xch_off = a.sfb_off + static_cast<int>(r1k(2 * sfb));
  a.tab_off = a.xch_off + static_cast<int>(r1k(xch));
  const size_t smem = 1024 + a.tab_off + r1k(tab);
  auto kern = grouped_kernel<kRouted, kGateUp>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_check(e, "grouped kernel smem attribute");
  int grid = num_sms();
  if (items_max < grid) grid = items_max;
  if (grid < 1) return LG_OK;
  kern<<<grid, kThreads, smem, s>>>(a, m.A0, m.A1, m.B, m.B80, m.SA0, m.SA1, m.SB, m.SB80);
  return cuda_check(cudaGetLastError(), "grouped kernel launch");
}

bool map_3d_swz(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t n, uint64_t n_stride,
                uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz);

// Tensor-core calls whose experts average at least this many routes run the
// routed products with the weights widened to bf16 (grouped_dq.cuh): four
// K = 16 MMAs per 64 values instead of one K = 64 kind::mxf4 MMA per term,
// but no activation terms and 256-route tiles.  LIVGLM_BATCHED_DQ=0 / 1
// forces it off / on for every tensor-core call.
constexpr int kDqMinRoutesPerExpert = 128;
bool dq_mode(const lg_moe_config* c, int M) {
  static const int env = [] {
    const char* v = std::getenv("LIVGLM_BATCHED_DQ");
    return v && v[0] == '0' ? 0 : (v && v[0] == '1' ? 1 : -1);
  }();
  if (env >= 0) return env == 1;
  return static_cast<long long>(M) * c->num_experts_per_tok >=
         static_cast<long long>(kDqMinRoutesPerExpert) * c->n_routed_experts;
}

template <bool kGateUp, bool kBf16A = false>
int launch_dq(const lg::gdq::Args& a0, long long items_max, const CUtensorMap& A0, const CUtensorMap& A1,
              const CUtensorMap& B, cudaStream_t s) {
  using namespace lg::gdq;
  Args a = a0;
  const size_t smem = 1024 + kSmemBytes;  // 1024-byte alignment slack
  auto kern = grouped_dq_kernel<kGateUp, kBf16A>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_check(e, "grouped bf16 kernel smem attribute");
  long long grid = num_sms();
  if (items_max < grid) grid = items_max;
  if (grid < 1) return LG_OK;
  kern<<<static_cast<int>(grid), kThreads, smem, s>>>(a, A0, A1, B);
  return cuda_check(cudaGetLastError(), "grouped bf16 kernel launch");
}

// Routed gate/up (kGateUp) or down with the bf16-widened weights: route
// chunks, the token rows gathered to dispatch order (gate/up), the kernel.
int launch_routed_dq(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M, const int* offsets,
                     const int* perm, void* ws, const Layout& L, uint16_t* y, bool gate_up, cudaStream_t s) {
  const int d = c->hidden_size, F = c->moe_intermediate_size, E = c->n_routed_experts, k = c->num_experts_per_tok;
  const int R = M * k;
  lg::gdq::Args q{};
  q.d = d; q.F = F; q.E = E; q.R = R;
  q.limit = c->swiglu_limit;
  q.offsets = offsets; q.perm = perm; q.chunk_start = at<int>(ws, L.tiles);
  q.act = at<uint16_t>(ws, L.act); q.y = y;
  q.silu = at<uint16_t>(ws, L.silu);
  q.status = at<int>(ws, L.status);
  uint16_t* xp = at<uint16_t>(ws, L.xterm);  // [R][d] bf16: fits the token-term region
  const long long chunks_max = static_cast<long long>(R) / lg::gdq::kNMax + std::min(E, R);
  CUtensorMap A0, A1, B;
  if (gate_up) {
    lg::gdq::chunk_table_kernel<<<1, 1024, 0, s>>>(offsets, E, at<int>(ws, L.tiles));
    lg::gdq::silu_table_kernel<<<256, 256, 0, s>>>(at<uint16_t>(ws, L.silu));
    // a warp per dispatched row, eight warps per CTA
    lg::gdq::gather_rows_kernel<<<static_cast<int>(std::min<long long>((R + 7) / 8, 8LL * num_sms())), 256, 0,
                                  s>>>(x, d, k, perm, offsets, E, xp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_check(e, "route gather launch");
    q.ks_count = d / 64; q.rb_count = F / 128; q.rb_rows = 128; q.acc1_rows = 0;
    q.pk0 = w->gate_packed; q.pk1 = w->up_packed;
    q.pk0_stride = static_cast<long long>(w->gate_packed_stride);
    q.pk1_stride = static_cast<long long>(w->up_packed_stride);
    q.pk_row = d / 2;
    q.sc0 = w->gate_scale; q.sc1 = w->up_scale;
    q.sc0_stride = static_cast<long long>(w->gate_scale_stride); q.sc1_stride = static_cast<long long>(w->up_scale_stride);
    q.sc_row = d / 32;
    if (!map_3d_swz(&A0, w->gate_packed, d / 2, F, E, w->gate_packed_stride, 32, 128, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !map_3d_swz(&A1, w->up_packed, d / 2, F, E, w->up_packed_stride, 32, 128, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !map_2d(&B, xp, static_cast<uint64_t>(d) * 2, R, 128, lg::gdq::kBoxRows, true))
      return fail(LG_ERR_CUDA, "batched bf16 gate/up: tensor map encoding failed");
    return launch_dq<true>(q, chunks_max * q.rb_count, A0, A1, B, s);
  }
  q.ks_count = F / 64; q.rb_count = d / 256; q.rb_rows = 256; q.acc1_rows = 128;
  q.pk0 = q.pk1 = w->down_packed;
  q.pk0_stride = q.pk1_stride = static_cast<long long>(w->down_packed_stride);
  q.pk_row = F / 2;
  q.sc0 = q.sc1 = w->down_scale;
  q.sc0_stride = q.sc1_stride = static_cast<long long>(w->down_scale_stride);
  q.sc_row = F / 32;
  if (!map_3d_swz(&A0, w->down_packed, F / 2, d, E, w->down_packed_stride, 32, 128, CU_TENSOR_MAP_SWIZZLE_32B) ||
      !map_2d(&B, q.act, static_cast<uint64_t>(F) * 2, R, 128, lg::gdq::kBoxRows, true))
    return fail(LG_ERR_CUDA, "batched bf16 down: tensor map encoding failed");
  return launch_dq<false>(q, chunks_max * q.rb_count, A0, A0, B, s);
}

// Token chunks of the shared expert on the widened-weight kernel: every chunk
// makes rb_count work items for `grid` CTAs, so the chunk width that costs
// the fewest rounds x MMA cycles wins (118 cycles per M = 128 MMA up to
// N = 160, rising to 166 at N = 256, measured), larger chunks on a tie.  The
// chunk count returned is ceil(M / width), so that no chunk is empty.
int shared_chunks(int M, int rb_count, int grid) {
  int best_n = (M + lg::gdq::kNMax - 1) / lg::gdq::kNMax;
  double best = 1e300;
  for (int c = lg::gdq::kNMax; c >= 128; c -= lg::gdq::kBoxRows) {
    const int n = (M + c - 1) / c;
    const int width = ((M + n - 1) / n + lg::gdq::kBoxRows - 1) / lg::gdq::kBoxRows * lg::gdq::kBoxRows;
    const long long rounds = (static_cast<long long>(n) * rb_count + grid - 1) / grid;
    const double cost = static_cast<double>(rounds) * (width <= 160 ? 118.0 : 118.0 + 0.5 * (width - 160));
    if (cost < best - 1e-9) {
      best = cost;
      best_n = n;
    }
  }
  return best_n;
}

// The shared expert of a large batch on the same kernel (kBf16A): its bf16
// weight rows TMA-loaded as the A tiles, the tokens (gate/up) or act_s (down)
// in order as B, token chunks of at most 256 (shared_chunks).  Needs
// Fs % 128 == 0.
int launch_shared_dq(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M, void* ws,
                     const Layout& L, uint16_t* ys, bool gate_up, bool fill_silu, cudaStream_t s) {
  const int d = c->hidden_size, Fs = c->moe_intermediate_size * c->n_shared_experts;
  lg::gdq::Args q{};
  int* tab = at<int>(ws, L.shtab);
  q.d = d; q.F = Fs; q.E = 1; q.R = M;
  q.limit = c->swiglu_limit;
  q.offsets = tab; q.perm = nullptr; q.chunk_start = tab + 2;
  q.silu = at<uint16_t>(ws, L.silu);
  q.act = at<uint16_t>(ws, L.act_s); q.y = ys;
  q.status = at<int>(ws, L.status);
  CUtensorMap A0, A1, B;
  if (gate_up) {
    const int nch = shared_chunks(M, Fs / 128, num_sms());
    lg::gdq::shared_table_kernel<<<1, 32, 0, s>>>(M, nch, tab);
    if (fill_silu) lg::gdq::silu_table_kernel<<<256, 256, 0, s>>>(at<uint16_t>(ws, L.silu));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_check(e, "shared tables launch");
    q.ks_count = d / 64; q.rb_count = Fs / 128; q.rb_rows = 128; q.acc1_rows = 0;
    if (!map_2d(&A0, w->shared_gate, static_cast<uint64_t>(d) * 2, Fs, 128, 128, true) ||
        !map_2d(&A1, w->shared_up, static_cast<uint64_t>(d) * 2, Fs, 128, 128, true) ||
        !map_2d(&B, x, static_cast<uint64_t>(d) * 2, M, 128, lg::gdq::kBoxRows, true))
      return fail(LG_ERR_CUDA, "batched shared gate/up: tensor map encoding failed");
    return launch_dq<true, true>(q, static_cast<long long>(nch) * q.rb_count, A0, A1, B, s);
  }
  q.ks_count = Fs / 64; q.rb_count = d / 256; q.rb_rows = 256; q.acc1_rows = 128;
  const int nch = shared_chunks(M, q.rb_count, num_sms());
  lg::gdq::shared_table_kernel<<<1, 32, 0, s>>>(M, nch, tab);  // after the gate/up kernel read it
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_check(e, "shared table launch");
  if (!map_2d(&A0, w->shared_down, static_cast<uint64_t>(Fs) * 2, d, 128, 128, true) ||
      !map_2d(&B, q.act, static_cast<uint64_t>(Fs) * 2, M, 128, lg::gdq::kBoxRows, true))
    return fail(LG_ERR_CUDA, "batched shared down: tensor map encoding failed");
  return launch_dq<false, true>(q, static_cast<long long>(nch) * q.rb_count, A0, A0, B, s);
}

// The batched expert passes on the tensor core: token split, route tiles,
// routed and/or shared gate/up, then routed and/or shared down.  Routing
// tables (offsets, perm) must be ready; y gets the routed outputs in slot
// order, ys the shared output.
int launch_experts_tc(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M, const int* offsets,
                      const int* perm, void* ws, const Layout& L, uint16_t* y, uint16_t* ys, bool with_routed,
                      bool with_shared, cudaStream_t s, int slot = -1) {
  using namespace lg::gtc;
  const int d = c->hidden_size, F = c->moe_intermediate_size, E = c->n_routed_experts, k = c->num_experts_per_tok;
  const int Fs = F * c->n_shared_experts, T = kTcTerms, R = M * k;
  const bool sh = with_shared && Fs > 0;
  Args a{};
  a.M = M; a.d = d; a.F = F; a.Fs = Fs; a.E = E; a.k = k; a.R = R;
  a.limit = c->swiglu_limit;
  a.offsets = offsets; a.perm = perm; a.tile_start = at<int>(ws, L.tiles);
  a.act_terms = at<uint8_t>(ws, L.aterm); a.act_tsc = at<uint8_t>(ws, L.atsc);
  a.act_s = at<uint16_t>(ws, L.act_s); a.y = y; a.ys = ys;
  a.status = at<int>(ws, L.status);
  uint8_t* xterm = at<uint8_t>(ws, L.xterm);
  uint8_t* xtsc = at<uint8_t>(ws, L.xtsc);
  int* inv = at<int>(ws, L.inv);
  const int tok_tiles = (M + kNtShared - 1) / kNtShared;
  // routed tiles: at most one partial tile per expert beyond R / kNtMax full ones
  const long long tiles_max = static_cast<long long>(R) / kNtMax + std::min(E, R);
  const uint64_t rt = static_cast<uint64_t>(R) * T;  // term rows
  GgMaps m;
  int rc;
  cudaError_t e;
  const bool dq = with_routed && dq_mode(c, M);
  if (dq) {
    if ((rc = launch_routed_dq(c, w, x, M, offsets, perm, ws, L, y, true, s))) return rc;
  } else if (with_routed) {
    tile_table_kernel<<<1, 1024, 0, s>>>(offsets, E, at<int>(ws, L.tiles));
    cudaMemsetAsync(inv, 0xFF, static_cast<size_t>(R) * 4, s);
    inverse_perm_kernel<<<std::min((R + 255) / 256, 4 * num_sms()), 256, 0, s>>>(perm, offsets, E, inv);
    const long long warps = static_cast<long long>(M) * (d / 256);
    split_routes_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, s>>>(x, M, d, k, inv, xterm, xtsc);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_check(e, "route split launch");
    Args g = a;
    g.kb_count = d / 256; g.rb_count = F / 64; g.sc_bytes = d / 32; g.sc_swz = d / 32 == 128;
    if (!map_3d(&m.A0, w->gate_packed, d / 2, F, E, w->gate_packed_stride, 128, 64, true) ||
        !map_3d(&m.A1, w->up_packed, d / 2, F, E, w->up_packed_stride, 128, 64, true) ||
        !map_2d(&m.B, xterm, d / 2, rt, 128, kTerms * kNtMax, true) ||
        !map_2d(&m.B80, xterm, d / 2, rt, 128, kTerms * kNtMax / 2, true) ||
        !map_3d(&m.SA0, w->gate_scale, d / 32, F, E, w->gate_scale_stride, d / 32, 64, g.sc_swz) ||
        !map_3d(&m.SA1, w->up_scale, d / 32, F, E, w->up_scale_stride, d / 32, 64, g.sc_swz) ||
        !map_2d(&m.SB, xtsc, d / 32, rt, d / 32, kTerms * kNtMax, g.sc_swz) ||
        !map_2d(&m.SB80, xtsc, d / 32, rt, d / 32, kTerms * kNtMax / 2, g.sc_swz))
      return fail(LG_ERR_CUDA, "batched gate/up: tensor map encoding failed");
    const long long items = tiles_max * g.rb_count;
    if ((rc = launch_grouped<true, true>(g, static_cast<int>(std::min<long long>(items, 1 << 30)), m, s))) return rc;
  }
  // large batches: the shared expert on the widened-weight kernel (256-token tiles)
  const bool sdq = sh && Fs % 128 == 0 && dq_mode(c, M);
  if (sdq) {
    if ((rc = launch_shared_dq(c, w, x, M, ws, L, ys, true, !dq, s))) return rc;
  } else if (sh) {
    Args g = a;
    g.kb_count = d / 64; g.rb_count = Fs / 64; g.n_tok_tiles = tok_tiles;
    if (!map_2d(&m.A0, w->shared_gate, static_cast<uint64_t>(d) * 2, Fs, 128, 64, true) ||
        !map_2d(&m.A1, w->shared_up, static_cast<uint64_t>(d) * 2, Fs, 128, 64, true) ||
        !map_2d(&m.B, x, static_cast<uint64_t>(d) * 2, M, 128, kNtShared, true))
      return fail(LG_ERR_CUDA, "batched shared gate/up: tensor map encoding failed");
    m.B80 = m.SA0 = m.SA1 = m.SB = m.SB80 = m.A0;  // unused by the shared kernels
    if ((rc = launch_grouped<false, true>(g, g.rb_count * tok_tiles, m, s))) return rc;
  }
  trace_mark(slot, 3, s);
  if (dq) {
    if ((rc = launch_routed_dq(c, w, x, M, offsets, perm, ws, L, y, false, s))) return rc;
  } else if (with_routed) {
    Args g = a;
    g.kb_count = F / 256; g.rb_count = d / 128; g.sc_bytes = F / 32; g.sc_swz = F / 32 == 128;
    if (!map_3d(&m.A0, w->down_packed, F / 2, d, E, w->down_packed_stride, 128, 128, true) ||
        !map_2d(&m.B, a.act_terms, F / 2, rt, 128, kTerms * kNtMax, true) ||
        !map_2d(&m.B80, a.act_terms, F / 2, rt, 128, kTerms * kNtMax / 2, true) ||
        !map_3d(&m.SA0, w->down_scale, F / 32, d, E, w->down_scale_stride, F / 32, 128, g.sc_swz) ||
        !map_2d(&m.SB, a.act_tsc, F / 32, rt, F / 32, kTerms * kNtMax, g.sc_swz) ||
        !map_2d(&m.SB80, a.act_tsc, F / 32, rt, F / 32, kTerms * kNtMax / 2, g.sc_swz))
      return fail(LG_ERR_CUDA, "batched down: tensor map encoding failed");
    m.A1 = m.SA1 = m.A0;
    const long long items = tiles_max * g.rb_count;
    if ((rc = launch_grouped<true, false>(g, static_cast<int>(std::min<long long>(items, 1 << 30)), m, s))) return rc;
  }
  if (sdq) {
    if ((rc = launch_shared_dq(c, w, x, M, ws, L, ys, false, false, s))) return rc;
  } else if (sh) {
    Args g = a;
    g.kb_count = Fs / 64; g.rb_count = d / 128; g.n_tok_tiles = tok_tiles;
    if (!map_2d(&m.A0, w->shared_down, static_cast<uint64_t>(Fs) * 2, d, 128, 128, true) ||
        !map_2d(&m.B, a.act_s, static_cast<uint64_t>(Fs) * 2, M, 128, kNtShared, true))
      return fail(LG_ERR_CUDA, "batched shared down: tensor map encoding failed");
    m.A1 = m.B80 = m.SA0 = m.SA1 = m.SB = m.SB80 = m.A0;
    if ((rc = launch_grouped<false, false>(g, g.rb_count * tok_tiles, m, s))) return rc;
  }
  trace_mark(slot, 4, s);
  return LG_OK;
}

// Gate/up (+ SwiGLU) pass over routed experts and, when `with_shared`, the
// shared expert.  Routing tables must be ready.
int launch_gate_up(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M,
                   const int* offsets, const int* perm, const int* active, uint16_t* act,
                   uint16_t* act_s, bool with_routed, bool with_shared, cudaStream_t s) {
  const int d = c->hidden_size, F = c->moe_intermediate_size, k = c->num_experts_per_tok;
  const int Fs = F * c->n_shared_experts;
  const bool sh = with_shared && Fs > 0;
  lg::GemvArgs a{};
  a.K = d; a.N = F; a.Ks = d; a.Ns = sh ? Fs : 0; a.k = k; a.M = M; a.pair = 1;
  a.limit = c->swiglu_limit;
  if (with_routed) {
    a.a_packed = w->gate_packed; a.a_scale = w->gate_scale; a.b_packed = w->up_packed; a.b_scale = w->up_scale;
    a.a_pstride = w->gate_packed_stride; a.a_sstride = w->gate_scale_stride;
    a.b_pstride = w->up_packed_stride; a.b_sstride = w->up_scale_stride;
  }
  a.sa = sh ? w->shared_gate : nullptr; a.sb = sh ? w->shared_up : nullptr;
  a.xin = x; a.xin_by_token = 1; a.xin_s = x;
  a.offsets = offsets; a.perm = perm; a.active = active;
  a.out = act; a.out_by_slot = 0; a.out_s = act_s;
  return launch_gemv(a, M, M, with_routed ? c->n_routed_experts : 0, s);
}

// Down pass: routed outputs land in slot order (row t*k + j of y).
int launch_down(const lg_moe_config* c, const lg_moe_weights* w, int M, const int* offsets,
                const int* perm, const int* active, const uint16_t* act, const uint16_t* act_s,
                uint16_t* y, uint16_t* ys, bool with_routed, bool with_shared, cudaStream_t s) {
  const int d = c->hidden_size, F = c->moe_intermediate_size, k = c->num_experts_per_tok;
  const int Fs = F * c->n_shared_experts;
  const bool sh = with_shared && Fs > 0;
  lg::GemvArgs b{};
  b.K = F; b.N = d; b.Ks = sh ? Fs : F; b.Ns = sh ? d : 0; b.k = k; b.M = M; b.pair = 0;
  b.limit = c->swiglu_limit;
  if (with_routed) {
    b.a_packed = w->down_packed; b.a_scale = w->down_scale;
    b.a_pstride = w->down_packed_stride; b.a_sstride = w->down_scale_stride;
  }
  b.sa = sh ? w->shared_down : nullptr;
  b.xin = act; b.xin_by_token = 0; b.xin_s = act_s;
  b.offsets = offsets; b.perm = perm; b.active = active;
  b.out = y; b.out_by_slot = 1; b.out_s = ys;
  return launch_gemv(b, M, M, with_routed ? c->n_routed_experts : 0, s);
}

int launch_experts(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M,
                   const int* offsets, const int* perm, const int* active, uint16_t* act,
                   uint16_t* act_s, uint16_t* y, uint16_t* ys, bool with_routed, bool with_shared,
                   cudaStream_t s) {
  int rc = launch_gate_up(c, w, x, M, offsets, perm, active, act, act_s, with_routed, with_shared, s);
  if (rc) return rc;
  return launch_down(c, w, M, offsets, perm, active, act, act_s, y, ys, with_routed, with_shared, s);
}

void trace_mark(int slot, int i, cudaStream_t s);

// ---- decode chain (M <= lg::kDecodeMaxTokens) ----------------------------------
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename K>
int occupancy(K kernel, int threads, size_t smem) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem);
  return occ < 1 ? 1 : occ;
}

constexpr size_t kSmemBudget = 227 * 1024 - 2048;  // dynamic bytes left after static shared

struct StreamPlan {
  lg::StreamCfg gu, dn;
  size_t gu_smem, dn_smem;
};

bool plan_stream(const lg_moe_config* c, int M, int TT, StreamPlan* P) {
  const size_t d = c->hidden_size, F = c->moe_intermediate_size, Fs = F * c->n_shared_experts;
  const size_t G = d / 32, KI = (G + 31) / 32, WPL = (d / 4 / 8 + 31) / 32;
  const size_t GF = F / 32, WS = (Fs / 8 + 31) / 32, R = static_cast<size_t>(M) * c->num_experts_per_tok;
  // gate/up
  const size_t gu_stage = std::max<size_t>(Fs > 0 ? 2 * lg::kGuRowsShared * d * 2 : 0,
                                           2 * lg::kGuRowsRouted * (d / 2) + 2 * lg::kGuRowsRouted * G);
  const size_t gu_x = TT * KI * 128 * 16 + TT * 4 * WPL * 32 * 16;
  const size_t tables = (2 * ((static_cast<size_t>(c->n_routed_experts) + 1 + 3) & ~size_t(3)) + R + 4) * 4;
  const size_t gu_aux = lg::kGroups * 2 * lg::kGuRowsShared * 4 * TT * 2 * 4 + tables;
  const size_t gu_fixed = gu_x + gu_aux;
  if (gu_fixed + 2 * gu_stage > kSmemBudget) return false;
  P->gu.stages = static_cast<int>(std::min<size_t>(lg::kMaxStages, (kSmemBudget - gu_fixed) / gu_stage));
  P->gu.stage_bytes = static_cast<int>(gu_stage);
  P->gu.x_off = P->gu.stages * P->gu.stage_bytes;
  P->gu.aux_off = static_cast<int>(P->gu.x_off + gu_x);
  P->gu_smem = P->gu.aux_off + gu_aux;
  // down
  const size_t dn_stage = std::max<size_t>(Fs > 0 ? lg::kDnRowsShared * Fs * 2 : 0,
                                           lg::kDnRowsRouted * (F / 2) + lg::kDnRowsRouted * GF);
  const size_t dn_x = R * F * 2 + static_cast<size_t>(M) * WS * 32 * 16;
  const size_t dn_aux = ((R + 3) & ~size_t(3)) * 4 + tables;
  if (dn_x + dn_aux + 2 * dn_stage > kSmemBudget) return false;
  P->dn.stages = static_cast<int>(std::min<size_t>(lg::kMaxStages, (kSmemBudget - dn_x - dn_aux) / dn_stage));
  P->dn.stage_bytes = static_cast<int>(dn_stage);
  P->dn.x_off = P->dn.stages * P->dn.stage_bytes;
  P->dn.aux_off = static_cast<int>(P->dn.x_off + dn_x);
  P->dn_smem = P->dn.aux_off + dn_aux;
  return true;
}

// One-token down kernel plan: routed chunks of kRows rows (scale copies start
// on 16 bytes: rows in units of 16/gcd(F/32, 16)), shared chunks of kShRows
// rows; activations in registers need F <= 1536 with F % 128 == 0 (scale
// words) and Fs <= 1536.
bool plan_down1(const lg_moe_config* c, lg::down1::Cfg* D, size_t* smem) {
  using namespace lg::down1;
  const size_t F = c->moe_intermediate_size, Fs = F * c->n_shared_experts, G2 = F / 32;
  if (F % 128 || F > 16 * 32 * kDcg || Fs > 32 * 8 * kScg || Fs % 8) return false;
  size_t stage = kRows * (F / 2 + G2);
  if (Fs > 0) stage = std::max<size_t>(stage, kShRows * Fs * 2);
  stage = (stage + 127) / 128 * 128;
  int g = static_cast<int>(G2), h = 16;
  while (h) { const int t = g % h; g = h; h = t; }
  D->unit = 16 / g;
  if (c->hidden_size % D->unit) return false;
  // routes one CTA's routed slice can span: ceil((slice + unit - 1) / d) + 1
  const size_t d = c->hidden_size, R = c->num_experts_per_tok;
  const size_t slice = (R * d + num_sms() - 1) / num_sms() + D->unit;
  const size_t span = (slice + d - 1) / d + 1;  // routes one slice can touch
  if (span > 4) return false;                    // down1 kernel's kMaxSpan
  const size_t act = span * F * 2;
  const size_t tail = (act + 127) / 128 * 128 + (slice + (d + num_sms() - 1) / num_sms()) * 2;
  const int stages = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemBudget - tail) / stage));
  if (stages < 2) return false;
  D->stages = stages;
  D->stage_bytes = static_cast<int>(stage);
  D->act_off = static_cast<int>(static_cast<size_t>(stages) * stage);
  D->yb_off = D->act_off + static_cast<int>((act + 127) / 128 * 128);
  D->yb_rows = static_cast<int>(slice);
  *smem = D->yb_off + (slice + (d + num_sms() - 1) / num_sms()) * 2;
  return true;
}

// ---- tensor-core one-token down ------------------------------------------------
// Default for one-token calls whose geometry fits plan_down_tc; LIVGLM_TC_DOWN=0
// (read once per process) selects the CUDA-core down1 kernel instead.
bool tc_down_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LIVGLM_TC_DOWN");
    return !(v && v[0] == '0');
  }();
  return on;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2-D byte tensor [rows][inner] (row stride = inner bytes), boxes of
// box_inner bytes x 128 rows, 128-byte swizzle or none
bool map_bytes(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner, bool sw128) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
  if (!fn || !aligned(base, 16) || inner % 16) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner};
  const cuuint32_t box[2] = {box_inner, static_cast<cuuint32_t>(lg::dtc::kTile)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Byte tensor maps of the batched tensor-core kernels: 2-D [rows][inner] or
// 3-D [n][rows][inner] (expert banks, n_stride bytes between experts), boxes of
// box_inner bytes x box_rows rows (x 1 expert), 128-byte swizzle or none.
bool map_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
            bool sw128) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
  if (!fn || !aligned(base, 16) || inner % 16) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
bool map_3d_swz(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t n, uint64_t n_stride,
                uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
  if (!fn || !aligned(base, 16) || inner % 16 || n_stride % 16) return false;
  const cuuint64_t dims[3] = {inner, rows, n};
  const cuuint64_t strides[2] = {inner, n_stride};
  const cuuint32_t box[3] = {box_inner, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
bool map_3d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t n, uint64_t n_stride,
            uint32_t box_inner, uint32_t box_rows, bool sw128) {
  return map_3d_swz(m, base, inner, rows, n, n_stride, box_inner, box_rows,
                    sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Needs: one token, d % 128 == 0, F a multiple of 512 up to 1536 (whole
// 256-value atom columns, 16-byte scale rows), Fs a multiple of 64 up to 1536,
// contiguous banks, every CTA of the routed share with at most kMaxUnits tiles
// over at most two routes.
bool plan_down_tc(const lg_moe_config* c, const lg_moe_weights* w, lg::dtc::Cfg* D, size_t* smem) {
  using namespace lg::dtc;
  const int d = c->hidden_size, F = c->moe_intermediate_size, Fs = F * c->n_shared_experts, k = c->num_experts_per_tok;
  if (d % kTile || F % 512 || F > 1536 || (Fs > 0 && (Fs % 64 || Fs > 1536))) return false;
  if (w->down_packed_stride != static_cast<int64_t>(d) * F / 2 || w->down_scale_stride != static_cast<int64_t>(d) * F / 32)
    return false;
  const int blocks = d / kTile, P = num_sms();
  D->n_sh = Fs > 0 ? blocks : 0;
  D->n_units = k * blocks;
  const int q = P - D->n_sh;
  if (q < 1) return false;
  for (int i = 0; i < q; ++i) {
    const int lo = static_cast<int>(static_cast<long long>(i) * D->n_units / q);
    const int hi = static_cast<int>(static_cast<long long>(i + 1) * D->n_units / q);
    if (hi - lo > kMaxUnits || (hi > lo && (hi - 1) / blocks - lo / blocks > 1)) return false;
  }
  D->cols = F / 256;
  D->sh_cols = Fs / 64;
  D->sc_bytes = F / 32;
  const size_t bsize = std::max<size_t>(2 * D->cols * kBRows * 128, static_cast<size_t>(D->sh_cols) * kShBRows * 128);
  const size_t scale = 2 * kTile * static_cast<size_t>(D->sc_bytes);
  const size_t budget = 227 * 1024 - 4096 - 1024;  // less static shared memory and the 1024-byte alignment slack
  const size_t fixed = (scale + 1023) / 1024 * 1024 + bsize;
  if (fixed + 2 * kBox > budget) return false;
  D->stages = static_cast<int>(std::min<size_t>(kMaxStages, (budget - fixed) / kBox));
  D->ring_off = 0;
  D->scale_off = D->stages * kBox;
  D->b_off = D->scale_off + static_cast<int>((scale + 1023) / 1024 * 1024);
  *smem = 1024 + D->b_off + bsize;
  return true;
}

// The decode chain needs bulk-copyable chunks: 16-byte aligned bases and
// expert strides (scales included), d % 64 == 0.
bool decode_fits(const lg_moe_config* c, const lg_moe_weights* w, int64_t M) {
  if (M < 1 || M > lg::kDecodeMaxTokens) return false;
  if (c->hidden_size % 64) return false;
  if (static_cast<size_t>(lg::kRouterExperts) * c->hidden_size * 4 > 200 * 1024) return false;
  // register-staged activation rows: d*M/8 <= 4 * 512 uint4, F/8 <= 8 * 32
  if (static_cast<size_t>(c->hidden_size) * M / 8 > 4 * 512 || c->moe_intermediate_size / 8 > 8 * 32) return false;
  if (c->num_experts_per_tok * M > lg::kDecodeMaxTokens * 32) return false;
  if (!aligned(w->gate_scale, 16) || !aligned(w->up_scale, 16) || !aligned(w->down_scale, 16)) return false;
  if (w->gate_scale_stride % 16 || w->up_scale_stride % 16 || w->down_scale_stride % 16) return false;
  StreamPlan P;
  const int TT = M <= 1 ? 1 : M <= 2 ? 2 : 4;
  return plan_stream(c, static_cast<int>(M), TT, &P);
}

template <int TT>
int launch_decode_t(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M, float* out,
                    float* wts, uint32_t* idx, void* ws, const Layout& L, bool x_host, int slot, cudaStream_t s) {
  using namespace lg;
  const int d = c->hidden_size, F = c->moe_intermediate_size, E = c->n_routed_experts, k = c->num_experts_per_tok;
  const int Fs = F * c->n_shared_experts;
  StreamPlan P;
  if (!plan_stream(c, M, TT, &P)) return fail(LG_ERR_UNSUPPORTED, "decode chain does not fit in shared memory");
  DecodeArgs a{};
  a.M = M; a.d = d; a.F = F; a.Fs = Fs; a.E = E; a.k = k; a.G = c->n_group; a.g = c->topk_group;
  a.norm = c->norm_topk_prob; a.scale = c->routed_scaling_factor; a.limit = c->swiglu_limit;
  a.x = x; a.Wr = w->router_weight; a.bias = w->router_bias;
  a.gate_p = w->gate_packed; a.gate_s = w->gate_scale; a.up_p = w->up_packed; a.up_s = w->up_scale;
  a.down_p = w->down_packed; a.down_s = w->down_scale;
  a.gate_ps = w->gate_packed_stride; a.gate_ss = w->gate_scale_stride;
  a.up_ps = w->up_packed_stride; a.up_ss = w->up_scale_stride;
  a.down_ps = w->down_packed_stride; a.down_ss = w->down_scale_stride;
  a.sh_gate = w->shared_gate; a.sh_up = w->shared_up; a.sh_down = w->shared_down;
  a.logits = at<float>(ws, L.logits); a.weights = wts; a.indices = idx;
  a.counts = at<int>(ws, L.counts); a.offsets = at<int>(ws, L.offsets); a.perm = at<int>(ws, L.perm);
  a.active = at<int>(ws, L.active);
  a.act = at<uint16_t>(ws, L.act); a.act_s = at<uint16_t>(ws, L.act_s);
  a.y = at<uint16_t>(ws, L.y); a.ys = at<uint16_t>(ws, L.ys);
  a.tickets = at<unsigned>(ws, L.tickets); a.out = out;
  a.status = at<int>(ws, L.status);
  a.lpr_down = pick_lpr(F);
  const int n_tickets = d / kDnRowsRouted;
  const int sms = num_sms();
  const bool pdl = slot < 0;
  cudaError_t e;
  // 0. tokens in page-locked host memory: one read over the host link, into HBM
  if (x_host) {
    uint16_t* xs = at<uint16_t>(ws, L.xs);
    const int n16 = M * d / 8;
    const int blocks = std::min((n16 + 255) / 256, sms);
    e = launch_ex(stage_tokens_kernel, dim3(blocks), dim3(256), 0, s, pdl, reinterpret_cast<const uint4*>(x),
                  reinterpret_cast<uint4*>(xs), n16);
    if (e != cudaSuccess) return cuda_check(e, "token staging launch");
    a.x = xs;
  }
  // 1. router logits
  const size_t smem_rl = static_cast<size_t>(kRouterExperts) * d * 4;
  occupancy(router_logits_decode_kernel<TT>, kRouterExperts * 32, smem_rl);
  e = launch_ex(router_logits_decode_kernel<TT>, dim3((E + kRouterExperts - 1) / kRouterExperts),
                dim3(kRouterExperts * 32), smem_rl, s, pdl, a);
  if (e != cudaSuccess) return cuda_check(e, "router logits launch");
  // 2. select + dispatch
  const int G = c->n_group;
  const size_t smem_sel = (2 * E + 3 * G) * 4 + G * 4 + kDecodeMaxTokens * 32 * 4 + 32 * 4 + (3 * E + 2) * 4;
  e = launch_ex(router_select_dispatch_kernel, dim3(1), dim3(256), smem_sel, s, pdl, a, n_tickets);
  if (e != cudaSuccess) return cuda_check(e, "router select launch");
  trace_mark(slot, 1, s);
  trace_mark(slot, 2, s);
  // 3. gate/up
  occupancy(gate_up_stream_kernel<TT>, kStreamThreads, P.gu_smem);
  e = launch_ex(gate_up_stream_kernel<TT>, dim3(sms), dim3(kStreamThreads), P.gu_smem, s, pdl, a, P.gu);
  if (e != cudaSuccess) return cuda_check(e, "gate/up launch");
  trace_mark(slot, 3, s);
  // 4. down + combine
  lg::down1::Cfg D1;
  lg::dtc::Cfg DT;
  size_t d1_smem = 0, dt_smem = 0;
  CUtensorMap tm_w, tm_s, tm_sh;
  if (TT == 1 && M == 1 && tc_down_enabled() && plan_down_tc(c, w, &DT, &dt_smem) &&
      map_bytes(&tm_w, w->down_packed, F / 2, static_cast<uint64_t>(E) * d, 128, true) &&
      map_bytes(&tm_s, w->down_scale, F / 32, static_cast<uint64_t>(E) * d, F / 32, false) &&
      (Fs == 0 ? map_bytes(&tm_sh, w->down_packed, F / 2, static_cast<uint64_t>(E) * d, 128, true)
               : map_bytes(&tm_sh, w->shared_down, static_cast<uint64_t>(Fs) * 2, d, 128, true))) {
    DT.bimg = at<uint8_t>(ws, L.bimg);
    DT.bsc = at<uint8_t>(ws, L.bsc);
    const int halves = M * k * DT.cols * 8;  // one half-warp per 32-value block
    e = launch_ex(lg::dtc::split_act_kernel, dim3((halves * 16 + 63) / 64), dim3(64), 0, s, pdl, a, DT);
    if (e != cudaSuccess) return cuda_check(e, "activation split launch");
    occupancy(lg::dtc::down_tc_kernel, lg::dtc::kThreads, dt_smem);
    e = launch_ex(lg::dtc::down_tc_kernel, dim3(sms), dim3(lg::dtc::kThreads), dt_smem, s, pdl, a, DT, tm_w, tm_s,
                  tm_sh);
  } else if (TT == 1 && M == 1 && plan_down1(c, &D1, &d1_smem)) {
    occupancy(lg::down1::down1_stream_kernel, lg::down1::kThreads, d1_smem);
    e = launch_ex(lg::down1::down1_stream_kernel, dim3(sms), dim3(lg::down1::kThreads), d1_smem, s, pdl, a, D1);
  } else {
    occupancy(down_stream_kernel<TT>, kStreamThreads, P.dn_smem);
    e = launch_ex(down_stream_kernel<TT>, dim3(sms), dim3(kStreamThreads), P.dn_smem, s, pdl, a, P.dn);
  }
  if (e != cudaSuccess) return cuda_check(e, "down launch");
  trace_mark(slot, 4, s);
  // 5. combine
  const int n4 = M * (d / 4);
  e = launch_ex(combine_decode_kernel, dim3((n4 + 255) / 256 < 2 * sms ? (n4 + 255) / 256 : 2 * sms), dim3(256), 0, s,
                pdl, a);
  if (e != cudaSuccess) return cuda_check(e, "combine launch");
  trace_mark(slot, 5, s);
  return LG_OK;
}

int launch_decode(const lg_moe_config* c, const lg_moe_weights* w, const uint16_t* x, int M, float* out,
                  float* wts, uint32_t* idx, void* ws, const Layout& L, bool x_host, int slot, cudaStream_t s) {
  if (M <= 1) return launch_decode_t<1>(c, w, x, M, out, wts, idx, ws, L, x_host, slot, s);
  if (M <= 2) return launch_decode_t<2>(c, w, x, M, out, wts, idx, ws, L, x_host, slot, s);
  return launch_decode_t<4>(c, w, x, M, out, wts, idx, ws, L, x_host, slot, s);
}

// ---- bounded-wait check ---------------------------------------------------------
// Runs the library's bounded waits, each with the given limit, against an
// mbarrier that never completes (initialised for one arrival that nobody
// makes) and a global flag that nothing sets: every wait must give up, record
// 6 | site in its status word and let the kernel return, leaving the context
// usable.  status[0]: the warp-wide wait of the streaming kernels (warp 0);
// status[1]: the hinted wait of the tensor-core kernels (warp 1, one lane);
// status[2]: the flag wait (warp 1, one lane); status[3]: the flag, zero.
__global__ void wait_timeout_kernel(unsigned long long limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    lg::mbar_init(&bar, 1);
    lg::mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    lg::mbar_wait_warp(&bar, 0, status, lg::kSiteSelfTestBar, limit_ns);
  } else if (threadIdx.x == 32) {
    lg::dtc::wait1(&bar, 0, status + 1, lg::kSiteSelfTestBar, limit_ns);
    lg::flag_wait(reinterpret_cast<const unsigned*>(status + 3), status + 2, lg::kSiteSelfTestFlag, limit_ns);
  }
}

// ---- stage tracing ------------------------------------------------------------
// When enabled, lg_moe_forward records a CUDA event before its first stage and
// after each stage (router, dispatch, gate/up, down, combine) into a ring of
// per-call slots, the device-side counterpart of the reference's trace spans
// (moe.py:97-197).  Not thread-safe; meant for measurement runs.
constexpr int kStages = 5;
struct Trace {
  int cap = 0, next = 0, recorded = 0;
  cudaEvent_t* ev = nullptr;  // cap * (kStages + 1)
};
Trace g_trace;

int trace_slot() {
  if (!g_trace.cap) return -1;
  const int slot = g_trace.next;
  g_trace.next = (g_trace.next + 1) % g_trace.cap;
  if (g_trace.recorded < g_trace.cap) ++g_trace.recorded;
  return slot;
}
void trace_mark(int slot, int i, cudaStream_t s) {
  if (slot < 0) return;
  cudaEvent_t ev = g_trace.ev[slot * (kStages + 1) + i];
  // Under stream capture a plain record becomes an internal graph edge; the
  // external flag makes each replay record the event where the host sees it.
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &st);
  if (st == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal);
  else cudaEventRecord(ev, s);
}

}  // namespace

// Sets this thread's lg_moe_last_error() message from other translation units
// of the library (not exported: hidden visibility).
__attribute__((visibility("hidden"))) int lg_internal_set_error(int code, const char* msg) {
  return fail(code, "%s", msg);
}

extern "C" {

int lg_moe_trace_enable(int capacity_calls) {
  if (g_trace.ev) {
    for (int i = 0; i < g_trace.cap * (kStages + 1); ++i) cudaEventDestroy(g_trace.ev[i]);
    delete[] g_trace.ev;
    g_trace = Trace{};
  }
  if (capacity_calls <= 0) return LG_OK;
  if (capacity_calls > (1 << 16)) return fail(LG_ERR_INVALID_ARG, "trace capacity too large");
  g_trace.ev = new cudaEvent_t[capacity_calls * (kStages + 1)];
  for (int i = 0; i < capacity_calls * (kStages + 1); ++i) {
    const cudaError_t e = cudaEventCreate(&g_trace.ev[i]);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(g_trace.ev[j]);
      delete[] g_trace.ev;
      g_trace = Trace{};
      return cuda_check(e, "trace event create");
    }
  }
  g_trace.cap = capacity_calls;
  return LG_OK;
}

int lg_moe_trace_read(float* stage_ms, int max_calls) {
  if (!stage_ms && max_calls > 0) return -fail(LG_ERR_INVALID_ARG, "trace: NULL output");
  const int n = g_trace.recorded < max_calls ? g_trace.recorded : max_calls;
  for (int c = 0; c < n; ++c) {
    const int slot = (g_trace.next - g_trace.recorded + c + g_trace.cap) % g_trace.cap;
    cudaEvent_t* e = g_trace.ev + slot * (kStages + 1);
    if (cudaEventSynchronize(e[kStages]) != cudaSuccess) return -fail(LG_ERR_CUDA, "trace: event sync failed");
    for (int i = 0; i < kStages; ++i) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, e[i], e[i + 1]) != cudaSuccess) ms = -1.f;
      stage_ms[c * kStages + i] = ms;
    }
  }
  return n;
}


int lg_moe_abi_version(void) { return LG_MOE_ABI_VERSION; }

int lg_moe_check_wait_timeout(int64_t limit_ns, int32_t* status, void* stream) {
  if (!status || !aligned(status, 16)) return fail(LG_ERR_INVALID_ARG, "wait check: status must be 16-byte aligned");
  if (limit_ns < 1000 || limit_ns > 2000000000LL)
    return fail(LG_ERR_INVALID_ARG, "wait check: limit %lld ns outside 1 us .. 2 s", static_cast<long long>(limit_ns));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(status, 0, 16, s);
  if (e != cudaSuccess) return cuda_check(e, "wait check memset");
  wait_timeout_kernel<<<1, 64, 0, s>>>(static_cast<unsigned long long>(limit_ns), status);
  return cuda_check(cudaGetLastError(), "wait check launch");
}

const char* lg_moe_last_error(void) { return g_err; }

size_t lg_moe_workspace_size(const lg_moe_config* cfg, int64_t max_tokens) {
  if (validate_cfg(cfg) || validate_tokens(max_tokens, cfg)) return 0;
  return layout(cfg, max_tokens).total;
}

int lg_moe_router(const lg_moe_config* cfg, const uint16_t* x, int64_t M, const float* router_weight,
                  const float* router_bias, float* logits, float* weights, uint32_t* indices,
                  void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if (!x || !router_weight || !router_bias || !weights || !indices)
    return fail(LG_ERR_INVALID_ARG, "router: NULL tensor pointer");
  if (!aligned(x, 16) || !aligned(router_weight, 16))
    return fail(LG_ERR_INVALID_ARG, "router: x and router_weight must be 16-byte aligned");
  if (!logits) {
    if ((rc = check_ws(cfg, M, workspace, workspace_bytes))) return rc;
    logits = at<float>(workspace, layout(cfg, M).logits);
  }
  return launch_router(cfg, x, static_cast<int>(M), router_weight, router_bias, logits, weights, indices,
                       nullptr, static_cast<cudaStream_t>(stream));
}

int lg_moe_dispatch(const lg_moe_config* cfg, const uint32_t* indices, int64_t M, int32_t* counts,
                    int32_t* offsets, int32_t* perm, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (!indices || !counts || !offsets || !perm) return fail(LG_ERR_INVALID_ARG, "dispatch: NULL pointer");
  if ((rc = check_ws(cfg, M, workspace, workspace_bytes))) return rc;
  const Layout L = layout(cfg, M);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0) {
    cudaMemsetAsync(counts, 0, cfg->n_routed_experts * sizeof(int), s);
    cudaMemsetAsync(offsets, 0, (cfg->n_routed_experts + 1) * sizeof(int), s);
    return cuda_check(cudaGetLastError(), "dispatch memset");
  }
  return launch_dispatch(cfg, indices, static_cast<int>(M), counts, offsets, perm,
                         at<int>(workspace, L.active), true, s);
}

int lg_moe_experts(const lg_moe_config* cfg, const lg_moe_weights* w, const uint16_t* x,
                   const uint32_t* indices, int64_t M, uint16_t* y, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if ((rc = validate_weights(cfg, w, true, false))) return rc;
  if (!x || !indices || !y) return fail(LG_ERR_INVALID_ARG, "experts: NULL tensor pointer");
  if (!aligned(x, 16) || !aligned(y, 16)) return fail(LG_ERR_INVALID_ARG, "experts: x and y must be 16-byte aligned");
  if ((rc = check_ws(cfg, M, workspace, workspace_bytes))) return rc;
  const Layout L = layout(cfg, M);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* counts = at<int>(workspace, L.counts);
  int* offsets = at<int>(workspace, L.offsets);
  int* perm = at<int>(workspace, L.perm);
  int* active = at<int>(workspace, L.active);
  if ((rc = launch_dispatch(cfg, indices, static_cast<int>(M), counts, offsets, perm, active, true, s))) return rc;
  if (L.tc && tc_batched_env() && tc_weights_fit(cfg, w, true, false))
    return launch_experts_tc(cfg, w, x, static_cast<int>(M), offsets, perm, workspace, L, y, nullptr, true, false, s);
  return launch_experts(cfg, w, x, static_cast<int>(M), offsets, perm, active, at<uint16_t>(workspace, L.act),
                        nullptr, y, nullptr, true, false, s);
}

int lg_moe_shared(const lg_moe_config* cfg, const lg_moe_weights* w, const uint16_t* x, int64_t M,
                  uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (cfg->n_shared_experts < 1) return fail(LG_ERR_INVALID_ARG, "shared: n_shared_experts is 0");
  if (M == 0) return LG_OK;
  if ((rc = validate_weights(cfg, w, false, true))) return rc;
  if (!x || !out) return fail(LG_ERR_INVALID_ARG, "shared: NULL tensor pointer");
  if (!aligned(x, 16)) return fail(LG_ERR_INVALID_ARG, "shared: x must be 16-byte aligned");
  if ((rc = check_ws(cfg, M, workspace, workspace_bytes))) return rc;
  const Layout L = layout(cfg, M);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* active = at<int>(workspace, L.active);
  if (L.tc && tc_batched_env())
    return launch_experts_tc(cfg, w, x, static_cast<int>(M), nullptr, nullptr, workspace, L, nullptr, out, false,
                             true, s);
  cudaMemsetAsync(active, 0, sizeof(int), s);
  return launch_experts(cfg, w, x, static_cast<int>(M), at<int>(workspace, L.offsets), at<int>(workspace, L.perm),
                        active, nullptr, at<uint16_t>(workspace, L.act_s), nullptr, out, false, true, s);
}

int lg_moe_combine(const lg_moe_config* cfg, const uint16_t* y, const float* weights, const uint16_t* shared,
                   int64_t M, float* out, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if (!y || !weights || !out) return fail(LG_ERR_INVALID_ARG, "combine: NULL tensor pointer");
  if (!aligned(y, 16) || !aligned(out, 16) || (shared && !aligned(shared, 16)))
    return fail(LG_ERR_INVALID_ARG, "combine: misaligned tensor");
  const int d = cfg->hidden_size;
  const long long n8 = M * (d / 8);
  const int grid = static_cast<int>(n8 / 256 + 1 < 8 * num_sms() ? n8 / 256 + 1 : 8 * num_sms());
  lg::combine_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      y, weights, shared, static_cast<int>(M), cfg->num_experts_per_tok, d, out);
  return cuda_check(cudaGetLastError(), "combine launch");
}

int lg_moe_combine_gather(const lg_moe_config* cfg, const uint16_t* y_disp, const int32_t* inv, const float* weights,
                          const uint16_t* shared, int64_t M, float* out, void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if (!y_disp || !inv || !weights || !out) return fail(LG_ERR_INVALID_ARG, "combine_gather: NULL tensor pointer");
  if (!aligned(y_disp, 16) || !aligned(out, 16) || (shared && !aligned(shared, 16)))
    return fail(LG_ERR_INVALID_ARG, "combine_gather: misaligned tensor");
  const int d = cfg->hidden_size;
  const long long n8 = M * (d / 8);
  const int grid = static_cast<int>(n8 / 256 + 1 < 8 * num_sms() ? n8 / 256 + 1 : 8 * num_sms());
  lg::combine_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      y_disp, weights, shared, static_cast<int>(M), cfg->num_experts_per_tok, d, out, inv);
  return cuda_check(cudaGetLastError(), "combine_gather launch");
}

int lg_moe_ep_pack(const lg_moe_config* cfg, const uint16_t* x, int64_t M, const uint32_t* indices,
                   const int32_t* perm, int32_t n_ranks, uint16_t* x_send, int32_t* e_send, int32_t* inv,
                   void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if (n_ranks < 1 || cfg->n_routed_experts % n_ranks)
    return fail(LG_ERR_INVALID_ARG, "ep_pack: %d experts do not split over %d ranks", cfg->n_routed_experts,
                n_ranks);
  if (!x || !indices || !perm || !x_send || !e_send || !inv) return fail(LG_ERR_INVALID_ARG, "ep_pack: NULL pointer");
  if (!aligned(x, 16) || !aligned(x_send, 16)) return fail(LG_ERR_INVALID_ARG, "ep_pack: rows must be 16-byte aligned");
  const int d = cfg->hidden_size, k = cfg->num_experts_per_tok;
  const long long R = M * k, n = R * (d / 8);
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, 8LL * num_sms()));
  lg::ep_pack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, indices, perm, static_cast<int>(R), k, d, cfg->n_routed_experts / n_ranks, x_send, e_send, inv);
  return cuda_check(cudaGetLastError(), "ep_pack launch");
}

int lg_fp8_block_dequant(const uint8_t* weight, const float* scale_inv, int64_t rows, int64_t cols, int32_t block,
                         uint16_t* out, int32_t* nonfinite, void* stream) {
  if (!weight || !scale_inv || !out || !nonfinite) return fail(LG_ERR_INVALID_ARG, "fp8 dequant: NULL pointer");
  if (rows < 1 || cols < 8 || block < 8 || block % 8 || rows % block || cols % block)
    return fail(LG_ERR_INVALID_ARG, "fp8 dequant: shape %lld x %lld not a multiple of block %d",
                static_cast<long long>(rows), static_cast<long long>(cols), block);
  if (!aligned(weight, 8) || !aligned(out, 16) || !aligned(scale_inv, 4))
    return fail(LG_ERR_INVALID_ARG, "fp8 dequant: misaligned tensor");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(nonfinite, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_check(e, "fp8 dequant memset");
  const long long n = rows * (cols / 8);
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, 8LL * num_sms()));
  lg::fp8_block_dequant_kernel<<<grid, 256, 0, s>>>(weight, scale_inv, rows, cols, block, out, nonfinite);
  return cuda_check(cudaGetLastError(), "fp8 dequant launch");
}

int lg_mx_requantize(const uint16_t* weight, int64_t rows, int64_t cols, int32_t bits, uint16_t* out, void* stream) {
  if (!weight || !out) return fail(LG_ERR_INVALID_ARG, "mx requantize: NULL pointer");
  if (bits != 4 && bits != 8) return fail(LG_ERR_INVALID_ARG, "mx requantize: bits %d not 4 or 8", bits);
  if (rows < 1 || cols < 32 || cols % 32) return fail(LG_ERR_INVALID_ARG, "mx requantize: cols %lld not a multiple of 32",
                                                      static_cast<long long>(cols));
  if (!aligned(weight, 16) || !aligned(out, 16)) return fail(LG_ERR_INVALID_ARG, "mx requantize: misaligned tensor");
  const long long groups = rows * (cols / 32);
  const int grid = static_cast<int>(std::min<long long>((groups + 255) / 256, 8LL * num_sms()));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bits == 8) lg::mx_requantize_kernel<8><<<grid, 256, 0, s>>>(weight, groups, out);
  else lg::mx_requantize_kernel<4><<<grid, 256, 0, s>>>(weight, groups, out);
  return cuda_check(cudaGetLastError(), "mx requantize launch");
}

int lg_moe_forward(const lg_moe_config* cfg, const lg_moe_weights* w, const uint16_t* x, int64_t M, float* out,
                   float* weights_out, uint32_t* indices_out, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int rc;
  if ((rc = validate_cfg(cfg)) || (rc = validate_tokens(M, cfg))) return rc;
  if (M == 0) return LG_OK;
  if ((rc = validate_weights(cfg, w, true, true))) return rc;
  if (!x || !out || !w->router_weight || !w->router_bias) return fail(LG_ERR_INVALID_ARG, "forward: NULL pointer");
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w->router_weight, 16))
    return fail(LG_ERR_INVALID_ARG, "forward: x, out and router_weight must be 16-byte aligned");
  if ((rc = check_ws(cfg, M, workspace, workspace_bytes))) return rc;
  // x and the outputs may be device memory or page-locked host memory (read
  // and written through the device mapping; host tokens are staged into HBM)
  bool x_host = false, host = false;
  {
    const void* p = nullptr;
    if ((rc = resolve(x, "forward: x", &p, &x_host))) return rc;
    x = static_cast<const uint16_t*>(p);
    if ((rc = resolve(out, "forward: out", &p, &host))) return rc;
    out = static_cast<float*>(const_cast<void*>(p));
    if (weights_out) {
      if ((rc = resolve(weights_out, "forward: weights_out", &p, &host))) return rc;
      weights_out = static_cast<float*>(const_cast<void*>(p));
    }
    if (indices_out) {
      if ((rc = resolve(indices_out, "forward: indices_out", &p, &host))) return rc;
      indices_out = static_cast<uint32_t*>(const_cast<void*>(p));
    }
  }
  const Layout L = layout(cfg, M);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int m = static_cast<int>(M);
  float* wts = weights_out ? weights_out : at<float>(workspace, L.weights);
  uint32_t* idx = indices_out ? indices_out : at<uint32_t>(workspace, L.indices);
  int* counts = at<int>(workspace, L.counts);
  int* offsets = at<int>(workspace, L.offsets);
  int* perm = at<int>(workspace, L.perm);
  int* active = at<int>(workspace, L.active);
  const int slot = trace_slot();
  trace_mark(slot, 0, s);
  if (decode_fits(cfg, w, M))
    return launch_decode(cfg, w, x, m, out, wts, idx, workspace, L, x_host, slot, s);
  if (x_host) {  // the other paths read x many times: one copy into HBM first
    uint16_t* xs = at<uint16_t>(workspace, L.xs);
    if ((rc = cuda_check(cudaMemcpyAsync(xs, x, static_cast<size_t>(M) * cfg->hidden_size * 2,
                                         cudaMemcpyDefault, s), "token staging copy")))
      return rc;
    x = xs;
  }
  if ((rc = cuda_check(cudaMemsetAsync(counts, 0, cfg->n_routed_experts * sizeof(int), s), "memset"))) return rc;
  if ((rc = launch_router(cfg, x, m, w->router_weight, w->router_bias, at<float>(workspace, L.logits), wts, idx,
                          counts, s)))
    return rc;
  trace_mark(slot, 1, s);
  if ((rc = launch_dispatch(cfg, idx, m, counts, offsets, perm, active, false, s))) return rc;
  trace_mark(slot, 2, s);
  uint16_t* act = at<uint16_t>(workspace, L.act);
  uint16_t* act_s = at<uint16_t>(workspace, L.act_s);
  uint16_t* y = at<uint16_t>(workspace, L.y);
  uint16_t* ys = cfg->n_shared_experts > 0 ? at<uint16_t>(workspace, L.ys) : nullptr;
  if (L.tc && tc_batched_env() && tc_weights_fit(cfg, w, true, true)) {
    if ((rc = launch_experts_tc(cfg, w, x, m, offsets, perm, workspace, L, y, ys, true, true, s, slot))) return rc;
  } else {
    if ((rc = launch_gate_up(cfg, w, x, m, offsets, perm, active, act, act_s, true, true, s))) return rc;
    trace_mark(slot, 3, s);
    if ((rc = launch_down(cfg, w, m, offsets, perm, active, act, act_s, y, ys, true, true, s))) return rc;
    trace_mark(slot, 4, s);
  }
  rc = lg_moe_combine(cfg, y, wts, ys, M, out, stream);
  trace_mark(slot, 5, s);
  return rc;
}

}  // extern "C"
