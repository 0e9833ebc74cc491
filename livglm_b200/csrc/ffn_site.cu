// FFN site of a GLM MoE decoder layer: manifold-constrained hyper-connections
// around the MoE block (kg36/livglm src/glm53flash/model.py:132-136):
//
//   post, comb, collapsed = ffn_hc(streams)                  mhc.py:23-48
//   x   = post_attention_layernorm(collapsed)                layers.py:119-131
//   out = hyper_residual(streams, moe(x), post, comb)        mhc.py:51-60
//
// streams are bf16 [M, hc, d] (M tokens, hc residual streams each).  Three
// small kernels around lg_moe_forward:
//   hc_mix_kernel     partial dot products of every token's hc*d streams with
//                     the hc*(hc+2) rows of fn, and partial sums of squares,
//                     per 256-element slice (fn is read once per token pair);
//   hc_finish_kernel  one CTA per token: the partials (fixed order), the
//                     unweighted RMS factor, pre / post gates, the Sinkhorn-
//                     normalised comb matrix, collapsed = sum_h pre_h * stream_h
//                     (bf16), and the weighted RMSNorm of collapsed (bf16);
//   hc_post_kernel    out = bf16(post) * moe_out + bf16(bf16(comb)^T @ streams).
// All bound by launch latency at decode widths (under 1.6 MB of fn, 64 KB of
// streams at hc = 4, d = 4096, two tokens).

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>

#include "livglm_moe.h"

int lg_internal_set_error(int code, const char* msg);

namespace {

int fail(int code, const char* fmt, ...) {
  char msg[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof msg, fmt, ap);
  va_end(ap);
  return lg_internal_set_error(code, msg);
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LG_OK;
  return fail(LG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr int kMaxHc = 4;
constexpr int kSlice = 256;                      // fn columns per mix CTA
constexpr int kMixThreads = 128;
constexpr int kTokTile = 2;                      // tokens per mix CTA
constexpr size_t kAlign = 256;
size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t to_bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float round_bf(float f) { return bf(to_bf(f)); }

// partial[(t * S + s) * (R + 1) + r]: sum over slice s of streams[t] * fn[r]
// (r < R) and of streams[t]^2 (r = R).
template <int HC>
__global__ void __launch_bounds__(kMixThreads) hc_mix_kernel(const uint16_t* __restrict__ streams,
                                                             const float* __restrict__ fn, int M, int K,
                                                             float* __restrict__ partial) {
  constexpr int R = HC * (HC + 2);
  constexpr int V = R + 1;
  const int s = blockIdx.x, S = gridDim.x;
  const int t0 = blockIdx.y * kTokTile;
  float acc[kTokTile][V];
#pragma unroll
  for (int a = 0; a < kTokTile; ++a)
#pragma unroll
    for (int v = 0; v < V; ++v) acc[a][v] = 0.f;
  const int k_end = min(K, (s + 1) * kSlice);
  for (int k = s * kSlice + threadIdx.x; k < k_end; k += kMixThreads) {
    float xv[kTokTile];
#pragma unroll
    for (int a = 0; a < kTokTile; ++a) {
      xv[a] = t0 + a < M ? bf(streams[static_cast<size_t>(t0 + a) * K + k]) : 0.f;
      acc[a][R] = fmaf(xv[a], xv[a], acc[a][R]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float f = fn[static_cast<size_t>(r) * K + k];
#pragma unroll
      for (int a = 0; a < kTokTile; ++a) acc[a][r] = fmaf(xv[a], f, acc[a][r]);
    }
  }
  __shared__ float red[kMixThreads / 32][kTokTile][V];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int a = 0; a < kTokTile; ++a)
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float x = acc[a][v];
#pragma unroll
      for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) red[warp][a][v] = x;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < kTokTile * V; i += kMixThreads) {
    const int a = i / V, v = i % V;
    if (t0 + a >= M) continue;
    float x = 0.f;
#pragma unroll
    for (int w = 0; w < kMixThreads / 32; ++w) x += red[w][a][v];
    partial[(static_cast<size_t>(t0 + a) * S + s) * V + v] = x;
  }
}

__device__ __forceinline__ float sigmoidf(float z) { return 1.f / (1.f + expf(-z)); }

__device__ float block_sum(float x, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  __syncthreads();
  if (lane == 0) sh[warp] = x;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s += sh[w];
  return s;
}

constexpr int kFinishThreads = 1024;
constexpr int kMaxHidden = 16384;  // collapsed row staged in shared memory (32 KB)

template <int HC>
__global__ void __launch_bounds__(kFinishThreads) hc_finish_kernel(const float* __restrict__ partial, int S, int d,
                                                        const uint16_t* __restrict__ streams,
                                                        const float* __restrict__ base,
                                                        const float* __restrict__ scale,
                                                        const uint16_t* __restrict__ norm_weight, int iters,
                                                        float hc_eps, float rms_eps, float* __restrict__ post,
                                                        float* __restrict__ comb, uint16_t* __restrict__ collapsed,
                                                        uint16_t* __restrict__ x_norm) {
  constexpr int R = HC * (HC + 2);
  constexpr int V = R + 1;
  const int t = blockIdx.x;
  const int K = HC * d;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float red[8][V];
  __shared__ float mixed[V];
  __shared__ float pre[HC];
  __shared__ float cm[HC * HC];
  __shared__ float sh[32];
  // the slice partials: warp w < 8 sums slices w, w + 8, ... (eight loads in
  // flight per lane), then the eight warp sums in warp order
  if (warp < 8 && lane < V) {
    float acc = 0.f;
    for (int s0 = warp; s0 < S; s0 += 64) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int s = s0 + 8 * j;
        v[j] = s < S ? partial[(static_cast<size_t>(t) * S + s) * V + lane] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc += v[j];
    }
    red[warp][lane] = acc;
  }
  __syncthreads();
  if (threadIdx.x < V) {
    float x = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) x += red[w][threadIdx.x];
    mixed[threadIdx.x] = x;
  }
  __syncthreads();
  if (warp == 0) {
    // UnweightedRMSNorm of the flattened streams scales every dot product
    const float inv = 1.f / sqrtf(mixed[R] / static_cast<float>(K) + rms_eps);
    if (lane < HC) {
      pre[lane] = sigmoidf(mixed[lane] * inv * scale[0] + base[lane]) + hc_eps;
      post[static_cast<size_t>(t) * HC + lane] = 2.f * sigmoidf(mixed[HC + lane] * inv * scale[1] + base[HC + lane]);
    }
    // comb: lane i*HC + j holds element (i, j); row and column sums run in
    // index order through shared memory
    const bool act = lane < HC * HC;
    const int i = act ? lane / HC : 0, j = act ? lane % HC : 0;
    float c = act ? mixed[2 * HC + lane] * inv * scale[2] + base[2 * HC + lane] : 0.f;
    if (act) cm[lane] = c;
    __syncwarp();
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < HC; ++q) mx = fmaxf(mx, cm[i * HC + q]);
    const float e = act ? expf(c - mx) : 0.f;
    __syncwarp();
    if (act) cm[lane] = e;
    __syncwarp();
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < HC; ++q) sum += cm[i * HC + q];
    c = e / sum + hc_eps;
    for (int it = 0; it < iters; ++it) {
      if (it > 0) {  // rows, then columns, each iteration after the first
        __syncwarp();
        if (act) cm[lane] = c;
        __syncwarp();
        sum = 0.f;
#pragma unroll
        for (int q = 0; q < HC; ++q) sum += cm[i * HC + q];
        c = c / (sum + hc_eps);
      }
      __syncwarp();
      if (act) cm[lane] = c;
      __syncwarp();
      sum = 0.f;
#pragma unroll
      for (int q = 0; q < HC; ++q) sum += cm[q * HC + j];
      c = c / (sum + hc_eps);
    }
    if (act) comb[static_cast<size_t>(t) * HC * HC + lane] = c;
  }
  __syncthreads();
  // collapsed = sum_h pre_h * stream_h, rounded to bf16 and kept in shared
  // memory; then RMSNorm with weight.  Four elements per thread in flight.
  extern __shared__ uint16_t col[];  // [d]
  const uint16_t* st = streams + static_cast<size_t>(t) * K;
  float ss = 0.f;
  for (int i0 = threadIdx.x; i0 < d; i0 += 4 * blockDim.x) {
    float v[4][HC];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
#pragma unroll
      for (int h = 0; h < HC; ++h) v[u][h] = i < d ? bf(st[static_cast<size_t>(h) * d + i]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= d) break;
      float c = __fmul_rn(pre[0], v[u][0]);
#pragma unroll
      for (int h = 1; h < HC; ++h) c = __fadd_rn(c, __fmul_rn(pre[h], v[u][h]));
      const uint16_t cb = to_bf(c);
      col[i] = cb;
      if (collapsed) collapsed[static_cast<size_t>(t) * d + i] = cb;
      ss = fmaf(bf(cb), bf(cb), ss);
    }
  }
  if (!x_norm) return;
  const float n = 1.f / sqrtf(block_sum(ss, sh) / static_cast<float>(d) + rms_eps);  // syncs: col is complete
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float y = round_bf(__fmul_rn(bf(col[i]), n));
    x_norm[static_cast<size_t>(t) * d + i] = to_bf(__fmul_rn(bf(norm_weight[i]), y));
  }
}

// out[t, h, i] = bf16(post[t, h]) * sub[t, i] + bf16(sum_g bf16(comb[t, g, h]) * res[t, g, i])
template <int HC>
__global__ void __launch_bounds__(256) hc_post_kernel(const uint16_t* __restrict__ res, const float* __restrict__ sub,
                                                      const float* __restrict__ post, const float* __restrict__ comb,
                                                      int M, int d, float* __restrict__ out) {
  const long long n = static_cast<long long>(M) * d;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / d), i = static_cast<int>(e % d);
    const uint16_t* rt = res + static_cast<size_t>(t) * HC * d;
    float r[HC];
#pragma unroll
    for (int g = 0; g < HC; ++g) r[g] = bf(rt[static_cast<size_t>(g) * d + i]);
    const float f = sub[e];
#pragma unroll
    for (int h = 0; h < HC; ++h) {
      float m = 0.f;
#pragma unroll
      for (int g = 0; g < HC; ++g) m = fmaf(round_bf(comb[(static_cast<size_t>(t) * HC + g) * HC + h]), r[g], m);
      const float placed = __fmul_rn(round_bf(post[static_cast<size_t>(t) * HC + h]), f);
      out[(static_cast<size_t>(t) * HC + h) * d + i] = __fadd_rn(placed, round_bf(m));
    }
  }
}

int validate_hc(const lg_hc_config* hc, int d) {
  if (!hc) return fail(LG_ERR_INVALID_ARG, "hyper-connection config is NULL");
  if (hc->hc_mult < 1 || hc->hc_mult > kMaxHc)
    return fail(LG_ERR_UNSUPPORTED, "hc_mult %d outside 1..%d", hc->hc_mult, kMaxHc);
  if (hc->sinkhorn_iters < 1 || hc->sinkhorn_iters > 1000)
    return fail(LG_ERR_INVALID_ARG, "hc_sinkhorn_iters %d outside 1..1000", hc->sinkhorn_iters);
  if (d < 2 || d > kMaxHidden) return fail(LG_ERR_UNSUPPORTED, "hidden size %d outside 2..%d", d, kMaxHidden);
  return LG_OK;
}

int slices(const lg_hc_config* hc, int d) { return (hc->hc_mult * d + kSlice - 1) / kSlice; }

size_t partial_bytes(const lg_hc_config* hc, int d, int64_t M) {
  const int R = hc->hc_mult * (hc->hc_mult + 2);
  return up(static_cast<size_t>(M) * slices(hc, d) * (R + 1) * sizeof(float));
}

template <int HC>
int launch_pre_t(const lg_hc_config* hc, const lg_hc_weights* w, int d, const uint16_t* streams, int M, float* post,
                 float* comb, uint16_t* collapsed, uint16_t* x_norm, float* partial, cudaStream_t s) {
  const int S = slices(hc, d);
  hc_mix_kernel<HC><<<dim3(S, (M + kTokTile - 1) / kTokTile), kMixThreads, 0, s>>>(streams, w->fn, M, HC * d, partial);
  hc_finish_kernel<HC><<<M, kFinishThreads, d * sizeof(uint16_t), s>>>(partial, S, d, streams, w->base, w->scale, w->norm_weight,
                                         hc->sinkhorn_iters, hc->hc_eps, hc->rms_norm_eps, post, comb, collapsed,
                                         x_norm);
  return cuda_check(cudaGetLastError(), "hyper-connection launch");
}

int launch_pre(const lg_hc_config* hc, const lg_hc_weights* w, int d, const uint16_t* streams, int M, float* post,
               float* comb, uint16_t* collapsed, uint16_t* x_norm, float* partial, cudaStream_t s) {
  switch (hc->hc_mult) {
    case 1: return launch_pre_t<1>(hc, w, d, streams, M, post, comb, collapsed, x_norm, partial, s);
    case 2: return launch_pre_t<2>(hc, w, d, streams, M, post, comb, collapsed, x_norm, partial, s);
    case 3: return launch_pre_t<3>(hc, w, d, streams, M, post, comb, collapsed, x_norm, partial, s);
    default: return launch_pre_t<4>(hc, w, d, streams, M, post, comb, collapsed, x_norm, partial, s);
  }
}

int launch_post(const lg_hc_config* hc, int d, const uint16_t* res, const float* sub, const float* post,
                const float* comb, int M, float* out, cudaStream_t s) {
  const long long n = static_cast<long long>(M) * d;
  const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, 4096));
  switch (hc->hc_mult) {
    case 1: hc_post_kernel<1><<<grid, 256, 0, s>>>(res, sub, post, comb, M, d, out); break;
    case 2: hc_post_kernel<2><<<grid, 256, 0, s>>>(res, sub, post, comb, M, d, out); break;
    case 3: hc_post_kernel<3><<<grid, 256, 0, s>>>(res, sub, post, comb, M, d, out); break;
    default: hc_post_kernel<4><<<grid, 256, 0, s>>>(res, sub, post, comb, M, d, out); break;
  }
  return cuda_check(cudaGetLastError(), "hyper-residual launch");
}

bool aligned(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

}  // namespace

extern "C" {

size_t lg_hc_workspace_size(const lg_hc_config* hc, int32_t d, int64_t max_tokens) {
  if (validate_hc(hc, d) || max_tokens < 1 || max_tokens > (1 << 24)) return 0;
  return partial_bytes(hc, d, max_tokens);
}

int lg_hc_pre(const lg_hc_config* hc, const lg_hc_weights* w, int32_t d, const uint16_t* streams, int64_t M,
              float* post, float* comb, uint16_t* collapsed, uint16_t* x_norm, void* workspace,
              size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate_hc(hc, d))) return rc;
  if (M < 0 || M > (1 << 24)) return fail(LG_ERR_INVALID_ARG, "hyper-connection: token count %lld", (long long)M);
  if (M == 0) return LG_OK;
  if (!w || !w->fn || !w->base || !w->scale || !streams || !post || !comb)
    return fail(LG_ERR_INVALID_ARG, "hyper-connection: NULL pointer");
  if (x_norm && !w->norm_weight) return fail(LG_ERR_INVALID_ARG, "hyper-connection: norm_weight is NULL");
  if (!workspace || !aligned(workspace, kAlign) || workspace_bytes < partial_bytes(hc, d, M))
    return fail(LG_ERR_WORKSPACE, "hyper-connection: workspace needs %zu bytes, 256-byte aligned",
                partial_bytes(hc, d, M));
  return launch_pre(hc, w, d, streams, static_cast<int>(M), post, comb, collapsed, x_norm,
                    static_cast<float*>(workspace), static_cast<cudaStream_t>(stream));
}

int lg_hc_post(const lg_hc_config* hc, int32_t d, const uint16_t* residual, const float* sublayer, const float* post,
               const float* comb, int64_t M, float* out, void* stream) {
  int rc;
  if ((rc = validate_hc(hc, d))) return rc;
  if (M < 0 || M > (1 << 24)) return fail(LG_ERR_INVALID_ARG, "hyper-residual: token count %lld", (long long)M);
  if (M == 0) return LG_OK;
  if (!residual || !sublayer || !post || !comb || !out) return fail(LG_ERR_INVALID_ARG, "hyper-residual: NULL pointer");
  return launch_post(hc, d, residual, sublayer, post, comb, static_cast<int>(M), out,
                     static_cast<cudaStream_t>(stream));
}

size_t lg_moe_ffn_site_workspace_size(const lg_moe_config* cfg, const lg_hc_config* hc, int64_t max_tokens) {
  if (!cfg || validate_hc(hc, cfg->hidden_size) || max_tokens < 1 || max_tokens > (1 << 24)) return 0;
  const size_t moe = lg_moe_workspace_size(cfg, max_tokens);
  if (!moe) return 0;
  const size_t M = max_tokens, d = cfg->hidden_size, H = hc->hc_mult;
  return up(moe) + partial_bytes(hc, cfg->hidden_size, max_tokens) + up(M * H * 4) + up(M * H * H * 4) +
         up(M * d * 2) + up(M * d * 4);
}

int lg_moe_ffn_site(const lg_moe_config* cfg, const lg_moe_weights* w, const lg_hc_config* hc,
                    const lg_hc_weights* hw, const uint16_t* streams, int64_t M, float* out, float* weights_out,
                    uint32_t* indices_out, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if (!cfg) return fail(LG_ERR_INVALID_ARG, "config is NULL");
  const int d = cfg->hidden_size;
  if ((rc = validate_hc(hc, d))) return rc;
  if (M < 0 || M > (1 << 24)) return fail(LG_ERR_INVALID_ARG, "ffn site: token count %lld", (long long)M);
  if (M == 0) return LG_OK;
  const size_t need = lg_moe_ffn_site_workspace_size(cfg, hc, M);
  if (!need) return LG_ERR_INVALID_ARG;  // the message is already set
  if (!workspace || !aligned(workspace, kAlign) || workspace_bytes < need)
    return fail(LG_ERR_WORKSPACE, "ffn site: workspace needs %zu bytes, 256-byte aligned", need);
  if (!out || !streams) return fail(LG_ERR_INVALID_ARG, "ffn site: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t H = hc->hc_mult;
  char* base = static_cast<char*>(workspace);
  const size_t moe = up(lg_moe_workspace_size(cfg, M));  // status word first
  size_t o = moe;
  float* partial = reinterpret_cast<float*>(base + o);
  o += partial_bytes(hc, d, M);
  float* post = reinterpret_cast<float*>(base + o);
  o += up(M * H * 4);
  float* comb = reinterpret_cast<float*>(base + o);
  o += up(M * H * H * 4);
  uint16_t* x = reinterpret_cast<uint16_t*>(base + o);
  o += up(static_cast<size_t>(M) * d * 2);
  float* ffn = reinterpret_cast<float*>(base + o);
  if ((rc = lg_hc_pre(hc, hw, d, streams, M, post, comb, nullptr, x, partial, partial_bytes(hc, d, M), stream)))
    return rc;
  if ((rc = lg_moe_forward(cfg, w, x, M, ffn, weights_out, indices_out, workspace, moe, stream))) return rc;
  return launch_post(hc, d, streams, ffn, post, comb, static_cast<int>(M), out, s);
}

}  // extern "C"
