/*
 * livglm_moe.h -- C ABI of the B200-native GLM MoE block.
 *
 * One MoE block of GLM-5.3-Flash as in kg36/livglm: sigmoid router with
 * e_score_correction_bias and group-limited top-k, token-to-expert dispatch,
 * routed limited-SwiGLU experts read straight from the checkpoint's group-32
 * MXFP4 records, and the weighted combine with the shared expert added.
 *
 * Conventions
 *  - Every pointer argument is a DEVICE pointer unless its comment says
 *    "host".  bf16 tensors are passed as uint16_t bit patterns.
 *  - Every call is stream-ordered on `stream` (a cudaStream_t passed as
 *    void*; NULL is the legacy default stream), performs no host
 *    synchronisation and allocates no device memory: scratch comes from the
 *    caller's `workspace` (size from lg_moe_workspace_size), which must be
 *    256-byte aligned and must not be shared by calls that overlap on the GPU.
 *  - Return value: LG_OK (0) or an LG_ERR_* code; lg_moe_last_error() gives
 *    a message for the calling thread.  Argument errors are detected on the
 *    host before any launch and leave the stream untouched.
 *  - Device-side failures cannot be returned from a stream-ordered call: the
 *    first 4 bytes of the workspace are a status word that kernels set when a
 *    bounded wait gives up (LG_ERR_TIMEOUT in the low byte, the waiting site
 *    above it) or when a routing table holds an expert id outside [0, E)
 *    (LG_ERR_INVALID_ARG in the low byte).  Zero it once after allocating the
 *    workspace.  The library never clears it: it stays set until the caller
 *    clears it, so one read after a batch of calls reports any of them.
 *  - Routed expert tensors are banks: expert e's tensor starts at
 *    base + e * stride (bytes) and is byte-identical to the checkpoint's
 *      model.language_model.layers.{L}.mlp.experts.{e}.{gate,up}_proj.weight_packed  U8 [F, d/2]
 *      ...{gate,up}_proj.weight_scale   U8 [F, d/32]
 *      ...down_proj.weight_packed       U8 [d, F/2]
 *      ...down_proj.weight_scale        U8 [d, F/32]
 *    (kg36/livglm src/glm53flash/expert_source.py:189-229, contract.py:47-50).
 *    E2M1 nibbles: the low nibble of byte i is column 2i.  E8M0 scale s means
 *    2^(s-127); 255 is NaN.
 */
#ifndef LIVGLM_MOE_H
#define LIVGLM_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LG_MOE_ABI_VERSION 1

enum {
  LG_OK = 0,
  LG_ERR_INVALID_ARG = 1, /* bad shape, null pointer, misalignment */
  LG_ERR_UNSUPPORTED = 2, /* geometry outside what the kernels handle */
  LG_ERR_WORKSPACE = 3,   /* workspace missing or too small */
  LG_ERR_CUDA = 4,        /* a CUDA launch or runtime call failed */
  LG_ERR_NCCL = 5,        /* a collective failed */
  LG_ERR_TIMEOUT = 6      /* a bounded device wait gave up */
};

/* MoE geometry; field names follow GLMTextConfig
 * (kg36/livglm src/glm53flash/model_config.py:11-54). */
typedef struct lg_moe_config {
  int32_t hidden_size;           /* d */
  int32_t moe_intermediate_size; /* F, width of one routed expert */
  int32_t n_routed_experts;      /* E */
  int32_t num_experts_per_tok;   /* k */
  int32_t n_shared_experts;      /* shared width Fs = F * n_shared_experts */
  int32_t n_group;               /* G */
  int32_t topk_group;            /* g */
  int32_t norm_topk_prob;        /* 0 or 1 */
  float routed_scaling_factor;
  float swiglu_limit; /* <= 0 disables the clamp (expert_ssd.py:103-107) */
} lg_moe_config;

/* Resident weights of one MoE layer (all device pointers). */
typedef struct lg_moe_weights {
  const float *router_weight; /* mlp.gate.weight                 f32 [E, d] */
  const float *router_bias;   /* mlp.gate.e_score_correction_bias f32 [E] */
  const uint8_t *gate_packed, *gate_scale;
  const uint8_t *up_packed, *up_scale;
  const uint8_t *down_packed, *down_scale;
  int64_t gate_packed_stride, gate_scale_stride; /* bytes between experts */
  int64_t up_packed_stride, up_scale_stride;
  int64_t down_packed_stride, down_scale_stride;
  const uint16_t *shared_gate; /* mlp.shared_experts.gate_proj.weight bf16 [Fs, d] */
  const uint16_t *shared_up;   /* mlp.shared_experts.up_proj.weight   bf16 [Fs, d] */
  const uint16_t *shared_down; /* mlp.shared_experts.down_proj.weight bf16 [d, Fs] */
} lg_moe_weights;

int lg_moe_abi_version(void);

/* Message for the last failed call on this thread ("" if none). */
const char *lg_moe_last_error(void);

/* Bytes of scratch one call needs for up to `max_tokens` tokens
 * (router, dispatch, experts, forward all fit in this size). 0 on error. */
size_t lg_moe_workspace_size(const lg_moe_config *cfg /* host */, int64_t max_tokens);

/*
 * Router.  Replaces TopKRouter.__call__ (kg36/livglm src/glm53flash/moe.py:36-63).
 *   x       bf16 [M, d]
 *   logits  f32  [M, E]   (may be NULL)
 *   weights f32  [M, k]   normalised, scaled route weights
 *   indices u32  [M, k]   ascending choice order, best expert last (moe.py:58)
 */
int lg_moe_router(const lg_moe_config *cfg, const uint16_t *x, int64_t M,
                  const float *router_weight, const float *router_bias,
                  float *logits, float *weights, uint32_t *indices,
                  void *workspace, size_t workspace_bytes, void *stream);

/*
 * Dispatch.  Replaces the first-occurrence compaction of routed ids
 * (expert_ssd.py:162-170) and the native route plan's unique/compact mapping
 * (native_expert_ssd.py:475-525) with a stable counting sort of the route
 * slots s = t*k + j by expert id:
 *   counts  i32 [E]      routes per expert
 *   offsets i32 [E + 1]  exclusive prefix sum, offsets[E] = M*k
 *   perm    i32 [M*k]    perm[offsets[e] + r] = r-th slot (increasing) routed to e
 * Route slots whose index is >= E are skipped: they are not counted, do not
 * appear in perm, and (in lg_moe_experts) their output rows stay unwritten.
 */
int lg_moe_dispatch(const lg_moe_config *cfg, const uint32_t *indices, int64_t M,
                    int32_t *counts, int32_t *offsets, int32_t *perm,
                    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Routed experts.  Replaces the expert backend call
 * ExpertSSD.__call__(x, indices) -> [M, k, d] (expert_ssd.py:159-188) and the
 * native pair QMV + masked QMV (native_expert_ssd.py:698-712):
 *   y[t, j] = down_e( limited_swiglu( gate_e(x_t), up_e(x_t) ) ), e = indices[t, j]
 * with bf16 results for gate, up, every SwiGLU op and down.
 *   x bf16 [M, d]; indices u32 [M, k]; y bf16 [M, k, d]
 */
int lg_moe_experts(const lg_moe_config *cfg, const lg_moe_weights *w,
                   const uint16_t *x, const uint32_t *indices, int64_t M,
                   uint16_t *y, void *workspace, size_t workspace_bytes,
                   void *stream);

/*
 * Shared expert.  Replaces DenseMLP.__call__ with bf16 weights
 * (layers.py:66-67, 160-171): out = down(limited_swiglu(gate(x), up(x))), bf16.
 *   x bf16 [M, d]; out bf16 [M, d]
 */
int lg_moe_shared(const lg_moe_config *cfg, const lg_moe_weights *w,
                  const uint16_t *x, int64_t M, uint16_t *out,
                  void *workspace, size_t workspace_bytes, void *stream);

/*
 * Combine.  Replaces the merge of ExpertSSDMoE._call_impl (moe.py:199-201):
 *   out[t] = sum_j f32(y[t, j]) * weights[t, j]  (+ f32(shared[t]))
 * summed in j order; shared may be NULL.  out f32 [M, d].
 */
int lg_moe_combine(const lg_moe_config *cfg, const uint16_t *y,
                   const float *weights, const uint16_t *shared, int64_t M,
                   float *out, void *stream);

/* Expert parallelism (no counterpart in the reference, whose experts stream
 * from SSD on one device; the multi-GPU form of ExpertSSDMoE.__call__,
 * moe.py:96-201).  The exchange itself runs on the caller's NCCL group.
 *
 * lg_moe_ep_pack: for the route slots sorted by expert id (perm from
 * lg_moe_dispatch; sorted by expert is also sorted by owning rank when rank
 * r owns experts [r*E/n_ranks, (r+1)*E/n_ranks)), write the send buffers of
 * the dispatch exchange: x_send[p] = x[perm[p] / k] (bf16 [M*k, d]),
 * e_send[p] = indices[perm[p]] % (E / n_ranks) (int32 [M*k], the expert id
 * local to its owner) and inv[perm[p]] = p (int32 [M*k]). */
int lg_moe_ep_pack(const lg_moe_config *cfg, const uint16_t *x, int64_t M,
                   const uint32_t *indices, const int32_t *perm, int32_t n_ranks,
                   uint16_t *x_send, int32_t *e_send, int32_t *inv, void *stream);

/* lg_moe_combine with the routed outputs in dispatch order (as the reverse
 * exchange returns them): the output of route slot s is row inv[s] of
 * y_disp.  Same arithmetic and order as lg_moe_combine. */
int lg_moe_combine_gather(const lg_moe_config *cfg, const uint16_t *y_disp,
                          const int32_t *inv, const float *weights,
                          const uint16_t *shared, int64_t M, float *out,
                          void *stream);

/* Checkpoint loading: block-FP8 weights to bf16, the resident plan's
 * block_fp8_to_bf16 transform for the shared expert (fp8.py:43-78,
 * resident_plan.py:177-220).  weight: E4M3FN bytes [rows, cols] (device);
 * scale_inv: f32 [rows/block, cols/block] (device); out: bf16 [rows, cols]
 * (device), out = bf16_rn(e4m3fn(w) * scale) with the product in f32;
 * *nonfinite (device int32) receives the number of non-finite products (the
 * reference refuses such a checkpoint).  rows and cols multiples of block,
 * block a multiple of 8. */
int lg_fp8_block_dequant(const uint8_t *weight, const float *scale_inv,
                         int64_t rows, int64_t cols, int32_t block,
                         uint16_t *out, int32_t *nonfinite, void *stream);

/* Resident-linear quantisation (layers.py:67-104: mx.quantize with group
 * size 32, mode "mxfp8" (bits 8) or "mxfp4" (bits 4)) of a bf16 [rows, cols]
 * matrix: per 32-value group the shared exponent floor(log2 amax) - emax
 * (8 for E4M3, 2 for E2M1), elements rounded to nearest even and saturated;
 * out (bf16, may equal weight) holds the quantised values, which bf16 holds
 * exactly.  cols % 32 == 0. */
int lg_mx_requantize(const uint16_t *weight, int64_t rows, int64_t cols,
                     int32_t bits, uint16_t *out, void *stream);

/*
 * Whole block.  Replaces ExpertSSDMoE.__call__ (moe.py:96-201) for bf16
 * hidden states: returns the f32 merge the MLX graph produces.
 *   x bf16 [M, d]; out f32 [M, d]
 *   weights_out f32 [M, k] and indices_out u32 [M, k] may be NULL; when given
 *   they receive the router's outputs (the reference's last_route record).
 *   x, out, weights_out and indices_out may each be device memory of the
 *   current device, managed memory, or page-locked host memory
 *   (cudaHostAlloc / cudaHostRegister) mapped for the current device: the
 *   reference's hidden states live in unified memory, and a caller whose
 *   tokens sit on the host passes them as they are.  Host tokens are read
 *   once over the host link into the workspace; host outputs are written in
 *   place by the kernels.  Pageable host memory or another device's memory
 *   returns LG_ERR_INVALID_ARG.
 */
int lg_moe_forward(const lg_moe_config *cfg, const lg_moe_weights *w,
                   const uint16_t *x, int64_t M, float *out,
                   float *weights_out, uint32_t *indices_out,
                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Whole block without a workspace.  No counterpart in the reference.
 * For callers that cannot allocate device memory when they run the block
 * (a host framework that owns all device memory and gives plugins no
 * allocator, a decode loop where cudaMalloc could synchronise the device,
 * code holding a lock the allocator also takes): same arguments and result
 * as lg_moe_forward, but the scratch lives in a fixed 4 MiB device array
 * inside the library, so this call performs no cudaMalloc/cudaFree and no
 * other allocation.
 *  - Limit: M must fit in 4 MiB of scratch (lg_moe_workspace_size(cfg, M)
 *    <= 4194304; about 37 tokens at d=4096, E=128, k=8, F=1536); larger M
 *    returns LG_ERR_UNSUPPORTED with a message saying so.
 *  - The first call on a device resolves the array's device address for the
 *    current device (cudaGetSymbolAddress); make that first call before any
 *    stream capture.  The current device must own `stream` and the tensors.
 *  - Every call on a device shares the one array and it keeps the last
 *    call's contents; calls that overlap on the GPU (different streams, or
 *    threads without ordering) race on it.  Each call zeroes what must start
 *    at zero for that call itself.  The array's first 4 bytes are the status
 *    word of the workspace convention above: no call clears it, and since the
 *    array is private, read and clear it with lg_moe_static_scratch_status.
 *  - The array occupies 4 MiB on every GPU where the library's device code
 *    is loaded, until the process exits.  The resolved address is cached per
 *    device for the life of the process, so a cudaDeviceReset between calls
 *    is not supported.
 */
int lg_moe_forward_static_scratch(const lg_moe_config *cfg, const lg_moe_weights *w,
                                  const uint16_t *x, int64_t M, float *out,
                                  float *weights_out, uint32_t *indices_out,
                                  void *stream);

/*
 * Status word of the fixed scratch used by lg_moe_forward_static_scratch on
 * the current device.  No counterpart in the reference.  Waits for `stream`,
 * copies the word into *status_out (host) and, if `clear` is nonzero, zeroes
 * it.  0 means no device-side failure since the last clear.  Allocates
 * nothing.
 */
int lg_moe_static_scratch_status(int clear, int32_t *status_out, void *stream);

/*
 * Check of the device-side failure reporting.  No counterpart in the
 * reference (its waits are host-side MLX evaluations).  Launches one kernel
 * whose bounded waits (the same wait routines the MoE kernels use, with a
 * limit of `limit_ns`, 1 us .. 2 s) wait on an mbarrier that never completes
 * and on a flag that nothing sets: they give up after the limit and the
 * kernel returns, the context staying usable.  status: device, 16-byte
 * aligned, four int32 words, zeroed here first; afterwards status[0] (the
 * warp-wide wait of the streaming kernels) and status[1] (the hinted wait of
 * the tensor-core kernels) hold LG_ERR_TIMEOUT | 30 << 8, status[2] (a flag
 * wait) LG_ERR_TIMEOUT | 31 << 8, and status[3] is the flag, still 0.
 */
int lg_moe_check_wait_timeout(int64_t limit_ns, int32_t *status, void *stream);

/*
 * Stage tracing.  Counterpart of the reference's per-layer trace spans
 * (DecodeTrace spans "router_graph_construct", "moe_merge_graph_construct",
 * moe.py:97-197; trace.py:43-310), measured on the device: while enabled,
 * every lg_moe_forward records CUDA events around its five stages (router,
 * dispatch, gate/up, down, combine) into a ring of `capacity_calls` slots
 * (works inside CUDA graph capture; a replay re-records the captured slot).
 * capacity_calls <= 0 disables tracing.  Process-wide, not thread-safe.
 */
int lg_moe_trace_enable(int capacity_calls);

/* Copies up to max_calls recorded calls, oldest first, as
 * stage_ms[call * 5 + stage] (milliseconds).  Waits for the events.  Returns
 * the number of calls copied, or a negative LG_ERR_* code. */
int lg_moe_trace_read(float *stage_ms /* host */, int max_calls);

/*
 * FFN site of a MoE decoder layer with manifold-constrained hyper-connections
 * (kg36/livglm src/glm53flash/model.py:132-136; the width-two MTP verify,
 * runtime.py:657-661, calls it with two tokens):
 *   post, comb, collapsed = ffn_hc(streams)          (HyperConnection, mhc.py:23-48)
 *   x   = post_attention_layernorm(collapsed)        (RMSNorm, layers.py:119-131)
 *   out = hyper_residual(streams, moe(x), post, comb) (mhc.py:51-60)
 * streams: bf16 [M, hc, d], the hc residual streams of M tokens.  Rounding
 * points are MLX's for bf16 streams: the mix and gates in f32, collapsed
 * cast to bf16, rms_norm's normalised value rounded to bf16 before and after
 * the weight, bf16(post) * moe(x) in f32 plus the bf16 matmul comb^T @ streams.
 */
typedef struct lg_hc_config {
  int32_t hc_mult;        /* streams per token, 1..4 (GLMTextConfig.hc_mult) */
  int32_t sinkhorn_iters; /* hc_sinkhorn_iters, >= 1 */
  float hc_eps;
  float rms_norm_eps;
} lg_hc_config;

typedef struct lg_hc_weights {
  const float *fn;             /* layers.{L}.hc_ffn_fn    f32 [hc*(hc+2), hc*d] */
  const float *base;           /* layers.{L}.hc_ffn_base  f32 [hc*(hc+2)] */
  const float *scale;          /* layers.{L}.hc_ffn_scale f32 [3] */
  const uint16_t *norm_weight; /* layers.{L}.post_attention_layernorm.weight bf16 [d] */
} lg_hc_weights;

/* Scratch of lg_hc_pre for up to max_tokens tokens (0 on error). */
size_t lg_hc_workspace_size(const lg_hc_config *hc /* host */, int32_t d, int64_t max_tokens);

/* HyperConnection.__call__ (mhc.py:23-48) and, when x_norm is not NULL,
 * the post-attention RMSNorm of its collapsed output (layers.py:126-131).
 *   post f32 [M, hc]; comb f32 [M, hc, hc]; collapsed bf16 [M, d] (may be
 *   NULL); x_norm bf16 [M, d] (may be NULL; needs w->norm_weight). */
int lg_hc_pre(const lg_hc_config *hc, const lg_hc_weights *w, int32_t d, const uint16_t *streams, int64_t M,
              float *post, float *comb, uint16_t *collapsed, uint16_t *x_norm, void *workspace,
              size_t workspace_bytes, void *stream);

/* hyper_residual (mhc.py:51-60): residual bf16 [M, hc, d], sublayer f32
 * [M, d] (the MoE output), post / comb from lg_hc_pre -> out f32 [M, hc, d]. */
int lg_hc_post(const lg_hc_config *hc, int32_t d, const uint16_t *residual, const float *sublayer,
               const float *post, const float *comb, int64_t M, float *out, void *stream);

/* Workspace of lg_moe_ffn_site (its first 4 bytes are the MoE status word). */
size_t lg_moe_ffn_site_workspace_size(const lg_moe_config *cfg /* host */, const lg_hc_config *hc /* host */,
                                      int64_t max_tokens);

/* The whole FFN site: lg_hc_pre, lg_moe_forward on the normalised collapsed
 * rows, lg_hc_post.  out f32 [M, hc, d]; weights_out / indices_out as in
 * lg_moe_forward. */
int lg_moe_ffn_site(const lg_moe_config *cfg, const lg_moe_weights *w, const lg_hc_config *hc,
                    const lg_hc_weights *hw, const uint16_t *streams, int64_t M, float *out, float *weights_out,
                    uint32_t *indices_out, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LIVGLM_MOE_H */
