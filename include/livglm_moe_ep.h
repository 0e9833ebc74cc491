/*
 * livglm_moe_ep.h -- C ABI of the expert-parallel MoE block (one call per
 * layer per rank), built as liblivglm_moe_ep.so over liblivglm_moe.so and
 * NCCL.
 *
 * No counterpart in the reference: kg36/livglm runs the block on one device
 * and streams experts from SSD (src/glm53flash/moe.py:96-201).  This is the
 * multi-GPU form of lg_moe_forward for batched work.  Rank r of W ranks
 * holds the routed experts r, r + W, r + 2W, ... (expert e lives on rank
 * e mod W as local expert e / W) and a replica of the router and the shared
 * expert; every rank brings its own token rows.  One lg_moe_ep_forward:
 *
 *   1. route the local rows (lg_moe_router), renumber the chosen experts to
 *      exchange ids (owner * E/W + local index) and sort the route slots by
 *      them (lg_moe_dispatch): slots grouped by destination rank, then by
 *      local expert; pack one bf16 row per slot (lg_moe_ep_pack);
 *   2. all-gather every rank's message (W + 2 int64: slots bound for each
 *      rank, its token count, a status word) and read the table on the host
 *      (the only host synchronisation of the call: NCCL's send/recv take
 *      host counts); every rank checks the whole table;
 *   3. send the rows and their local expert ids to their owners (NCCL
 *      send/recv on the communicator's own stream) while the shared expert
 *      runs on the caller's stream;
 *   4. run the received rows through the local experts (lg_moe_experts with
 *      top-1 over the E/W local experts);
 *   5. send the outputs back and merge them with the shared expert in the
 *      single-GPU combine's route order (lg_moe_combine_gather).
 *
 * The per-route arithmetic is the single-GPU kernels', so routing is
 * bit-identical to lg_moe_forward on the same rows and the output matches it
 * up to the batched kernels' rounding order.
 *
 * Conventions are those of livglm_moe.h (device pointers, bf16 as uint16_t,
 * LG_OK / LG_ERR_* return codes, status word in the first 4 bytes of the
 * workspace), except that lg_moe_ep_forward synchronises the host with
 * `stream` once (step 2) and so cannot be captured in a CUDA graph.
 *
 * Collective consistency: every rank must call lg_moe_ep_forward for the
 * same layer in the same order.  A rank whose arguments are bad (M above the
 * communicator's max_tokens, a null pointer, a small workspace) still takes
 * part in step 2 with a non-zero status, and then every rank returns
 * without further collectives (that rank its own error code, the others
 * LG_ERR_INVALID_ARG naming it).  A failure after step 2 on
 * one rank (a launch error) does not skip the remaining exchanges, so the
 * other ranks are not left waiting; the call returns the first error.  An
 * NCCL error returns LG_ERR_NCCL: abort the communicator
 * (lg_ep_comm_destroy) and build a new one.
 */
#ifndef LIVGLM_MOE_EP_H
#define LIVGLM_MOE_EP_H

#include "livglm_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lg_ep_comm lg_ep_comm;

/* Bytes of the opaque id that rank 0 creates and every rank passes to
 * lg_ep_comm_init (an NCCL unique id). */
int lg_ep_unique_id_bytes(void);

/* Rank 0 only: write a fresh id to `out` (host, lg_ep_unique_id_bytes()
 * bytes); the caller ships it to the other ranks (a store, a broadcast). */
int lg_ep_get_unique_id(void *out /* host */);

/* Join the communicator of `world` ranks as `rank` on the CURRENT device
 * (blocks until every rank has joined).  max_tokens bounds M of every
 * rank's lg_moe_ep_forward and so the rows one rank can receive
 * (world * max_tokens * k). */
int lg_ep_comm_init(const void *unique_id /* host */, int32_t world, int32_t rank,
                    int64_t max_tokens, lg_ep_comm **comm /* host out */);

/* Abort the NCCL communicator and free the communicator's stream, events
 * and host buffer.  NULL is a no-op. */
int lg_ep_comm_destroy(lg_ep_comm *comm);

/* Message for the last failed lg_ep_* / lg_moe_ep_* call on this thread. */
const char *lg_ep_last_error(void);

/* Workspace bytes of lg_moe_ep_forward on a communicator of `world` ranks
 * whose max_tokens is `max_tokens` (covers the worst case: every rank
 * sends all its route slots here).  0 on error. */
size_t lg_moe_ep_workspace_size(const lg_moe_config *cfg /* host */, int64_t max_tokens,
                                int32_t world);

/*
 * One expert-parallel MoE layer on this rank's rows.
 *   cfg          the full layer geometry (E = all routed experts)
 *   w            router and shared expert of the layer; routed banks holding
 *                only this rank's E/W experts, in the order rank, rank + W,
 *                rank + 2W, ... (strides as in livglm_moe.h)
 *   x            bf16 [M, d], 0 <= M <= max_tokens
 *   out          f32 [M, d]
 *   weights_out  f32 [M, k] route weights; indices_out uint32 [M, k] expert
 *                ids (global), as lg_moe_router writes them
 *   workspace    lg_moe_ep_workspace_size(cfg, max_tokens, world) bytes,
 *                256-byte aligned, status word zeroed once
 */
int lg_moe_ep_forward(lg_ep_comm *comm, const lg_moe_config *cfg, const lg_moe_weights *w,
                      const uint16_t *x, int64_t M, float *out, float *weights_out,
                      uint32_t *indices_out, void *workspace, size_t workspace_bytes,
                      void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LIVGLM_MOE_EP_H */
