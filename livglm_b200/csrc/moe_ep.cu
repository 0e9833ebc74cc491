// Expert-parallel MoE layer as one C call (include/livglm_moe_ep.h).
//
// A separate library over liblivglm_moe.so's public C ABI and NCCL: the
// router, dispatch, pack, shared expert, local experts and gathered combine
// are the single-GPU library's calls; this file adds the exchange plumbing
// (exchange-id renumbering, per-destination counts, NCCL send/recv on the
// communicator's stream overlapped with the shared expert).  It is the C form
// of livglm_b200/ep.py's ExpertParallelMoE.  No counterpart in kg36/livglm,
// whose block runs on one device (src/glm53flash/moe.py:96-201).

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "livglm_moe_ep.h"

struct lg_ep_comm {
  ncclComm_t nccl = nullptr;
  int world = 0, rank = 0, device = -1;
  int64_t max_tokens = 0;
  cudaStream_t xfer = nullptr;  // the dispatch exchange runs here
  cudaEvent_t packed = nullptr, sent = nullptr;
  int64_t* d_msg = nullptr;     // device: this rank's message, then all ranks' [world][kMsg]
  int64_t* h_msg = nullptr;     // pinned host copy of all ranks' messages
};

namespace {

// Per-rank message of the count exchange: slots bound for each rank, the
// rank's token count, its status (0 = ok, else an LG_ERR_* code).
int msg_len(int world) { return world + 2; }

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int from_lib(int rc, const char* what) {
  if (rc == LG_OK) return LG_OK;
  return fail(rc, "%s: %s", what, lg_moe_last_error());
}

int cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LG_OK;
  return fail(LG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int nccl_fail(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return LG_OK;
  return fail(LG_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

constexpr size_t kAlign = 256;
size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// The local experts' geometry: top-1 over E/W experts, no routing groups,
// no shared part.
lg_moe_config local_config(const lg_moe_config& c, int world) {
  lg_moe_config l = c;
  l.n_routed_experts = c.n_routed_experts / world;
  l.num_experts_per_tok = 1;
  l.n_group = 1;
  l.topk_group = 1;
  l.n_shared_experts = 0;
  return l;
}

struct Layout {
  size_t core = 0, core_bytes = 0;  // the single-GPU calls' workspace (status word first)
  size_t xidx, counts, offsets, perm, x_send, e_send, inv, shared, x_recv, e_recv, y_recv, y_back, total;
};

// Worst case of every buffer: this rank sends max_tokens * k slots and
// receives up to world * max_tokens * k rows.
bool layout(const lg_moe_config* c, int64_t max_tokens, int world, Layout* L) {
  if (!c || world < 1 || max_tokens < 1 || c->n_routed_experts % world) return false;
  const lg_moe_config l = local_config(*c, world);
  const size_t d = c->hidden_size, E = c->n_routed_experts, k = c->num_experts_per_tok;
  const size_t R = max_tokens * k, cap = R * world;
  const size_t a = lg_moe_workspace_size(c, max_tokens);
  const size_t b = lg_moe_workspace_size(&l, static_cast<int64_t>(cap));
  if (!a || !b) return false;
  size_t o = up(std::max(a, b));
  L->core_bytes = o;
  auto take = [&o](size_t bytes) { size_t at = o; o += up(bytes); return at; };
  L->xidx = take(R * 4);
  L->counts = take(E * 4);
  L->offsets = take((E + 1) * 4);
  L->perm = take(R * 4);
  L->x_send = take(R * d * 2);
  L->e_send = take(R * 4);
  L->inv = take(R * 4);
  L->shared = take(static_cast<size_t>(max_tokens) * d * 2);
  L->x_recv = take(cap * d * 2);
  L->e_recv = take(cap * 4);
  L->y_recv = take(cap * d * 2);
  L->y_back = take(R * d * 2);
  L->total = o;
  return true;
}

template <typename T>
T* at(void* base, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(base) + off); }

// Expert id -> exchange id: expert e lives on rank e mod W as local expert
// e / W, and exchange id = owner * (E/W) + local index, so that sorting the
// route slots by exchange id groups them by owner and then by local expert.
__global__ void exchange_id_kernel(const uint32_t* __restrict__ idx, int64_t R, int world, int per_rank,
                                   uint32_t* __restrict__ xidx) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < R;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t e = idx[i];
    xidx[i] = (e % world) * per_rank + e / world;
  }
}

// This rank's message: slots per destination (from the dispatch offsets of
// the exchange ids), token count, status.
__global__ void message_kernel(const int* __restrict__ offsets, int world, int per_rank, int64_t M,
                               int64_t* __restrict__ msg) {
  const int p = threadIdx.x;
  if (p < world) msg[p] = offsets[(p + 1) * per_rank] - offsets[p * per_rank];
  if (p == 0) {
    msg[world] = M;
    msg[world + 1] = 0;
  }
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace

extern "C" {

const char* lg_ep_last_error(void) { return g_err; }

int lg_ep_unique_id_bytes(void) { return static_cast<int>(sizeof(ncclUniqueId)); }

int lg_ep_get_unique_id(void* out) {
  if (!out) return fail(LG_ERR_INVALID_ARG, "unique id: NULL output");
  ncclUniqueId id;
  int rc = nccl_fail(ncclGetUniqueId(&id), "ncclGetUniqueId");
  if (rc) return rc;
  std::memcpy(out, &id, sizeof id);
  return LG_OK;
}

int lg_ep_comm_destroy(lg_ep_comm* c) {
  if (!c) return LG_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (c->device >= 0) cudaSetDevice(c->device);
  if (c->nccl) ncclCommAbort(c->nccl);
  if (c->xfer) cudaStreamDestroy(c->xfer);
  if (c->packed) cudaEventDestroy(c->packed);
  if (c->sent) cudaEventDestroy(c->sent);
  if (c->d_msg) cudaFree(c->d_msg);
  if (c->h_msg) cudaFreeHost(c->h_msg);
  delete c;
  if (prev >= 0) cudaSetDevice(prev);
  return LG_OK;
}

int lg_ep_comm_init(const void* unique_id, int32_t world, int32_t rank, int64_t max_tokens, lg_ep_comm** out) {
  if (!unique_id || !out) return fail(LG_ERR_INVALID_ARG, "comm init: NULL argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return fail(LG_ERR_INVALID_ARG, "comm init: rank %d of %d", rank, world);
  if (max_tokens < 1) return fail(LG_ERR_INVALID_ARG, "comm init: max_tokens %lld < 1", (long long)max_tokens);
  lg_ep_comm* c = new lg_ep_comm;
  c->world = world;
  c->rank = rank;
  c->max_tokens = max_tokens;
  int rc = cuda_fail(cudaGetDevice(&c->device), "cudaGetDevice");
  const size_t L = msg_len(world);
  if (!rc) rc = cuda_fail(cudaStreamCreateWithFlags(&c->xfer, cudaStreamNonBlocking), "exchange stream");
  if (!rc) rc = cuda_fail(cudaEventCreateWithFlags(&c->packed, cudaEventDisableTiming), "event");
  if (!rc) rc = cuda_fail(cudaEventCreateWithFlags(&c->sent, cudaEventDisableTiming), "event");
  if (!rc) rc = cuda_fail(cudaMalloc(&c->d_msg, (L + L * world) * sizeof(int64_t)), "message buffer");
  if (!rc) rc = cuda_fail(cudaMallocHost(&c->h_msg, (L + L * world) * sizeof(int64_t)), "pinned message buffer");
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  if (!rc) rc = nccl_fail(ncclCommInitRank(&c->nccl, world, id, rank), "ncclCommInitRank");
  if (rc) {
    lg_ep_comm_destroy(c);
    return rc;
  }
  *out = c;
  return LG_OK;
}

size_t lg_moe_ep_workspace_size(const lg_moe_config* cfg, int64_t max_tokens, int32_t world) {
  Layout L;
  if (!layout(cfg, max_tokens, world, &L)) {
    fail(LG_ERR_INVALID_ARG, "ep workspace: invalid geometry (E %% world, max_tokens or config)");
    return 0;
  }
  return L.total;
}

int lg_moe_ep_forward(lg_ep_comm* comm, const lg_moe_config* cfg, const lg_moe_weights* w, const uint16_t* x,
                      int64_t M, float* out, float* weights_out, uint32_t* indices_out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!comm) return fail(LG_ERR_INVALID_ARG, "ep forward: communicator is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int W = comm->world, me = comm->rank;
  const size_t ML = msg_len(W);
  int64_t* d_mine = comm->d_msg;
  int64_t* d_all = comm->d_msg + ML;
  int64_t* h_all = comm->h_msg + ML;

  // 1. local checks and the routing half; any failure becomes this rank's
  //    status in the count exchange, which every rank still joins.
  int rc = LG_OK;
  Layout L{};
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != comm->device)
    rc = fail(LG_ERR_INVALID_ARG, "ep forward: current device %d is not the communicator's %d", dev, comm->device);
  else if (!cfg || !layout(cfg, comm->max_tokens, W, &L))
    rc = fail(LG_ERR_INVALID_ARG, "ep forward: invalid config for %d ranks (E %% world, local experts >= 2)", W);
  else if (M < 0 || M > comm->max_tokens)
    rc = fail(LG_ERR_INVALID_ARG, "ep forward: M=%lld outside [0, %lld]", (long long)M, (long long)comm->max_tokens);
  else if (!workspace || reinterpret_cast<uintptr_t>(workspace) % kAlign || workspace_bytes < L.total)
    rc = fail(LG_ERR_WORKSPACE, "ep forward: workspace needs %zu bytes, 256-byte aligned", L.total);
  else if (M > 0 && (!w || !x || !out || !weights_out || !indices_out))
    rc = fail(LG_ERR_INVALID_ARG, "ep forward: NULL pointer");
  const int k = cfg ? cfg->num_experts_per_tok : 0;
  const int per_rank = rc ? 0 : cfg->n_routed_experts / W;
  const int64_t R = M * k;
  void* core = workspace;
  const size_t core_bytes = L.core_bytes;
  if (!rc && M > 0) {
    uint32_t* xidx = at<uint32_t>(workspace, L.xidx);
    rc = from_lib(lg_moe_router(cfg, x, M, w->router_weight, w->router_bias, nullptr, weights_out, indices_out, core,
                                core_bytes, s), "lg_moe_router");
    if (!rc) {
      const int blocks = static_cast<int>(std::min<int64_t>((R + 255) / 256, 4 * num_sms()));
      exchange_id_kernel<<<blocks, 256, 0, s>>>(indices_out, R, W, per_rank, xidx);
      rc = cuda_fail(cudaGetLastError(), "exchange id launch");
    }
    if (!rc)
      rc = from_lib(lg_moe_dispatch(cfg, xidx, M, at<int32_t>(workspace, L.counts), at<int32_t>(workspace, L.offsets),
                                    at<int32_t>(workspace, L.perm), core, core_bytes, s), "lg_moe_dispatch");
    if (!rc)
      rc = from_lib(lg_moe_ep_pack(cfg, x, M, xidx, at<int32_t>(workspace, L.perm), W, at<uint16_t>(workspace, L.x_send),
                                   at<int32_t>(workspace, L.e_send), at<int32_t>(workspace, L.inv), s), "lg_moe_ep_pack");
  }
  if (!rc && M > 0) {
    message_kernel<<<1, 32 * ((W + 31) / 32), 0, s>>>(at<int32_t>(workspace, L.offsets), W, per_rank, M, d_mine);
    rc = cuda_fail(cudaGetLastError(), "message launch");
  }
  if (rc || M == 0) {  // nothing to send (or a failure to report): the message comes from the host
    int64_t* h_mine = comm->h_msg;
    for (int p = 0; p < W; ++p) h_mine[p] = 0;
    h_mine[W] = rc ? 0 : M;
    h_mine[W + 1] = rc;
    cudaMemcpyAsync(d_mine, h_mine, ML * sizeof(int64_t), cudaMemcpyHostToDevice, s);
  }

  // 2. every rank's message to every rank; the host reads them.
  int xrc = nccl_fail(ncclAllGather(d_mine, d_all, ML, ncclInt64, comm->nccl, s), "count exchange");
  if (xrc) return xrc;
  cudaMemcpyAsync(h_all, d_all, ML * W * sizeof(int64_t), cudaMemcpyDeviceToHost, s);
  if ((xrc = cuda_fail(cudaStreamSynchronize(s), "count exchange"))) return xrc;
  // The same table on every rank, so every rank reaches the same verdict.
  if (rc) return rc;  // this rank's own failure (its status was sent as such)
  for (int p = 0; p < W; ++p) {
    const int64_t* row = h_all + p * ML;
    if (row[W + 1] != 0) {
      return fail(LG_ERR_INVALID_ARG, "ep forward: rank %d reported error %lld before the exchange", p,
                  (long long)row[W + 1]);
    }
    int64_t sum = 0;
    bool bad = row[W] < 0 || row[W] > comm->max_tokens;
    for (int q = 0; q < W; ++q) {
      bad |= row[q] < 0;
      sum += row[q];
    }
    if (bad || sum != row[W] * k)
      return fail(LG_ERR_INVALID_ARG, "ep forward: rank %d sent an inconsistent count table", p);
  }
  std::vector<int64_t> nsend(W), nrecv(W), soff(W + 1, 0), roff(W + 1, 0);
  for (int p = 0; p < W; ++p) {
    nsend[p] = h_all[me * ML + p];
    nrecv[p] = h_all[p * ML + me];
    soff[p + 1] = soff[p] + nsend[p];
    roff[p + 1] = roff[p] + nrecv[p];
  }
  const int64_t n_recv = roff[W];
  const size_t d = cfg->hidden_size, row_bytes = d * 2;

  // 3. rows and local expert ids to their owners on the exchange stream,
  //    the shared expert meanwhile on the caller's stream.
  char* x_send = at<char>(workspace, L.x_send);
  int32_t* e_send = at<int32_t>(workspace, L.e_send);
  char* x_recv = at<char>(workspace, L.x_recv);
  int32_t* e_recv = at<int32_t>(workspace, L.e_recv);
  char* y_recv = at<char>(workspace, L.y_recv);
  char* y_back = at<char>(workspace, L.y_back);
  if ((xrc = cuda_fail(cudaEventRecord(comm->packed, s), "event record"))) return xrc;
  if ((xrc = cuda_fail(cudaStreamWaitEvent(comm->xfer, comm->packed, 0), "stream wait"))) return xrc;
  ncclGroupStart();
  for (int p = 0; p < W && !xrc; ++p) {
    if (nsend[p]) {
      xrc = nccl_fail(ncclSend(x_send + soff[p] * row_bytes, nsend[p] * row_bytes, ncclUint8, p, comm->nccl, comm->xfer),
                      "dispatch send");
      if (!xrc) xrc = nccl_fail(ncclSend(e_send + soff[p], nsend[p], ncclInt32, p, comm->nccl, comm->xfer), "dispatch send");
    }
    if (nrecv[p] && !xrc) {
      xrc = nccl_fail(ncclRecv(x_recv + roff[p] * row_bytes, nrecv[p] * row_bytes, ncclUint8, p, comm->nccl, comm->xfer),
                      "dispatch recv");
      if (!xrc) xrc = nccl_fail(ncclRecv(e_recv + roff[p], nrecv[p], ncclInt32, p, comm->nccl, comm->xfer), "dispatch recv");
    }
  }
  const int grc = nccl_fail(ncclGroupEnd(), "dispatch exchange");
  if (xrc || grc) return xrc ? xrc : grc;
  if ((xrc = cuda_fail(cudaEventRecord(comm->sent, comm->xfer), "event record"))) return xrc;

  uint16_t* shared = nullptr;
  if (M > 0 && cfg->n_shared_experts > 0) {
    shared = at<uint16_t>(workspace, L.shared);
    rc = from_lib(lg_moe_shared(cfg, w, x, M, shared, core, core_bytes, s), "lg_moe_shared");
  }
  if ((xrc = cuda_fail(cudaStreamWaitEvent(s, comm->sent, 0), "stream wait"))) return xrc;

  // 4. the received rows through this rank's experts (top-1, local ids).
  if (!rc && n_recv > 0) {
    const lg_moe_config lc = local_config(*cfg, W);
    rc = from_lib(lg_moe_experts(&lc, w, reinterpret_cast<const uint16_t*>(x_recv),
                                 reinterpret_cast<const uint32_t*>(e_recv), n_recv, reinterpret_cast<uint16_t*>(y_recv),
                                 core, core_bytes, s), "lg_moe_experts (local)");
  }

  // 5. outputs back to the rows' ranks (even after a local failure, so that
  //    no peer waits for them), then the combine in route order.
  ncclGroupStart();
  for (int p = 0; p < W && !xrc; ++p) {
    if (nrecv[p])
      xrc = nccl_fail(ncclSend(y_recv + roff[p] * row_bytes, nrecv[p] * row_bytes, ncclUint8, p, comm->nccl, s),
                      "return send");
    if (nsend[p] && !xrc)
      xrc = nccl_fail(ncclRecv(y_back + soff[p] * row_bytes, nsend[p] * row_bytes, ncclUint8, p, comm->nccl, s),
                      "return recv");
  }
  const int grc2 = nccl_fail(ncclGroupEnd(), "return exchange");
  if (xrc || grc2) return xrc ? xrc : grc2;
  if (rc) return rc;
  if (M > 0)
    rc = from_lib(lg_moe_combine_gather(cfg, reinterpret_cast<const uint16_t*>(y_back), at<int32_t>(workspace, L.inv),
                                        weights_out, shared, M, out, s), "lg_moe_combine_gather");
  return rc;
}

}  // extern "C"
