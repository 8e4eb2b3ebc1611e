// comm.cu -- data-parallel gradient exchange over NCCL (NVLink / NVSwitch).
//
// The reference trains on one device and has no collective; the data-parallel
// form here follows the one-exchange-step design of the training step: every
// rank computes the gradients of its own batch, the gradient pool is summed
// over ranks (AdamW then applies grad_scale = 1/world), and every rank takes
// the identical optimizer step.
//
// NCCL is loaded with dlopen("libnccl.so.2") on first use, so the library loads
// and runs single-GPU where NCCL is absent.  In a process that already loaded
// NCCL (e.g. through torch.distributed) the same shared object is reused.
// Collectives run on a dedicated high-priority stream; ordering against the
// compute stream is by events only (no host synchronisation).
//
// Failure handling: the communicator is created non-blocking, every NCCL call
// that reports ncclInProgress is polled to completion against a deadline, and
// ne_sync waits for the streams by polling (cudaStreamQuery plus
// ncclCommGetAsyncError) instead of blocking.  When a deadline passes -- a rank
// that never joined, an exchange some rank never entered -- the communicator is
// aborted (ncclCommAbort makes its kernels return), the streams drain, and the
// call returns NE_ERR_TIMEOUT instead of holding the GPUs.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>

#include "ne_comm.h"
#include "ne_ctx.h"
#include "ne_fault.h"

namespace ne {

namespace {

struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                                ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api;
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
    return api;
  }
  auto sym = [&](const char* n) { return dlsym(h, n); };
  api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
  api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
  api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
  api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
  api.ReduceScatter = reinterpret_cast<decltype(api.ReduceScatter)>(sym("ncclReduceScatter"));
  api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
  api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
  api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
  api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
  api.CommInitRankConfig =
      reinterpret_cast<decltype(api.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
  api.CommGetAsyncError =
      reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
  api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
  api.Broadcast = reinterpret_cast<decltype(api.Broadcast)>(sym("ncclBroadcast"));
  if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.AllGather ||
      !api.ReduceScatter || !api.GroupStart || !api.GroupEnd || !api.CommDestroy ||
      !api.GetErrorString || !api.CommInitRankConfig || !api.CommGetAsyncError ||
      !api.CommAbort || !api.Broadcast) {
    api.error = "libnccl.so.2 lacks a required symbol";
    return api;
  }
  api.loaded = true;
  return api;
}

ne_status nccl_fail(ne_ctx* ctx, ncclResult_t r, const char* what) {
  return fail(ctx, NE_ERR_CUDA, std::string(what) + ": " + nccl().GetErrorString(r));
}

using Clock = std::chrono::steady_clock;

// Default deadline of one wait on the exchange: NE_COMM_TIMEOUT_MS, else 120 s.
int default_timeout_ms() {
  static const int ms = [] {
    const char* e = std::getenv("NE_COMM_TIMEOUT_MS");
    const int v = e ? std::atoi(e) : 0;
    return v > 0 ? v : 120000;
  }();
  return ms;
}

// Back-off of the host polling loops: spin briefly, then sleep a little.
void poll_pause(int iter) {
  if (iter < 2000) std::this_thread::yield();
  else std::this_thread::sleep_for(std::chrono::microseconds(50));
}

// The communicator ran into a deadline or an asynchronous error: abort it (its
// kernels in flight return), let both streams drain (bounded), drop it.
ne_status comm_abort(ne_ctx* ctx, ne_status why, const std::string& msg) {
  Comm* c = ctx->comm;
  if (c->comm) nccl().CommAbort(reinterpret_cast<ncclComm_t>(c->comm));
  c->comm = nullptr;
  c->aborted = true;
  const auto until = Clock::now() + std::chrono::seconds(30);
  for (int i = 0; Clock::now() < until; ++i) {
    const bool idle = cudaStreamQuery(ctx->st) != cudaErrorNotReady &&
                      (!c->cs || cudaStreamQuery(c->cs) != cudaErrorNotReady);
    if (idle) break;
    poll_pause(i);
  }
  return fail(ctx, why, msg + "; communicator aborted");
}

// Poll a non-blocking NCCL call that returned ncclInProgress until its host
// side finished (or failed, or the deadline passed).
ne_status comm_settle(ne_ctx* ctx, ncclResult_t r, const char* what) {
  Comm* c = ctx->comm;
  if (r == ncclSuccess) return NE_OK;
  if (r != ncclInProgress) return nccl_fail(ctx, r, what);
  const auto until = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (int i = 0;; ++i) {
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(reinterpret_cast<ncclComm_t>(c->comm), &st);
    if (st == ncclSuccess) return NE_OK;
    if (st != ncclInProgress)
      return comm_abort(ctx, NE_ERR_CUDA, std::string(what) + ": " + nccl().GetErrorString(st));
    if (Clock::now() > until)
      return comm_abort(ctx, NE_ERR_TIMEOUT,
                        std::string(what) + " did not complete within " +
                            std::to_string(c->timeout_ms) + " ms");
    poll_pause(i);
  }
}

ne_status comm_usable(ne_ctx* ctx) {
  if (!ctx->comm || ctx->comm->aborted || !ctx->comm->comm)
    return fail(ctx, NE_ERR_STATE, "the communicator was aborted after a failed exchange");
  return NE_OK;
}

}  // namespace

// Wait for the compute and comm streams with the exchange's deadline, watching
// the communicator for asynchronous errors (ne_sync with a communicator).
ne_status comm_sync(ne_ctx* ctx) {
  Comm* c = ctx->comm;
  if (c->aborted || !c->comm) {
    NE_CUDA(cudaStreamSynchronize(ctx->st));
    return NE_OK;
  }
  const auto until = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (int i = 0;; ++i) {
    const cudaError_t a = cudaStreamQuery(ctx->st);
    const cudaError_t b = cudaStreamQuery(c->cs);
    if (a != cudaErrorNotReady && b != cudaErrorNotReady) {
      NE_CUDA(a);
      NE_CUDA(b);
      return NE_OK;
    }
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(reinterpret_cast<ncclComm_t>(c->comm), &st);
    if (st != ncclSuccess && st != ncclInProgress)
      return comm_abort(ctx, NE_ERR_CUDA, std::string("gradient exchange: ") +
                                              nccl().GetErrorString(st));
    if (Clock::now() > until)
      return comm_abort(ctx, NE_ERR_TIMEOUT,
                        "the gradient exchange did not complete within " +
                            std::to_string(c->timeout_ms) + " ms (a rank did not take part)");
    poll_pause(i);
  }
}

void comm_free(ne_ctx* ctx) {
  if (!ctx || !ctx->comm) return;
  Comm* c = ctx->comm;
  // bounded: a communicator whose work cannot finish is aborted, not destroyed
  const bool idle = c->comm && nccl().loaded && comm_sync(ctx) == NE_OK && c->comm;
  // captured steps hold NCCL work of this communicator: release them first
  train_drop_step_graph(ctx);
  if (c->cs) cudaStreamSynchronize(c->cs);
  px_free(ctx);
  if (idle) nccl().CommDestroy(reinterpret_cast<ncclComm_t>(c->comm));
  c->comm = nullptr;
  for (cudaEvent_t e : c->ev)
    if (e) cudaEventDestroy(e);
  if (c->cs) cudaStreamDestroy(c->cs);
  if (c->gather) cudaFree(c->gather);
  delete c;
  ctx->comm = nullptr;
}

// Event recorded on the compute stream; the comm stream waits for it.
ne_status comm_fence_in(ne_ctx* ctx) {
  Comm* c = ctx->comm;
  cudaEvent_t e = c->ev[c->next_ev];
  c->next_ev = (c->next_ev + 1) % (int)c->ev.size();
  NE_CUDA(cudaEventRecord(e, ctx->st));
  NE_CUDA(cudaStreamWaitEvent(c->cs, e, 0));
  return NE_OK;
}

// The compute stream waits for everything enqueued on the comm stream so far.
ne_status comm_fence_out(ne_ctx* ctx) {
  Comm* c = ctx->comm;
  cudaEvent_t e = c->ev[c->next_ev];
  c->next_ev = (c->next_ev + 1) % (int)c->ev.size();
  NE_CUDA(cudaEventRecord(e, c->cs));
  NE_CUDA(cudaStreamWaitEvent(ctx->st, e, 0));
  return NE_OK;
}

ne_status comm_allreduce(ne_ctx* ctx, float* buf, size_t n) {
  ne_status s = comm_usable(ctx);
  if (s != NE_OK) return s;
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum,
                                    reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  return comm_settle(ctx, r, "ncclAllReduce");
}

// In place: rank r keeps the sum over ranks of buf[r * n_per_rank, +n_per_rank).
ne_status comm_reduce_scatter(ne_ctx* ctx, float* buf, size_t n_per_rank) {
  ne_status s = comm_usable(ctx);
  if (s != NE_OK) return s;
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().ReduceScatter(buf, buf + (size_t)c->rank * n_per_rank, n_per_rank,
                                        ncclFloat32, ncclSum,
                                        reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  return comm_settle(ctx, r, "ncclReduceScatter");
}

ne_status comm_group(ne_ctx* ctx, bool start) {
  ne_status s = comm_usable(ctx);
  if (s != NE_OK) return s;
  ncclResult_t r = start ? nccl().GroupStart() : nccl().GroupEnd();
  return comm_settle(ctx, r, start ? "ncclGroupStart" : "ncclGroupEnd");
}

ne_status comm_allgather(ne_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank) {
  ne_status s = comm_usable(ctx);
  if (s != NE_OK) return s;
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().AllGather(send, recv, bytes_per_rank, ncclUint8,
                                    reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  return comm_settle(ctx, r, "ncclAllGather");
}

// In place: every rank receives root's `bytes` at buf.
ne_status comm_broadcast(ne_ctx* ctx, void* buf, size_t bytes, int root) {
  ne_status s = comm_usable(ctx);
  if (s != NE_OK) return s;
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().Broadcast(buf, buf, bytes, ncclUint8, root,
                                    reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  return comm_settle(ctx, r, "ncclBroadcast");
}

// Unmap the other ranks' buffers and free the exchange's own (no work of it
// may be in flight).
void px_free(ne_ctx* ctx) {
  if (!ctx->comm) return;
  PxState& x = ctx->comm->pxs;
  for (void* p : x.mapped)
    if (p) cudaIpcCloseMemHandle(p);
  x.mapped.clear();
  for (cudaEvent_t e : x.ag_ev)
    if (e) cudaEventDestroy(e);
  x.ag_ev.clear();
  for (void* p : {(void*)x.flags, (void*)x.d_wsrc, (void*)x.d_asrc, (void*)x.d_chunks})
    if (p) cudaFree(p);
  x = PxState();
}

}  // namespace ne

using namespace ne;

extern "C" {

NE_API ne_status ne_comm_unique_id(void* id_out) {
  if (!id_out) return NE_ERR_INVALID;
  NcclApi& api = nccl();
  if (!api.loaded) return NE_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (api.GetUniqueId(&id) != ncclSuccess) return NE_ERR_CUDA;
  static_assert(sizeof(ncclUniqueId) == NE_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return NE_OK;
}

NE_API ne_status ne_comm_init(ne_ctx* ctx, const void* id, int rank, int world) {
  if (!ctx || !id || world < 1 || rank < 0 || rank >= world) return NE_ERR_INVALID;
  NE_FAULT_POINT(ctx, "ne_comm_init");
  NcclApi& api = nccl();
  if (!api.loaded) return fail(ctx, NE_ERR_UNSUPPORTED, api.error);
  NE_CUDA(cudaSetDevice(ctx->device));
  train_drop_step_graph(ctx);
  comm_free(ctx);
  Comm* c = new Comm();
  ctx->comm = c;
  c->rank = rank;
  c->world = world;
  int lo = 0, hi = 0;
  NE_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  NE_CUDA(cudaStreamCreateWithPriority(&c->cs, cudaStreamNonBlocking, hi));
  c->ev.resize(64, nullptr);
  for (cudaEvent_t& e : c->ev) NE_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  c->timeout_ms = ctx->comm_timeout_ms > 0 ? ctx->comm_timeout_ms : default_timeout_ms();
  {
    const char* e = std::getenv("NE_COMM_PX");
    c->px = !(e && e[0] == '0');
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;   // every wait is ours, with a deadline
  ncclComm_t comm = nullptr;
  ncclResult_t r = api.CommInitRankConfig(&comm, world, uid, rank, &cfg);
  c->comm = comm;
  if (r != ncclSuccess && r != ncclInProgress) {
    c->comm = nullptr;
    c->aborted = true;
    if (comm) api.CommAbort(comm);
    return nccl_fail(ctx, r, "ncclCommInitRankConfig");
  }
  // the init runs in the background until every rank has joined
  return comm_settle(ctx, r, "ncclCommInitRankConfig (every rank must join)");
}

NE_API ne_status ne_comm_set_timeout(ne_ctx* ctx, int timeout_ms) {
  if (!ctx || timeout_ms < 0) return NE_ERR_INVALID;
  ctx->comm_timeout_ms = timeout_ms;
  if (ctx->comm) ctx->comm->timeout_ms = timeout_ms > 0 ? timeout_ms : default_timeout_ms();
  return NE_OK;
}

NE_API ne_status ne_comm_set_reduce(ne_ctx* ctx, int on) {
  if (!ctx || !ctx->comm) return NE_ERR_STATE;
  ctx->comm->reduce = on != 0;   // the training step keeps one captured graph per mode
  return NE_OK;
}

NE_API ne_status ne_comm_set_sharding(ne_ctx* ctx, int on) {
  if (!ctx || !ctx->comm) return NE_ERR_STATE;
  if (ctx->comm->shard != (on != 0)) train_drop_step_graph(ctx);
  ctx->comm->shard = on != 0;
  return NE_OK;
}

}  // extern "C"
