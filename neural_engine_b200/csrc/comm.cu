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
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <string>

#include "ne_comm.h"
#include "ne_ctx.h"

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
  if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.AllGather ||
      !api.ReduceScatter || !api.GroupStart || !api.GroupEnd || !api.CommDestroy ||
      !api.GetErrorString) {
    api.error = "libnccl.so.2 lacks a required symbol";
    return api;
  }
  api.loaded = true;
  return api;
}

ne_status nccl_fail(ne_ctx* ctx, ncclResult_t r, const char* what) {
  return fail(ctx, NE_ERR_CUDA, std::string(what) + ": " + nccl().GetErrorString(r));
}

}  // namespace

void comm_free(ne_ctx* ctx) {
  if (!ctx || !ctx->comm) return;
  train_drop_step_graph(ctx);
  Comm* c = ctx->comm;
  if (c->cs) cudaStreamSynchronize(c->cs);
  if (c->comm && nccl().loaded) nccl().CommDestroy(reinterpret_cast<ncclComm_t>(c->comm));
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
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum,
                                    reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllReduce");
  return NE_OK;
}

// In place: rank r keeps the sum over ranks of buf[r * n_per_rank, +n_per_rank).
ne_status comm_reduce_scatter(ne_ctx* ctx, float* buf, size_t n_per_rank) {
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().ReduceScatter(buf, buf + (size_t)c->rank * n_per_rank, n_per_rank,
                                        ncclFloat32, ncclSum,
                                        reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclReduceScatter");
  return NE_OK;
}

ne_status comm_group(ne_ctx* ctx, bool start) {
  ncclResult_t r = start ? nccl().GroupStart() : nccl().GroupEnd();
  if (r != ncclSuccess) return nccl_fail(ctx, r, start ? "ncclGroupStart" : "ncclGroupEnd");
  return NE_OK;
}

ne_status comm_allgather(ne_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank) {
  Comm* c = ctx->comm;
  ncclResult_t r = nccl().AllGather(send, recv, bytes_per_rank, ncclUint8,
                                    reinterpret_cast<ncclComm_t>(c->comm), c->cs);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllGather");
  return NE_OK;
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
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  ncclResult_t r = api.CommInitRank(&comm, world, uid, rank);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclCommInitRank");
  c->comm = comm;
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
