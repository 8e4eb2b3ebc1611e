// ne_comm.h -- internal interface of the NCCL gradient exchange (comm.cu).
#pragma once
#include <cuda_runtime.h>

#include <vector>

#include "../../include/ne.h"
#include "ne_internal.h"
#include "ne_px.h"

namespace ne {

// Peer-memory ZeRO-1 exchange (px.cu): the other ranks' pools mapped through
// CUDA IPC, this rank's flag words, and the chunk lists of every exchange.
struct PxState {
  bool ready = false;
  uint32_t* flags = nullptr;           // this rank's flag words (device)
  std::vector<void*> mapped;           // the other ranks' mapped buffers
  PxTables T;                          // flag and gradient bases of every rank
  const char** d_wsrc = nullptr;       // [world] weight pool of each rank (device table)
  const char** d_asrc = nullptr;       // [world] activation pool of each rank
  PxChunk* d_chunks = nullptr;         // every chunk list below, one allocation
  std::vector<int> rs_first, rs_count; // per bucket (0 = tail, 1 + layer)
  int ag_first = 0, ag_count = 0;      // weight all-gather (every bucket)
  std::vector<int> ag_bfirst, ag_bcount;   // the same per bucket (0 = tail, 1 + layer)
  std::vector<cudaEvent_t> ag_ev;      // per bucket: its all-gather done (comm stream)
  // fused dW reduction: the layer matrices' dW products add straight into
  // their owners' gradients (EPI_RESID_PEER); their reduce-scatter is skipped
  bool fused = false;                  // set up for it (NE_PX_FUSED_DW, eligible shapes)
  bool fused_now = false;              // the current micro-step uses it
  bool owned_clean = false;            // owned fused parts zeroed and PX_ZEROED published
  std::vector<GemmPeerOut> peer_out;   // per training segment (used where fused_seg)
  std::vector<char> fused_seg;
  std::vector<int> rsf_first, rsf_count;   // per bucket: reduce-scatter without the fused segments
  int zf_first = 0, zf_count = 0;      // this rank's owned parts of the fused segments
  int zr_first = 0, zr_count = 0;      // every other gradient float (zeroed after the all-gather)
  int em_first = 0, em_count = 0;      // (token id, dY row) gather
};

struct Comm {
  void* comm = nullptr;            // ncclComm_t
  int rank = 0, world = 1;
  cudaStream_t cs = nullptr;       // collective stream (highest priority)
  std::vector<cudaEvent_t> ev;     // ring of ordering events
  int next_ev = 0;
  bool reduce = true;              // the training step reduces its gradients
  bool shard = false;              // ZeRO-1: reduce-scatter, sharded AdamW, weight all-gather
  void* gather = nullptr;          // all-gathered (token id, dY row) pairs
  size_t gather_bytes = 0;
  int timeout_ms = 120000;         // deadline of one wait on the exchange
  bool aborted = false;            // a deadline passed or NCCL failed: no more exchanges
  bool px = true;                  // ZeRO-1 over peer memory (NE_COMM_PX=0: NCCL collectives)
  PxState pxs;
};

void comm_free(ne_ctx* ctx);
// ne_train.cu: before the communicator or the exchange mode changes (drops the
// captured step and the optimizer work list).
void train_drop_step_graph(ne_ctx* ctx);
ne_status comm_fence_in(ne_ctx* ctx);    // comm stream waits for the compute stream
ne_status comm_fence_out(ne_ctx* ctx);   // compute stream waits for the comm stream
ne_status comm_allreduce(ne_ctx* ctx, float* buf, size_t n);
ne_status comm_allgather(ne_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank);
ne_status comm_reduce_scatter(ne_ctx* ctx, float* buf, size_t n_per_rank);   // in place
ne_status comm_group(ne_ctx* ctx, bool start);   // ncclGroupStart / ncclGroupEnd
// Wait for the compute and comm streams within the exchange's deadline; on
// expiry or an NCCL error the communicator is aborted (NE_ERR_TIMEOUT / CUDA).
ne_status comm_sync(ne_ctx* ctx);
ne_status comm_broadcast(ne_ctx* ctx, void* buf, size_t bytes, int root);   // in place
void px_free(ne_ctx* ctx);   // unmap the other ranks' buffers (streams idle)

}  // namespace ne
