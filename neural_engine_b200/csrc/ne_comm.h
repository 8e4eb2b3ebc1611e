// ne_comm.h -- internal interface of the NCCL gradient exchange (comm.cu).
#pragma once
#include <cuda_runtime.h>

#include <vector>

#include "../../include/ne.h"

namespace ne {

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

}  // namespace ne
