// comm.cuh - the library's NCCL communicator (host side, internal).
//
// libannb200 drives NCCL through its C API, loaded at run time (dlopen of
// libnccl.so.2, preferring a copy the process already has loaded), so the
// library loads and serves single-GPU calls on machines without NCCL. One
// AnnB200Comm is one rank: one device of a row-sharded search.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <mutex>

struct AnnB200Comm {
  ncclComm_t nccl = nullptr;
  int device = 0;
  int rank = 0;
  int nranks = 1;
  bool broken = false;      // aborted after a time-out: every later call fails
  std::mutex mu;            // one sharded search at a time on a rank
  // grow-only exchange buffers: this rank's packet, every rank's packets,
  // and a pinned copy of every rank's packet header
  void *send = nullptr;
  size_t send_bytes = 0;
  void *recv = nullptr;
  size_t recv_bytes = 0;
  uint8_t *host_heads = nullptr;
  size_t host_heads_bytes = 0;
  int32_t *host_status = nullptr;   // pinned: this rank's status, copied into its packet
  cudaEvent_t done = nullptr;
  // the mid-search exchange of per-query bounds: this rank's, then every rank's
  double *bounds = nullptr;
  size_t bounds_bytes = 0;
};

namespace annb200 {

// All-gather `bytes` of send from every rank into recv ([nranks][bytes]) on
// stream. Returns an AnnStatus (and sets the error message) on failure.
int comm_allgather(AnnB200Comm *c, const void *send, void *recv, size_t bytes, cudaStream_t st);

// Wait for everything queued on st so far, at most the communicator's time
// limit (ANN_B200_COMM_TIMEOUT_MS, default 60 s). A rank whose peers never
// join the exchange would otherwise wait for ever: on expiry the
// communicator is aborted (its kernels end) and marked broken.
int comm_wait(AnnB200Comm *c, cudaStream_t st);

// Grow-only device / pinned buffers of the communicator.
int comm_reserve(AnnB200Comm *c, size_t packet_bytes, size_t head_bytes);

// Grow-only device buffer of the bounds exchange: nq doubles of this rank's
// followed by nranks x nq of everyone's.
int comm_reserve_bounds(AnnB200Comm *c, uint32_t nq);

}  // namespace annb200
