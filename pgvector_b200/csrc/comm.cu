// comm.cu - NCCL communicators for the row-sharded search.
//
// The reference merges per-shard top-k lists on the host after copying each
// GPU's lists back (AnnIndexTreeMerge, ann/server/indexfile.c:3235-3258;
// MergeJob, ann/server/cuvs.c:3446-3455). Here the ranks of a row-sharded
// search exchange their lists with one NCCL all-gather over NVLink and merge
// them on the device (AnnB200SearchSharded, shard.cu). This file owns the
// communicators: NCCL's C API loaded at run time, one AnnB200Comm per rank
// (multi-process: AnnB200CommId + AnnB200CommCreate; one process over several
// devices: AnnB200CommCreateAll), their exchange buffers, and the bounded
// wait that aborts a communicator whose peers never arrive.
#include <dlfcn.h>
#include <sched.h>
#include <time.h>

#include <cstdlib>
#include <cstring>
#include <new>

#include "../../include/annb200.h"
#include "comm.cuh"
#include "internal.cuh"

namespace {

enum Status { OK = 0, INVALID = 1, UNSUPPORTED = 2, NOMEM = 4, BACKEND_ERROR = 5 };

// NCCL's entry points, resolved once.
struct Nccl {
  bool ok = false;
  const char *why = "NCCL not loaded";
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommInitAll)(ncclComm_t *, int, const int *) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

template <typename F>
bool sym(void *h, const char *name, F *f) {
  *f = reinterpret_cast<F>(dlsym(h, name));
  return *f != nullptr;
}

// libnccl.so.2: the copy already in the process if there is one (a torch
// or MPI program has loaded its own), else the one the loader finds.
const Nccl &nccl() {
  static Nccl n = [] {
    Nccl x;
    const char *env = getenv("ANN_B200_NCCL_LIBRARY");
    void *h = nullptr;
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      x.why = "libnccl.so.2 could not be loaded";
      return x;
    }
    x.ok = sym(h, "ncclGetUniqueId", &x.GetUniqueId) && sym(h, "ncclCommInitRank", &x.CommInitRank) &&
           sym(h, "ncclCommInitAll", &x.CommInitAll) && sym(h, "ncclCommDestroy", &x.CommDestroy) &&
           sym(h, "ncclCommAbort", &x.CommAbort) && sym(h, "ncclCommGetAsyncError", &x.CommGetAsyncError) &&
           sym(h, "ncclAllGather", &x.AllGather) && sym(h, "ncclGroupStart", &x.GroupStart) &&
           sym(h, "ncclGroupEnd", &x.GroupEnd) && sym(h, "ncclGetErrorString", &x.GetErrorString);
    if (!x.ok) x.why = "libnccl.so.2 lacks an entry point this library calls";
    return x;
  }();
  return n;
}

// Connections between the ranks are made while the group is created, all
// ranks present: NCCL otherwise makes them at a collective's first use,
// inside the host call, where a rank whose peers never arrive would wait
// for ever before any time limit could act. (Unless the caller chose.)
void eager_connect() { setenv("NCCL_RUNTIME_CONNECT", "0", 0); }

int nccl_fail(ncclResult_t r, const char *what) {
  return annb200::report_error(BACKEND_ERROR, "%s: %s", what, nccl().GetErrorString ? nccl().GetErrorString(r) : "");
}

double now_ms() {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

long timeout_ms() {
  const char *v = getenv("ANN_B200_COMM_TIMEOUT_MS");
  long t = v && *v ? strtol(v, nullptr, 10) : 60000;
  return t > 0 ? t : 60000;
}

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

AnnB200Comm *make_comm(int device, int rank, int nranks, ncclComm_t c) {
  AnnB200Comm *x = new (std::nothrow) AnnB200Comm();
  if (!x) return nullptr;
  x->nccl = c;
  x->device = device;
  x->rank = rank;
  x->nranks = nranks;
  DevGuard g(device);
  if (cudaMallocHost(&x->host_status, sizeof(int32_t)) != cudaSuccess ||
      cudaEventCreateWithFlags(&x->done, cudaEventDisableTiming) != cudaSuccess) {
    cudaGetLastError();
    if (x->host_status) cudaFreeHost(x->host_status);
    delete x;
    return nullptr;
  }
  return x;
}

// One small all-gather on every new rank while the whole group is there:
// its connections are made and proven before any search relies on them.
int warm_up(AnnB200Comm **comms, int n) {
  cudaStream_t st[64] = {};
  void *buf[64] = {};
  int status = OK;
  ncclResult_t r = ncclSuccess;
  for (int i = 0; i < n && status == OK; i++) {
    DevGuard g(comms[i]->device);
    if (cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&buf[i], 16 * (size_t)(comms[i]->nranks + 1)) != cudaSuccess) {
      cudaGetLastError();
      status = annb200::report_error(NOMEM, "communicator warm-up buffers");
    }
  }
  if (status == OK) {
    if (n > 1) nccl().GroupStart();
    for (int i = 0; i < n && r == ncclSuccess; i++) {
      DevGuard g(comms[i]->device);
      r = nccl().AllGather(buf[i], (uint8_t *)buf[i] + 16, 16, ncclUint8, comms[i]->nccl, st[i]);
    }
    if (n > 1) {
      ncclResult_t e = nccl().GroupEnd();
      if (r == ncclSuccess) r = e;
    }
    if (r != ncclSuccess) status = nccl_fail(r, "communicator warm-up");
  }
  for (int i = 0; i < n && status == OK; i++) {
    DevGuard g(comms[i]->device);
    status = annb200::comm_wait(comms[i], st[i]);
  }
  for (int i = 0; i < n; i++) {
    DevGuard g(comms[i]->device);
    if (st[i]) {
      cudaStreamSynchronize(st[i]);
      cudaStreamDestroy(st[i]);
    }
    if (buf[i]) cudaFree(buf[i]);
  }
  return status;
}

}  // namespace

extern "C" int AnnB200CommId(void *id) {
  if (!id) return annb200::report_error(INVALID, "id pointer is NULL");
  if (!nccl().ok) return annb200::report_error(UNSUPPORTED, "%s", nccl().why);
  ncclUniqueId u;
  ncclResult_t r = nccl().GetUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id, &u, sizeof(u));
  return OK;
}

extern "C" int AnnB200CommCreate(int device, int nranks, int rank, const void *id, AnnB200Comm **out) {
  if (!out || !id) return annb200::report_error(INVALID, "NULL id or output pointer");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) return annb200::report_error(INVALID, "rank %d of %d", rank, nranks);
  if (device < 0 || device >= AnnB200DeviceCount()) return annb200::report_error(INVALID, "no CUDA device %d", device);
  if (!nccl().ok) return annb200::report_error(UNSUPPORTED, "%s", nccl().why);
  DevGuard g(device);
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  eager_connect();
  ncclResult_t r = nccl().CommInitRank(&c, nranks, u, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  AnnB200Comm *x = make_comm(device, rank, nranks, c);
  if (!x) {
    nccl().CommAbort(c);
    return annb200::report_error(NOMEM, "communicator");
  }
  int status = warm_up(&x, 1);
  if (status != OK) {
    x->broken = true;
    AnnB200CommDestroy(x);
    return status;
  }
  *out = x;
  return OK;
}

extern "C" int AnnB200CommCreateAll(int ndev, const int *devices, AnnB200Comm **out) {
  if (!out || !devices || ndev < 1) return annb200::report_error(INVALID, "NULL device list or output");
  for (int i = 0; i < ndev; i++) {
    out[i] = nullptr;
    if (devices[i] < 0 || devices[i] >= AnnB200DeviceCount())
      return annb200::report_error(INVALID, "no CUDA device %d", devices[i]);
    for (int j = 0; j < i; j++)
      if (devices[j] == devices[i]) return annb200::report_error(INVALID, "device %d listed twice", devices[i]);
  }
  if (!nccl().ok) return annb200::report_error(UNSUPPORTED, "%s", nccl().why);
  ncclComm_t *c = new (std::nothrow) ncclComm_t[ndev];
  if (!c) return annb200::report_error(NOMEM, "communicators");
  int prev = 0;
  cudaGetDevice(&prev);
  eager_connect();
  ncclResult_t r = nccl().CommInitAll(c, ndev, devices);
  cudaSetDevice(prev);
  if (r != ncclSuccess) {
    delete[] c;
    return nccl_fail(r, "ncclCommInitAll");
  }
  int status = OK;
  for (int i = 0; i < ndev && status == OK; i++) {
    out[i] = make_comm(devices[i], i, ndev, c[i]);
    if (!out[i]) status = NOMEM;
  }
  if (status != OK) {
    // the group is incomplete: end every rank of it without waiting
    for (int i = 0; i < ndev; i++) {
      if (out[i]) out[i]->broken = true;
      else nccl().CommAbort(c[i]);
      AnnB200CommDestroy(out[i]);
      out[i] = nullptr;
    }
    delete[] c;
    return annb200::report_error(NOMEM, "communicator");
  }
  delete[] c;
  status = ndev <= 64 ? warm_up(out, ndev) : OK;
  if (status != OK) {
    for (int i = 0; i < ndev; i++) {
      if (out[i]) out[i]->broken = true;
      AnnB200CommDestroy(out[i]);
      out[i] = nullptr;
    }
    return status;
  }
  return OK;
}

extern "C" void AnnB200CommDestroy(AnnB200Comm *c) {
  if (!c) return;
  {
    DevGuard g(c->device);
    if (c->nccl) (c->broken ? nccl().CommAbort : nccl().CommDestroy)(c->nccl);
    if (c->send) cudaFree(c->send);
    if (c->recv) cudaFree(c->recv);
    if (c->host_heads) cudaFreeHost(c->host_heads);
    if (c->host_status) cudaFreeHost(c->host_status);
    if (c->done) cudaEventDestroy(c->done);
    if (c->bounds) cudaFree(c->bounds);
  }
  delete c;
}

extern "C" void AnnB200CommAbort(AnnB200Comm *c) {
  if (!c) return;
  std::lock_guard<std::mutex> lock(c->mu);
  if (c->nccl) {
    DevGuard g(c->device);
    nccl().CommAbort(c->nccl);
  }
  c->nccl = nullptr;
  c->broken = true;
}

extern "C" int AnnB200CommRank(const AnnB200Comm *c) { return c ? c->rank : -1; }
extern "C" int AnnB200CommSize(const AnnB200Comm *c) { return c ? c->nranks : 0; }

namespace annb200 {

int comm_reserve(AnnB200Comm *c, size_t packet_bytes, size_t head_bytes) {
  auto grow = [](void **p, size_t *have, size_t want, bool host) -> cudaError_t {
    if (want <= *have) return cudaSuccess;
    if (*p) host ? cudaFreeHost(*p) : cudaFree(*p);
    *p = nullptr;
    *have = 0;
    cudaError_t e = host ? cudaMallocHost(p, want) : cudaMalloc(p, want);
    if (e == cudaSuccess) *have = want;
    return e;
  };
  cudaError_t e = grow(&c->send, &c->send_bytes, packet_bytes, false);
  if (e == cudaSuccess) e = grow(&c->recv, &c->recv_bytes, packet_bytes * c->nranks, false);
  if (e == cudaSuccess)
    e = grow(reinterpret_cast<void **>(&c->host_heads), &c->host_heads_bytes, head_bytes * c->nranks, true);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return report_error(e == cudaErrorMemoryAllocation ? NOMEM : BACKEND_ERROR, "exchange buffers: %s",
                        cudaGetErrorString(e));
  }
  return OK;
}

int comm_reserve_bounds(AnnB200Comm *c, uint32_t nq) {
  const size_t want = (size_t)nq * (1 + (size_t)c->nranks) * sizeof(double);
  if (want <= c->bounds_bytes) return OK;
  if (c->bounds) cudaFree(c->bounds);
  c->bounds = nullptr;
  c->bounds_bytes = 0;
  cudaError_t e = cudaMalloc(reinterpret_cast<void **>(&c->bounds), want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return report_error(e == cudaErrorMemoryAllocation ? NOMEM : BACKEND_ERROR, "bounds exchange: %s",
                        cudaGetErrorString(e));
  }
  c->bounds_bytes = want;
  return OK;
}

int comm_allgather(AnnB200Comm *c, const void *send, void *recv, size_t bytes, cudaStream_t st) {
  if (c->broken) return report_error(BACKEND_ERROR, "communicator was aborted after a time-out");
  ncclResult_t r = nccl().AllGather(send, recv, bytes, ncclUint8, c->nccl, st);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
  return OK;
}

int comm_wait(AnnB200Comm *c, cudaStream_t st) {
  cudaError_t e = cudaEventRecord(c->done, st);
  if (e != cudaSuccess) return report_error(BACKEND_ERROR, "event: %s", cudaGetErrorString(e));
  const double t0 = now_ms(), limit = (double)timeout_ms();
  for (uint64_t spins = 0;; spins++) {
    e = cudaEventQuery(c->done);
    if (e == cudaSuccess) return OK;
    if (e != cudaErrorNotReady) return report_error(BACKEND_ERROR, "sharded search: %s", cudaGetErrorString(e));
    if ((spins & 255) == 0) {
      ncclResult_t ar = ncclSuccess;
      if (nccl().CommGetAsyncError(c->nccl, &ar) == ncclSuccess && ar != ncclSuccess && ar != ncclInProgress) {
        nccl().CommAbort(c->nccl);
        c->nccl = nullptr;
        c->broken = true;
        return nccl_fail(ar, "all-gather");
      }
      if (now_ms() - t0 > limit) {
        // a peer never joined: end the collective's kernels, retire the communicator
        nccl().CommAbort(c->nccl);
        c->nccl = nullptr;
        c->broken = true;
        return report_error(BACKEND_ERROR, "sharded search: the ranks' exchange did not finish within %ld ms",
                            timeout_ms());
      }
    }
    if (spins > 2000) sched_yield();
  }
}

}  // namespace annb200
