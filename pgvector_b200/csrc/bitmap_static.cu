// bitmap_static.cu - filter-bitmap expansion that allocates no device memory.
//
// AnnB200BitmapRows keeps the per-block offsets of its three kernels in a
// device buffer it allocates the first time a thread calls it, and grows it
// for larger bitmaps. Some callers cannot do that on their call path: a
// worker that serves requests from a device-memory budget it reserved up
// front, or a latency-critical caller for whom cudaMalloc / cudaFree (which
// synchronise the device) are not acceptable between requests. For them,
// AnnB200BitmapRowsStatic runs the same kernels with that scratch in a
// file-scope __device__ array of fixed size, which every GPU that loads this
// library holds until the process exits.
//
// The array holds kMaxBlocks block offsets (one per 32,768 bitmap bits) and
// the 64-bit row count after them: 256 KB + 8 B, enough for bitmaps of up to
// 2^31 rows. Larger bitmaps are rejected with ANN_INVALID. Every call shares
// the one array; calls whose kernels overlap on a device (different
// streams, or threads, at the same time) race on it and must be serialised
// by the caller. Nothing in the array has to start at zero: each call
// overwrites every offset and the count it reads.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/annb200.h"
#include "internal.cuh"

namespace {

constexpr uint32_t kMaxBlocks = 65536;                          // bitmap blocks of 1,024 words
constexpr uint64_t kMaxBits = (uint64_t)kMaxBlocks * 1024 * 32;  // 2^31 rows

// [0, kMaxBlocks): per-block offsets; [kMaxBlocks, kMaxBlocks + 2): the count (u64)
static __device__ __align__(256) uint32_t g_bitmap_scratch[kMaxBlocks + 2];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint32_t *g_scratch_addr[kMaxDevices];  // the array's device address, per device

// The array's device address on the current device, looked up once per
// device (host code cannot take the address of a __device__ variable; the
// runtime gives it here).
int scratch_for_current_device(uint32_t **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return annb200::report_error(5, "no current CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return annb200::report_error(2, "device %d is beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bitmap_scratch);
    if (e != cudaSuccess || !p)
      return annb200::report_error(5, "scratch address on device %d: %s", dev, cudaGetErrorString(e));
    g_scratch_addr[dev] = static_cast<uint32_t *>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" int AnnB200BitmapRowsStatic(const uint32_t *words, uint64_t nbits, uint32_t *rows, uint64_t *count,
                                       void *stream) {
  if (!count) return annb200::report_error(1, "count pointer is NULL");
  *count = 0;
  if (nbits == 0) return 0;
  if (!words || !rows) return annb200::report_error(1, "NULL pointer");
  if (nbits > kMaxBits)
    return annb200::report_error(1, "bitmap of %llu rows exceeds the static scratch limit of %llu rows",
                                 (unsigned long long)nbits, (unsigned long long)kMaxBits);
  uint32_t *scratch = nullptr;
  int r = scratch_for_current_device(&scratch);
  if (r != 0) return r;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long *total = reinterpret_cast<unsigned long long *>(scratch + kMaxBlocks);
  annb200::launch_bitmap_rows(words, nbits, rows, scratch, total, st);
  annb200::count_launches(3);
  cudaError_t e = cudaGetLastError();
  unsigned long long found = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&found, total, sizeof(found), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return annb200::report_error(5, "bitmap rows: %s", cudaGetErrorString(e));
  *count = found;
  return 0;
}
