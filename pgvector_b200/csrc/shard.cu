// shard.cu - host side of libannb200.so: shards, search orchestration, merge.
//
// One AnnB200Search call is the device half of the reference's SearchGather
// (ann/server/cuvs.c:4585-4930) for one shard, with the host re-score and
// CPU repair steps removed: selection, exact rescoring and ordering all run
// on the device, and the only host decisions are buffer sizes (a candidate
// list that overflows its capacity is grown and the chunk re-scanned).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/annb200.h"
#include "comm.cuh"
#include "internal.cuh"

using namespace annb200;

namespace {

enum Status { OK = 0, INVALID = 1, UNSUPPORTED = 2, NOMEM = 4, BACKEND_ERROR = 5 };

thread_local std::string g_error;

int fail(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(e == cudaErrorMemoryAllocation ? NOMEM : BACKEND_ERROR, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(expr, what)                            \
  do {                                            \
    cudaError_t e_ = (expr);                      \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Grow-only device allocation.
struct DeviceBuffer {
  void *p = nullptr;
  size_t n = 0;
  ~DeviceBuffer() {
    if (p) cudaFree(p);
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  cudaError_t reserve(size_t bytes) {
    if (bytes <= n) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) n = bytes;
    return e;
  }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

uint64_t row_bytes_of(uint32_t dtype, uint32_t dims) {
  switch (dtype) {
    case DT_F32: return (uint64_t)dims * 4;
    case DT_F16: return (uint64_t)dims * 2;
    case DT_E4M3: return ((uint64_t)dims + 15) / 16 * 16;
    case DT_NVFP4: return ((uint64_t)dims + 15) / 16 * 8;
    case DT_BIT: return ((uint64_t)dims + 7) / 8;
  }
  return 0;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Carves one allocation into 256-byte-aligned pieces.
struct Carver {
  size_t off = 0;
  template <typename T>
  size_t take(size_t count) {
    size_t o = off;
    off = align256(off + count * sizeof(T));
    return o;
  }
};

// ---- launch counting and stage timing (ANN_B200_KERNEL_TIMING=1)
std::atomic<unsigned long long> g_launches{0};
enum Stage { ST_PREP, ST_SAMPLE, ST_BOUND, ST_FILTER, ST_TIGHTEN, ST_FINAL, ST_BITMAP, ST_MERGE, ST_GATHER, ST_PROBE,
             ST_COUNT };
// A call that books every stage of the work it runs to one stage (the
// coarse probe's centroid search) sets this for its duration.
thread_local int g_stage_override = -1;
std::mutex g_stage_mu;
double g_stage_ms[ST_COUNT];
unsigned long long g_stage_calls[ST_COUNT];

bool debug_on() {
  static const int on = [] {
    const char *v = getenv("ANN_B200_DEBUG");
    return v && *v && *v != '0';
  }();
  return on;
}

// Stage timing: ANN_B200_KERNEL_TIMING at the first call, then AnnB200StageTiming.
std::atomic<int> &timing_state() {
  static std::atomic<int> on([] {
    const char *v = getenv("ANN_B200_KERNEL_TIMING");
    return (v && *v && *v != '0') ? 1 : 0;
  }());
  return on;
}

bool timing_on() { return timing_state().load(std::memory_order_relaxed) != 0; }

// Recorded stage spans whose events have not been read yet. A call never
// waits for its stage events: they are read once complete -- at the start of
// a later call, or all of them (waiting) when AnnB200StageTimes reports --
// so the timing adds no host synchronisation to the calls it times.
struct Span {
  int stage, dev;
  cudaEvent_t a, b;
};
std::vector<Span> g_pending;   // under g_stage_mu

// Events of read spans go back to a pool per device instead of being
// destroyed: creating and destroying two events a span cost more host time
// than the shorter stages themselves.
std::vector<std::pair<int, cudaEvent_t>> g_event_pool;   // (device, event), under g_stage_mu

cudaEvent_t pooled_event(int dev) {
  {
    std::lock_guard<std::mutex> lock(g_stage_mu);
    for (size_t i = g_event_pool.size(); i-- > 0;)
      if (g_event_pool[i].first == dev) {
        cudaEvent_t e = g_event_pool[i].second;
        g_event_pool[i] = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
      }
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void pool_event(int dev, cudaEvent_t e) {   // under g_stage_mu
  if (g_event_pool.size() < 4096) g_event_pool.push_back({dev, e});
  else cudaEventDestroy(e);
}

// Fold completed spans into the totals (all of them, waiting, when `wait`).
void collect_spans(bool wait) {
  std::lock_guard<std::mutex> lock(g_stage_mu);
  size_t keep = 0;
  for (size_t i = 0; i < g_pending.size(); i++) {
    Span &sp = g_pending[i];
    cudaError_t e = wait ? cudaEventSynchronize(sp.b) : cudaEventQuery(sp.b);
    if (e == cudaErrorNotReady) {
      g_pending[keep++] = sp;
      continue;
    }
    float ms = 0;
    if (e == cudaSuccess && cudaEventElapsedTime(&ms, sp.a, sp.b) == cudaSuccess) {
      g_stage_ms[sp.stage] += ms;
      g_stage_calls[sp.stage] += 1;
    }
    cudaGetLastError();
    pool_event(sp.dev, sp.a);
    pool_event(sp.dev, sp.b);
  }
  g_pending.resize(keep);
}

// CUDA events around stages of one call, on the call's stream; handed to
// the pending list when the call returns.
struct StageClock {
  cudaStream_t st;
  bool on;
  int dev = 0;
  std::vector<Span> spans;
  explicit StageClock(cudaStream_t s) : st(s), on(timing_on()) {
    if (!on) return;
    cudaGetDevice(&dev);
    collect_spans(false);
  }
  int begin(int stage) {
    if (!on) return -1;
    if (g_stage_override >= 0) stage = g_stage_override;
    Span sp{stage, dev, pooled_event(dev), pooled_event(dev)};
    cudaEventRecord(sp.a, st);
    spans.push_back(sp);
    return (int)spans.size() - 1;
  }
  void end(int h) {
    if (h >= 0) cudaEventRecord(spans[h].b, st);
  }
  ~StageClock() {
    if (!on || spans.empty()) return;
    std::lock_guard<std::mutex> lock(g_stage_mu);
    g_pending.insert(g_pending.end(), spans.begin(), spans.end());
  }
};

void counted(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 2-D FP16 tensor [outer][inner] (row pitch in bytes) read in boxes of
// box_rows x 64 elements with the 128-byte swizzle tcgen05 operands use.
// FP32 rows [outer][inner] in unswizzled boxes of 64 floats x 128 rows (the
// split FP32 tensor scan's raw stage).
bool encode_f32_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_f16_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch,
                    uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw codes of a quantized shard as a 2-D byte tensor [outer][inner bytes]
// (row pitch in bytes), read in unswizzled boxes of box_x bytes x 128 rows;
// bytes past `inner` read as zero.
bool encode_u8_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch,
                   uint32_t box_x) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_x, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A byte tensor [outer][inner] in boxes of 128 bytes x box_rows rows with
// the 128-byte swizzle (the IVF tensor scan's raw segments, box_rows = 128;
// the int8 query block of bit vectors); bytes past `inner` read as zero.
bool encode_u8_seg_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch,
                       uint32_t box_rows = 128) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Formats the tensor scan reads (row pitch a multiple of 16 bytes, as TMA
// needs): FP16 rows, and E4M3 / NVFP4 codes converted to FP16 on chip.
bool tc_format(uint32_t dtype, uint32_t dims, uint64_t row_bytes) {
  switch (dtype) {
    case DT_F32: return row_bytes % 16 == 0;
    case DT_F16: return dims % 8 == 0;
    case DT_E4M3: return row_bytes % 16 == 0;
    case DT_NVFP4: return row_bytes % 16 == 0;
    case DT_BIT: return row_bytes % 16 == 0;
    default: return false;
  }
}

// The tensor map the tensor scan reads `rows` rows of this format from.
bool encode_rows_map(CUtensorMap *map, uint32_t dtype, const void *base, uint32_t dims, uint64_t rows,
                     uint64_t pitch) {
  switch (dtype) {
    case DT_F32: return encode_f32_map(map, base, dims, rows, pitch);
    case DT_F16: return encode_f16_map(map, base, dims, rows, pitch, 128);
    case DT_E4M3: return encode_u8_map(map, base, dims, rows, pitch, 64);
    case DT_NVFP4: return encode_u8_map(map, base, (dims + 1) / 2, rows, pitch, 32);
    case DT_BIT: return encode_u8_map(map, base, ((uint64_t)dims + 7) / 8, rows, pitch, 16);
    default: return false;
  }
}

// The tensor scan's query block: elements a query row (FP16 halves, a
// multiple of 64; for bit vectors the +-1 int8 expansion of the row's bits,
// a multiple of 128), bytes an element, and the block's tensor map
// (128-byte boxes of bn rows, 128-byte swizzle) over nq_pad rows.
uint32_t tc_kpad(const ShardView &v) {
  return v.dtype == DT_BIT ? (uint32_t)((v.row_bytes * 8 + 127) / 128 * 128) : (v.dims + 63) / 64 * 64;
}
size_t tc_qelem(const ShardView &v) { return v.dtype == DT_BIT ? 1 : 2; }
// Queries a tensor-scan tile: at most 128 for FP32 rows (four tiles a stage).
uint32_t tc_bn(const ShardView &v, uint32_t nq) {
  return std::min<uint32_t>(v.dtype == DT_F32 ? 128 : 256, (nq + 31) / 32 * 32);
}
// Whether the tensor scan serves this shard and metric: FP32 rows only for
// L2 and inner product (their split's bound has absolute terms a cosine
// would divide by the row's norm).
bool tc_metric(const ShardView &v, uint32_t metric) { return v.dtype != DT_F32 || metric != M_COS; }
bool encode_query_map(CUtensorMap *map, const ShardView &v, const void *q, uint32_t kpad, uint32_t nq_pad,
                      uint32_t bn) {
  if (v.dtype == DT_BIT) return encode_u8_seg_map(map, q, kpad, nq_pad, kpad, bn);
  return encode_f16_map(map, q, kpad, nq_pad, (uint64_t)kpad * 2, bn);
}

// Relative bound on the approximate dot product's accumulation error (times
// sum |x_i q_i| <= ||x|| ||q||). Tensor scan: each tcgen05.mma (K=16) adds an
// exactly formed FP16 product sum into the FP32 accumulator, so K/16 rounding
// steps, each allowed 4 ulps (2^-21) of the magnitudes involved. CUDA-core
// scan: one FP32 rounding per fused multiply-add, allowed 2 ulps each.
// FP8 scan: two MMAs (the query's two terms) a 32-element K step, each
// allowed 16 ulps (2^-19) of the magnitudes involved -- four times the FP16
// scan's allowance, for an accumulator whose FP8 product alignment the
// documents leave open; tests/test_error_model_gpu.py measures the margin.
double scan_gamma(bool bits, bool tc, uint32_t kpad, uint32_t dims, bool split = false, bool f8 = false) {
  if (bits) return 0.0;
  if (tc && f8) return (2.0 * kpad / 32.0 + 2.0) * std::ldexp(1.0, -19);
  if (tc && split) return (3.0 * kpad / 16.0 + 2.0) * std::ldexp(1.0, -21);   // three MMAs a K step
  if (tc) return ((double)kpad / 16.0 + 2.0) * std::ldexp(1.0, -21);
  return (double)dims * std::ldexp(1.0, -22);
}

constexpr uint64_t kChunkRows = 589824;     // most rows one gathered tensor-scan chunk covers
constexpr uint64_t kNoSampleRows = 32768;  // at most this many candidates: no sample pass
constexpr uint64_t kSampleRows = 16384;    // sample size of the bound

// The bound's sample size: kSampleRows, or ANN_B200_SAMPLE_ROWS (a tuning
// knob, at least 1,024), read once.
uint64_t sample_rows() {
  static const uint64_t n = [] {
    const char *v = getenv("ANN_B200_SAMPLE_ROWS");
    const long long x = v && *v ? atoll(v) : 0;
    return x >= 1024 ? (uint64_t)x : kSampleRows;
  }();
  return n;
}
constexpr uint32_t kBaseCap = 16384;       // initial candidate capacity a query

}  // namespace

struct AnnB200Shard {
  int device = 0;
  int sms = 148;
  ShardView view{};
  int64_t first = 0;
  void *owned[3] = {nullptr, nullptr, nullptr};
  float *n2 = nullptr;
  float *rn = nullptr;
  double *n2x = nullptr;
  uint32_t *maxn2 = nullptr;
  uint64_t norm_rows = 0;     // capacity of n2 / rn
  std::mutex mu;
  DeviceBuffer ws;      // per-search scratch
  DeviceBuffer cand;    // candidate lists
  DeviceBuffer big;     // survivor sort scratch of the rare large case
  uint32_t *hflags = nullptr;  // pinned: flags readback
  CUtensorMap rows_map;        // the shard's FP16 rows, box 64 x 128, for the tensor scan
  bool rows_map_ok = false;
  CUtensorMap scales_map;      // NVFP4 block scales [rows][bblocks], box 16 x 128 (IVF tensor scan)
  bool scales_map_ok = false;
  CUtensorMap seg_map;         // E4M3 / NVFP4 codes, 128-byte swizzled boxes 128 x 128 (IVF tensor scan)
  bool seg_map_ok = false;
  DeviceBuffer staging;        // gathered candidate rows (contiguous) for the tensor scan
  std::mutex rows_mu;          // AnnB200SearchBitmap's row list
  DeviceBuffer bitmap_rows;
  cudaStream_t side = nullptr; // gathers the next chunk's rows while the current one is scanned
  cudaEvent_t ev[5] = {};      // [0,1] slot gathered, [2,3] slot scanned, [4] pass start
};

namespace {
// E4M3 rows go to the FP8 tensor scan when TMA can read their codes in
// 128-byte swizzled boxes (the shard's seg map), unless the call asks for
// the FP16 conversion (ANNB200_FORCE_F16).
bool use_f8(const AnnB200Shard *sh, uint32_t flags) {
  return sh->view.dtype == DT_E4M3 && sh->seg_map_ok && !(flags & ANNB200_FORCE_F16);
}
}  // namespace

namespace annb200 {
int report_error(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return status;
}
void count_launches(unsigned long long n) { counted(n); }
}  // namespace annb200

extern "C" const char *AnnB200LastError(void) { return g_error.c_str(); }

extern "C" int AnnB200DeviceCount(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

extern "C" void AnnB200ShardDestroy(AnnB200Shard *s) {
  if (!s) return;
  {
    DeviceGuard g(s->device);
    for (void *p : s->owned)
      if (p) cudaFree(p);
    if (s->n2) cudaFree(s->n2);
    if (s->rn) cudaFree(s->rn);
    if (s->n2x) cudaFree(s->n2x);
    if (s->maxn2) cudaFree(s->maxn2);
    if (s->hflags) cudaFreeHost(s->hflags);
    for (cudaEvent_t &e : s->ev)
      if (e) cudaEventDestroy(e);
    if (s->side) cudaStreamDestroy(s->side);
    s->ws.release();
    s->cand.release();
    s->big.release();
    s->staging.release();
  }
  delete s;
}

// Point shard s at rows stored on its device (owning nothing) or copy them
// from the host (owned), and compute the per-row norms.
static int shard_bind(AnnB200Shard *s, uint32_t dtype, uint32_t dims, uint64_t rows, const void *codes,
                      const void *block_scales, const float *row_scales, int64_t first_id, bool host,
                      cudaStream_t st, bool sync = true, bool to_half = false) {
  if (dtype > DT_BIT) return fail(INVALID, "unknown storage format %u", dtype);
  if (dims == 0 || dims > (dtype == DT_BIT ? 65536u : 16000u)) return fail(INVALID, "dimensions %u out of range", dims);
  if (rows > 0xffffffffull) return fail(INVALID, "a shard holds at most 2^32-1 rows");
  if (rows && !codes) return fail(INVALID, "rows without codes");
  if ((dtype == DT_E4M3 || dtype == DT_NVFP4) && rows && !row_scales) return fail(INVALID, "row scales missing");
  if (dtype == DT_NVFP4 && rows && !block_scales) return fail(INVALID, "block scales missing");
  if (!host && ((uintptr_t)codes & 15)) return fail(INVALID, "codes must be 16-byte aligned");
  for (void *&p : s->owned)
    if (p) {
      cudaFree(p);
      p = nullptr;
    }
  s->first = first_id;
  ShardView &v = s->view;
  v.dims = dims;
  v.dtype = dtype;
  v.rows = rows;
  v.row_bytes = row_bytes_of(dtype, dims);
  v.bblocks = (dims + 15) / 16;
  const size_t code_bytes = rows * v.row_bytes;
  const size_t bs_bytes = dtype == DT_NVFP4 ? rows * v.bblocks : 0;
  const size_t rs_bytes = (dtype == DT_E4M3 || dtype == DT_NVFP4) ? rows * sizeof(float) : 0;
  cudaError_t e = cudaSuccess;
  if (host && to_half) {
    // host FP32 rows kept as FP16: copied in chunks through a device buffer
    // and rounded to nearest on the device
    const uint64_t chunk_rows = std::max<uint64_t>(1, (64ull << 20) / ((uint64_t)dims * 4));
    void *tmp = nullptr;
    e = cudaMalloc(&s->owned[0], code_bytes);
    if (e == cudaSuccess && rows) e = cudaMalloc(&tmp, std::min<uint64_t>(rows, chunk_rows) * dims * 4);
    for (uint64_t r0 = 0; e == cudaSuccess && r0 < rows; r0 += chunk_rows) {
      const uint64_t m = std::min<uint64_t>(chunk_rows, rows - r0);
      e = cudaMemcpyAsync(tmp, (const float *)codes + r0 * dims, m * dims * 4, cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) {
        launch_f32_to_f16((const float *)tmp, (__half *)s->owned[0] + r0 * dims, m * dims, st);
        counted(1);
        e = cudaGetLastError();
      }
    }
    if (tmp) {
      cudaError_t e2 = cudaStreamSynchronize(st);
      if (e == cudaSuccess) e = e2;
      cudaFree(tmp);
    }
    v.codes = (const uint8_t *)s->owned[0];
    v.bscales = nullptr;
    v.rowscale = nullptr;
  } else if (host) {
    const void *src[3] = {codes, block_scales, row_scales};
    const size_t bytes[3] = {code_bytes, bs_bytes, rs_bytes};
    for (int i = 0; i < 3 && e == cudaSuccess; i++) {
      if (!bytes[i]) continue;
      e = cudaMalloc(&s->owned[i], bytes[i]);
      if (e == cudaSuccess) e = cudaMemcpyAsync(s->owned[i], src[i], bytes[i], cudaMemcpyHostToDevice, st);
    }
    v.codes = (const uint8_t *)s->owned[0];
    v.bscales = (const uint8_t *)s->owned[1];
    v.rowscale = (const float *)s->owned[2];
  } else {
    v.codes = (const uint8_t *)codes;
    v.bscales = (const uint8_t *)block_scales;
    v.rowscale = row_scales;
  }
  if (e == cudaSuccess && dtype != DT_BIT && rows > s->norm_rows) {
    if (s->n2) cudaFree(s->n2);
    if (s->rn) cudaFree(s->rn);
    if (s->n2x) cudaFree(s->n2x);
    s->n2 = s->rn = nullptr;
    s->n2x = nullptr;
    s->norm_rows = 0;
    e = cudaMalloc(&s->n2, rows * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->rn, rows * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->n2x, rows * sizeof(double));
    if (e == cudaSuccess) s->norm_rows = rows;
  }
  if (e == cudaSuccess) e = cudaMemsetAsync(s->maxn2, 0, 16, st);
  if (e == cudaSuccess) {
    v.n2 = s->n2;
    v.rn = s->rn;
    v.n2x = s->n2x;
    launch_shard_stats(v, s->n2, s->rn, s->n2x, s->maxn2, st);
    if (dtype != DT_BIT && rows) counted(2);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && sync) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "shard upload");
  // the tensor scan gathers 128-byte row pieces by TMA (row pitch a multiple of 16 bytes)
  s->rows_map_ok = tc_format(dtype, dims, v.row_bytes) && rows > 0 && rows < (1ull << 31) &&
                   encode_rows_map(&s->rows_map, dtype, v.codes, dims, rows, v.row_bytes);
  // the IVF tensor scan reads NVFP4 block scales by TMA: 16 bytes (four
  // k-blocks) a row a box, so the scale pitch must be a multiple of 16
  s->scales_map_ok = s->rows_map_ok && dtype == DT_NVFP4 && v.bblocks % 16 == 0 &&
                     encode_u8_map(&s->scales_map, v.bscales, v.bblocks, rows, v.bblocks, 16);
  // and quantized codes in 128-byte row pieces (128 bytes = 2 E4M3 / 4 NVFP4 k-blocks)
  s->seg_map_ok = s->rows_map_ok && (dtype == DT_E4M3 || dtype == DT_NVFP4) &&
                  encode_u8_seg_map(&s->seg_map, v.codes, dtype == DT_E4M3 ? dims : (dims + 1) / 2, rows,
                                    v.row_bytes);
  return OK;
}

extern "C" int AnnB200ShardCreate(int device, uint32_t dtype, uint32_t dims, uint64_t rows, const void *codes,
                                  const void *block_scales, const float *row_scales, int64_t first_id,
                                  uint32_t flags, void *stream, AnnB200Shard **out) {
  if (!out) return fail(INVALID, "shard output pointer is NULL");
  *out = nullptr;
  if (device < 0 || device >= AnnB200DeviceCount()) return fail(INVALID, "no CUDA device %d", device);
  DeviceGuard g(device);
  AnnB200Shard *s = new AnnB200Shard();
  s->device = device;
  cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, device);
  cudaError_t e = cudaMalloc(&s->maxn2, 16);
  if (e == cudaSuccess) e = cudaMallocHost(&s->hflags, 64);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking);
  for (int i = 0; i < 5 && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&s->ev[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    int r = cuda_fail(e, "shard");
    AnnB200ShardDestroy(s);
    return r;
  }
  const bool to_half = (flags & ANNB200_SHARD_F32_TO_F16) != 0;
  if (to_half && (dtype != DT_F16 || !(flags & ANNB200_SHARD_HOST))) {
    AnnB200ShardDestroy(s);
    return fail(INVALID, "FP32 rows kept as FP16 need storage format F16 and host rows");
  }
  int r = shard_bind(s, dtype, dims, rows, codes, block_scales, row_scales, first_id, flags & ANNB200_SHARD_HOST,
                     (cudaStream_t)stream, true, to_half);
  if (r != OK) {
    std::string keep = g_error;
    AnnB200ShardDestroy(s);
    g_error = keep;
    return r;
  }
  *out = s;
  return OK;
}

extern "C" int AnnB200ShardAssign(AnnB200Shard *s, uint32_t dtype, uint32_t dims, uint64_t rows, const void *codes,
                                  const void *block_scales, const float *row_scales, int64_t first_id,
                                  void *stream) {
  if (!s) return fail(INVALID, "shard is NULL");
  DeviceGuard g(s->device);
  std::lock_guard<std::mutex> lock(s->mu);
  return shard_bind(s, dtype, dims, rows, codes, block_scales, row_scales, first_id, false, (cudaStream_t)stream);
}

namespace {

// Queries whose survivors outgrew the shared-memory sort: rescored and sorted
// one at a time in a global scratch.
int big_sorts(AnnB200Shard *sh, const SelectLaunch &sl, const uint32_t *big, uint32_t nq, cudaStream_t st) {
  std::vector<uint32_t> hbig(nq);
  CK(cudaMemcpyAsync(hbig.data(), big, nq * sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "big list");
  CK(cudaStreamSynchronize(st), "big list");
  for (uint32_t q = 0; q < nq; q++) {
    if (!hbig[q]) continue;
    uint32_t p2 = 1;
    while (p2 < hbig[q]) p2 <<= 1;
    CK(sh->big.reserve((size_t)p2 * 16), "sort scratch");
    launch_finalize_big(sl, q, (unsigned long long *)sh->big.p, (unsigned long long *)sh->big.p + p2, p2, st);
    counted(1);
    CK(cudaGetLastError(), "large sort");
    CK(cudaStreamSynchronize(st), "large sort");
  }
  return OK;
}

// The bounds exchange in the middle of a deferred sharded search. Each
// query block's survivors kernel writes this rank's bound U of every
// query's k-th exact distance (from its own candidates), one all-gather
// shares them, and survivors_global cuts every rank's survivors again at
// the smallest: with R ranks a rank then re-scores, sorts and sends about
// k / R survivors a query instead of k. Every rank takes part in exactly one
// exchange a query block whatever happens to its own search -- a block that
// failed, or had nothing to search, sends NaN (no bound) -- so the ranks'
// collectives stay paired.
struct BoundsExchange {
  AnnB200Comm *comm;
  uint32_t nq;         // doubles a rank sends: the largest query block
  uint32_t done = 0;   // exchanges taken part in
  double *send() const { return comm->bounds; }
  double *recv() const { return comm->bounds + nq; }
  int run(cudaStream_t st) {
    done++;
    return comm_allgather(comm, send(), recv(), (size_t)nq * sizeof(double), st);
  }
  int skip(cudaStream_t st) {
    cudaMemsetAsync(send(), 0xff, (size_t)nq * sizeof(double), st);   // all-ones bytes: NaN
    return run(st);
  }
};

// One search over queries [q0, q0+nq) (nq within one tensor-scan launch).
//
// defer_flags (device, 8 words) selects the deferred form the sharded search
// uses: everything is enqueued on st with no host synchronisation, and the
// search's flag words are copied to defer_flags when its kernels end; the
// caller inspects them later and runs the search again synchronously if a
// candidate list overflowed or a query needs the large sort. A deferred
// search with `bx` takes part in the bounds exchange once, between its
// survivors and their exact re-score (or not at all if it ends earlier).
int search_block(AnnB200Shard *sh, const void *queries, uint32_t nq, const uint32_t *rows, uint64_t nrows,
                 uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
                 uint32_t *out_count, int32_t *status, cudaStream_t st, bool *any_invalid,
                 uint32_t *defer_flags = nullptr, BoundsExchange *bx = nullptr) {
  const ShardView &v = sh->view;
  const bool bits = v.dtype == DT_BIT;
  const bool window = flags & ANNB200_WINDOW;
  const uint64_t n = rows ? nrows : v.rows;
  const bool tc = sh->rows_map_ok && !(flags & ANNB200_FORCE_SIMT) && nq >= 16 && tc_metric(v, metric);
  const bool split = tc && v.dtype == DT_F32;   // FP32 rows: BF16 halves of rows and queries
  const bool f8 = tc && use_f8(sh, flags);      // E4M3 rows: FP8 MMAs, queries as two E4M3 terms
  const uint32_t kpad = tc ? (f8 ? (v.dims + 127) / 128 * 128 : tc_kpad(v)) : 0;
  const uint32_t bn = tc ? tc_bn(v, nq) : 0;
  const uint32_t qtiles = tc ? (nq + bn - 1) / bn : 0;
  const uint32_t nq_pad = qtiles * bn;
  const uint64_t lo_off = split ? (uint64_t)nq_pad * kpad : 0;   // the low halves' block
  const double gamma = scan_gamma(bits, tc, kpad, v.dims, split, f8);
  // the bound's sample: 16,384 rows (at least 8k), or a sixteenth of the
  // candidates when that is fewer -- a row-sharded rank's smaller share
  // needs no larger sample for the same bound quality (its k-th sampled
  // score sits near the 16k-th row either way), and the sample scan and its
  // selection are fixed costs of every rank
  const bool sample = k > 0 && n > kNoSampleRows;
  const uint64_t target = std::min<uint64_t>(std::max<uint64_t>(sample_rows(), 8ull * k),
                                             std::max<uint64_t>(8ull * k, n / 16));
  const uint64_t stride = sample ? std::max<uint64_t>(1, n / target) : 1;
  const uint64_t S = sample ? n / stride : 0;

  // ---- workspace
  Carver c;
  const size_t o_qn2 = c.take<float>(nq), o_rnq = c.take<float>(nq), o_qn2d = c.take<double>(nq),
               o_err = c.take<double>(nq), o_thr = c.take<float>(nq), o_status = c.take<int32_t>(nq),
               o_q16 = c.take<__half>((size_t)nq_pad * kpad * (split ? 2 : 1)), o_mat = c.take<float>((size_t)S * nq),
               o_cnt = c.take<uint32_t>(nq), o_thr0 = c.take<float>(nq), o_flags = c.take<uint32_t>(16),
               o_big = c.take<uint32_t>(nq), o_exact = c.take<double>((size_t)nq * kSortCap),
               o_qsc = c.take<float>(nq);
  CK(sh->ws.reserve(c.off), "workspace");
  uint8_t *w = (uint8_t *)sh->ws.p;
  double *exact = (double *)(w + o_exact);
  QueryState qs;
  qs.qn2 = (float *)(w + o_qn2);
  qs.rnq = (float *)(w + o_rnq);
  qs.qn2d = (double *)(w + o_qn2d);
  qs.err = (double *)(w + o_err);
  qs.thr = (float *)(w + o_thr);
  qs.status = (int32_t *)(w + o_status);
  qs.q16 = (__half *)(w + o_q16);
  qs.qscale = (float *)(w + o_qsc);
  float *mat = (float *)(w + o_mat);
  uint32_t *cnt = (uint32_t *)(w + o_cnt);
  float *thr0 = (float *)(w + o_thr0);
  uint32_t *dflags = (uint32_t *)(w + o_flags);
  uint32_t *big = (uint32_t *)(w + o_big);

  uint32_t cap = (uint32_t)std::min<uint64_t>(std::max<uint64_t>(n, 1), std::max<uint64_t>(kBaseCap, 8ull * k));
  if (!sample) cap = (uint32_t)std::max<uint64_t>(n, 1);
  CK(sh->cand.reserve((size_t)nq * cap * sizeof(uint2)), "candidate lists");

  CK(cudaMemsetAsync(dflags, 0, 64, st), "memset");
  CK(cudaMemsetAsync(big, 0, nq * sizeof(uint32_t), st), "memset");
  CK(cudaMemsetAsync(cnt, 0, nq * sizeof(uint32_t), st), "memset");
  if (f8 && nq_pad > nq)
    for (int term = 0; term < 2; term++)   // padding query rows of both E4M3 terms score zero
      CK(cudaMemsetAsync((uint8_t *)qs.q16 + ((size_t)term * nq_pad + nq) * kpad, 0, (size_t)(nq_pad - nq) * kpad, st),
         "memset");
  else if (tc && nq_pad > nq)
    for (int half = 0; half < (split ? 2 : 1); half++)   // padding query rows (of both halves) score zero
      CK(cudaMemsetAsync((uint8_t *)qs.q16 + ((size_t)half * lo_off + (size_t)nq * kpad) * tc_qelem(v), 0,
                         (size_t)(nq_pad - nq) * kpad * tc_qelem(v), st),
         "memset");
  StageClock clock(st);
  if (rows) {
    // kernels clamp list entries to the shard; a bad list is reported at the end
    launch_check_rows(rows, nrows, v.rows, dflags, st);
    counted(1);
  }
  int h = clock.begin(ST_PREP);
  launch_prep_queries((const float *)queries, nq, v.dims, metric, kpad, tc && !f8, gamma, sh->maxn2, qs, bits, dflags,
                      st, f8 ? (uint64_t)nq_pad * kpad : lo_off, f8);
  clock.end(h);
  counted(bits && tc ? 2 : 1);
  CK(cudaGetLastError(), "query preparation");

  ScanArgs a{};
  a.s = v;
  a.ids = rows;
  a.queries = (const float *)queries;
  a.nq = nq;
  a.metric = metric;
  a.raw_scale = tc && (v.dtype == DT_E4M3 || v.dtype == DT_NVFP4);   // scores on raw codes
  a.f8 = f8;
  a.qscale = qs.qscale;
  a.thr = qs.thr;
  a.cnt = cnt;
  a.flags = dflags;

  CUtensorMap query_map, query_lo_map;
  if (f8 ? !encode_u8_seg_map(&query_map, qs.q16, kpad, 2ull * nq_pad, kpad, bn)
         : (tc && (!encode_query_map(&query_map, v, qs.q16, kpad, nq_pad, bn) ||
                   (split && !encode_query_map(&query_lo_map, v, qs.q16 + lo_off, kpad, nq_pad, bn)))))
    return fail(BACKEND_ERROR, "tensor map of the query block could not be encoded");
  // One scan launch timed as `stage`. Tensor path: rows come from the shard
  // itself when the candidates are a contiguous run, else from `staged`
  // (virtual row 0 at its first row, filled by gather_rows); FP16 row lists
  // are gathered by the scan itself.
  auto tc_launch = [&](const CUtensorMap &rows_map, int64_t row0) -> cudaError_t {
    return launch_tc_scan(a, rows_map, row0, query_map, split ? &query_lo_map : nullptr, kpad, bn, sh->sms, st);
  };
  auto scan = [&](int stage, const void *staged) -> cudaError_t {
    int hk = clock.begin(stage);
    cudaError_t e;
    if (tc && !staged) {
      e = tc_launch(f8 ? sh->seg_map : sh->rows_map, (int64_t)a.base);
    } else if (tc) {
      CUtensorMap staged_map;
      if (!(f8 ? encode_u8_seg_map(&staged_map, staged, v.dims, a.count, v.row_bytes)
               : encode_rows_map(&staged_map, v.dtype, staged, v.dims, a.count, v.row_bytes)))
        return cudaErrorInvalidValue;
      e = tc_launch(staged_map, 0);
    } else {
      launch_simt_scan(a, st);
      e = cudaGetLastError();
    }
    clock.end(hk);
    counted(1);
    return e;
  };
  // gather candidate rows [base + i*stride] into `slot` on stream gst
  auto gather = [&](uint64_t base, uint64_t stride, uint64_t count, void *slot, cudaStream_t gst) {
    int hg = gst == st ? clock.begin(ST_GATHER) : -1;
    launch_gather_rows(v.codes, v.row_bytes, v.rows, rows, base, stride, count, (uint8_t *)slot, gst);
    clock.end(hg);
    counted(1);
  };

  SelectLaunch sl{};
  sl.s = v;
  sl.ids = rows;
  sl.queries = (const float *)queries;
  sl.nq = nq;
  sl.k = k;
  sl.metric = metric;
  sl.window = window;
  sl.qbytes = bits ? (uint32_t)v.row_bytes : v.dims * 4;
  sl.qs = qs;
  sl.cnt = cnt;
  sl.flags = dflags;
  sl.big = big;
  sl.out_dist = out_dist;
  sl.out_id = out_id;
  sl.out_count = out_count;
  sl.out_cap = out_cap;
  sl.first_id = sh->first;
  sl.index_form = (flags & ANNB200_INDEX_L2) && metric == M_L2;

  // FP16 candidate rows are gathered by the tensor scan itself; quantized
  // rows are copied to a contiguous staging buffer its TMA reads
  const bool stage_rows = tc && v.dtype != DT_F16;
  if (k > 0 && n > 0) {
    // staging: the pass's gathered candidate rows, then the sample's
    if (stage_rows && (rows || sample))
      CK(sh->staging.reserve(((rows ? n : 0) + (sample ? S : 0)) * v.row_bytes), "staging");
    if (sample) {
      a.mode = MODE_MATRIX;
      a.count = S;
      a.base = 0;
      a.stride = stride;
      a.mat = mat;
      a.mat_ld = S;
      const void *staged = nullptr;
      if (stage_rows && (rows || stride > 1)) {
        uint8_t *sample_rows = (uint8_t *)sh->staging.p + (rows ? n * v.row_bytes : 0);
        gather(0, stride, S, sample_rows, st);
        staged = sample_rows;
      }
      CK(scan(ST_SAMPLE, staged), "sample scan");
      h = clock.begin(ST_BOUND);
      launch_kth_bound(mat, S, S, nq, k, metric, window, qs, st);
      clock.end(h);
      counted(2);
    } else {
      launch_fill_thresholds(nq, qs, st);
      counted(1);
    }
    CK(cudaGetLastError(), "bound");
    // ---- filter pass, survivors, exact rescoring and ordering, enqueued with
    // one host synchronisation at the end. Chunks of the filter pass are
    // sized so each appends at most about cap/2 entries a query (tighten
    // after each such capacity chunk); a tensor scan over a row list splits
    // them into overlap chunks growing 3x from 64k rows, gathering chunk i+1
    // on the side stream while chunk i is scanned (two staging slots). If a
    // list overflowed, the whole pass runs again with larger lists.
    CK(cudaMemcpyAsync(thr0, qs.thr, nq * sizeof(float), cudaMemcpyDeviceToDevice, st), "thresholds");
    a.mode = MODE_FILTER;
    a.stride = 1;
    const bool staged_pass = stage_rows && rows;
    for (int attempt = 0;; attempt++) {
      std::vector<std::pair<uint64_t, uint64_t>> chunks;
      std::vector<char> tighten_after;
      uint64_t seen = sample ? S : n;
      for (uint64_t start = 0; start < n;) {
        uint64_t len = n - start;
        if (sample) {
          double room = (double)seen * (double)cap / (2.0 * (double)k);
          len = std::min<uint64_t>(len, std::max<uint64_t>(65536, (uint64_t)room));
          if (start == 0) {
            // head window: its rows pass the sample's bound at about k/S of
            // them, the rows after the tighten at about k/(S + head); head =
            // sqrt(S n) - S minimises the appends of the two
            const double head = std::sqrt((double)S * (double)n) - (double)S;
            len = std::min<uint64_t>(len, std::max<uint64_t>(65536, (uint64_t)head / 128 * 128));
          }
        }
        uint64_t piece = staged_pass ? std::min<uint64_t>(len, 65536) : len;
        for (uint64_t off = 0; off < len;) {
          uint64_t m = std::min(piece, len - off);
          chunks.push_back({start + off, m});
          tighten_after.push_back(0);
          off += m;
          piece = std::min<uint64_t>(piece * 3, kChunkRows);
        }
        tighten_after.back() = 1;
        seen += len;
        start += len;
      }
      // the staging copy holds every candidate row of the pass at its
      // position (exact rescoring reads survivors from it); the sample's
      // copy sits after it
      uint8_t *stage_base = nullptr;
      if (staged_pass) {
        stage_base = (uint8_t *)sh->staging.p;
        // the side stream starts after everything queued so far
        CK(cudaEventRecord(sh->ev[4], st), "event");
        CK(cudaStreamWaitEvent(sh->side, sh->ev[4], 0), "event");
        gather(chunks[0].first, 1, chunks[0].second, stage_base + chunks[0].first * v.row_bytes, sh->side);
        CK(cudaEventRecord(sh->ev[0], sh->side), "event");
      }
      sl.staged = staged_pass ? stage_base : nullptr;
      a.cand = (uint2 *)sh->cand.p;
      a.cap = cap;
      sl.cand = (uint2 *)sh->cand.p;
      sl.cap = cap;
      for (size_t i = 0; i < chunks.size(); i++) {
        const int cur = (int)(i & 1), nxt = (int)((i + 1) & 1);
        if (staged_pass && i + 1 < chunks.size()) {
          gather(chunks[i + 1].first, 1, chunks[i + 1].second, stage_base + chunks[i + 1].first * v.row_bytes,
                 sh->side);
          CK(cudaEventRecord(sh->ev[nxt], sh->side), "event");
        }
        if (staged_pass) CK(cudaStreamWaitEvent(st, sh->ev[cur], 0), "event");
        a.count = chunks[i].second;
        a.base = chunks[i].first;
        CK(scan(ST_FILTER, staged_pass ? stage_base + chunks[i].first * v.row_bytes : nullptr), "filter scan");
        if (i + 1 < chunks.size() && tighten_after[i]) {
          h = clock.begin(ST_TIGHTEN);
          launch_tighten(sl, st);
          clock.end(h);
          counted(1);
        }
      }
      const bool mid = bx && defer_flags;
      h = clock.begin(ST_TIGHTEN);
      sl.upper = mid ? bx->send() : nullptr;
      launch_survivors(sl, st);
      clock.end(h);
      if (mid) {
        h = clock.begin(ST_MERGE);
        int r = bx->run(st);
        clock.end(h);
        if (r != OK) return r;
        h = clock.begin(ST_TIGHTEN);
        launch_survivors_global(sl, bx->recv(), (uint32_t)bx->comm->nranks, bx->nq, st);
        clock.end(h);
        counted(1);
      }
      h = clock.begin(ST_FINAL);
      CK(launch_finalize(sl, exact, st), "finalize");
      clock.end(h);
      counted(3);
      if (defer_flags) {
        CK(cudaMemcpyAsync(defer_flags, dflags, 32, cudaMemcpyDeviceToDevice, st), "flags");
        if (status)
          CK(cudaMemcpyAsync(status, qs.status, nq * sizeof(int32_t), cudaMemcpyDeviceToDevice, st), "status");
        return OK;
      }
      CK(cudaMemcpyAsync(sh->hflags, dflags, 32, cudaMemcpyDeviceToHost, st), "flags");
      CK(cudaStreamSynchronize(st), "search");
      if (sh->hflags[0] & FLAG_TIMEOUT) return fail(BACKEND_ERROR, "tensor scan pipeline timed out");
      if (!(sh->hflags[0] & FLAG_OVERFLOW)) break;
      // run the pass again with lists sized for the largest count seen
      uint64_t need = std::max<uint64_t>(sh->hflags[1], (uint64_t)cap * 2);
      uint32_t ncap = (uint32_t)std::min<uint64_t>(std::max<uint64_t>(n, 1), need + need / 4);
      if (ncap <= cap) ncap = cap + 1;
      cap = ncap;
      CK(sh->cand.reserve((size_t)nq * cap * sizeof(uint2)), "candidate lists");
      CK(cudaMemsetAsync(cnt, 0, nq * sizeof(uint32_t), st), "memset");
      CK(cudaMemsetAsync(big, 0, nq * sizeof(uint32_t), st), "memset");
      CK(cudaMemcpyAsync(qs.thr, thr0, nq * sizeof(float), cudaMemcpyDeviceToDevice, st), "thresholds");
      CK(cudaMemsetAsync(dflags, 0, 8, st), "memset");
      CK(cudaMemsetAsync(dflags + 2, 0, 12, st), "memset");
    }
    if (debug_on())
      fprintf(stderr, "annb200: nq=%u n=%llu k=%u tensor=%d sample=%llu cap=%u candidates=%u survivors=%u\n", nq,
              (unsigned long long)n, k, (int)tc, (unsigned long long)S, cap, sh->hflags[3], sh->hflags[4]);
    if (sh->hflags[0] & FLAG_BIGSORT) {
      int r = big_sorts(sh, sl, big, nq, st);
      if (r != OK) return r;
    }
    if (sh->hflags[0] & FLAG_OUT_CAP) return fail(INVALID, "window results exceed out_cap");
  } else {
    CK(cudaMemsetAsync(out_count, 0, nq * sizeof(uint32_t), st), "memset");
    if (defer_flags) {
      CK(cudaMemcpyAsync(defer_flags, dflags, 32, cudaMemcpyDeviceToDevice, st), "flags");
      if (status)
        CK(cudaMemcpyAsync(status, qs.status, nq * sizeof(int32_t), cudaMemcpyDeviceToDevice, st), "status");
      return OK;
    }
    CK(cudaMemcpyAsync(sh->hflags, dflags, 32, cudaMemcpyDeviceToHost, st), "flags");
    CK(cudaStreamSynchronize(st), "search");
  }
  if (sh->hflags[0] & FLAG_BAD_ROWS)
    return fail(INVALID, "candidate rows must be increasing and < %llu", (unsigned long long)v.rows);
  if (status) CK(cudaMemcpyAsync(status, qs.status, nq * sizeof(int32_t), cudaMemcpyDeviceToDevice, st), "status");
  if (sh->hflags[5]) *any_invalid = true;   // queries prep_queries marked invalid
  return OK;
}

}  // namespace

extern "C" int AnnB200Search(AnnB200Shard *sh, const void *queries, uint32_t nq, const uint32_t *rows, uint64_t nrows,
                             uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap, double *out_dist,
                             int64_t *out_id, uint32_t *out_count, int32_t *status, void *stream) {
  if (!sh) return fail(INVALID, "shard is NULL");
  const ShardView &v = sh->view;
  if (v.dtype == DT_BIT ? metric != M_HAM : metric > M_COS)
    return fail(UNSUPPORTED, "metric %u does not apply to storage format %u", metric, v.dtype);
  if (nq == 0) return OK;
  if (!queries || !out_dist || !out_id || !out_count) return fail(INVALID, "NULL query or result pointer");
  if (!(flags & ANNB200_WINDOW) && out_cap < k) return fail(INVALID, "out_cap %u < k %u", out_cap, k);
  if (rows && nrows > v.rows) return fail(INVALID, "more candidate rows than the shard holds");
  DeviceGuard g(sh->device);
  std::lock_guard<std::mutex> lock(sh->mu);
  cudaStream_t st = (cudaStream_t)stream;
  const uint32_t block = tc_scan_max_queries();
  const uint64_t qbytes = v.dtype == DT_BIT ? v.row_bytes : (uint64_t)v.dims * 4;
  bool any_invalid = false;
  for (uint32_t q0 = 0; q0 < nq; q0 += block) {
    uint32_t m = std::min(block, nq - q0);
    int r = search_block(sh, (const uint8_t *)queries + q0 * qbytes, m, rows, nrows, k, metric, flags, out_cap,
                         out_dist + (uint64_t)q0 * out_cap, out_id + (uint64_t)q0 * out_cap, out_count + q0,
                         status ? status + q0 : nullptr, st, &any_invalid);
    if (r != OK) return r;
  }
  if (any_invalid) return fail(INVALID, "a query is not finite, or has zero norm under cosine");
  return OK;
}

// ---------------------------------------------------------------- batches of independent searches

namespace {

// A 4-byte word per job: nonzero when the job's rows hold a non-finite value.
__global__ void nonfinite_rows(const float *v, uint64_t n, uint32_t *flag) {
  bool bad = false;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    bad |= !isfinite(v[i]);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

constexpr size_t kJobWords = 16;   // a job's flag words: the search's 8, then the rows check

}  // namespace

extern "C" int AnnB200SearchBatch(AnnB200Shard *sh, AnnB200BatchJob *jobs, uint32_t n, void *stream) {
  if (!sh) return fail(INVALID, "shard is NULL");
  if (n && !jobs) return fail(INVALID, "jobs is NULL");
  if (n == 0) return OK;
  DeviceGuard g(sh->device);
  std::lock_guard<std::mutex> lock(sh->mu);
  cudaStream_t st = (cudaStream_t)stream;
  static thread_local DeviceBuffer fl[64];
  static thread_local std::vector<uint32_t> hfl;
  if (sh->device < 0 || sh->device >= 64) return fail(UNSUPPORTED, "device %d", sh->device);
  DeviceBuffer &words = fl[sh->device];
  CK(words.reserve((size_t)n * kJobWords * 4), "batch flags");
  CK(cudaMemsetAsync(words.p, 0, (size_t)n * kJobWords * 4, st), "memset");
  hfl.assign((size_t)n * kJobWords, 0);
  uint32_t *w = (uint32_t *)words.p;
  // every job's rows, then its search, all enqueued; one synchronisation
  std::vector<char> queued(n, 0);
  for (uint32_t j = 0; j < n; j++) {
    AnnB200BatchJob &b = jobs[j];
    b.result = OK;
    if (b.dims == 0 || b.dims > 16000u || b.metric > M_COS || !b.queries || !b.out_dist || !b.out_id ||
        !b.out_count || (b.nrows && !b.rows)) {
      b.result = fail(INVALID, "batch job %u: bad dimensions, metric or pointer", j);
      continue;
    }
    if (b.nq > tc_scan_max_queries()) {
      b.result = fail(UNSUPPORTED, "batch job %u: more than %u queries", j, tc_scan_max_queries());
      continue;
    }
    if (!(b.flags & ANNB200_WINDOW) && b.out_cap < b.k) {
      b.result = fail(INVALID, "batch job %u: out_cap < k", j);
      continue;
    }
    if (b.nq == 0) continue;
    if ((b.flags & ANNB200_REJECT_NONFINITE) && b.nrows) {
      const uint64_t vals = (uint64_t)b.nrows * b.dims;
      const unsigned blocks = (unsigned)std::min<uint64_t>((vals + 255) / 256, (uint64_t)sh->sms * 8);
      nonfinite_rows<<<blocks, 256, 0, st>>>(b.rows, vals, w + (size_t)j * kJobWords + 8);
      counted(1);
    }
    int r = shard_bind(sh, DT_F32, b.dims, b.nrows, b.rows, nullptr, nullptr, 0, false, st, false);
    bool any_invalid = false;
    if (r == OK)
      r = search_block(sh, b.queries, b.nq, nullptr, 0, b.k, b.metric, b.flags & ~ANNB200_REJECT_NONFINITE,
                       b.out_cap, b.out_dist, b.out_id, b.out_count, b.status, st, &any_invalid,
                       w + (size_t)j * kJobWords);
    if (r != OK) {
      b.result = r;
      continue;
    }
    queued[j] = 1;
  }
  CK(cudaMemcpyAsync(hfl.data(), w, (size_t)n * kJobWords * 4, cudaMemcpyDeviceToHost, st), "batch flags");
  CK(cudaStreamSynchronize(st), "batch");
  for (uint32_t j = 0; j < n; j++) {
    if (!queued[j]) continue;
    AnnB200BatchJob &b = jobs[j];
    const uint32_t *f = hfl.data() + (size_t)j * kJobWords;
    if (f[8]) {
      b.result = fail(INVALID, "batch job %u: a row holds a non-finite value", j);
      continue;
    }
    if (f[0] & FLAG_TIMEOUT) {
      b.result = fail(BACKEND_ERROR, "tensor scan pipeline timed out");
      continue;
    }
    if (f[0] & (FLAG_OVERFLOW | FLAG_BIGSORT)) {
      // the rare case: this job again, synchronously (larger lists, the large sort)
      bool any_invalid = false;
      int r = shard_bind(sh, DT_F32, b.dims, b.nrows, b.rows, nullptr, nullptr, 0, false, st);
      if (r == OK)
        r = search_block(sh, b.queries, b.nq, nullptr, 0, b.k, b.metric, b.flags & ~ANNB200_REJECT_NONFINITE,
                         b.out_cap, b.out_dist, b.out_id, b.out_count, b.status, st, &any_invalid);
      if (r == OK && any_invalid) r = fail(INVALID, "a query is not finite, or has zero norm under cosine");
      b.result = r;
      continue;
    }
    if (f[0] & FLAG_OUT_CAP) b.result = fail(INVALID, "window results exceed out_cap");
    else if (f[5]) b.result = fail(INVALID, "a query is not finite, or has zero norm under cosine");
  }
  return OK;
}

// ---------------------------------------------------------------- row-sharded search over NCCL
//
// Every rank searches its own shard (global ids first_id + row) for the
// same queries, then one all-gather moves each rank's packet -- a header
// (its status and its search's flag words), its counts, distances and ids
// -- to every rank, and each rank merges the lists on its device. The
// search is enqueued without a host round trip (the deferred form of
// search_block); the one synchronisation comes after the merge, when every
// rank reads every rank's header. Because all ranks see the same headers,
// they take the same decision: fail together, or -- when some rank's
// candidate list overflowed or needs the large sort -- all search again
// synchronously and exchange a second time. No rank ever leaves a
// collective the others enter.

namespace {

constexpr uint32_t kShardBlocks = 8;                  // query blocks a sharded call (8 x 4,096 queries)
constexpr size_t kHead = 16 + 32 * kShardBlocks;      // status word + 8 flag words a block

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct Packet {
  size_t counts, dist, ids, bytes;
  Packet(uint32_t nq, uint32_t k) {
    counts = kHead;
    dist = counts + align16((size_t)nq * 4);
    ids = dist + (size_t)nq * k * 8;
    bytes = align16(ids + (size_t)nq * k * 8);
  }
};

// This rank's search of the queries into its packet: deferred (flags to the
// header) or synchronous (overflow and large sorts handled here). Returns a
// local status; the caller puts it in the header.
int local_search(AnnB200Shard *sh, uint8_t *pk, const Packet &pl, const void *queries, uint32_t nq,
                 const uint32_t *rows, uint64_t nrows, uint32_t k, uint32_t metric, uint32_t flags, int32_t *status,
                 cudaStream_t st, bool deferred, BoundsExchange *bx) {
  const ShardView &v = sh->view;
  const uint32_t block = tc_scan_max_queries();
  const uint64_t qbytes = v.dtype == DT_BIT ? v.row_bytes : (uint64_t)v.dims * 4;
  bool any_invalid = false;
  for (uint32_t b = 0, q0 = 0; q0 < nq; q0 += block, b++) {
    const uint32_t m = std::min(block, nq - q0);
    int r = search_block(sh, (const uint8_t *)queries + q0 * qbytes, m, rows, nrows, k, metric, flags, k,
                         (double *)(pk + pl.dist) + (uint64_t)q0 * k, (int64_t *)(pk + pl.ids) + (uint64_t)q0 * k,
                         (uint32_t *)(pk + pl.counts) + q0, status ? status + q0 : nullptr, st, &any_invalid,
                         deferred ? (uint32_t *)(pk + 16 + 32 * b) : nullptr, deferred ? bx : nullptr);
    if (r != OK) return r;
    // a block that ended before its exchange (nothing to search) still takes part
    while (deferred && bx && bx->done < b + 1) {
      r = bx->skip(st);
      if (r != OK) return r;
    }
  }
  if (any_invalid) return fail(INVALID, "a query is not finite, or has zero norm under cosine");
  return OK;
}

}  // namespace

namespace {

// The exchange both sharded searches share: `local(pk, deferred, bx)`
// searches this rank's shard into its packet (deferred: enqueued only, flags
// to the header) and returns a local status; `local` is this rank's argument
// check. A deferred local search that uses the bounds exchange takes part in
// `bound_blocks` of them (bx); whichever it did not reach run here, with no
// bounds, so that every rank's collectives pair up. See AnnB200SearchSharded.
template <typename Local>
int sharded_exchange(AnnB200Shard *sh, AnnB200Comm *comm, int local, uint32_t nq, uint32_t k, uint32_t out_cap,
                     double *out_dist, int64_t *out_id, uint32_t *out_count, cudaStream_t st, uint32_t bound_blocks,
                     uint32_t bound_nq, Local local_fn) {
  if (nq == 0) return local;        // every rank sees the same nq: no exchange at all
  DeviceGuard g(sh->device);
  std::lock_guard<std::mutex> lock_comm(comm->mu);
  std::lock_guard<std::mutex> lock(sh->mu);
  const Packet pl(nq, k);
  // without room for the exchange this rank cannot join it: the others end
  // by the communicator's time limit
  int r = comm_reserve(comm, pl.bytes, kHead);
  if (r == OK && bound_blocks) r = comm_reserve_bounds(comm, bound_nq);
  if (r != OK) return r;
  uint8_t *pk = (uint8_t *)comm->send;
  const uint8_t *all = (const uint8_t *)comm->recv;
  std::string local_msg;
  for (int round = 0; round < 2; round++) {
    CK(cudaMemsetAsync(pk, 0, pl.dist, st), "memset");       // header and counts
    BoundsExchange bx{comm, bound_nq};
    if (local == OK) {
      local = local_fn(pk, pl, round == 0, bound_blocks ? &bx : nullptr);
      if (local != OK) CK(cudaMemsetAsync(pk, 0, pl.dist, st), "memset");
    }
    if (local != OK) local_msg = g_error;
    if (round == 0)
      while (bx.done < bound_blocks) {
        r = bx.skip(st);
        if (r != OK) return r;   // this rank's NCCL failed: the others end by the time limit
      }
    *comm->host_status = local;
    CK(cudaMemcpyAsync(pk, comm->host_status, 4, cudaMemcpyHostToDevice, st), "status");
    StageClock clock(st);
    int h = clock.begin(ST_MERGE);
    r = comm_allgather(comm, pk, comm->recv, pl.bytes, st);
    if (r != OK) return r;       // this rank's NCCL failed: the others end by the time limit
    if (out_dist && out_id && out_count && out_cap >= k) {
      CK(launch_merge_ranked(all + pl.dist, pl.bytes, all + pl.ids, pl.bytes, all + pl.counts, pl.bytes,
                             (uint32_t)comm->nranks, nq, k, k, out_cap, out_dist, out_id, out_count, st),
         "merge");
      counted(1);
    }
    clock.end(h);
    CK(cudaMemcpy2DAsync(comm->host_heads, kHead, all, pl.bytes, kHead, comm->nranks, cudaMemcpyDeviceToHost, st),
       "headers");
    r = comm_wait(comm, st);
    if (r != OK) return r;
    // every rank now holds every rank's header: the same decision everywhere
    bool again = false, timeout = false, bad_rows = false, invalid_q = false;
    int first_bad = OK, bad_rank = -1;
    for (int rk = 0; rk < comm->nranks; rk++) {
      const uint8_t *hd = comm->host_heads + (size_t)rk * kHead;
      const int32_t rs = *(const int32_t *)hd;
      if (rs != OK && first_bad == OK) {
        first_bad = rs;
        bad_rank = rk;
      }
      for (uint32_t b = 0; b < kShardBlocks; b++) {
        const uint32_t *fw = (const uint32_t *)(hd + 16 + 32 * b);
        if (round == 0 && (fw[0] & (FLAG_OVERFLOW | FLAG_BIGSORT))) again = true;
        if (fw[0] & FLAG_TIMEOUT) timeout = true;
        if (fw[0] & FLAG_BAD_ROWS) bad_rows = true;
        if (fw[5]) invalid_q = true;
      }
    }
    if (first_bad != OK) {
      if (bad_rank == comm->rank) return fail(first_bad, "%s", local_msg.c_str());
      return fail(first_bad, "rank %d of the sharded search failed", bad_rank);
    }
    if (timeout) return fail(BACKEND_ERROR, "tensor scan pipeline timed out on a rank of the sharded search");
    if (bad_rows) return fail(INVALID, "candidate rows must be increasing and within each rank's shard");
    if (invalid_q) return fail(INVALID, "a query is not finite, or has zero norm under cosine");
    if (!again) return OK;
  }
  return OK;
}

}  // namespace

namespace {

// AnnB200SearchSharded with `local` the caller's own status of this rank
// (a failure of its own preparation: the rank still joins the exchange).
int sharded_search(AnnB200Shard *sh, AnnB200Comm *comm, int local, const void *queries, uint32_t nq,
                   const uint32_t *rows, uint64_t nrows, uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap,
                   double *out_dist, int64_t *out_id, uint32_t *out_count, int32_t *status, void *stream) {
  if (!comm) {
    if (local != OK) return local;
    return AnnB200Search(sh, queries, nq, rows, nrows, k, metric, flags, out_cap, out_dist, out_id, out_count, status,
                         stream);
  }
  if (!sh) return fail(INVALID, "shard is NULL");
  if (comm->device != sh->device)
    return fail(INVALID, "the communicator's device %d is not the shard's %d", comm->device, sh->device);
  // Checks that depend on this rank alone become its status: the rank still
  // joins the exchange, and every rank returns the failure.
  const ShardView &v = sh->view;
  if (local != OK) {
  } else if (flags & ANNB200_WINDOW) local = fail(UNSUPPORTED, "a sharded search returns the strict top k");
  else if (v.dtype == DT_BIT ? metric != M_HAM : metric > M_COS)
    local = fail(UNSUPPORTED, "metric %u does not apply to storage format %u", metric, v.dtype);
  else if (!queries || !out_dist || !out_id || !out_count) local = fail(INVALID, "NULL query or result pointer");
  else if (out_cap < k) local = fail(INVALID, "out_cap %u < k %u", out_cap, k);
  else if (rows && nrows > v.rows) local = fail(INVALID, "more candidate rows than the shard holds");
  else if ((uint64_t)comm->nranks * k > (uint64_t)kSortCap)
    local = fail(UNSUPPORTED, "ranks x k must not exceed %d", kSortCap);
  else if (nq > kShardBlocks * tc_scan_max_queries())
    local = fail(UNSUPPORTED, "at most %u queries a sharded call", kShardBlocks * tc_scan_max_queries());
  // the bounds exchange only when asked (every rank passes the same flags):
  // by default the ranks' lists cross in the one all-gather
  const uint32_t block = tc_scan_max_queries();
  const bool bounds = flags & ANNB200_BOUNDS_EXCHANGE;
  return sharded_exchange(sh, comm, local, nq, k, out_cap, out_dist, out_id, out_count, (cudaStream_t)stream,
                          bounds ? (nq + block - 1) / block : 0, bounds ? std::min(nq, block) : 0,
                          [&](uint8_t *pk, const Packet &pl, bool deferred, BoundsExchange *bx) {
                            return local_search(sh, pk, pl, queries, nq, rows, nrows, k, metric, flags, status,
                                                (cudaStream_t)stream, deferred, bx);
                          });
}

}  // namespace

extern "C" int AnnB200SearchSharded(AnnB200Shard *sh, AnnB200Comm *comm, const void *queries, uint32_t nq,
                                    const uint32_t *rows, uint64_t nrows, uint32_t k, uint32_t metric, uint32_t flags,
                                    uint32_t out_cap, double *out_dist, int64_t *out_id, uint32_t *out_count,
                                    int32_t *status, void *stream) {
  return sharded_search(sh, comm, OK, queries, nq, rows, nrows, k, metric, flags, out_cap, out_dist, out_id,
                        out_count, status, stream);
}

// The coarse probe: each query's nprobe nearest centroids, as a search of
// the centroid shard with k = nprobe (exact distances, ties by list number),
// then the results' ids as list numbers. Scratch for those results is a
// buffer of this host thread on this device, so the shard's lock is taken
// only by the search.
extern "C" int AnnB200ProbeLists(AnnB200Shard *centroids, const float *queries, uint32_t nq, uint32_t nprobe,
                                 uint32_t metric, uint32_t *probes, int32_t *status, void *stream) {
  if (!centroids) return fail(INVALID, "centroid shard is NULL");
  if (nq == 0) return OK;
  if (!queries || !probes) return fail(INVALID, "NULL query or probe pointer");
  if (nprobe == 0 || nprobe > kMaxProbes) return fail(UNSUPPORTED, "nprobe %u outside 1 .. %u", nprobe, kMaxProbes);
  if (centroids->view.dtype == DT_BIT || metric > M_COS)
    return fail(UNSUPPORTED, "coarse probe takes vector centroids and metric L2, IP or cosine");
  DeviceGuard g(centroids->device);
  static thread_local DeviceBuffer scratch[64];
  if (centroids->device < 0 || centroids->device >= 64) return fail(UNSUPPORTED, "device %d", centroids->device);
  DeviceBuffer &w = scratch[centroids->device];
  const size_t pairs = (size_t)nq * nprobe;
  CK(w.reserve(pairs * (sizeof(double) + sizeof(int64_t)) + (size_t)nq * sizeof(uint32_t)), "probe scratch");
  double *dist = (double *)w.p;
  int64_t *ids = (int64_t *)(dist + pairs);
  uint32_t *counts = (uint32_t *)(ids + pairs);
  g_stage_override = ST_PROBE;
  int r = AnnB200Search(centroids, queries, nq, nullptr, 0, nprobe, metric, 0, nprobe, dist, ids, counts, status,
                        stream);
  g_stage_override = -1;
  if (r != OK) return r;
  launch_probe_table(ids, counts, nq, nprobe, centroids->first, probes, (cudaStream_t)stream);
  counted(1);
  CK(cudaGetLastError(), "probe table");
  // the scratch is reused by this thread's next call, on whatever stream
  CK(cudaStreamSynchronize((cudaStream_t)stream), "probe table");
  return OK;
}

namespace {

// One IVF search over queries [q0, q0+nq): plan (probe inversion), then the
// probed lists' rows in windows of growing depth -- rows [0, S) of every
// list (S >= k, so one list alone can supply a bound), then [S, 8S),
// [8S, 64S) ... -- each window appending the rows that pass the current
// thresholds and each followed by a tighten that lowers them from the k-th
// candidate so far (a window appends about 7k rows a query once k rows of
// its lists have been seen). Then the flat search's survivor selection,
// exact rescoring and ordering.
int search_lists_block(AnnB200Shard *sh, const float *queries, uint32_t nq, const uint64_t *offsets,
                       uint32_t nlists, const uint32_t *probes, uint32_t nprobe, const int64_t *row_ids, uint32_t k,
                       uint32_t metric, uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
                       uint32_t *out_count, int32_t *status, cudaStream_t st, bool *any_invalid) {
  const ShardView &v = sh->view;
  // tensor cores when the rows can be read by TMA (and NVFP4's scales too)
  const bool tc = !(flags & ANNB200_FORCE_SIMT) && sh->rows_map_ok &&
                  (v.dtype == DT_F16 || sh->seg_map_ok) && (v.dtype != DT_NVFP4 || sh->scales_map_ok);
  const uint32_t kpad = tc ? (v.dims + 63) / 64 * 64 : 0;
  const double gamma = scan_gamma(false, tc, kpad, v.dims);
  // first window: k rows a list rounded up to the item's row tile (256 rows
  // on tensor cores, 64 on CUDA cores), so every later window (x8) starts on
  // a tile boundary
  const uint64_t tile = tc ? 256 : 64;
  const uint64_t S = std::max<uint64_t>(tile, ((uint64_t)k + tile - 1) / tile * tile);

  Carver c;
  const size_t o_qn2 = c.take<float>(nq), o_rnq = c.take<float>(nq), o_qn2d = c.take<double>(nq),
               o_err = c.take<double>(nq), o_thr = c.take<float>(nq), o_status = c.take<int32_t>(nq),
               o_cnt = c.take<uint32_t>(nq), o_flags = c.take<uint32_t>(16), o_big = c.take<uint32_t>(nq),
               o_exact = c.take<double>((size_t)nq * kSortCap), o_lcount = c.take<uint64_t>(nlists),
               o_lfill = c.take<uint64_t>(nlists), o_tiles = c.take<uint64_t>(nlists),
               o_qoff = c.take<uint64_t>((size_t)nlists + 1), o_toff = c.take<uint64_t>((size_t)nlists + 1),
               o_bsum = c.take<uint64_t>(kMaxLists / 4096), o_qlist = c.take<uint32_t>((size_t)nq * nprobe),
               o_q16 = c.take<__half>((size_t)nq * kpad), o_nzl = c.take<uint32_t>(tc ? nlists : 0),
               o_nzoff = c.take<uint64_t>(tc ? (size_t)nlists + 1 : 0);
  CK(sh->ws.reserve(c.off), "workspace");
  uint8_t *w = (uint8_t *)sh->ws.p;
  double *exact = (double *)(w + o_exact);
  QueryState qs{};
  qs.qn2 = (float *)(w + o_qn2);
  qs.rnq = (float *)(w + o_rnq);
  qs.qn2d = (double *)(w + o_qn2d);
  qs.err = (double *)(w + o_err);
  qs.thr = (float *)(w + o_thr);
  qs.status = (int32_t *)(w + o_status);
  qs.q16 = (__half *)(w + o_q16);
  uint32_t *cnt = (uint32_t *)(w + o_cnt);
  uint32_t *dflags = (uint32_t *)(w + o_flags);
  uint32_t *big = (uint32_t *)(w + o_big);
  ListPlan p{};
  p.offsets = offsets;
  p.nlists = nlists;
  p.rows = v.rows;
  p.probes = probes;
  p.nprobe = nprobe;
  p.nq = nq;
  p.lcount = (unsigned long long *)(w + o_lcount);
  p.lfill = (unsigned long long *)(w + o_lfill);
  p.tiles = (unsigned long long *)(w + o_tiles);
  p.qoff = (unsigned long long *)(w + o_qoff);
  p.toff = (unsigned long long *)(w + o_toff);
  p.bsum = (unsigned long long *)(w + o_bsum);
  p.qlist = (uint32_t *)(w + o_qlist);
  p.bm = tc ? 256 : 64;   // an item: 256 rows x 64 queries on tensor cores, 64 x 16 on CUDA cores
  p.bq = tc ? 64 : 16;
  p.nzl = tc ? (uint32_t *)(w + o_nzl) : nullptr;
  p.nzoff = tc ? (unsigned long long *)(w + o_nzoff) : nullptr;

  // the first window appends at most nprobe * S rows a query: it never overflows
  uint32_t cap = (uint32_t)std::max<uint64_t>({kBaseCap, 8ull * k, (uint64_t)nprobe * S});
  CK(sh->cand.reserve((size_t)nq * cap * sizeof(uint2)), "candidate lists");
  CK(cudaMemsetAsync(dflags, 0, 64, st), "memset");
  CK(cudaMemsetAsync(big, 0, nq * sizeof(uint32_t), st), "memset");
  CK(cudaMemsetAsync(cnt, 0, nq * sizeof(uint32_t), st), "memset");
  if (nlists) {
    CK(cudaMemsetAsync(p.lcount, 0, (size_t)nlists * 8, st), "memset");
    CK(cudaMemsetAsync(p.lfill, 0, (size_t)nlists * 8, st), "memset");
  }
  StageClock clock(st);
  int h = clock.begin(ST_PREP);
  launch_prep_queries(queries, nq, v.dims, metric, kpad, tc, gamma, sh->maxn2, qs, 0, dflags, st);
  launch_list_plan(p, qs, dflags, st);
  clock.end(h);
  counted(1 + (nlists ? 1 : 0) + 2 + list_plan_scan_launches(nlists));
  CK(cudaGetLastError(), "list plan");

  ScanArgs a{};
  a.s = v;
  a.queries = queries;
  a.nq = nq;
  a.metric = metric;
  a.mode = MODE_FILTER;
  a.raw_scale = tc && v.dtype != DT_F16;   // tensor scan of quantized rows: scores on raw codes
  a.thr = qs.thr;
  a.cnt = cnt;
  a.flags = dflags;

  SelectLaunch sl{};
  sl.s = v;
  sl.row_ids = row_ids;
  sl.queries = queries;
  sl.nq = nq;
  sl.k = k;
  sl.metric = metric;
  sl.qbytes = v.dims * 4;
  sl.qs = qs;
  sl.cnt = cnt;
  sl.flags = dflags;
  sl.big = big;
  sl.out_dist = out_dist;
  sl.out_id = out_id;
  sl.out_count = out_count;
  sl.out_cap = out_cap;
  sl.first_id = sh->first;

  auto pass = [&](int stage, uint64_t rbegin, uint64_t rend) -> cudaError_t {
    int hk = clock.begin(stage);
    launch_list_items(p, rbegin, rend, st);
    cudaError_t e = cudaSuccess;
    if (tc)
      e = launch_tc_scan_lists(a, p, rbegin, rend, v.dtype == DT_F16 ? sh->rows_map : sh->seg_map, sh->scales_map,
                               qs.q16, kpad, sh->sms, st);
    else launch_simt_scan_lists(p, rbegin, rend, a, sh->sms, st);
    clock.end(hk);
    counted((nlists ? 1 : 0) + list_plan_scan_launches(nlists) + 1 +
            (tc ? (nlists ? 2 : 0) + list_plan_scan_launches(nlists) : 0));
    return e != cudaSuccess ? e : cudaGetLastError();
  };

  for (;;) {
    a.cand = (uint2 *)sh->cand.p;
    a.cap = cap;
    sl.cand = a.cand;
    sl.cap = cap;
    launch_fill_thresholds(nq, qs, st);
    counted(1);
    for (uint64_t rb = 0, re = S;; rb = re, re = std::min<uint64_t>(re * 8, v.rows)) {
      CK(pass(rb == 0 ? ST_SAMPLE : ST_FILTER, rb, re), "list pass");
      if (re >= v.rows) break;
      h = clock.begin(rb == 0 ? ST_BOUND : ST_TIGHTEN);
      launch_tighten(sl, st);
      clock.end(h);
      counted(1);
    }
    h = clock.begin(ST_TIGHTEN);
    launch_survivors(sl, st);
    clock.end(h);
    h = clock.begin(ST_FINAL);
    CK(launch_finalize(sl, exact, st), "finalize");
    clock.end(h);
    counted(3);
    CK(cudaMemcpyAsync(sh->hflags, dflags, 32, cudaMemcpyDeviceToHost, st), "flags");
    CK(cudaStreamSynchronize(st), "list search");
    if (!(sh->hflags[0] & FLAG_OVERFLOW)) break;
    uint64_t need = std::max<uint64_t>(sh->hflags[1], (uint64_t)cap * 2);
    cap = (uint32_t)std::min<uint64_t>(std::max<uint64_t>(v.rows, 1), need + need / 4);
    CK(sh->cand.reserve((size_t)nq * cap * sizeof(uint2)), "candidate lists");
    CK(cudaMemsetAsync(cnt, 0, nq * sizeof(uint32_t), st), "memset");
    CK(cudaMemsetAsync(big, 0, nq * sizeof(uint32_t), st), "memset");
    CK(cudaMemsetAsync(dflags, 0, 8, st), "memset");
    CK(cudaMemsetAsync(dflags + 2, 0, 12, st), "memset");
  }
  if (debug_on())
    fprintf(stderr, "annb200: lists nq=%u nlists=%u nprobe=%u k=%u sample=%llu cap=%u candidates=%u survivors=%u\n",
            nq, nlists, nprobe, k, (unsigned long long)S, cap, sh->hflags[3], sh->hflags[4]);
  if (sh->hflags[0] & FLAG_BIGSORT) {
    int r = big_sorts(sh, sl, big, nq, st);
    if (r != OK) return r;
  }
  if (sh->hflags[0] & FLAG_BAD_ROWS)
    return fail(INVALID, "list offsets must be non-decreasing and <= %llu", (unsigned long long)v.rows);
  if (status) CK(cudaMemcpyAsync(status, qs.status, nq * sizeof(int32_t), cudaMemcpyDeviceToDevice, st), "status");
  if (sh->hflags[5]) *any_invalid = true;
  return OK;
}

}  // namespace

namespace {

// The argument checks of a list search (the shard's, the call's).
int lists_check(const AnnB200Shard *sh, const float *queries, uint32_t nq, const uint64_t *list_offsets,
                uint32_t nlists, const uint32_t *probes, uint32_t nprobe, uint32_t k, uint32_t metric, uint32_t flags,
                uint32_t out_cap, const double *out_dist, const int64_t *out_id, const uint32_t *out_count) {
  const ShardView &v = sh->view;
  if (v.dtype == DT_BIT || metric > M_COS)
    return fail(UNSUPPORTED, "list search takes L2, inner product or cosine over vector rows");
  if (flags & ANNB200_WINDOW) return fail(UNSUPPORTED, "list search returns the strict top k only");
  if (nq == 0) return OK;
  if (!queries || !out_dist || !out_id || !out_count || !list_offsets || (nprobe && !probes))
    return fail(INVALID, "NULL query, list, probe or result pointer");
  if (out_cap < k) return fail(INVALID, "out_cap %u < k %u", out_cap, k);
  if (nlists > kMaxLists) return fail(UNSUPPORTED, "more than %u lists", kMaxLists);
  if (nprobe > kMaxProbes) return fail(UNSUPPORTED, "more than %u probes a query", kMaxProbes);
  return OK;
}

// Every query's list search, in blocks of 4,096 queries (the shard's lock held).
int search_lists_all(AnnB200Shard *sh, const float *queries, uint32_t nq, const uint64_t *list_offsets,
                     uint32_t nlists, const uint32_t *probes, uint32_t nprobe, const int64_t *row_ids, uint32_t k,
                     uint32_t metric, uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
                     uint32_t *out_count, int32_t *status, cudaStream_t st) {
  const ShardView &v = sh->view;
  const uint32_t block = 4096;
  bool any_invalid = false;
  for (uint32_t q0 = 0; q0 < nq; q0 += block) {
    const uint32_t m = std::min(block, nq - q0);
    int r;
    if (k == 0) {
      CK(cudaMemsetAsync(out_count + q0, 0, m * sizeof(uint32_t), st), "memset");
      r = OK;
    } else {
      r = search_lists_block(sh, queries + (uint64_t)q0 * v.dims, m, list_offsets, nlists, probes + (uint64_t)q0 * nprobe,
                             nprobe, row_ids, k, metric, flags, out_cap, out_dist + (uint64_t)q0 * out_cap,
                             out_id + (uint64_t)q0 * out_cap, out_count + q0, status ? status + q0 : nullptr, st,
                             &any_invalid);
    }
    if (r != OK) return r;
  }
  CK(cudaStreamSynchronize(st), "list search");
  if (any_invalid) return fail(INVALID, "a query is not finite, has zero norm under cosine, or probes a bad list");
  return OK;
}

}  // namespace

extern "C" int AnnB200SearchLists(AnnB200Shard *sh, const float *queries, uint32_t nq, const uint64_t *list_offsets,
                                  uint32_t nlists, const uint32_t *probes, uint32_t nprobe, const int64_t *row_ids,
                                  uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap, double *out_dist,
                                  int64_t *out_id, uint32_t *out_count, int32_t *status, void *stream) {
  if (!sh) return fail(INVALID, "shard is NULL");
  int r = lists_check(sh, queries, nq, list_offsets, nlists, probes, nprobe, k, metric, flags, out_cap, out_dist,
                      out_id, out_count);
  if (r != OK || nq == 0) return r;
  DeviceGuard g(sh->device);
  std::lock_guard<std::mutex> lock(sh->mu);
  return search_lists_all(sh, queries, nq, list_offsets, nlists, probes, nprobe, row_ids, k, metric, flags, out_cap,
                          out_dist, out_id, out_count, status, (cudaStream_t)stream);
}

extern "C" int AnnB200SearchListsSharded(AnnB200Shard *sh, AnnB200Comm *comm, const float *queries, uint32_t nq,
                                         const uint64_t *list_offsets, uint32_t nlists, const uint32_t *probes,
                                         uint32_t nprobe, const int64_t *row_ids, uint32_t k, uint32_t metric,
                                         uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
                                         uint32_t *out_count, int32_t *status, void *stream) {
  if (!comm)
    return AnnB200SearchLists(sh, queries, nq, list_offsets, nlists, probes, nprobe, row_ids, k, metric, flags, out_cap,
                              out_dist, out_id, out_count, status, stream);
  if (!sh) return fail(INVALID, "shard is NULL");
  if (comm->device != sh->device)
    return fail(INVALID, "the communicator's device %d is not the shard's %d", comm->device, sh->device);
  int local = lists_check(sh, queries, nq, list_offsets, nlists, probes, nprobe, k, metric, flags, out_cap, out_dist,
                          out_id, out_count);
  if (local == OK && (uint64_t)comm->nranks * k > (uint64_t)kSortCap)
    local = fail(UNSUPPORTED, "ranks x k must not exceed %d", kSortCap);
  // the list search synchronises on its own (its windows): the exchange's
  // header carries only its status
  return sharded_exchange(sh, comm, local, nq, k, out_cap, out_dist, out_id, out_count, (cudaStream_t)stream, 0, 0,
                          [&](uint8_t *pk, const Packet &pl, bool, BoundsExchange *) {
                            return search_lists_all(sh, queries, nq, list_offsets, nlists, probes, nprobe, row_ids, k,
                                                    metric, flags, k, (double *)(pk + pl.dist),
                                                    (int64_t *)(pk + pl.ids), (uint32_t *)(pk + pl.counts), status,
                                                    (cudaStream_t)stream);
                          });
}

extern "C" int AnnB200MergeTopk(const double *dist, const int64_t *ids, const uint32_t *counts, uint32_t nlists,
                                uint32_t nq, uint32_t list_cap, uint32_t k, uint32_t flags, uint32_t out_cap,
                                double *out_dist, int64_t *out_id, uint32_t *out_count, void *stream) {
  if (nq == 0) return OK;
  if (!dist || !ids || !counts || !out_dist || !out_id || !out_count) return fail(INVALID, "NULL pointer");
  if (nlists == 0 || nlists > 64 || (uint64_t)nlists * list_cap > (uint64_t)kSortCap)
    return fail(UNSUPPORTED, "merge takes at most 64 lists and 4096 entries a query");
  if (!(flags & ANNB200_WINDOW) && out_cap < k) return fail(INVALID, "out_cap %u < k %u", out_cap, k);
  cudaStream_t st = (cudaStream_t)stream;
  StageClock clock(st);
  if (!(flags & ANNB200_WINDOW)) {
    // the k best of sorted lists, by rank; queued on the stream with no host
    // round trip (k <= out_cap was checked)
    const uint64_t per = (uint64_t)nq * list_cap;
    int h = clock.begin(ST_MERGE);
    CK(launch_merge_ranked(dist, per * sizeof(double), ids, per * sizeof(int64_t), counts, (uint64_t)nq * 4, nlists,
                           nq, list_cap, k, out_cap, out_dist, out_id, out_count, st),
       "merge");
    clock.end(h);
    counted(1);
    return OK;
  }
  // a buffer of this host thread on the current device (a thread may merge on several)
  static thread_local DeviceBuffer fls[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(UNSUPPORTED, "device %d", dev);
  DeviceBuffer &fl = fls[dev];
  CK(fl.reserve(64), "merge flags");
  CK(cudaMemsetAsync(fl.p, 0, 16, st), "memset");
  int h = clock.begin(ST_MERGE);
  CK(launch_merge(dist, ids, counts, nlists, nq, list_cap, k, flags & ANNB200_WINDOW, out_cap, out_dist, out_id,
                  out_count, (uint32_t *)fl.p, st),
     "merge");
  clock.end(h);
  counted(1);
  uint32_t hf = 0;
  CK(cudaMemcpyAsync(&hf, fl.p, 4, cudaMemcpyDeviceToHost, st), "merge flags");
  CK(cudaStreamSynchronize(st), "merge");
  if (hf & FLAG_OUT_CAP) return fail(INVALID, "window results exceed out_cap");
  return OK;
}

extern "C" int AnnB200RescoreRows(const float *queries, uint32_t nq, uint32_t dims, const float *rows,
                                  uint32_t stride, const uint32_t *counts, float *out, void *stream) {
  if (nq == 0 || stride == 0) return OK;
  if (!queries || !rows || !out) return fail(INVALID, "NULL pointer");
  if (dims == 0) return fail(INVALID, "dimensions 0");
  if ((uint64_t)nq * stride > 0xffffffffull) return fail(INVALID, "more than 2^32 candidates");
  cudaStream_t st = (cudaStream_t)stream;
  launch_rescore_rows(queries, nq, dims, rows, stride, counts, out, st);
  CK(cudaGetLastError(), "rescore rows");
  counted(1);
  return OK;
}

extern "C" int AnnB200RescoreGather(const float *queries, uint32_t nq, uint32_t dims, const float *rows,
                                    const uint64_t *ords, uint32_t stride, const uint32_t *counts, float *out,
                                    void *stream) {
  if (nq == 0 || stride == 0) return OK;
  if (!queries || !rows || !ords || !out) return fail(INVALID, "NULL pointer");
  if (dims == 0) return fail(INVALID, "dimensions 0");
  if ((uint64_t)nq * stride > 0xffffffffull) return fail(INVALID, "more than 2^32 candidates");
  cudaStream_t st = (cudaStream_t)stream;
  launch_rescore_gather(queries, nq, dims, rows, ords, stride, counts, out, st);
  CK(cudaGetLastError(), "rescore gather");
  counted(1);
  return OK;
}

namespace {

int bitmap_rows_at(const uint32_t *words, uint64_t nbits, uint32_t base, uint32_t *rows, uint64_t *count,
                   cudaStream_t st) {
  if (!count) return fail(INVALID, "count pointer is NULL");
  *count = 0;
  if (nbits == 0) return OK;
  if (!words || !rows) return fail(INVALID, "NULL pointer");
  if (nbits > 0xffffffffull || (uint64_t)base + nbits > 0x100000000ull)
    return fail(INVALID, "row numbers past 2^32");
  // a buffer of this host thread on the current device (a thread may expand on several)
  static thread_local DeviceBuffer scratches[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(UNSUPPORTED, "device %d", dev);
  DeviceBuffer &scratch = scratches[dev];
  const uint32_t nb = bitmap_blocks(nbits);
  CK(scratch.reserve(align256((size_t)nb * 4) + 8), "bitmap scratch");
  unsigned long long *total = (unsigned long long *)((uint8_t *)scratch.p + align256((size_t)nb * 4));
  StageClock clock(st);
  int h = clock.begin(ST_BITMAP);
  launch_bitmap_rows(words, nbits, rows, (uint32_t *)scratch.p, total, st, base);
  clock.end(h);
  counted(3);
  CK(cudaGetLastError(), "bitmap rows");
  // the count comes back through pinned memory: a pageable destination
  // costs the copy a staging pass through the driver
  struct PinnedCount {
    unsigned long long *p = nullptr;
    PinnedCount() {
      void *v = nullptr;
      if (cudaMallocHost(&v, 8) == cudaSuccess) p = (unsigned long long *)v;
      else cudaGetLastError();
    }
    ~PinnedCount() {
      if (p) cudaFreeHost(p);
    }
  };
  static thread_local PinnedCount found;
  unsigned long long pageable = 0;
  unsigned long long *dst = found.p ? found.p : &pageable;
  CK(cudaMemcpyAsync(dst, total, 8, cudaMemcpyDeviceToHost, st), "bitmap count");
  CK(cudaStreamSynchronize(st), "bitmap rows");
  *count = *dst;
  return OK;
}

}  // namespace

extern "C" int AnnB200BitmapRows(const uint32_t *words, uint64_t nbits, uint32_t *rows, uint64_t *count,
                                 void *stream) {
  return bitmap_rows_at(words, nbits, 0, rows, count, (cudaStream_t)stream);
}

extern "C" int AnnB200BitmapRowsFrom(const uint32_t *words, uint64_t nbits, uint32_t first_row, uint32_t *rows,
                                     uint64_t *count, void *stream) {
  return bitmap_rows_at(words, nbits, first_row, rows, count, (cudaStream_t)stream);
}

// The bitmap's rows go to a buffer of the shard (its own lock: the search
// takes the shard's), then the search over them -- one call, so the host
// turns from the count's read-back straight to the search's launches.
extern "C" int AnnB200SearchBitmap(AnnB200Shard *sh, AnnB200Comm *comm, const void *queries, uint32_t nq,
                                   const uint32_t *words, uint64_t nbits, uint32_t k, uint32_t metric, uint32_t flags,
                                   uint32_t out_cap, double *out_dist, int64_t *out_id, uint32_t *out_count,
                                   int32_t *status, uint64_t *nrows_out, void *stream) {
  if (nrows_out) *nrows_out = 0;
  if (!sh) return fail(INVALID, "shard is NULL");
  std::lock_guard<std::mutex> lock(sh->rows_mu);
  DeviceGuard g(sh->device);
  uint64_t n = 0;
  int local = OK;
  if (nbits > sh->view.rows) local = fail(INVALID, "the bitmap has more bits than the shard has rows");
  else if (nbits && !words) local = fail(INVALID, "bitmap words are NULL");
  else if (cudaError_t e = sh->bitmap_rows.reserve(std::max<uint64_t>(nbits, 1) * sizeof(uint32_t)))
    local = fail(e == cudaErrorMemoryAllocation ? NOMEM : BACKEND_ERROR, "bitmap rows: %s", cudaGetErrorString(e));
  else
    local = bitmap_rows_at(words, nbits, 0, (uint32_t *)sh->bitmap_rows.p, &n, (cudaStream_t)stream);
  if (local != OK) cudaGetLastError();
  if (nrows_out) *nrows_out = n;
  // an empty row list is a search over no rows (not over the whole shard)
  return sharded_search(sh, comm, local, queries, nq, (const uint32_t *)sh->bitmap_rows.p, n, k, metric, flags,
                        out_cap, out_dist, out_id, out_count, status, stream);
}

extern "C" unsigned long long AnnB200LaunchCount(void) { return g_launches.load(); }

extern "C" int AnnB200StageTiming(int on) {
  if (on < 0) return timing_on() ? 1 : 0;
  return timing_state().exchange(on ? 1 : 0);
}

extern "C" int AnnB200StageTimes(double *ms, unsigned long long *calls, uint32_t n, int reset) {
  collect_spans(true);
  std::lock_guard<std::mutex> lock(g_stage_mu);
  for (uint32_t i = 0; i < n && i < (uint32_t)ST_COUNT; i++) {
    if (ms) ms[i] = g_stage_ms[i];
    if (calls) calls[i] = g_stage_calls[i];
  }
  if (reset)
    for (int i = 0; i < ST_COUNT; i++) {
      g_stage_ms[i] = 0;
      g_stage_calls[i] = 0;
    }
  return timing_on() ? ST_COUNT : 0;
}

extern "C" int AnnB200ScoreMatrix(AnnB200Shard *sh, const void *queries, uint32_t nq, const uint32_t *rows,
                                  uint64_t nrows, uint32_t metric, uint32_t flags, float *out, double *err,
                                  void *stream) {
  if (!sh) return fail(INVALID, "shard is NULL");
  const ShardView &v = sh->view;
  if (v.dtype == DT_BIT ? metric != M_HAM : metric > M_COS)
    return fail(UNSUPPORTED, "metric %u does not apply to storage format %u", metric, v.dtype);
  const uint64_t n = rows ? nrows : v.rows;
  if (nq == 0 || n == 0) return OK;
  if (!queries || !out) return fail(INVALID, "NULL query or output pointer");
  if (nq > tc_scan_max_queries()) return fail(UNSUPPORTED, "at most %u queries a call", tc_scan_max_queries());
  DeviceGuard g(sh->device);
  std::lock_guard<std::mutex> lock(sh->mu);
  cudaStream_t st = (cudaStream_t)stream;
  const bool bits = v.dtype == DT_BIT;
  const bool tc = sh->rows_map_ok && !(flags & ANNB200_FORCE_SIMT) && nq >= 16 && tc_metric(v, metric);
  const bool split = tc && v.dtype == DT_F32;   // FP32 rows: BF16 halves of rows and queries
  const bool f8 = tc && use_f8(sh, flags);
  const uint32_t kpad = tc ? (f8 ? (v.dims + 127) / 128 * 128 : tc_kpad(v)) : 0;
  const uint32_t bn = tc ? tc_bn(v, nq) : 0;
  const uint32_t nq_pad = tc ? (nq + bn - 1) / bn * bn : 0;
  const uint64_t lo_off = split ? (uint64_t)nq_pad * kpad : 0;
  Carver c;
  const size_t o_qn2 = c.take<float>(nq), o_rnq = c.take<float>(nq), o_qn2d = c.take<double>(nq),
               o_err = c.take<double>(nq), o_thr = c.take<float>(nq), o_status = c.take<int32_t>(nq),
               o_q16 = c.take<__half>((size_t)nq_pad * kpad * (split ? 2 : 1)), o_flags = c.take<uint32_t>(16),
               o_qsc = c.take<float>(nq);
  CK(sh->ws.reserve(c.off), "workspace");
  uint8_t *w = (uint8_t *)sh->ws.p;
  QueryState qs;
  qs.qn2 = (float *)(w + o_qn2);
  qs.rnq = (float *)(w + o_rnq);
  qs.qn2d = (double *)(w + o_qn2d);
  qs.err = (double *)(w + o_err);
  qs.thr = (float *)(w + o_thr);
  qs.status = (int32_t *)(w + o_status);
  qs.q16 = (__half *)(w + o_q16);
  qs.qscale = (float *)(w + o_qsc);
  uint32_t *dflags = (uint32_t *)(w + o_flags);
  CK(cudaMemsetAsync(dflags, 0, 64, st), "memset");
  if (f8 && nq_pad > nq)
    for (int term = 0; term < 2; term++)
      CK(cudaMemsetAsync((uint8_t *)qs.q16 + ((size_t)term * nq_pad + nq) * kpad, 0, (size_t)(nq_pad - nq) * kpad, st),
         "memset");
  else if (tc && nq_pad > nq)
    for (int half = 0; half < (split ? 2 : 1); half++)
      CK(cudaMemsetAsync((uint8_t *)qs.q16 + ((size_t)half * lo_off + (size_t)nq * kpad) * tc_qelem(v), 0,
                         (size_t)(nq_pad - nq) * kpad * tc_qelem(v), st),
         "memset");
  if (rows) launch_check_rows(rows, nrows, v.rows, dflags, st);
  launch_prep_queries((const float *)queries, nq, v.dims, metric, kpad, tc && !f8,
                      scan_gamma(bits, tc, kpad, v.dims, split, f8), sh->maxn2, qs, bits, dflags, st,
                      f8 ? (uint64_t)nq_pad * kpad : lo_off, f8);
  counted(bits && tc ? 2 : 1);
  ScanArgs a{};
  a.s = v;
  a.ids = rows;
  a.count = n;
  a.base = 0;
  a.stride = 1;
  a.queries = (const float *)queries;
  a.nq = nq;
  a.metric = metric;
  a.mode = MODE_MATRIX;
  a.mat = out;
  a.mat_ld = n;
  a.flags = dflags;
  a.raw_scale = tc && (v.dtype == DT_E4M3 || v.dtype == DT_NVFP4);
  a.f8 = f8;
  a.qscale = qs.qscale;
  if (tc) {
    CUtensorMap query_map, query_lo_map;
    if (f8 ? !encode_u8_seg_map(&query_map, qs.q16, kpad, 2ull * nq_pad, kpad, bn)
           : (!encode_query_map(&query_map, v, qs.q16, kpad, nq_pad, bn) ||
              (split && !encode_query_map(&query_lo_map, v, qs.q16 + lo_off, kpad, nq_pad, bn))))
      return fail(BACKEND_ERROR, "tensor map of the query block could not be encoded");
    auto tc_launch = [&](const CUtensorMap &rows_map) -> cudaError_t {
      return launch_tc_scan(a, rows_map, 0, query_map, split ? &query_lo_map : nullptr, kpad, bn, sh->sms, st);
    };
    if (!rows || v.dtype == DT_F16) {
      CK(tc_launch(f8 ? sh->seg_map : sh->rows_map), "score scan");   // FP16 row lists: gathered by the scan
    } else {
      CK(sh->staging.reserve(n * v.row_bytes), "staging");
      launch_gather_rows(v.codes, v.row_bytes, v.rows, rows, 0, 1, n, (uint8_t *)sh->staging.p, st);
      CUtensorMap staged;
      if (!(f8 ? encode_u8_seg_map(&staged, sh->staging.p, v.dims, n, v.row_bytes)
               : encode_rows_map(&staged, v.dtype, sh->staging.p, v.dims, n, v.row_bytes)))
        return fail(BACKEND_ERROR, "tensor map of the staged rows could not be encoded");
      CK(tc_launch(staged), "score scan");
      counted(1);
    }
  } else {
    launch_simt_scan(a, st);
    CK(cudaGetLastError(), "score scan");
  }
  counted(1);
  launch_v_to_distance(out, n, nq, metric, qs, st);
  counted(1);
  if (err) CK(cudaMemcpyAsync(err, qs.err, nq * sizeof(double), cudaMemcpyDeviceToDevice, st), "err");
  CK(cudaMemcpyAsync(sh->hflags, dflags, 4, cudaMemcpyDeviceToHost, st), "flags");
  CK(cudaStreamSynchronize(st), "score matrix");
  if (sh->hflags[0] & FLAG_TIMEOUT) return fail(BACKEND_ERROR, "tensor scan pipeline timed out");
  if (sh->hflags[0] & FLAG_BAD_ROWS) return fail(INVALID, "candidate rows must be increasing and < rows");
  return OK;
}
