// internal.cuh - shared definitions of the B200 gather-scan kernels.
//
// Pipeline of one AnnB200Search call (all on the caller's stream):
//   1. prep_queries: per-query squared norm, FP16 copy for the tensor scan,
//      and the error bound of the approximate score.
//   2. sample scan (MATRIX mode) over every stride-th candidate, then
//      kth_bound: per query the k-th smallest approximate score of the sample
//      bounds the k-th exact distance from above.
//   3. filter scan (FILTER mode), in chunks of the candidate list: every
//      (row, query) whose approximate score can still reach the final answer,
//      given the bound and the error margin, is appended to the query's
//      candidate list. Between chunks, tighten: the k-th smallest score of the
//      list so far lowers the bound and drops entries that can no longer win.
//   4. finalize: per query, the exact reference-order distance of each
//      surviving candidate, sort by (distance, id), top-k or tolerance window.
// The approximate scores never decide a result: they only prune, with margins
// that bound their error, so the result equals the exact scan bit for bit.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace annb200 {

enum Dtype : uint32_t { DT_F32 = 0, DT_F16 = 1, DT_E4M3 = 2, DT_NVFP4 = 3, DT_BIT = 4 };
enum Metric : uint32_t { M_L2 = 0, M_IP = 1, M_COS = 2, M_HAM = 3 };
enum ScanMode : int { MODE_MATRIX = 0, MODE_FILTER = 1 };

// Error flags a search's kernels raise in its workspace.
enum Flag : uint32_t {
  FLAG_OVERFLOW = 1u,    // a query's candidate list outgrew its capacity
  FLAG_BIGSORT = 2u,     // a query kept more survivors than shared memory sorts
  FLAG_TIMEOUT = 4u,     // a pipeline wait in the tensor scan ran out
  FLAG_BAD_ROWS = 8u,    // the candidate row list is not strictly increasing / in range
  FLAG_OUT_CAP = 16u,    // a window result set was cut at out_cap
};

constexpr double kTolerance = 1e-3;   // ANN_GATHERED_TOLERANCE
constexpr int kSortCap = 4096;        // survivors sorted in shared memory per query

// Per-query state written by prep_queries and the bound kernels.
struct QueryState {
  float *qn2;      // FP32 squared norm (rounded from FP64)
  float *rnq;      // FP32 1/||q|| (0 for a zero query)
  double *qn2d;    // FP64 squared norm in dimension order (cosine's queryNorm)
  double *err;     // bound on |approximate - exact| in the distance domain
  float *thr;      // v-domain threshold of the filter scan
  int32_t *status; // ANN_OK / ANN_INVALID
  __half *q16;     // [nq_pad][kpad] FP16 queries for the tensor scan (FP8 scan: E4M3 bytes, see qscale)
  float *qscale;   // FP8 scan: per query the power of two s with q ~ s * (hi + lo), hi and lo
                   // E4M3 terms at q16 (bytes [nq_pad][kpad]) and lo_off bytes further
};

// A shard's rows and per-row statistics on the device.
struct ShardView {
  const uint8_t *codes;
  const uint8_t *bscales;   // NVFP4 block scales
  const float *rowscale;    // E4M3 / NVFP4 row scales
  const float *n2;          // decoded squared norm, FP32
  const float *rn;          // 1/sqrt(n2), 0 for a zero row
  const double *n2x;        // FP64 squared norm summed in dimension order (the reference's cosine norm)
  uint64_t row_bytes;
  uint64_t rows;
  uint32_t dims;
  uint32_t dtype;
  uint32_t bblocks;         // NVFP4 blocks a row (ceil(dims/16))
};

// Arguments shared by both scan kernels.
struct ScanArgs {
  ShardView s;
  const uint32_t *ids;      // candidate list, or NULL for rows 0..n-1
  uint64_t count;           // virtual rows to scan
  uint64_t base;            // virtual row i is candidate position base + i*stride
  uint64_t stride;
  const float *queries;     // FP32 [nq][dims] (bits for Hamming, as bytes)
  uint32_t nq;
  uint32_t metric;
  int mode;
  int raw_scale;            // scores are on raw codes: multiply by the row scale
  int f8;                   // E4M3 rows scored by FP8 MMAs against the queries' two E4M3 terms
  const float *qscale;      // f8: [nq] the terms' power-of-two scales
  const float *thr;         // [nq] v-domain thresholds (FILTER)
  float *mat;               // MATRIX: mat[q * mat_ld + i]
  uint64_t mat_ld;
  uint32_t *cnt;            // FILTER: per-query append counters
  uint2 *cand;              // FILTER: [nq][cap] (v bits, candidate position)
  uint32_t cap;
  uint32_t *flags;          // [0] Flag bits, [1] largest count seen (overflow)
};

// IVF list gather (ivf.cu): the shard holds lists l = 0..nlists-1 as row
// runs [offsets[l], offsets[l+1]); probes [nq][nprobe] name each query's
// lists. The plan arrays are device workspace.
constexpr uint32_t kMaxProbes = 4096;
constexpr uint32_t kNoProbe = 0xffffffffu;  // probe table padding
constexpr uint32_t kMaxLists = 1u << 24;
struct ListPlan {
  const uint64_t *offsets;    // [nlists + 1]
  uint32_t nlists;
  uint64_t rows;              // shard rows
  const uint32_t *probes;     // [nq][nprobe]
  uint32_t nprobe, nq;
  unsigned long long *lcount; // [nlists] queries probing each list
  unsigned long long *lfill;  // [nlists] fill cursors
  unsigned long long *qoff;   // [nlists + 1] start of each list's queries in qlist
  uint32_t *qlist;            // [nq * nprobe] query numbers, list-major
  unsigned long long *tiles;  // [nlists] work items of each list
  unsigned long long *toff;   // [nlists + 1] prefix sums of tiles (toff[nlists] = items)
  unsigned long long *bsum;   // [kMaxLists / 4096] prefix-sum block totals
  uint32_t bm, bq;            // rows and queries of a work item (the scan kernel's tile)
  uint32_t *nzl;              // [nlists] the lists with work items, in order (tensor scan; or NULL)
  unsigned long long *nzoff;  // [nlists + 1] their prefix counts (nzoff[nlists] = how many)
};

// Row range [lo, hi) of list l, clamped to the shard; bad offsets (decreasing,
// or past the shard) are flagged by check_offsets and read as empty here.
__device__ __forceinline__ void list_range(const ListPlan &p, uint32_t l, uint64_t &lo, uint64_t &hi) {
  lo = p.offsets[l];
  hi = p.offsets[l + 1];
  if (hi > p.rows) hi = p.rows;
  if (lo > hi) lo = hi;
}

// Rows [lo + rbegin, lo + rend) of list l, clipped to the list.
__device__ __forceinline__ void list_window(const ListPlan &p, uint32_t l, uint64_t rbegin, uint64_t rend,
                                            uint64_t &b, uint64_t &e) {
  uint64_t lo, hi;
  list_range(p, l, lo, hi);
  const uint64_t len = hi - lo;
  b = lo + (rbegin < len ? rbegin : len);
  e = lo + (rend < len ? rend : len);
}

// Largest l with toff[l] <= item (toff non-decreasing, toff[0] = 0).
__device__ __forceinline__ uint32_t find_list(const unsigned long long *toff, uint32_t nlists, uint64_t item) {
  uint32_t lo = 0, hi = nlists;  // toff[lo] <= item < toff[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (toff[mid] <= item) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Row id of candidate position pos: ids[pos], or pos when there is no list.
// A list entry past the shard is clamped to its last row, so a bad list can
// never address memory outside the shard; check_rows flags such a list and
// the search then fails with ANN_INVALID.
__device__ __forceinline__ uint64_t cand_row(const uint32_t *ids, uint64_t pos, uint64_t rows) {
  if (!ids) return pos;
  const uint64_t id = __ldg(ids + pos);
  return id < rows ? id : rows - 1;
}

// Append (v, position) to query q's candidate list; FILTER mode.
__device__ __forceinline__ void append_candidate(const ScanArgs &a, float v, uint64_t pos, uint32_t q) {
  uint32_t idx = atomicAdd(a.cnt + q, 1u);
  if (idx < a.cap) a.cand[(uint64_t)q * a.cap + idx] = make_uint2(__float_as_uint(v), (uint32_t)pos);
  else {
    atomicOr(a.flags, FLAG_OVERFLOW);
    atomicMax(a.flags + 1, idx + 1);
  }
}

// ---------------------------------------------------------------- decoding

// E4M3 magnitude from its 7-bit code: exponent bits 6..3 (bias 7), mantissa
// bits 2..0, subnormal at exponent 0, code 127 NaN. Exact in FP32.
__device__ __forceinline__ float e4m3_value(uint32_t code) {
  uint32_t mag = code & 0x7fu;
  uint32_t e = mag >> 3, m = mag & 7u;
  float v;
  if (mag == 0x7fu) v = __int_as_float(0x7fc00000);
  else if (e == 0) v = (float)m * 0.001953125f;  // m * 2^-9
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return (code & 0x80u) ? -v : v;
}

// E2M1 value of a nibble: magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, bit 3 sign.
__device__ __forceinline__ float e2m1_value(uint32_t nib) {
  const uint32_t m = nib & 7u;
  // 0,0.5,1,1.5 for m < 4; 2,3,4,6 for m >= 4
  float v = (m < 4u) ? 0.5f * (float)m : (m == 7u ? 6.0f : (float)(m - 2u));
  return (nib & 8u) ? -v : v;
}

// Eight decoded values of row `id` at dimensions d0..d0+7 (d0 % 8 == 0),
// zero beyond the row's dimensions.
template <int DT>
__device__ __forceinline__ void decode8(const ShardView &s, uint64_t id, uint32_t d0, float v[8]) {
  const uint8_t *row = s.codes + id * s.row_bytes;
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = 0.0f;
  if (d0 >= s.dims) return;
  const bool full = d0 + 8 <= s.dims;
  if (DT == DT_F32) {
    const float *r = reinterpret_cast<const float *>(row);
    if (full && (s.row_bytes & 15) == 0) {
      float4 a = __ldg(reinterpret_cast<const float4 *>(r + d0));
      float4 b = __ldg(reinterpret_cast<const float4 *>(r + d0 + 4));
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (d0 + j < s.dims) v[j] = __ldg(r + d0 + j);
    }
  } else if (DT == DT_F16) {
    const __half *r = reinterpret_cast<const __half *>(row);
    if (full && (s.row_bytes & 15) == 0) {
      uint4 w = __ldg(reinterpret_cast<const uint4 *>(r + d0));
      const __half2 *h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float2 f = __half22float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (d0 + j < s.dims) v[j] = __half2float(r[d0 + j]);
    }
  } else if (DT == DT_E4M3) {
    // rows are padded to 16 bytes: d0..d0+7 lies inside the row
    uint2 w = __ldg(reinterpret_cast<const uint2 *>(row + d0));
    float rs = __ldg(s.rowscale + id);
    uint32_t lo = w.x, hi = w.y;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint32_t code = ((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xffu;
      if (d0 + j < s.dims) v[j] = __fmul_rn(e4m3_value(code), rs);
    }
  } else if (DT == DT_NVFP4) {
    // 8 dims = 4 bytes of nibble pairs, all in one 16-dim block
    uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(row + d0 / 2));
    float rs = __ldg(s.rowscale + id);
    float bs = __fmul_rn(e4m3_value(__ldg(s.bscales + id * s.bblocks + d0 / 16)), rs);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint32_t nib = (w >> (4 * j)) & 0xfu;
      if (d0 + j < s.dims) v[j] = __fmul_rn(e2m1_value(nib), bs);
    }
  }
}

// ---------------------------------------------------------------- ordering

// Map a float to an unsigned key with the same order; NaN sorts last.
__device__ __forceinline__ uint32_t float_key(float v) {
  uint32_t b = __float_as_uint(v);
  if (v != v) return 0xffffffffu;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}
__device__ __forceinline__ unsigned long long double_key(double v) {
  unsigned long long b = (unsigned long long)__double_as_longlong(v);
  return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}
__device__ __forceinline__ double key_double(unsigned long long k) {
  unsigned long long b = (k & 0x8000000000000000ull) ? (k & 0x7fffffffffffffffull) : ~k;
  return __longlong_as_double((long long)b);
}

// ---------------------------------------------------------------- score domains
//
// The scans compute v = acc * alpha(row) + beta(row) per (row, query), where
// acc is the approximate dot product (or XOR popcount) and v orders rows
// like the distance for a fixed query:
//   L2      v = n2 - 2 acc           distance^2 = v + ||q||^2
//   IP      v = -acc (* row scale)   distance   = v
//   cosine  v = -acc * rn            distance   = 1 + v / ||q||
//   Hamming v = popcount             distance   = v
// Zero-norm rows under cosine get v = NaN, which never passes a threshold.

__device__ __forceinline__ void row_affine(const ShardView &s, uint64_t id, uint32_t metric,
                                           int raw_scale, float &alpha, float &beta) {
  float rs = raw_scale ? s.rowscale[id] : 1.0f;
  switch (metric) {
    case M_L2: alpha = -2.0f * rs; beta = s.n2[id]; break;
    case M_IP: alpha = -rs; beta = 0.0f; break;
    case M_COS: {
      float r = s.rn[id];
      alpha = -r * rs;
      beta = (r == 0.0f) ? __int_as_float(0x7fc00000) : 0.0f;
      break;
    }
    default: alpha = 1.0f; beta = 0.0f; break;
  }
}

// Distance-domain value of a v-domain score, in FP64.
__device__ __forceinline__ double v_to_dist(uint32_t metric, double v, double qn2, double rnq) {
  switch (metric) {
    case M_L2: return v + qn2;            // squared distance
    case M_COS: return 1.0 + v * rnq;
    default: return v;
  }
}

// Inverse of v_to_dist.
__device__ __forceinline__ double dist_to_v(uint32_t metric, double d, double qn2, double rnq) {
  switch (metric) {
    case M_L2: return d - qn2;
    case M_COS: return (d - 1.0) / rnq;
    default: return d;
  }
}

// d + 1e-3*|d| + 1e-6 with the reference's rounding order (cpu.c:267-268).
__device__ __forceinline__ double widen(double d) {
  return __dadd_rn(d, __dadd_rn(__dmul_rn(kTolerance, fabs(d)), 1e-6));
}

// Given an approximate distance-domain value D that at least k rows reach
// (their approximate scores are <= D), an upper bound of the exact k-th
// distance: those k rows' exact distances are each within err of their
// approximate ones, so d_k <= U = D + err.
__device__ __forceinline__ double kth_upper(double D, double err) { return D + err; }

// The v-domain threshold every row of the final answer passes, given an
// upper bound U of the exact k-th distance (from this shard's rows or from
// any rank's of a sharded search): the answer keeps rows with exact distance
// <= C (C = d_k, or its widened window), and their approximate score is
// <= C + err (err: this shard's error bound of the query). For L2 the
// domain is the squared distance and the window applies to the distance
// itself.
__device__ __forceinline__ float threshold_upper(uint32_t metric, double U, double err, int window, double qn2,
                                                 double rnq) {
  if (!(U < __longlong_as_double(0x7ff0000000000000ll))) return __int_as_float(0x7f800000);
  double t;
  if (metric == M_L2) {
    double c = sqrt(U > 0.0 ? U : 0.0);
    if (window) c = widen(c);
    c = c * (1.0 + 1e-12) + 1e-300;
    t = c * c + err;
  } else {
    double c = U;
    if (window) c = widen(c);
    t = c + err + fabs(c) * 1e-12;
  }
  double v = dist_to_v(metric, t, qn2, rnq);
  float f = (float)v;
  if ((double)f < v) f = nextafterf(f, __int_as_float(0x7f800000));
  // one more step up for the FP32 rounding of the scan's own v
  return nextafterf(f, __int_as_float(0x7f800000));
}

// The threshold from this shard's own k-th approximate value D.
__device__ __forceinline__ float threshold_v(uint32_t metric, double D, double err, int window,
                                            double qn2, double rnq) {
  if (!(D < __longlong_as_double(0x7ff0000000000000ll))) return __int_as_float(0x7f800000);
  return threshold_upper(metric, kth_upper(D, err), err, window, qn2, rnq);
}

// Arguments of the per-query selection kernels (tighten, finalize).
struct SelectLaunch {
  ShardView s;
  const uint8_t *staged;    // candidate rows in position order (or NULL: read the shard)
  const int64_t *row_ids;   // global id of each shard row (or NULL: first_id + row)
  const uint32_t *ids;
  const float *queries;
  uint32_t nq, k, metric;
  int window;
  uint32_t qbytes;
  QueryState qs;
  uint32_t *cnt;
  uint2 *cand;
  uint32_t cap;
  uint32_t *flags;
  uint32_t *big;
  double *out_dist;
  int64_t *out_id;
  uint32_t *out_count;
  uint32_t out_cap;
  int64_t first_id;
  int index_form;           // L2 distances in the loaded-index form (FP32 sqrtf)
  double *upper;            // survivors: each query's bound U of its k-th exact distance (NaN: none), or NULL
};

// ---------------------------------------------------------------- launchers
// Record the calling thread's error message (AnnB200LastError) and return status.
int report_error(int status, const char *fmt, ...);
// Count kernels launched by this library (AnnB200LaunchCount).
void count_launches(unsigned long long n);
void launch_simt_scan(const ScanArgs &a, cudaStream_t st);
void launch_list_plan(const ListPlan &p, const QueryState &qs, uint32_t *flags, cudaStream_t st);
void launch_list_items(const ListPlan &p, uint64_t rbegin, uint64_t rend, cudaStream_t st);
void launch_simt_scan_lists(const ListPlan &p, uint64_t rbegin, uint64_t rend, const ScanArgs &a, int sms,
                            cudaStream_t st);
uint32_t list_plan_scan_launches(uint32_t nlists);
// ids/counts of a centroid search (out_cap = nprobe) -> u32 probe table.
void launch_probe_table(const int64_t *ids, const uint32_t *counts, uint32_t nq, uint32_t nprobe, int64_t first,
                        uint32_t *probes, cudaStream_t st);
// FP32 re-score (FP64 sum in dimension order) of gathered candidate rows.
void launch_rescore_rows(const float *queries, uint32_t nq, uint32_t dims, const float *rows, uint32_t stride,
                         const uint32_t *counts, float *out, cudaStream_t st);
// The same, each candidate's row fetched by ordinal (rows: device-readable).
void launch_rescore_gather(const float *queries, uint32_t nq, uint32_t dims, const float *rows,
                           const uint64_t *ords, uint32_t stride, const uint32_t *counts, float *out,
                           cudaStream_t st);
// query_lo_map: the low BF16 halves of the queries (FP32 rows only, else NULL).
cudaError_t launch_tc_scan(const ScanArgs &a, const CUtensorMap &rows_map, int64_t a_row0,
                           const CUtensorMap &query_map, const CUtensorMap *query_lo_map, uint32_t kpad, uint32_t bn,
                           int sms, cudaStream_t st);
void launch_gather_rows(const uint8_t *codes, uint64_t row_bytes, uint64_t rows, const uint32_t *ids, uint64_t base,
                        uint64_t stride, uint64_t count, uint8_t *out, cudaStream_t st);
uint32_t tc_scan_max_queries();
cudaError_t launch_tc_scan_lists(const ScanArgs &a, const ListPlan &p, uint64_t rbegin, uint64_t rend,
                                 const CUtensorMap &rows_map, const CUtensorMap &scales_map, const __half *q16,
                                 uint32_t kpad, int sms, cudaStream_t st);
void launch_shard_stats(const ShardView &s, float *n2, float *rn, double *n2x, uint32_t *maxn2, cudaStream_t st);
// lo_off: FP32 rows on tensor cores -- q16 receives the queries' BF16 high
// halves and, lo_off elements further, their low halves (0: an FP16 copy).
// f8: the queries as two E4M3 terms with a power-of-two scale each (the FP8
// tensor scan): hi bytes at q16, lo bytes lo_off bytes further.
void launch_prep_queries(const float *queries, uint32_t nq, uint32_t dims, uint32_t metric, uint32_t kpad,
                         int use_q16, double gamma, const uint32_t *maxn2, const QueryState &qs, int bits,
                         uint32_t *flags, cudaStream_t st, uint64_t lo_off = 0, int f8 = 0);
void launch_fill_thresholds(uint32_t nq, const QueryState &qs, cudaStream_t st);
void launch_check_rows(const uint32_t *ids, uint64_t n, uint64_t rows, uint32_t *flags, cudaStream_t st);
void launch_kth_bound(const float *mat, uint64_t ld, uint64_t n, uint32_t nq, uint32_t k, uint32_t metric,
                      int window, const QueryState &qs, cudaStream_t st);
void launch_tighten(const SelectLaunch &l, cudaStream_t st);
void launch_survivors(const SelectLaunch &l, cudaStream_t st);
// Second cut of a sharded search's survivors: every rank's bounds U
// ([nranks][ld] doubles, NaN where a rank has none) -> the smallest, and each
// query keeps only the survivors that can beat it.
void launch_survivors_global(const SelectLaunch &l, const double *upper_all, uint32_t nranks, uint32_t ld,
                             cudaStream_t st);
cudaError_t launch_finalize(const SelectLaunch &l, double *exact, cudaStream_t st);
void launch_finalize_big(const SelectLaunch &l, uint32_t q, unsigned long long *key, unsigned long long *pos,
                         uint32_t p2, cudaStream_t st);
cudaError_t launch_merge(const double *dist, const int64_t *ids, const uint32_t *counts, uint32_t nlists,
                         uint32_t nq, uint32_t list_cap, uint32_t k, int window, uint32_t out_cap,
                         double *out_dist, int64_t *out_id, uint32_t *out_count, uint32_t *flags,
                         cudaStream_t st);
// The non-window merge of sorted per-shard lists by rank (no sort), each
// array's lists `*_stride` bytes apart; nlists * list_cap <= kSortCap.
cudaError_t launch_merge_ranked(const void *dist, uint64_t dist_stride, const void *ids, uint64_t id_stride,
                                const void *counts, uint64_t count_stride, uint32_t nlists, uint32_t nq,
                                uint32_t list_cap, uint32_t k, uint32_t out_cap, double *out_dist, int64_t *out_id,
                                uint32_t *out_count, cudaStream_t st);
uint32_t bitmap_blocks(uint64_t nbits);
void launch_f32_to_f16(const float *in, __half *out, uint64_t n, cudaStream_t st);
void launch_v_to_distance(float *m, uint64_t n, uint32_t nq, uint32_t metric, const QueryState &qs, cudaStream_t st);
void launch_bitmap_rows(const uint32_t *words, uint64_t nbits, uint32_t *rows, uint32_t *blockcnt,
                        unsigned long long *total, cudaStream_t st,
                        uint32_t base = 0);

}  // namespace annb200
