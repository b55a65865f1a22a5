// select.cu - bounds, candidate pruning, exact rescoring and merging.
//
// Reference counterparts: the sampled-bound candidate lists of
// AnnBlackwellCandidates (stride_rows / select32 / merge32 / fuse_mma,
// ann/server/blackwell.c:1452-1548), the radix prune-select and final
// rank/bucket kernels (prune_select_s, final_rank, final_bucket,
// ann/server/cuvs.c:3882-4248), the FP64 rerank kernels (rerank8_*,
// rerank_final_*, ann/server/cuvs.c:3912-3990,4149-4248), the host merge of
// per-shard top-k lists (AnnIndexTreeMerge, ann/server/indexfile.c:3235-3258)
// and bitmap expansion (expand_*, ann/server/cuvs.c:1910-1968).
//
// Exactness: candidates are rescored with the reference CPU worker's own
// arithmetic on the rows decoded to FP32 (ann/server/cpu.c:82-175): L2 as
// eight FP32 partial sums combined ((sum + (s0+s1)+(s2+s3)) + ((s4+s5)+(s6+s7)))
// then a double square root; inner product and cosine as FP64 sums in
// dimension order. Every operation is an explicit round-to-nearest intrinsic
// so no multiply-add is fused, which makes each distance identical to the
// CPU's bit for bit.
#include <algorithm>

#include <cuda_bf16.h>

#include <cuda_fp8.h>

#include "internal.cuh"

namespace annb200 {

namespace {

constexpr int NT = 512;  // threads of the per-query bound / tighten / merge kernels
constexpr int NTF = 256; // threads of finalize (two blocks an SM at its register use)

// ---------------------------------------------------------------- block helpers

// Exclusive prefix sum of one value a thread over the block; *total gets the sum.
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *scratch, uint32_t *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nw ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) scratch[lane] = w;
  }
  __syncthreads();
  uint32_t before = (warp ? scratch[warp - 1] : 0) + x - v;
  *total = scratch[nw - 1];
  __syncthreads();
  return before;
}

// k-th smallest (1-based) 32-bit key among n, keys from key_at(i): three
// radix passes of 11, 11 and 10 bits with a shared histogram.
template <typename KeyAt>
__device__ uint32_t block_radix_select(KeyAt key_at, uint32_t n, uint32_t k, uint32_t *hist,
                                       uint32_t *scratch) {
  __shared__ uint32_t s_prefix, s_k;
  uint32_t prefix = 0, mask = 0;
  if (threadIdx.x == 0) s_k = k;
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
  __syncthreads();
  for (int p = 0; p < 3; p++) {
    const int shift = shifts[p], nb = 1 << widths[p];
    const uint32_t want = s_k;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    if (threadIdx.x == 0) s_prefix = prefix;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
      uint32_t key = key_at(i);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    // each thread owns a contiguous run of bins
    const int per = (nb + blockDim.x - 1) / blockDim.x;
    const int b0 = threadIdx.x * per;
    uint32_t local = 0;
    for (int b = b0; b < b0 + per && b < nb; b++) local += hist[b];
    uint32_t total;
    uint32_t before = block_exclusive_scan(local, scratch, &total);
    if (before < want && want <= before + local) {
      uint32_t c = before;
      for (int b = b0; b < b0 + per && b < nb; b++) {
        if (c + hist[b] >= want) {
          s_prefix = prefix | ((uint32_t)b << shift);
          s_k = want - c;
          break;
        }
        c += hist[b];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    mask |= (uint32_t)(nb - 1) << shift;
    __syncthreads();
  }
  return prefix;
}

// block_radix_select over keys held in registers: thread t holds elements
// t, t + blockDim.x, ... in kr[0..R); slots past n are not counted. Same
// passes, same result.
template <int R>
__device__ uint32_t block_radix_select_regs(const uint32_t (&kr)[R], uint32_t n, uint32_t k, uint32_t *hist,
                                            uint32_t *scratch) {
  __shared__ uint32_t s_prefix, s_k;
  uint32_t prefix = 0, mask = 0;
  if (threadIdx.x == 0) s_k = k;
  const int shifts[3] = {21, 10, 0};
  const int widths[3] = {11, 11, 10};
  __syncthreads();
  for (int p = 0; p < 3; p++) {
    const int shift = shifts[p], nb = 1 << widths[p];
    const uint32_t want = s_k;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    if (threadIdx.x == 0) s_prefix = prefix;
#pragma unroll
    for (int j = 0; j < R; j++) {
      const uint32_t i = threadIdx.x + j * blockDim.x;
      if (i < n && (kr[j] & mask) == prefix) atomicAdd(&hist[(kr[j] >> shift) & (nb - 1)], 1u);
    }
    __syncthreads();
    const int per = (nb + blockDim.x - 1) / blockDim.x;
    const int b0 = threadIdx.x * per;
    uint32_t local = 0;
    for (int b = b0; b < b0 + per && b < nb; b++) local += hist[b];
    uint32_t total;
    uint32_t before = block_exclusive_scan(local, scratch, &total);
    if (before < want && want <= before + local) {
      uint32_t c = before;
      for (int b = b0; b < b0 + per && b < nb; b++) {
        if (c + hist[b] >= want) {
          s_prefix = prefix | ((uint32_t)b << shift);
          s_k = want - c;
          break;
        }
        c += hist[b];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    mask |= (uint32_t)(nb - 1) << shift;
    __syncthreads();
  }
  return prefix;
}

// ---------------------------------------------------------------- exact distances

// Raw storage of 8 consecutive dimensions of a row, per format: loaded first,
// decoded later, so a thread keeps many loads in flight.
template <int DT> struct Raw8 { uint4 w; };
template <> struct Raw8<DT_F32> { float4 a, b; };
template <> struct Raw8<DT_E4M3> { uint2 w; };
template <> struct Raw8<DT_NVFP4> { uint32_t w; uint32_t sc; };

template <int DT>
__device__ __forceinline__ void load_raw8(const ShardView &s, const uint8_t *row, uint64_t id, uint32_t d0,
                                          Raw8<DT> &r) {
  if (DT == DT_F32) {
    Raw8<DT_F32> &x = reinterpret_cast<Raw8<DT_F32> &>(r);
    const float *f = reinterpret_cast<const float *>(row) + d0;
    if ((s.row_bytes & 15) == 0 && d0 + 8 <= s.dims) {
      x.a = __ldg(reinterpret_cast<const float4 *>(f));
      x.b = __ldg(reinterpret_cast<const float4 *>(f + 4));
    } else {
      float t[8];
#pragma unroll
      for (int j = 0; j < 8; j++) t[j] = d0 + j < s.dims ? __ldg(f + j) : 0.0f;
      x.a = make_float4(t[0], t[1], t[2], t[3]);
      x.b = make_float4(t[4], t[5], t[6], t[7]);
    }
  } else if (DT == DT_F16) {
    Raw8<DT_F16> &x = reinterpret_cast<Raw8<DT_F16> &>(r);
    const uint16_t *h = reinterpret_cast<const uint16_t *>(row) + d0;
    if ((s.row_bytes & 15) == 0 && d0 + 8 <= s.dims) x.w = __ldg(reinterpret_cast<const uint4 *>(h));
    else {
      uint32_t t[4] = {0, 0, 0, 0};
      for (int j = 0; j < 8; j++)
        if (d0 + j < s.dims) t[j / 2] |= (uint32_t)__ldg(h + j) << (16 * (j & 1));
      x.w = make_uint4(t[0], t[1], t[2], t[3]);
    }
  } else if (DT == DT_E4M3) {
    reinterpret_cast<Raw8<DT_E4M3> &>(r).w = __ldg(reinterpret_cast<const uint2 *>(row + d0));
  } else {
    Raw8<DT_NVFP4> &x = reinterpret_cast<Raw8<DT_NVFP4> &>(r);
    x.w = __ldg(reinterpret_cast<const uint32_t *>(row + d0 / 2));
    x.sc = __ldg(s.bscales + id * s.bblocks + d0 / 16);
  }
}

// Decode like decode8 (the FP32 values the reference would score).
template <int DT>
__device__ __forceinline__ void decode_raw8(const Raw8<DT> &r, float rs, float v[8]) {
  if (DT == DT_F32) {
    const Raw8<DT_F32> &x = reinterpret_cast<const Raw8<DT_F32> &>(r);
    v[0] = x.a.x; v[1] = x.a.y; v[2] = x.a.z; v[3] = x.a.w;
    v[4] = x.b.x; v[5] = x.b.y; v[6] = x.b.z; v[7] = x.b.w;
  } else if (DT == DT_F16) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&reinterpret_cast<const Raw8<DT_F16> &>(r).w);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float2 f = __half22float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else if (DT == DT_E4M3) {
    const uint2 w = reinterpret_cast<const Raw8<DT_E4M3> &>(r).w;
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fmul_rn(e4m3_value(((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xffu), rs);
  } else {
    const Raw8<DT_NVFP4> &x = reinterpret_cast<const Raw8<DT_NVFP4> &>(r);
    const float bs = __fmul_rn(e4m3_value(x.sc), rs);
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fmul_rn(e2m1_value((x.w >> (4 * j)) & 0xfu), bs);
  }
}

// Final L2 of the eight lane sums and the tail. Gathered jobs
// (ann/server/cpu.c L2Squared): sqrt in FP64 of (tail + left) + right.
// Loaded indexes (ann/server/indexfile.c Distance): sqrtf of
// tail + (left + right), an FP32 distance.
__device__ __forceinline__ double l2_finish(const float (&sums)[8], float tail, int index_form) {
  const float left = __fadd_rn(__fadd_rn(sums[0], sums[1]), __fadd_rn(sums[2], sums[3]));
  const float right = __fadd_rn(__fadd_rn(sums[4], sums[5]), __fadd_rn(sums[6], sums[7]));
  if (index_form) return (double)__fsqrt_rn(__fadd_rn(tail, __fadd_rn(left, right)));
  return __dsqrt_rn((double)__fadd_rn(__fadd_rn(tail, left), right));
}

// The reference CPU worker's distance of one decoded row (see file header),
// with the row streamed in batches of 64 dimensions: the next batch's loads
// are issued before the current batch is summed, and the sums keep the
// reference's exact operation order.
template <int DT>
__device__ double exact_distance(const ShardView &s, uint64_t id, const float *q, uint32_t metric,
                                 double qn2d, const uint8_t *row, int index_form) {
  const uint32_t dims = s.dims;
  if (DT == DT_BIT) {
    const uint8_t *qb = reinterpret_cast<const uint8_t *>(q);
    uint32_t d = 0;
    uint64_t b = 0;
    if ((s.row_bytes & 15) == 0)
      for (; b < s.row_bytes; b += 16) {
        const uint4 x = __ldg(reinterpret_cast<const uint4 *>(row + b));
        const uint4 y = *reinterpret_cast<const uint4 *>(qb + b);
        d += __popc(x.x ^ y.x) + __popc(x.y ^ y.y) + __popc(x.z ^ y.z) + __popc(x.w ^ y.w);
      }
    else if ((s.row_bytes & 3) == 0)
      for (; b < s.row_bytes; b += 4)
        d += __popc(__ldg(reinterpret_cast<const uint32_t *>(row + b)) ^ *reinterpret_cast<const uint32_t *>(qb + b));
    for (; b < s.row_bytes; b++) d += __popc((uint32_t)(__ldg(row + b) ^ qb[b]));
    return (double)d;
  } else {
    // 8-dimension groups a batch: 128 bytes of row per buffer
    constexpr int G = DT == DT_F32 ? 4 : (DT == DT_F16 ? 8 : 16);
    const float rs = (DT == DT_E4M3 || DT == DT_NVFP4) ? __ldg(s.rowscale + id) : 1.0f;
    const uint32_t groups = (dims + 7) / 8;
    // the whole row toward L2 first: every batch load below then hits L2
    for (uint64_t b = 0; b < s.row_bytes; b += 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(row + b));
    Raw8<DT> buf[G];
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float tail = 0.0f;
    double dot = 0.0;
    for (uint32_t g0 = 0; g0 < groups; g0 += G) {
#pragma unroll
      for (int g = 0; g < G; g++)
        if (g0 + g < groups) load_raw8<DT>(s, row, id, (g0 + g) * 8, buf[g]);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const uint32_t d0 = (g0 + g) * 8;
        if (d0 >= dims) break;
        float v[8];
        decode_raw8<DT>(buf[g], rs, v);
        if (metric == M_L2) {
          if (d0 + 8 <= dims) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
              float diff = __fsub_rn(v[j], q[d0 + j]);
              sums[j] = __fadd_rn(sums[j], __fmul_rn(diff, diff));
            }
          } else {
            for (int j = 0; d0 + j < dims; j++) {
              float diff = __fsub_rn(v[j], q[d0 + j]);
              tail = __fadd_rn(tail, __fmul_rn(diff, diff));
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++)
            if (d0 + j < dims) dot = __dadd_rn(dot, __dmul_rn((double)v[j], (double)q[d0 + j]));
        }
      }
    }
    if (metric == M_L2) return l2_finish(sums, tail, index_form);
    if (metric == M_IP) return -dot;
    const double nrm = s.n2x[id];
    double r = __ddiv_rn(dot, __dsqrt_rn(__dmul_rn(nrm, qn2d)));
    return __dsub_rn(1.0, fmax(-1.0, fmin(1.0, r)));
  }
}

// FP32 re-score of a quantized scan's candidates, as the reference's
// loaded-index scan route does it on the host (ExactDistance,
// ann/server/cuvs.c:2930-2942): each difference and square in FP64, summed
// in dimension order, the FP64 square root rounded to FP32. One thread a
// candidate row; rows [nq][stride][dims], only the first counts[q] of a
// query's stride are read and written.
__global__ void __launch_bounds__(256) rescore_rows(const float *__restrict__ queries, uint32_t nq, uint32_t dims,
                                                    const float *__restrict__ rows, uint32_t stride,
                                                    const uint32_t *__restrict__ counts, float *__restrict__ out,
                                                    int vec4) {
  const uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (t >= (uint64_t)nq * stride) return;
  const uint32_t q = (uint32_t)(t / stride), j = (uint32_t)(t % stride);
  if (counts && j >= counts[q]) return;
  const float *x = rows + t * dims;
  const float *v = queries + (uint64_t)q * dims;
  double sum = 0.0;
  uint32_t d = 0;
  if (vec4)
    for (; d < dims; d += 4) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(x + d));
      const float4 b = __ldg(reinterpret_cast<const float4 *>(v + d));
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const double delta = __dsub_rn((double)av[i], (double)bv[i]);
        sum = __dadd_rn(sum, __dmul_rn(delta, delta));
      }
    }
  for (; d < dims; d++) {
    const double delta = __dsub_rn((double)__ldg(x + d), (double)__ldg(v + d));
    sum = __dadd_rn(sum, __dmul_rn(delta, delta));
  }
  out[t] = __double2float_rn(__dsqrt_rn(sum));
}


// ---------------------------------------------------------------- shard stats

// Per row: FP64 squared norm of the decoded values -> n2 (FP32) and
// rn = 1/sqrt(n2) (0 for a zero row); the largest n2 goes to *maxn2 (as
// float bits, which order like integers for non-negative values).
template <int DT>
__global__ void shard_stats(ShardView s, float *n2, float *rn, uint32_t *maxn2) {
  const uint64_t row = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= s.rows) return;
  double acc = 0.0;
  float v[8];
  for (uint32_t d = lane * 8; d < s.dims; d += 256) {
    decode8<DT>(s, row, d, v);
#pragma unroll
    for (int j = 0; j < 8; j++) acc += (double)v[j] * (double)v[j];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    float f = (float)acc;
    n2[row] = f;
    rn[row] = acc > 0.0 ? (float)(1.0 / sqrt(acc)) : 0.0f;
    atomicMax(maxn2, __float_as_uint(f));
  }
}

// Per row, one thread: the FP64 squared norm of the decoded values summed in
// dimension order -- exactly the norm the reference's cosine accumulates
// (ann/server/cpu.c:118-126) -- so rescoring needs only the dot product.
template <int DT>
__global__ void exact_norms(ShardView s, double *n2x) {
  const uint64_t row = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= s.rows) return;
  double acc = 0.0;
  float v[8];
  for (uint32_t d = 0; d < s.dims; d += 8) {
    decode8<DT>(s, row, d, v);
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (d + j < s.dims) acc = __dadd_rn(acc, __dmul_rn((double)v[j], (double)v[j]));
  }
  n2x[row] = acc;
}

// ---------------------------------------------------------------- queries

struct PrepArgs {
  const float *queries;
  uint32_t nq, dims, metric, kpad;
  int use_q16;
  uint64_t lo_off;         // FP32 rows: the queries' low BF16 halves start lo_off elements after q16 (0: FP16 copy)
  double gamma;            // relative accumulation error of the approximate scan
  const uint32_t *maxn2;   // shard's largest squared row norm (float bits)
  QueryState qs;
  uint32_t *flags;         // [5] counts invalid queries
  int f8;                  // two E4M3 terms (bytes) instead of the FP16 copy; lo_off in bytes
};

// One block a query: validity, norms, the FP16 copy and the error bound
// (distance domain; squared distance for L2) of the approximate score:
//   |acc - dot| <= gamma*||x||*||q16|| + ||x||*||q - q16|| + FP32 epilogue
// rounding, with ||x|| <= sqrt(maxn2); the L2 bound also covers the rounding
// of the reference's own FP32 eight-lane sum.
constexpr uint32_t kPrepSqMax = 6144;   // dims whose squares fit the kernel's shared memory (48 KB)

__global__ void prep_queries(PrepArgs p) {
  const uint32_t q = blockIdx.x;
  const float *qv = p.queries + (uint64_t)q * p.dims;
  extern __shared__ double sq[];   // x[d]^2 (exact in FP64) when dims <= kPrepSqMax
  __shared__ double red[4][32];
  __shared__ int bad;
  __shared__ float s_scale;
  if (threadIdx.x == 0) bad = 0;
  if (p.f8) {
    // the FP8 scan's query terms share one power-of-two scale s with
    // max |q| / s <= 448 (E4M3's largest value): s * (hi + lo) holds q to
    // about 2^-8 of each element, and multiplying by s is exact
    float mx = 0.0f;
    for (uint32_t d = threadIdx.x; d < p.dims; d += blockDim.x) mx = fmaxf(mx, fabsf(qv[d]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[0][threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
      double m = 0.0;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmax(m, red[0][w]);
      double sc = 1.0;
      if (m > 0.0 && isfinite(m)) {
        const double v = m / 448.0;
        sc = ldexp(1.0, ilogb(v));
        if (sc < v) sc *= 2.0;
      }
      s_scale = (float)sc;
      p.qs.qscale[q] = (float)sc;
    }
  }
  __syncthreads();
  double r2 = 0.0, t2 = 0.0, n2 = 0.0, l2 = 0.0;
  for (uint32_t d = threadIdx.x; d < p.kpad || d < p.dims; d += blockDim.x) {
    float x = d < p.dims ? qv[d] : 0.0f;
    if (d < p.dims && !isfinite(x)) bad = 1;
    if (p.f8 && d < p.kpad) {
      // hi = RN_e4m3(x / s), lo = RN_e4m3(x / s - hi) (the difference is
      // exact: it is at most 2^-4 of x / s); the scan sees s * (hi + lo)
      const float sc = s_scale;
      const float y = isfinite(x) ? x / sc : 0.0f;
      const __nv_fp8_storage_t h = __nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
      const float hv = __half2float(__half(__nv_cvt_fp8_to_halfraw(h, __NV_E4M3)));
      const __nv_fp8_storage_t l = __nv_cvt_float_to_fp8(y - hv, __NV_SATFINITE, __NV_E4M3);
      const float lv = __half2float(__half(__nv_cvt_fp8_to_halfraw(l, __NV_E4M3)));
      uint8_t *q8 = reinterpret_cast<uint8_t *>(p.qs.q16);
      q8[(uint64_t)q * p.kpad + d] = h;
      q8[p.lo_off + (uint64_t)q * p.kpad + d] = l;
      const double t = (double)sc * ((double)hv + (double)lv);
      t2 += t * t;
      r2 += ((double)x - t) * ((double)x - t);
    } else if (p.use_q16 && d < p.kpad && p.lo_off) {
      // two BF16 halves: hi = RN(x), lo = RN(x - hi); the scan sees hi + lo
      const __nv_bfloat16 h = __float2bfloat16_rn(x);
      const float hf = __bfloat162float(h);
      const __nv_bfloat16 l = __float2bfloat16_rn(x - hf);
      const float lf = __bfloat162float(l);
      uint16_t *q16 = reinterpret_cast<uint16_t *>(p.qs.q16);
      q16[(uint64_t)q * p.kpad + d] = __bfloat16_as_ushort(h);
      q16[p.lo_off + (uint64_t)q * p.kpad + d] = __bfloat16_as_ushort(l);
      const double s = (double)hf + (double)lf;
      t2 += s * s;
      r2 += ((double)x - s) * ((double)x - s);
      l2 += (double)lf * (double)lf;
    } else if (p.use_q16 && d < p.kpad) {
      __half h = __float2half_rn(x);
      p.qs.q16[(uint64_t)q * p.kpad + d] = h;
      double hx = (double)__half2float(h);
      t2 += hx * hx;
      r2 += ((double)x - hx) * ((double)x - hx);
    }
    n2 += (double)x * (double)x;
    if (d < p.dims && p.dims <= kPrepSqMax) sq[d] = __dmul_rn((double)x, (double)x);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    r2 += __shfl_xor_sync(0xffffffffu, r2, o);
    t2 += __shfl_xor_sync(0xffffffffu, t2, o);
    n2 += __shfl_xor_sync(0xffffffffu, n2, o);
    l2 += __shfl_xor_sync(0xffffffffu, l2, o);
  }
  if (lane == 0) {
    red[0][warp] = r2;
    red[1][warp] = t2;
    red[2][warp] = n2;
    red[3][warp] = l2;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  r2 = t2 = n2 = l2 = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
    r2 += red[0][w];
    t2 += red[1][w];
    n2 += red[2][w];
    l2 += red[3][w];
  }
  // the reference's query norm: FP64, dimension order (cpu.c:96-101); the
  // squares (exact: FP32 x FP32 fits FP64) were formed in parallel above,
  // only the ordered sum is serial
  double qn = 0.0;
  if (p.dims <= kPrepSqMax)
    for (uint32_t d = 0; d < p.dims; d++) qn = __dadd_rn(qn, sq[d]);
  else
    for (uint32_t d = 0; d < p.dims; d++) qn = __dadd_rn(qn, __dmul_rn((double)qv[d], (double)qv[d]));
  if (!p.use_q16 && !p.f8) {
    t2 = n2;
    r2 = 0.0;
  }
  const double mx2 = (double)__uint_as_float(*p.maxn2);
  const double mx = sqrt(mx2), qnorm = sqrt(n2), tnorm = sqrt(t2), rnorm = sqrt(r2), lnorm = sqrt(l2);
  const double eps = 1.0 / 1048576.0;  // 2^-20
  // FP32 rows split into BF16 halves X' = hi + lo, |x - X'| <= 2^-16 |x| +
  // 2^-134 and |lo| <= 2^-8 |x| + 2^-134 an element; the scan computes
  // X'.Q' - lo_x.lo_q: |x.q - that| <= ||x|| ||r_q|| (in rnorm) + (2^-16 ||x||
  // + 2^-134 sqrt(d)) ||Q'|| + (2^-8 ||x|| + 2^-134 sqrt(d)) ||lo_q||, plus
  // 2^-126 for each of the 3 kpad products in case the tensor core flushes a
  // subnormal product. Zero for the FP16 copy. (Cosine over FP32 rows is
  // scored on CUDA cores: these absolute terms would scale with 1/||x||.)
  const double sd = sqrt((double)p.kpad);
  const bool split = p.lo_off && !p.f8;
  const double esplit =
      split ? ldexp(1.0, -16) * tnorm + ldexp(1.0, -8) * lnorm + ldexp(1.0, -134) * sd * (tnorm + lnorm) : 0.0;
  const double etiny = split ? 3.0 * p.kpad * ldexp(1.0, -126) : 0.0;
  double err;
  switch (p.metric) {
    case M_L2: {
      double edot = p.gamma * mx * tnorm + mx * rnorm + eps * mx * qnorm + mx * esplit + etiny;
      double span = (mx + qnorm) * (mx + qnorm);
      err = 2.0 * edot + eps * (mx2 + n2 + mx * qnorm) + ((double)p.dims / 8.0 + 8.0) * 1.2e-7 * span;
      break;
    }
    case M_IP: err = p.gamma * mx * tnorm + mx * rnorm + eps * mx * qnorm + mx * esplit + etiny; break;
    case M_COS: err = qnorm > 0.0 ? p.gamma * tnorm / qnorm + rnorm / qnorm + 2.0 * eps : 0.0; break;
    default: err = 0.0; break;
  }
  p.qs.err[q] = err * 1.0001 + 1e-30;
  p.qs.qn2d[q] = qn;
  p.qs.qn2[q] = (float)qn;
  p.qs.rnq[q] = qn > 0.0 ? (float)(1.0 / sqrt(qn)) : 0.0f;
  const int invalid = bad || (p.metric == M_COS && qn == 0.0);
  p.qs.status[q] = invalid;
  if (invalid) atomicAdd(p.flags + 5, 1u);
}

__global__ void prep_queries_bits(uint32_t nq, QueryState qs) {
  uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  qs.err[q] = 0.0;
  qs.qn2d[q] = 0.0;
  qs.qn2[q] = 0.0f;
  qs.rnq[q] = 0.0f;
  qs.status[q] = 0;
}

// Bit-vector queries -> the tensor scan's int8 block [q][kpad]: element b
// (byte b/8 of the row, bit b%8 from the least significant) is -1 if the bit
// is set, +1 if clear, 0 past the row's bytes -- the expansion the scan
// applies to the rows, so the S32 dot product is nbits - 2 x Hamming.
__global__ void expand_query_bits(const uint8_t *q, uint32_t row_bytes, uint32_t kpad, int8_t *out) {
  const uint64_t qi = blockIdx.x;
  for (uint32_t b = threadIdx.x; b < kpad; b += blockDim.x) {
    const uint32_t byte = b >> 3;
    int8_t v = 0;
    if (byte < row_bytes) v = ((q[qi * row_bytes + byte] >> (b & 7)) & 1u) ? (int8_t)-1 : (int8_t)1;
    out[qi * kpad + b] = v;
  }
}

// Threshold for queries without a sample bound: +inf (everything eligible).
__global__ void fill_thresholds(uint32_t nq, QueryState qs) {
  uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  qs.thr[q] = qs.status[q] ? __int_as_float(0x7fc00000) : __int_as_float(0x7f800000);
}

// ---------------------------------------------------------------- candidate rows

__global__ void check_rows(const uint32_t *ids, uint64_t n, uint64_t rows, uint32_t *flags) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t v = ids[i];
  if (v >= rows || (i && v <= ids[i - 1])) atomicOr(flags, FLAG_BAD_ROWS);
}

// ---------------------------------------------------------------- sample bound

struct BoundArgs {
  const float *mat;
  uint64_t ld, n;
  uint32_t k, metric;
  int window;
  QueryState qs;
};

// Per query: the k-th smallest sampled v bounds the k-th exact distance;
// thr = threshold_v of it (or +inf when the sample holds fewer than k rows).
// The query's sampled scores are read once, all loads in flight at once, into
// registers (KB_REG a thread: the whole sample up to NT * KB_REG scores); the
// three radix passes then read registers instead of re-reading the row.
constexpr int KB_REG = 32;

// BT threads a block: 256 when the sample fits 256 x KB_REG registers (a
// row-sharded rank's smaller sample), so four blocks share an SM instead of
// two (the registers hold the scores).
template <int BT>
__global__ void __launch_bounds__(BT, 1024 / BT) kth_bound(BoundArgs b) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t scratch[32];
  const uint32_t q = blockIdx.x;
  if (b.qs.status[q]) {
    if (threadIdx.x == 0) b.qs.thr[q] = __int_as_float(0x7fc00000);
    return;
  }
  const float *m = b.mat + (uint64_t)q * b.ld;
  uint32_t key = 0xffffffffu;
  if (b.n >= b.k && b.n <= (uint64_t)BT * KB_REG) {
    uint32_t kr[KB_REG];
#pragma unroll
    for (int j = 0; j < KB_REG; j++) {
      const uint32_t i = threadIdx.x + j * BT;
      kr[j] = i < b.n ? float_key(__ldg(m + i)) : 0xffffffffu;
    }
    // element i lives in thread i % BT, slot i / BT: the select visits a
    // thread's own elements only (i = threadIdx.x + j * BT), so it indexes
    // its registers with the unrolled j
    key = block_radix_select_regs<KB_REG>(kr, (uint32_t)b.n, b.k, hist, scratch);
  } else if (b.n >= b.k) {
    key = block_radix_select([&](uint32_t i) { return float_key(m[i]); }, (uint32_t)b.n, b.k, hist, scratch);
  }
  if (threadIdx.x == 0) {
    float v = key == 0xffffffffu ? __int_as_float(0x7f800000) : key_float(key);
    double rnq = (double)b.qs.rnq[q], qn2 = b.qs.qn2d[q];
    double D = v_to_dist(b.metric, (double)v, qn2, rnq);
    if (v != v || isinf(v)) b.qs.thr[q] = __int_as_float(0x7f800000);
    else b.qs.thr[q] = threshold_v(b.metric, D, b.qs.err[q], b.window, qn2, rnq);
  }
}

// ---------------------------------------------------------------- tighten / finalize

struct SelectArgs {
  ShardView s;
  const uint8_t *staged;  // candidate rows in position order (or NULL: read the shard)
  const int64_t *row_ids; // global id of each shard row (or NULL: first_id + row)
  const uint32_t *ids;
  const float *queries;
  uint32_t nq, k, metric;
  int window;
  uint32_t qbytes;        // bytes a query (Hamming) or 4*dims
  QueryState qs;
  uint32_t *cnt;
  uint2 *cand;
  uint32_t cap;
  uint32_t *flags;        // [0] flags, [1] largest count, [2] largest survivor set
  uint32_t *big;          // [nq] survivor count of queries left to the big sort
  double *out_dist;
  int64_t *out_id;
  uint32_t *out_count;
  uint32_t out_cap;
  int64_t first_id;
  int index_form;         // L2 distances in the loaded-index form (FP32 sqrtf)
  double *upper;          // survivors: the bound U of each query's k-th exact distance (NaN: none), or NULL
};

// Keep the entries of a candidate list (c entries at e) whose score is <= t,
// in place. Returns the kept count (all threads).
__device__ uint32_t compact_le(uint2 *e, uint32_t c, float t, uint32_t *scratch) {
  __shared__ uint32_t s_m;
  if (threadIdx.x == 0) s_m = 0;
  __syncthreads();
  for (uint32_t base = 0; base < c; base += blockDim.x) {
    uint32_t i = base + threadIdx.x;
    uint2 val = make_uint2(0, 0);
    uint32_t keep = 0;
    if (i < c) {
      val = e[i];
      keep = __uint_as_float(val.x) <= t;
    }
    uint32_t total;
    uint32_t off = block_exclusive_scan(keep, scratch, &total);
    const uint32_t m0 = s_m;
    if (keep) e[m0 + off] = val;
    __syncthreads();
    if (threadIdx.x == 0) s_m = m0 + total;
    __syncthreads();
  }
  return s_m;
}

// Lower a query's threshold with the k-th smallest v among its candidates and
// drop the entries above it. Returns the survivor count (all threads);
// *upper_out (thread 0, when given) gets the bound U of the k-th exact
// distance those candidates give (NaN when there are not more than k).
__device__ uint32_t tighten_one(const SelectArgs &a, uint32_t q, uint32_t c, uint32_t *hist, uint32_t *scratch,
                                float *thr_out, double *upper_out = nullptr) {
  __shared__ float s_thr;
  uint2 *e = a.cand + (uint64_t)q * a.cap;
  float t = a.qs.thr[q];
  if (upper_out && threadIdx.x == 0) *upper_out = __longlong_as_double(0x7ff8000000000000ll);
  if (c > a.k) {
    uint32_t key = block_radix_select([&](uint32_t i) { return float_key(__uint_as_float(e[i].x)); }, c, a.k, hist,
                                      scratch);
    if (threadIdx.x == 0) {
      double rnq = (double)a.qs.rnq[q], qn2 = a.qs.qn2d[q];
      float v = key_float(key);
      const double D = v_to_dist(a.metric, (double)v, qn2, rnq);
      float t2 = threshold_v(a.metric, D, a.qs.err[q], a.window, qn2, rnq);
      s_thr = t2 < t ? t2 : t;
      if (upper_out && D < __longlong_as_double(0x7ff0000000000000ll)) *upper_out = kth_upper(D, a.qs.err[q]);
    }
    __syncthreads();
    t = s_thr;
  }
  *thr_out = t;
  return compact_le(e, c, t, scratch);
}

__global__ void __launch_bounds__(NT) tighten(SelectArgs a) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t scratch[32];
  const uint32_t q = blockIdx.x;
  if (a.qs.status[q]) return;
  const uint32_t c = a.cnt[q];
  if (c > a.cap || c <= a.k) return;
  float t;
  uint32_t m = tighten_one(a, q, c, hist, scratch, &t);
  if (threadIdx.x == 0) {
    a.cnt[q] = m;
    a.qs.thr[q] = t;
  }
}

// Sort (key, gid) pairs in shared or global memory, ascending by key then by
// gid -- the ordered global row id, so ties fall in row-id order (bitonic
// network over the next power of two; entries past the count are padding
// with the largest key).
__device__ void bitonic_sort(unsigned long long *key, unsigned long long *pos, uint32_t p2) {
  for (uint32_t size = 2; size <= p2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = threadIdx.x; i < p2 / 2; i += blockDim.x) {
        uint32_t lo = 2 * i - (i & (stride - 1));
        uint32_t hi = lo + stride;
        bool up = (lo & size) == 0;
        unsigned long long ka = key[lo], kb = key[hi];
        unsigned long long pa = pos[lo], pb = pos[hi];
        bool greater = ka > kb || (ka == kb && pa > pb);
        if (greater == up) {
          key[lo] = kb;
          key[hi] = ka;
          pos[lo] = pb;
          pos[hi] = pa;
        }
      }
      __syncthreads();
    }
  }
}

// Global row id of candidate position p (row_ids map, else first_id + row),
// as an unsigned key with the order of the signed id.
__device__ __forceinline__ unsigned long long gid_key(const SelectArgs &a, uint32_t p) {
  const uint64_t row = cand_row(a.ids, p, a.s.rows);
  const int64_t g = a.row_ids ? a.row_ids[row] : a.first_id + (int64_t)row;
  return (unsigned long long)g ^ 0x8000000000000000ull;
}

// Write a sorted survivor list: the k best, or the gathered window.
__device__ void write_results(const SelectArgs &a, uint32_t q, const unsigned long long *key,
                              const unsigned long long *gid, uint32_t m) {
  __shared__ uint32_t s_n;
  if (threadIdx.x == 0) {
    uint32_t n = m < a.k ? m : a.k;
    if (a.window && m > a.k) {
      double c = widen(key_double(key[a.k - 1]));
      unsigned long long ck = double_key(c);
      uint32_t lo = a.k, hi = m;  // first index with key > ck
      while (lo < hi) {
        uint32_t mid = (lo + hi) / 2;
        if (key[mid] <= ck) lo = mid + 1;
        else hi = mid;
      }
      n = lo;
    }
    if (n > a.out_cap) {
      n = a.out_cap;
      if (a.window) atomicOr(a.flags, FLAG_OUT_CAP);
    }
    s_n = n;
    a.out_count[q] = n;
  }
  __syncthreads();
  const uint32_t n = s_n;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    a.out_dist[(uint64_t)q * a.out_cap + i] = key_double(key[i]);
    a.out_id[(uint64_t)q * a.out_cap + i] = (int64_t)(gid[i] ^ 0x8000000000000000ull);
  }
}

// Final pruning of each query's list: drop what the k-th approximate score
// rules out; cnt[q] becomes the survivor count (or the query is left to the
// large-sort path when more than kSortCap survive).
__global__ void __launch_bounds__(NT) survivors(SelectArgs a) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t scratch[32];
  const uint32_t q = blockIdx.x;
  const double none = __longlong_as_double(0x7ff8000000000000ll);
  if (a.qs.status[q]) {
    if (threadIdx.x == 0) {
      a.cnt[q] = 0;
      a.out_count[q] = 0;
      if (a.upper) a.upper[q] = none;
    }
    return;
  }
  const uint32_t c = a.cnt[q];
  if (c > a.cap) {
    if (threadIdx.x == 0) {
      atomicOr(a.flags, FLAG_OVERFLOW);
      atomicMax(a.flags + 1, c);
      a.cnt[q] = 0;
      a.out_count[q] = 0;
      if (a.upper) a.upper[q] = none;
    }
    return;
  }
  float t;
  const uint32_t m = tighten_one(a, q, c, hist, scratch, &t, a.upper ? a.upper + q : nullptr);
  if (threadIdx.x == 0) {
    atomicAdd(a.flags + 3, c);   // statistics: candidates and survivors
    atomicAdd(a.flags + 4, m);
    if (m > (uint32_t)kSortCap) {
      a.big[q] = m;
      atomicOr(a.flags, FLAG_BIGSORT);
      atomicMax(a.flags + 2, m);
      a.out_count[q] = 0;
      a.cnt[q] = 0;          // the large-sort path reads big[q]
    } else {
      a.cnt[q] = m;
    }
  }
}

// The sharded search's second cut: the smallest of every rank's bounds U of
// the query's k-th exact distance bounds the merged answer's k-th distance
// too, so a survivor whose approximate score cannot reach it is dropped
// here instead of being re-scored, sorted and sent. A query keeps its local
// cut when no rank has a bound (NaN everywhere), and queries left to the
// large sort or to a new pass (count 0) are untouched.
__global__ void __launch_bounds__(NT) survivors_global(SelectArgs a, const double *upper_all, uint32_t nranks,
                                                       uint32_t ld) {
  __shared__ uint32_t scratch[32];
  const uint32_t q = blockIdx.x;
  if (a.qs.status[q]) return;
  const uint32_t m = a.cnt[q];
  if (m == 0) return;
  double U = __longlong_as_double(0x7ff8000000000000ll);
  for (uint32_t r = 0; r < nranks; r++) U = fmin(U, upper_all[(uint64_t)r * ld + q]);   // NaN: no bound
  if (!(U < __longlong_as_double(0x7ff0000000000000ll))) return;
  const float t = threshold_upper(a.metric, U, a.qs.err[q], a.window, a.qs.qn2d[q], (double)a.qs.rnq[q]);
  const uint32_t m2 = compact_le(a.cand + (uint64_t)q * a.cap, m, t, scratch);
  if (threadIdx.x == 0) {
    a.cnt[q] = m2;
    atomicSub(a.flags + 4, m - m2);   // statistics: survivors
  }
}

// Exact distance of every survivor, one thread a survivor with its own
// (alignment-checked) row loads: the path for rows whose pitch is not a
// multiple of 16 bytes.
template <int DT>
__global__ void __launch_bounds__(128) rescore_thread(SelectArgs a, unsigned long long *exact) {
  const uint32_t q = blockIdx.y;
  const uint32_t m = a.cnt[q];
  const uint2 *e = a.cand + (uint64_t)q * a.cap;
  const float *qv = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.queries) +
                                                    (uint64_t)q * a.qbytes);
  const double qn2d = a.qs.qn2d[q];
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) {
    const uint32_t p = e[i].y;
    const uint64_t id = cand_row(a.ids, p, a.s.rows);
    const uint8_t *row = a.staged ? a.staged + (uint64_t)p * a.s.row_bytes : a.s.codes + id * a.s.row_bytes;
    exact[(uint64_t)q * kSortCap + i] = double_key(exact_distance<DT>(a.s, id, qv, a.metric, qn2d, row, a.index_form));
  }
}

// Exact distance of every survivor of every query. A warp owns 32 survivors
// (one a lane) and streams their rows through shared memory 128 bytes at a
// time: each load instruction reads 4 rows x 128 contiguous bytes (the rows
// are random in HBM, so per-lane 16-byte loads of 32 different rows would
// run at a fifth of this bandwidth); then every lane sums its own row's
// chunk in the reference's exact operation order. Chunks are double
// buffered. exact[q * kSortCap + i] receives ordered keys. Needs a row pitch
// that is a multiple of 16 bytes (and 16-byte aligned rows).
constexpr int RS_WARPS = 4;

// Four E4M3 codes -> their values (exact: every E4M3 value is an FP16 value).
__device__ __forceinline__ void e4m3x4_values(uint32_t w, float (&v)[4]) {
  uint32_t o0, o1;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(o0), "=r"(o1)
      : "r"(w));
  const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&o0));
  const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&o1));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
// Eight E2M1 codes (low nibble first) -> their values (exact in FP16).
__device__ __forceinline__ void e2m1x8_values(uint32_t w, float (&v)[8]) {
  uint32_t o[4];
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&o[j]));
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
constexpr int RS_STRIDE = 144;  // bytes a staged row chunk: 128 + 16 of padding (bank-conflict free)

// Inner product and cosine sum FP64 products of FP32 values in dimension
// order (ann/server/cpu.c:118-126: dot += (double) x * (double) q). Such a
// product is exact in FP64 (24-bit significands give at most 48 bits; no
// FP32 pair overflows or underflows it), so the fused multiply-add
// fma(x, q, dot) rounds exactly as the reference's add of the rounded
// product does: one FP64 operation a dimension instead of two. The query
// is converted to FP64 once a block (qd, shared memory) when it fits.
constexpr uint32_t kQdMax = 2048;

template <int DT>
__device__ void rescore_group(const SelectArgs &a, unsigned long long *exact, uint32_t q, uint32_t m, uint32_t i0,
                              uint8_t (*stage)[32 * RS_STRIDE], const double *qd) {
  const int lane = threadIdx.x & 31;
  const uint2 *e = a.cand + (uint64_t)q * a.cap;
  const float *qv = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.queries) +
                                                    (uint64_t)q * a.qbytes);
  const ShardView &s = a.s;
  const uint32_t i = i0 + lane;
  const bool mine = i < m;
  const uint32_t p = mine ? e[i].y : e[i0].y;
  const uint64_t id = cand_row(a.ids, p, s.rows);
  const uint8_t *row = a.staged ? a.staged + (uint64_t)p * s.row_bytes : s.codes + id * s.row_bytes;
  const uint32_t chunks = (uint32_t)((s.row_bytes + 127) / 128);
  // lane l loads, for t = 0..7, 16 bytes (segment l % 8) of warp row l / 8 + 4t
  auto load_chunk = [&](uint32_t c, uint4 (&v)[8]) {
#pragma unroll
    for (int t = 0; t < 8; t++) {
      const int r = lane / 8 + 4 * t;
      const uint8_t *src = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, (unsigned long long)row, r));
      const uint64_t off = (uint64_t)c * 128 + (lane % 8) * 16;
      v[t] = off + 16 <= s.row_bytes ? __ldg(reinterpret_cast<const uint4 *>(src + off)) : make_uint4(0, 0, 0, 0);
    }
  };
  auto store_chunk = [&](int buf, const uint4 (&v)[8]) {
#pragma unroll
    for (int t = 0; t < 8; t++)
      *reinterpret_cast<uint4 *>(&stage[buf][(lane / 8 + 4 * t) * RS_STRIDE + (lane % 8) * 16]) = v[t];
  };
  const float rs = (DT == DT_E4M3 || DT == DT_NVFP4) ? __ldg(s.rowscale + id) : 1.0f;
  float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float tail = 0.0f;
  double dot = 0.0;
  uint32_t ham = 0;
  const uint32_t dims = s.dims;
  const uint8_t *qb = reinterpret_cast<const uint8_t *>(qv);
  const bool qvec = (reinterpret_cast<uintptr_t>(qv) & 15u) == 0;   // the query read 16 bytes at a time
  float bs = 0.0f;                                                   // NVFP4: the current 16-dim block's scale
  // one staging buffer a warp: the next chunk's loads go to registers while
  // this one is summed, and are stored after every lane is done with it
  // (the loop's closing __syncwarp), which leaves room for 8 blocks an SM
  uint4 v[8];
  load_chunk(0, v);
  for (uint32_t c = 0; c < chunks; c++) {
    const int buf = 0;
    store_chunk(buf, v);
    __syncwarp();
    if (c + 1 < chunks) load_chunk(c + 1, v);   // in flight while this chunk is summed
    const uint8_t *mine_chunk = &stage[buf][lane * RS_STRIDE];
    if (DT == DT_BIT) {
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const uint64_t off = (uint64_t)c * 128 + u * 16;
        if (off < s.row_bytes) {
          const uint4 x = *reinterpret_cast<const uint4 *>(mine_chunk + u * 16);
          const uint32_t *y = reinterpret_cast<const uint32_t *>(qb + off);
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int w = 0; w < 4; w++)
            if (off + 4 * w < s.row_bytes) ham += __popc(xs[w] ^ y[w]);
        }
      }
    } else {
      constexpr uint32_t per = DT == DT_F32 ? 32 : (DT == DT_F16 ? 64 : (DT == DT_E4M3 ? 128 : 256));
      const uint32_t d0 = c * per;
#pragma unroll 1
      for (uint32_t g = 0; g < per / 8; g++) {
        const uint32_t d = d0 + g * 8;
        if (d >= dims) break;
        float x[8];
        if (DT == DT_F32) {
          const float4 a4 = *reinterpret_cast<const float4 *>(mine_chunk + g * 32);
          const float4 b4 = *reinterpret_cast<const float4 *>(mine_chunk + g * 32 + 16);
          x[0] = a4.x; x[1] = a4.y; x[2] = a4.z; x[3] = a4.w; x[4] = b4.x; x[5] = b4.y; x[6] = b4.z; x[7] = b4.w;
        } else if (DT == DT_F16) {
          const uint4 w = *reinterpret_cast<const uint4 *>(mine_chunk + g * 16);
          const __half2 *h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            float2 f = __half22float2(h[j]);
            x[2 * j] = f.x;
            x[2 * j + 1] = f.y;
          }
        } else if (DT == DT_E4M3) {
          // code values by the hardware conversion, then the reference's FP32 product with the row scale
          const uint2 w = *reinterpret_cast<const uint2 *>(mine_chunk + g * 8);
          float lo[4], hi[4];
          e4m3x4_values(w.x, lo);
          e4m3x4_values(w.y, hi);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            x[j] = __fmul_rn(lo[j], rs);
            x[4 + j] = __fmul_rn(hi[j], rs);
          }
        } else {
          const uint32_t w = *reinterpret_cast<const uint32_t *>(mine_chunk + g * 4);
          if ((d & 15u) == 0) bs = __fmul_rn(e4m3_value(__ldg(s.bscales + id * s.bblocks + d / 16)), rs);
          float e[8];
          e2m1x8_values(w, e);
#pragma unroll
          for (int j = 0; j < 8; j++) x[j] = __fmul_rn(e[j], bs);
        }
        float qx[8];
        if (qvec && d + 8 <= dims) {
          const float4 q0 = *reinterpret_cast<const float4 *>(qv + d);
          const float4 q1 = *reinterpret_cast<const float4 *>(qv + d + 4);
          qx[0] = q0.x; qx[1] = q0.y; qx[2] = q0.z; qx[3] = q0.w;
          qx[4] = q1.x; qx[5] = q1.y; qx[6] = q1.z; qx[7] = q1.w;
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) qx[j] = d + j < dims ? qv[d + j] : 0.0f;
        }
        if (a.metric == M_L2) {
          if (d + 8 <= dims) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
              float diff = __fsub_rn(x[j], qx[j]);
              sums[j] = __fadd_rn(sums[j], __fmul_rn(diff, diff));
            }
          } else {
            for (int j = 0; d + j < dims; j++) {
              float diff = __fsub_rn(x[j], qx[j]);
              tail = __fadd_rn(tail, __fmul_rn(diff, diff));
            }
          }
        } else if (qd && d + 8 <= dims) {
          const double2 *q2 = reinterpret_cast<const double2 *>(qd + d);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const double2 qq = q2[j];
            dot = __fma_rn((double)x[2 * j], qq.x, dot);
            dot = __fma_rn((double)x[2 * j + 1], qq.y, dot);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++)
            if (d + j < dims) dot = __fma_rn((double)x[j], (double)qx[j], dot);
        }
      }
    }
    __syncwarp();
  }
  if (!mine) return;
  double dist;
  if (DT == DT_BIT) {
    dist = (double)ham;
  } else if (a.metric == M_L2) {
    dist = l2_finish(sums, tail, a.index_form);
  } else if (a.metric == M_IP) {
    dist = -dot;
  } else {
    const double r = __ddiv_rn(dot, __dsqrt_rn(__dmul_rn(s.n2x[id], a.qs.qn2d[q])));
    dist = __dsub_rn(1.0, fmax(-1.0, fmin(1.0, r)));
  }
  exact[(uint64_t)q * kSortCap + i] = double_key(dist);
}

// A few blocks a query, each warp taking 32 survivors at a time: most
// queries keep about k survivors, so a grid sized for the largest possible
// count (4,096) would be mostly blocks with nothing to do.
template <int DT>
__global__ void __launch_bounds__(RS_WARPS * 32, 8) rescore(SelectArgs a, unsigned long long *exact, int use_qd) {
  __shared__ __align__(16) uint8_t stage[RS_WARPS][1][32 * RS_STRIDE];
  extern __shared__ double qd_dyn[];
  const uint32_t q = blockIdx.y;
  const uint32_t m = a.cnt[q];
  const int warp = threadIdx.x >> 5;
  if (use_qd) {
    if ((uint32_t)(blockIdx.x * RS_WARPS * 32) >= m) return;   // no survivors for this block (whole block)
    const float *qv = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.queries) +
                                                      (uint64_t)q * a.qbytes);
    for (uint32_t d = threadIdx.x; d < a.s.dims; d += blockDim.x) qd_dyn[d] = (double)qv[d];
    __syncthreads();
  }
  for (uint32_t i0 = (blockIdx.x * RS_WARPS + warp) * 32; i0 < m; i0 += gridDim.x * RS_WARPS * 32)
    rescore_group<DT>(a, exact, q, m, i0, stage[warp], use_qd ? qd_dyn : nullptr);
}

// Per query: sort the survivors by (exact distance, global row id) and write
// the k best or the gathered window.
__global__ void __launch_bounds__(NTF) order(SelectArgs a, const unsigned long long *exact) {
  extern __shared__ uint8_t dyn[];
  unsigned long long *key = reinterpret_cast<unsigned long long *>(dyn);
  unsigned long long *pos = key + kSortCap;
  const uint32_t q = blockIdx.x;
  if (a.qs.status[q] || a.big[q]) return;
  const uint32_t m = a.cnt[q];
  if (m == 0) {
    if (threadIdx.x == 0) a.out_count[q] = 0;
    return;
  }
  uint32_t p2 = 1;
  while (p2 < m) p2 <<= 1;
  const uint2 *e = a.cand + (uint64_t)q * a.cap;
  for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) {
    if (i < m) {
      key[i] = exact[(uint64_t)q * kSortCap + i];
      pos[i] = gid_key(a, e[i].y);
    } else {
      key[i] = ~0ull;
      pos[i] = ~0ull;
    }
  }
  __syncthreads();
  bitonic_sort(key, pos, p2);
  write_results(a, q, key, pos, m);
}

// The same for one query whose survivors outgrew shared memory: rescoring and
// sorting in a global scratch of p2 (key, gid) pairs.
template <int DT>
__global__ void __launch_bounds__(NT) finalize_big(SelectArgs a, uint32_t q, unsigned long long *key,
                                                   unsigned long long *pos, uint32_t p2) {
  const uint32_t m = a.big[q];
  const uint2 *e = a.cand + (uint64_t)q * a.cap;
  const float *qv = reinterpret_cast<const float *>(reinterpret_cast<const uint8_t *>(a.queries) +
                                                    (uint64_t)q * a.qbytes);
  const double qn2d = a.qs.qn2d[q];
  for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) {
    if (i < m) {
      uint32_t p = e[i].y;
      uint64_t id = cand_row(a.ids, p, a.s.rows);
      const uint8_t *row = a.staged ? a.staged + (uint64_t)p * a.s.row_bytes : a.s.codes + id * a.s.row_bytes;
      key[i] = double_key(exact_distance<DT>(a.s, id, qv, a.metric, qn2d, row, a.index_form));
      pos[i] = gid_key(a, p);
    } else {
      key[i] = ~0ull;
      pos[i] = ~0ull;
    }
  }
  __syncthreads();
  bitonic_sort(key, pos, p2);
  write_results(a, q, key, pos, m);
}

// ---------------------------------------------------------------- rank merge

// Lists of per-shard results, each sorted by (distance, id): list l of query
// q has counts[l][q] entries at dist[l][q][..], ids[l][q][..], where list l
// starts `*_stride` bytes after list l-1 (the [nlists][nq][cap] layout of
// AnnB200MergeTopk, or the per-rank packets of the sharded search's
// all-gather).
struct RankMergeArgs {
  const uint8_t *dist, *ids, *counts;
  uint64_t dist_stride, id_stride, count_stride;
  uint32_t nlists, nq, list_cap, k, out_cap;
  double *out_dist;
  int64_t *out_id;
  uint32_t *out_count;
};

constexpr int RM_NT = 256;

// (key, id, list) order: equal (distance, id) pairs -- which disjoint shards
// never produce -- still get distinct ranks.
__device__ __forceinline__ bool rank_before(unsigned long long ka, unsigned long long ia, uint32_t la,
                                            unsigned long long kb, unsigned long long ib, uint32_t lb) {
  return ka < kb || (ka == kb && (ia < ib || (ia == ib && la < lb)));
}

// Per query: each entry's place in the merged order is its position in its
// own list plus, for every other list, how many of that list's entries come
// before it (a binary search: the lists are sorted). Entries placed before k
// are written there. No sort: one pass over the lists in shared memory.
__global__ void __launch_bounds__(RM_NT) merge_ranked(RankMergeArgs a) {
  extern __shared__ uint8_t dyn[];
  unsigned long long *key = reinterpret_cast<unsigned long long *>(dyn);
  unsigned long long *idk = key + kSortCap;
  __shared__ uint32_t s_off[65];
  const uint32_t q = blockIdx.x;
  if (threadIdx.x == 0) {
    uint32_t o = 0;
    for (uint32_t l = 0; l < a.nlists; l++) {
      s_off[l] = o;
      const uint32_t c = reinterpret_cast<const uint32_t *>(a.counts + l * a.count_stride)[q];
      o += c < a.list_cap ? c : a.list_cap;
    }
    s_off[a.nlists] = o;
  }
  __syncthreads();
  const uint32_t total = s_off[a.nlists];
  for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
    uint32_t l = 0;
    while (s_off[l + 1] <= i) l++;
    const uint64_t src = (uint64_t)q * a.list_cap + (i - s_off[l]);
    key[i] = double_key(reinterpret_cast<const double *>(a.dist + l * a.dist_stride)[src]);
    idk[i] = (unsigned long long)reinterpret_cast<const int64_t *>(a.ids + l * a.id_stride)[src] ^
             0x8000000000000000ull;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
    uint32_t l = 0;
    while (s_off[l + 1] <= i) l++;
    const unsigned long long ki = key[i], ii = idk[i];
    uint32_t rank = i - s_off[l];
    for (uint32_t m = 0; m < a.nlists && rank < a.k; m++) {
      if (m == l) continue;
      uint32_t lo = s_off[m], hi = s_off[m + 1];   // first entry of list m not before entry i
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (rank_before(key[mid], idk[mid], m, ki, ii, l)) lo = mid + 1;
        else hi = mid;
      }
      rank += lo - s_off[m];
    }
    if (rank < a.k) {
      a.out_dist[(uint64_t)q * a.out_cap + rank] = key_double(ki);
      a.out_id[(uint64_t)q * a.out_cap + rank] = (int64_t)(ii ^ 0x8000000000000000ull);
    }
  }
  if (threadIdx.x == 0) a.out_count[q] = total < a.k ? total : a.k;
}

// ---------------------------------------------------------------- score matrix

// v-domain scores -> approximate distances (squared distance for L2).
__global__ void v_to_distance(float *m, uint64_t n, uint32_t nq, uint32_t metric, QueryState qs) {
  const uint32_t q = blockIdx.y;
  const double qn2 = qs.qn2d[q], rnq = qs.rnq[q];
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float *p = m + (uint64_t)q * n + i;
    *p = (float)v_to_dist(metric, (double)*p, qn2, rnq);
  }
}

// ---------------------------------------------------------------- merge

struct MergeArgs {
  const double *dist;
  const int64_t *ids;
  const uint32_t *counts;
  uint32_t nlists, nq, list_cap, k;
  int window;
  uint32_t out_cap;
  double *out_dist;
  int64_t *out_id;
  uint32_t *out_count;
  uint32_t *flags;
};

// Per query: gather every list's entries, sort by (distance, id), keep the k
// best (or the gathered window of the merged k-th distance).
__global__ void __launch_bounds__(NT) merge_lists(MergeArgs a) {
  extern __shared__ uint8_t dyn[];
  unsigned long long *key = reinterpret_cast<unsigned long long *>(dyn);
  unsigned long long *idk = key + kSortCap;
  __shared__ uint32_t s_off[65];
  __shared__ uint32_t s_n;
  const uint32_t q = blockIdx.x;
  if (threadIdx.x == 0) {
    uint32_t o = 0;
    for (uint32_t l = 0; l < a.nlists; l++) {
      s_off[l] = o;
      uint32_t c = a.counts[(uint64_t)l * a.nq + q];
      o += c < a.list_cap ? c : a.list_cap;
    }
    s_off[a.nlists] = o;
  }
  __syncthreads();
  const uint32_t total = s_off[a.nlists];
  uint32_t p2 = 1;
  while (p2 < total) p2 <<= 1;
  for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) {
    if (i < total) {
      uint32_t l = 0;
      while (s_off[l + 1] <= i) l++;
      uint64_t src = ((uint64_t)l * a.nq + q) * a.list_cap + (i - s_off[l]);
      key[i] = double_key(a.dist[src]);
      idk[i] = (unsigned long long)a.ids[src] ^ 0x8000000000000000ull;
    } else {
      key[i] = ~0ull;
      idk[i] = ~0ull;
    }
  }
  __syncthreads();
  // bitonic on (key, id) pairs
  for (uint32_t size = 2; size <= p2; size <<= 1)
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = threadIdx.x; i < p2 / 2; i += blockDim.x) {
        uint32_t lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        bool up = (lo & size) == 0;
        unsigned long long ka = key[lo], kb = key[hi], ia = idk[lo], ib = idk[hi];
        bool greater = ka > kb || (ka == kb && ia > ib);
        if (greater == up) {
          key[lo] = kb;
          key[hi] = ka;
          idk[lo] = ib;
          idk[hi] = ia;
        }
      }
      __syncthreads();
    }
  if (threadIdx.x == 0) {
    uint32_t n = total < a.k ? total : a.k;
    if (a.window && total > a.k) {
      unsigned long long ck = double_key(widen(key_double(key[a.k - 1])));
      uint32_t lo = a.k, hi = total;
      while (lo < hi) {
        uint32_t mid = (lo + hi) / 2;
        if (key[mid] <= ck) lo = mid + 1;
        else hi = mid;
      }
      n = lo;
    }
    if (n > a.out_cap) {
      n = a.out_cap;
      if (a.window) atomicOr(a.flags, FLAG_OUT_CAP);
    }
    s_n = n;
    a.out_count[q] = n;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < s_n; i += blockDim.x) {
    a.out_dist[(uint64_t)q * a.out_cap + i] = key_double(key[i]);
    a.out_id[(uint64_t)q * a.out_cap + i] = (int64_t)(idk[i] ^ 0x8000000000000000ull);
  }
}

// ---------------------------------------------------------------- bitmap rows

constexpr int BM_WORDS = 1024;  // words a block of the bitmap kernels

__global__ void bitmap_count(const uint32_t *words, uint64_t nwords, uint64_t nbits, uint32_t *blockcnt) {
  __shared__ uint32_t scratch[32];
  uint64_t w = (uint64_t)blockIdx.x * BM_WORDS + threadIdx.x;
  uint32_t c = 0;
  if (w < nwords) {
    uint32_t x = words[w];
    uint64_t b0 = w * 32;
    if (b0 + 32 > nbits) x &= (nbits - b0 >= 32) ? 0xffffffffu : ((1u << (nbits - b0)) - 1u);
    c = __popc(x);
  }
  uint32_t total;
  block_exclusive_scan(c, scratch, &total);
  if (threadIdx.x == 0) blockcnt[blockIdx.x] = total;
}

__global__ void bitmap_scan(uint32_t *blockcnt, uint32_t nblocks, unsigned long long *total_out) {
  __shared__ uint32_t scratch[32];
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (uint32_t base = 0; base < nblocks; base += blockDim.x) {
    uint32_t i = base + threadIdx.x;
    uint32_t v = i < nblocks ? blockcnt[i] : 0;
    uint32_t total;
    uint32_t before = block_exclusive_scan(v, scratch, &total);
    unsigned long long c = carry;
    if (i < nblocks) blockcnt[i] = (uint32_t)(c + before);
    __syncthreads();
    if (threadIdx.x == 0) carry = c + total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total_out = carry;
}

__global__ void bitmap_write(const uint32_t *words, uint64_t nwords, uint64_t nbits, const uint32_t *blockoff,
                             uint32_t *rows, uint32_t base) {
  __shared__ uint32_t scratch[32];
  uint64_t w = (uint64_t)blockIdx.x * BM_WORDS + threadIdx.x;
  uint32_t x = 0;
  if (w < nwords) {
    x = words[w];
    uint64_t b0 = w * 32;
    if (b0 + 32 > nbits) x &= (nbits - b0 >= 32) ? 0xffffffffu : ((1u << (nbits - b0)) - 1u);
  }
  uint32_t total;
  uint32_t before = block_exclusive_scan(__popc(x), scratch, &total);
  uint32_t o = blockoff[blockIdx.x] + before;
  while (x) {
    uint32_t b = __ffs(x) - 1;
    rows[o++] = base + (uint32_t)(w * 32 + b);
    x &= x - 1;
  }
}

// The same re-score with each candidate's row fetched by ordinal from a row
// array the device reads directly (device memory, or host memory mapped for
// the device): one warp a candidate, its row read in coalesced 128-byte
// pieces; every lane forms its dimensions' FP64 squared differences into
// shared memory, and lane 0 adds them in dimension order (the reference's
// order, so the sum is bit-identical).
constexpr int RG_WARPS = 8, RG_CHUNK = 256;

__global__ void __launch_bounds__(RG_WARPS * 32) rescore_gather(const float *__restrict__ queries, uint32_t nq,
                                                                uint32_t dims, const float *__restrict__ rows,
                                                                const uint64_t *__restrict__ ords, uint32_t stride,
                                                                const uint32_t *__restrict__ counts,
                                                                float *__restrict__ out) {
  __shared__ double buf[RG_WARPS][RG_CHUNK];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t w = (uint64_t)blockIdx.x * RG_WARPS + warp;
  if (w >= (uint64_t)nq * stride) return;                  // whole warps leave together
  const uint32_t q = (uint32_t)(w / stride), j = (uint32_t)(w % stride);
  if (counts && j >= counts[q]) return;
  const float *x = rows + ords[w] * (uint64_t)dims;
  const float *v = queries + (uint64_t)q * dims;
  double sum = 0.0;
  for (uint32_t d0 = 0; d0 < dims; d0 += RG_CHUNK) {
    const uint32_t n = min((uint32_t)RG_CHUNK, dims - d0);
    float r[RG_CHUNK / 32];
#pragma unroll
    for (int t = 0; t < RG_CHUNK / 32; t++) {
      const uint32_t i = lane + 32u * t;
      r[t] = i < n ? x[d0 + i] : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < RG_CHUNK / 32; t++) {
      const uint32_t i = lane + 32u * t;
      if (i < n) {
        const double delta = __dsub_rn((double)r[t], (double)__ldg(v + d0 + i));
        buf[warp][i] = __dmul_rn(delta, delta);
      }
    }
    __syncwarp();
    if (lane == 0)
      for (uint32_t t = 0; t < n; t++) sum = __dadd_rn(sum, buf[warp][t]);
    __syncwarp();
  }
  if (lane == 0) out[w] = __double2float_rn(__dsqrt_rn(sum));
}

// FP32 -> FP16 (round to nearest even): a shard made from FP32 rows but kept
// as halves (a loaded index whose manifest says dtype float16).
__global__ void f32_to_f16(const float *__restrict__ in, __half *__restrict__ out, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(in[i]);
}

}  // namespace

// ---------------------------------------------------------------- launchers

void launch_f32_to_f16(const float *in, __half *out, uint64_t n, cudaStream_t st) {
  if (n) f32_to_f16<<<(unsigned)std::min<uint64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(in, out, n);
}

void launch_rescore_rows(const float *queries, uint32_t nq, uint32_t dims, const float *rows, uint32_t stride,
                         const uint32_t *counts, float *out, cudaStream_t st) {
  const uint64_t n = (uint64_t)nq * stride;
  // 16-byte loads where every row and query starts on a 16-byte boundary
  const int vec4 = (dims & 3) == 0 && (((uintptr_t)queries | (uintptr_t)rows) & 15) == 0;
  if (n)
    rescore_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(queries, nq, dims, rows, stride, counts, out, vec4);
}

void launch_rescore_gather(const float *queries, uint32_t nq, uint32_t dims, const float *rows,
                           const uint64_t *ords, uint32_t stride, const uint32_t *counts, float *out,
                           cudaStream_t st) {
  const uint64_t n = (uint64_t)nq * stride;
  if (n)
    rescore_gather<<<(unsigned)((n + RG_WARPS - 1) / RG_WARPS), RG_WARPS * 32, 0, st>>>(queries, nq, dims, rows, ords,
                                                                                        stride, counts, out);
}

void launch_shard_stats(const ShardView &s, float *n2, float *rn, double *n2x, uint32_t *maxn2, cudaStream_t st) {
  if (s.rows == 0 || s.dtype == DT_BIT) return;
  dim3 grid((unsigned)((s.rows + 7) / 8));
  dim3 gridx((unsigned)((s.rows + 127) / 128));
  switch (s.dtype) {
    case DT_F32:
      shard_stats<DT_F32><<<grid, 256, 0, st>>>(s, n2, rn, maxn2);
      exact_norms<DT_F32><<<gridx, 128, 0, st>>>(s, n2x);
      break;
    case DT_F16:
      shard_stats<DT_F16><<<grid, 256, 0, st>>>(s, n2, rn, maxn2);
      exact_norms<DT_F16><<<gridx, 128, 0, st>>>(s, n2x);
      break;
    case DT_E4M3:
      shard_stats<DT_E4M3><<<grid, 256, 0, st>>>(s, n2, rn, maxn2);
      exact_norms<DT_E4M3><<<gridx, 128, 0, st>>>(s, n2x);
      break;
    case DT_NVFP4:
      shard_stats<DT_NVFP4><<<grid, 256, 0, st>>>(s, n2, rn, maxn2);
      exact_norms<DT_NVFP4><<<gridx, 128, 0, st>>>(s, n2x);
      break;
  }
}

void launch_prep_queries(const float *queries, uint32_t nq, uint32_t dims, uint32_t metric, uint32_t kpad,
                         int use_q16, double gamma, const uint32_t *maxn2, const QueryState &qs, int bits,
                         uint32_t *flags, cudaStream_t st, uint64_t lo_off, int f8) {
  if (bits) {
    prep_queries_bits<<<(nq + 255) / 256, 256, 0, st>>>(nq, qs);
    if (use_q16 && nq)
      expand_query_bits<<<nq, 256, 0, st>>>(reinterpret_cast<const uint8_t *>(queries), (dims + 7) / 8, kpad,
                                            reinterpret_cast<int8_t *>(qs.q16));
    return;
  }
  PrepArgs p{queries, nq, dims, metric, kpad, use_q16, lo_off, gamma, maxn2, qs, flags, f8};
  prep_queries<<<nq, 256, dims <= kPrepSqMax ? dims * sizeof(double) : 0, st>>>(p);
}

void launch_fill_thresholds(uint32_t nq, const QueryState &qs, cudaStream_t st) {
  fill_thresholds<<<(nq + 255) / 256, 256, 0, st>>>(nq, qs);
}

void launch_check_rows(const uint32_t *ids, uint64_t n, uint64_t rows, uint32_t *flags, cudaStream_t st) {
  if (n) check_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, rows, flags);
}

void launch_kth_bound(const float *mat, uint64_t ld, uint64_t n, uint32_t nq, uint32_t k, uint32_t metric,
                      int window, const QueryState &qs, cudaStream_t st) {
  BoundArgs b{mat, ld, n, k, metric, window, qs};
  if (n <= 256ull * KB_REG) kth_bound<256><<<nq, 256, 0, st>>>(b);
  else kth_bound<NT><<<nq, NT, 0, st>>>(b);
}

static SelectArgs to_args(const SelectLaunch &l) {
  SelectArgs a{l.s,   l.staged, l.row_ids, l.ids,   l.queries, l.nq,  l.k,        l.metric,   l.window,    l.qbytes,   l.qs,
               l.cnt, l.cand,  l.cap,     l.flags, l.big,    l.out_dist, l.out_id,    l.out_count, l.out_cap,
               l.first_id, l.index_form, l.upper};
  return a;
}

void launch_tighten(const SelectLaunch &l, cudaStream_t st) { tighten<<<l.nq, NT, 0, st>>>(to_args(l)); }

void launch_survivors(const SelectLaunch &l, cudaStream_t st) { survivors<<<l.nq, NT, 0, st>>>(to_args(l)); }

void launch_survivors_global(const SelectLaunch &l, const double *upper_all, uint32_t nranks, uint32_t ld,
                             cudaStream_t st) {
  survivors_global<<<l.nq, NT, 0, st>>>(to_args(l), upper_all, nranks, ld);
}

// Exact rescoring of the survivors (flat grid) and the per-query ordering.
cudaError_t launch_finalize(const SelectLaunch &l, double *exact, cudaStream_t st) {
  unsigned long long *ex = reinterpret_cast<unsigned long long *>(exact);
  const SelectArgs a = to_args(l);
  if (l.s.row_bytes % 16 != 0) {
    const dim3 g(2, l.nq);
    switch (l.s.dtype) {
      case DT_F32: rescore_thread<DT_F32><<<g, 128, 0, st>>>(a, ex); break;
      case DT_F16: rescore_thread<DT_F16><<<g, 128, 0, st>>>(a, ex); break;
      case DT_E4M3: rescore_thread<DT_E4M3><<<g, 128, 0, st>>>(a, ex); break;
      case DT_NVFP4: rescore_thread<DT_NVFP4><<<g, 128, 0, st>>>(a, ex); break;
      default: rescore_thread<DT_BIT><<<g, 128, 0, st>>>(a, ex); break;
    }
  } else {
    const dim3 grid(2, l.nq);
    const int use_qd = l.metric != M_L2 && l.s.dtype != DT_BIT && l.s.dims <= kQdMax;
    const size_t qsm = use_qd ? (size_t)l.s.dims * sizeof(double) : 0;
    switch (l.s.dtype) {
      case DT_F32: rescore<DT_F32><<<grid, RS_WARPS * 32, qsm, st>>>(a, ex, use_qd); break;
      case DT_F16: rescore<DT_F16><<<grid, RS_WARPS * 32, qsm, st>>>(a, ex, use_qd); break;
      case DT_E4M3: rescore<DT_E4M3><<<grid, RS_WARPS * 32, qsm, st>>>(a, ex, use_qd); break;
      case DT_NVFP4: rescore<DT_NVFP4><<<grid, RS_WARPS * 32, qsm, st>>>(a, ex, use_qd); break;
      default: rescore<DT_BIT><<<grid, RS_WARPS * 32, 0, st>>>(a, ex, 0); break;
    }
  }
  const size_t smem = (size_t)kSortCap * (8 + 8);
  cudaError_t e = cudaFuncSetAttribute(order, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  order<<<l.nq, NTF, smem, st>>>(a, ex);
  return cudaGetLastError();
}

void launch_finalize_big(const SelectLaunch &l, uint32_t q, unsigned long long *key, unsigned long long *pos,
                         uint32_t p2, cudaStream_t st) {
  switch (l.s.dtype) {
    case DT_F32: finalize_big<DT_F32><<<1, NT, 0, st>>>(to_args(l), q, key, pos, p2); break;
    case DT_F16: finalize_big<DT_F16><<<1, NT, 0, st>>>(to_args(l), q, key, pos, p2); break;
    case DT_E4M3: finalize_big<DT_E4M3><<<1, NT, 0, st>>>(to_args(l), q, key, pos, p2); break;
    case DT_NVFP4: finalize_big<DT_NVFP4><<<1, NT, 0, st>>>(to_args(l), q, key, pos, p2); break;
    default: finalize_big<DT_BIT><<<1, NT, 0, st>>>(to_args(l), q, key, pos, p2); break;
  }
}

cudaError_t launch_merge_ranked(const void *dist, uint64_t dist_stride, const void *ids, uint64_t id_stride,
                                const void *counts, uint64_t count_stride, uint32_t nlists, uint32_t nq,
                                uint32_t list_cap, uint32_t k, uint32_t out_cap, double *out_dist, int64_t *out_id,
                                uint32_t *out_count, cudaStream_t st) {
  if (nq == 0) return cudaSuccess;
  RankMergeArgs a{(const uint8_t *)dist, (const uint8_t *)ids, (const uint8_t *)counts, dist_stride, id_stride,
                  count_stride, nlists, nq, list_cap, k, out_cap, out_dist, out_id, out_count};
  const size_t smem = (size_t)kSortCap * 16;
  cudaError_t e = cudaFuncSetAttribute(merge_ranked, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  merge_ranked<<<nq, RM_NT, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_merge(const double *dist, const int64_t *ids, const uint32_t *counts, uint32_t nlists,
                         uint32_t nq, uint32_t list_cap, uint32_t k, int window, uint32_t out_cap,
                         double *out_dist, int64_t *out_id, uint32_t *out_count, uint32_t *flags,
                         cudaStream_t st) {
  MergeArgs a{dist, ids, counts, nlists, nq, list_cap, k, window, out_cap, out_dist, out_id, out_count, flags};
  const size_t smem = (size_t)kSortCap * 16;
  cudaError_t e = cudaFuncSetAttribute(merge_lists, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  merge_lists<<<nq, NT, smem, st>>>(a);
  return cudaGetLastError();
}

void launch_v_to_distance(float *m, uint64_t n, uint32_t nq, uint32_t metric, const QueryState &qs, cudaStream_t st) {
  dim3 grid((unsigned)std::min<uint64_t>((n + 255) / 256, 1024), nq);
  v_to_distance<<<grid, 256, 0, st>>>(m, n, nq, metric, qs);
}

uint32_t bitmap_blocks(uint64_t nbits) {
  uint64_t nwords = (nbits + 31) / 32;
  return (uint32_t)((nwords + BM_WORDS - 1) / BM_WORDS);
}

void launch_bitmap_rows(const uint32_t *words, uint64_t nbits, uint32_t *rows, uint32_t *blockcnt,
                        unsigned long long *total, cudaStream_t st, uint32_t base) {
  uint64_t nwords = (nbits + 31) / 32;
  uint32_t nb = bitmap_blocks(nbits);
  if (nb == 0) return;
  bitmap_count<<<nb, BM_WORDS, 0, st>>>(words, nwords, nbits, blockcnt);
  bitmap_scan<<<1, 1024, 0, st>>>(blockcnt, nb, total);
  bitmap_write<<<nb, BM_WORDS, 0, st>>>(words, nwords, nbits, blockcnt, rows, base);
}

}  // namespace annb200
