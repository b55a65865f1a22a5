// ivf.cu - IVF list gather: each query scans every row of the lists it probes.
//
// The reference's IVFFlat scan (src/ivfscan.c:124-186) visits the probed
// lists of one query, scores every entry and sorts them. Here a batch of
// queries is turned list-major: the probe table [nq][nprobe] is inverted on
// the device into, for each list, the queries that probe it (count, scan,
// fill), and one work item is a (list, 64-row tile, group of up to 16 of the
// list's queries). The rows of a list are contiguous in the shard, so a tile
// is one coalesced run read once for all the queries of its group, whatever
// the batch's probe pattern. A persistent grid walks the items through a
// prefix sum of per-list tile counts. The approximate scores only prune: the
// exact rescoring and ordering of the candidates are the flat search's own
// kernels.
#include "internal.cuh"

namespace annb200 {

namespace {

constexpr int BM = 64;          // rows a tile
constexpr int BK = 32;          // dimensions a shared-memory step
constexpr int BQ = 16;          // queries a tile
constexpr int SCAN_T = 1024;    // threads of the prefix-sum blocks
constexpr int SCAN_ITEMS = 4;   // values a thread
constexpr int SCAN_BLOCK = SCAN_T * SCAN_ITEMS;

// ---------------------------------------------------------------- prefix sum (u64)

__device__ unsigned long long warp_inclusive(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned long long u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

// Exclusive scan of one block's SCAN_BLOCK values; returns the block total.
__device__ unsigned long long block_scan_items(unsigned long long (&x)[SCAN_ITEMS]) {
  __shared__ unsigned long long warp_tot[SCAN_T / 32];
  __shared__ unsigned long long block_tot;
  unsigned long long t = 0;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++) {
    unsigned long long v = x[i];
    x[i] = t;
    t += v;
  }
  const unsigned long long inc = warp_inclusive(t);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long w = warp_tot[lane];
    warp_tot[lane] = warp_inclusive(w) - w;
  }
  __syncthreads();
  const unsigned long long off = warp_tot[warp] + inc - t;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++) x[i] += off;
  if (threadIdx.x == SCAN_T - 1) block_tot = off + t;
  __syncthreads();
  return block_tot;
}

__global__ void __launch_bounds__(SCAN_T) scan_blocks(const unsigned long long *in, uint64_t n,
                                                      unsigned long long *out, unsigned long long *bsum) {
  unsigned long long x[SCAN_ITEMS];
  const uint64_t base = (uint64_t)blockIdx.x * SCAN_BLOCK + (uint64_t)threadIdx.x * SCAN_ITEMS;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++) x[i] = base + i < n ? in[base + i] : 0ull;
  unsigned long long total = block_scan_items(x);
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++)
    if (base + i < n) out[base + i] = x[i];
  if (threadIdx.x == 0) bsum[blockIdx.x] = total;
}

// One block: exclusive scan of the nb <= SCAN_BLOCK block totals; the grand
// total goes to out[n].
__global__ void __launch_bounds__(SCAN_T) scan_sums(unsigned long long *bsum, uint32_t nb, unsigned long long *out,
                                                    uint64_t n) {
  unsigned long long x[SCAN_ITEMS];
  const uint32_t base = threadIdx.x * SCAN_ITEMS;
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++) x[i] = base + i < nb ? bsum[base + i] : 0ull;
  unsigned long long total = block_scan_items(x);
#pragma unroll
  for (int i = 0; i < SCAN_ITEMS; i++)
    if (base + i < nb) bsum[base + i] = x[i];
  if (threadIdx.x == 0) out[n] = total;
}

__global__ void scan_add(unsigned long long *out, uint64_t n, const unsigned long long *bsum) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] += bsum[i / SCAN_BLOCK];
}

// out[0..n] = exclusive prefix sums of in[0..n) and the total (n <= 2^24).
void exclusive_scan(const unsigned long long *in, uint64_t n, unsigned long long *out, unsigned long long *bsum,
                    cudaStream_t st) {
  const uint32_t nb = (uint32_t)((n + SCAN_BLOCK - 1) / SCAN_BLOCK);
  if (nb > 0) scan_blocks<<<nb, SCAN_T, 0, st>>>(in, n, out, bsum);
  scan_sums<<<1, SCAN_T, 0, st>>>(bsum, nb, out, n);
  if (nb > 1) scan_add<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(out, n, bsum);
}

// ---------------------------------------------------------------- probe table

__global__ void check_offsets(ListPlan p, uint32_t *flags) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= p.nlists) return;
  const uint64_t lo = p.offsets[l], hi = p.offsets[l + 1];
  if (hi < lo || hi > p.rows) atomicOr(flags, FLAG_BAD_ROWS);
}

// One block a query: a list number past nlists or a list probed twice makes
// the query invalid (status 1); a valid query counts itself into its lists.
// kNoProbe entries are padding (a query with fewer lists on this shard).
// Duplicates show as equal neighbours once the query's probes are sorted.
__global__ void __launch_bounds__(256) probe_count(ListPlan p, QueryState qs, uint32_t *flags) {
  __shared__ uint32_t s[kMaxProbes];
  __shared__ int bad;
  const uint32_t q = blockIdx.x;
  const uint32_t *pr = p.probes + (uint64_t)q * p.nprobe;
  uint32_t p2 = 1;
  while (p2 < p.nprobe) p2 <<= 1;
  if (threadIdx.x == 0) bad = 0;
  for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) s[i] = i < p.nprobe ? pr[i] : 0xffffffffu;
  __syncthreads();
  for (uint32_t size = 2; size <= p2; size <<= 1)
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = threadIdx.x; i < p2 / 2; i += blockDim.x) {
        const uint32_t lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint32_t x = s[lo], y = s[hi];
        if ((x > y) == up) {
          s[lo] = y;
          s[hi] = x;
        }
      }
      __syncthreads();
    }
  for (uint32_t i = threadIdx.x; i < p.nprobe; i += blockDim.x)
    if (s[i] != kNoProbe && (s[i] >= p.nlists || (i + 1 < p.nprobe && s[i] == s[i + 1]))) bad = 1;
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) {
      if (!qs.status[q]) atomicAdd(flags + 5, 1u);
      qs.status[q] = 1;
    }
    return;
  }
  if (qs.status[q]) return;
  for (uint32_t i = threadIdx.x; i < p.nprobe; i += blockDim.x)
    if (pr[i] != kNoProbe) atomicAdd(p.lcount + pr[i], 1ull);
}

__global__ void probe_fill(ListPlan p, QueryState qs) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= p.nq || qs.status[q]) return;
  const uint32_t *pr = p.probes + (uint64_t)q * p.nprobe;
  for (uint32_t i = 0; i < p.nprobe; i++) {
    const uint32_t l = pr[i];
    if (l == kNoProbe) continue;
    const unsigned long long slot = atomicAdd(p.lfill + l, 1ull);
    p.qlist[p.qoff[l] + slot] = q;
  }
}

// Work items of list l: row tiles (p.bm rows) of its rows [rbegin, rend) x
// query groups (p.bq queries).
__global__ void count_tiles(ListPlan p, uint64_t rbegin, uint64_t rend) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= p.nlists) return;
  uint64_t b, e;
  list_window(p, l, rbegin, rend, b, e);
  const uint64_t len = e - b;
  const uint64_t groups = (p.lcount[l] + p.bq - 1) / p.bq;
  p.tiles[l] = (len + p.bm - 1) / p.bm * groups;
}

__global__ void flag_nonempty(ListPlan p) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l < p.nlists) p.lfill[l] = p.tiles[l] > 0 ? 1ull : 0ull;
}

__global__ void scatter_nonempty(ListPlan p) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l < p.nlists && p.tiles[l] > 0) p.nzl[p.nzoff[l]] = l;
}

// ---------------------------------------------------------------- list scan

template <int DT>
__global__ void __launch_bounds__(256) simt_scan_lists(const ListPlan p, uint64_t rbegin, uint64_t rend,
                                                        const ScanArgs a) {
  __shared__ __align__(16) float xs[BK][BM + 4];
  __shared__ float qs[BK][BQ + 4];
  __shared__ uint32_t qidx[BQ];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int lr = tid / 4, lc = (tid % 4) * 8;
  const uint32_t dims = a.s.dims;
  const uint64_t items = p.toff[p.nlists];

  for (uint64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const uint32_t l = find_list(p.toff, p.nlists, item);
    const uint64_t t = item - p.toff[l];
    const uint64_t nql = p.lcount[l];
    const uint64_t groups = (nql + BQ - 1) / BQ;
    const uint64_t g = t % groups, rt = t / groups;
    uint64_t lo, hi;
    list_window(p, l, rbegin, rend, lo, hi);
    const uint64_t r0 = lo + rt * BM;
    const uint32_t nqt = (uint32_t)(nql - g * BQ < BQ ? nql - g * BQ : BQ);
    if (tid < BQ) qidx[tid] = tid < (int)nqt ? p.qlist[p.qoff[l] + g * BQ + tid] : 0u;
    __syncthreads();

    const uint64_t lrow = r0 + lr;
    const bool lvalid = lrow < hi;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t k0 = 0; k0 < dims; k0 += BK) {
      float v[8];
      if (lvalid) decode8<DT>(a.s, lrow, k0 + lc, v);
      else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; j++) xs[lc + j][lr] = v[j];
      // BQ x BK query values, two a thread
#pragma unroll
      for (int j = 0; j < BQ * BK / 256; j++) {
        const int e = tid * (BQ * BK / 256) + j;
        const int qi = e / BK, kk = e % BK;
        const uint32_t d = k0 + kk;
        qs[kk][qi] = (qi < (int)nqt && d < dims) ? __ldg(a.queries + (uint64_t)qidx[qi] * dims + d) : 0.0f;
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < BK; kk++) {
        const float4 x = *reinterpret_cast<const float4 *>(&xs[kk][ty * 4]);
        const float b = qs[kk][tx];
        acc[0] = fmaf(x.x, b, acc[0]);
        acc[1] = fmaf(x.y, b, acc[1]);
        acc[2] = fmaf(x.z, b, acc[2]);
        acc[3] = fmaf(x.w, b, acc[3]);
      }
      __syncthreads();
    }
    if (tx < (int)nqt) {
      const uint32_t q = qidx[tx];
      const float thr = __ldg(a.thr + q);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint64_t row = r0 + ty * 4 + i;
        if (row >= hi) continue;
        float al, be;
        row_affine(a.s, row, a.metric, 0, al, be);
        const float v = fmaf(acc[i], al, be);
        if (v <= thr) append_candidate(a, v, row, q);
      }
    }
    __syncthreads();  // qidx is rewritten by the next item
  }
}

// Probe table from a centroid search's results: entry j of query q is the
// list (id - first) of its j-th nearest centroid, UINT32_MAX past the count.
__global__ void probe_table(const int64_t *ids, const uint32_t *counts, uint32_t nq, uint32_t nprobe, int64_t first,
                            uint32_t *probes) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint64_t)nq * nprobe) return;
  const uint32_t q = (uint32_t)(i / nprobe), j = (uint32_t)(i % nprobe);
  probes[i] = j < counts[q] ? (uint32_t)(ids[i] - first) : kNoProbe;
}

}  // namespace

void launch_probe_table(const int64_t *ids, const uint32_t *counts, uint32_t nq, uint32_t nprobe, int64_t first,
                        uint32_t *probes, cudaStream_t st) {
  const uint64_t n = (uint64_t)nq * nprobe;
  if (n) probe_table<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, counts, nq, nprobe, first, probes);
}

// Invert the probe table: lcount, qoff, qlist (queries of each list). Marks
// queries with bad probes invalid and flags bad offsets.
void launch_list_plan(const ListPlan &p, const QueryState &qs, uint32_t *flags, cudaStream_t st) {
  if (p.nlists) check_offsets<<<(p.nlists + 255) / 256, 256, 0, st>>>(p, flags);
  probe_count<<<p.nq, 256, 0, st>>>(p, qs, flags);
  exclusive_scan(p.lcount, p.nlists, p.qoff, p.bsum, st);
  probe_fill<<<(p.nq + 127) / 128, 128, 0, st>>>(p, qs);
}

// Items of a pass over rows [rbegin, rend) of every probed list.
// With p.nzl set, also the compact list of lists that have work items
// (flags in lfill, free once the probe table is inverted).
void launch_list_items(const ListPlan &p, uint64_t rbegin, uint64_t rend, cudaStream_t st) {
  if (p.nlists) count_tiles<<<(p.nlists + 255) / 256, 256, 0, st>>>(p, rbegin, rend);
  exclusive_scan(p.tiles, p.nlists, p.toff, p.bsum, st);
  if (p.nzl) {
    if (p.nlists) flag_nonempty<<<(p.nlists + 255) / 256, 256, 0, st>>>(p);
    exclusive_scan(p.lfill, p.nlists, p.nzoff, p.bsum, st);
    if (p.nlists) scatter_nonempty<<<(p.nlists + 255) / 256, 256, 0, st>>>(p);
  }
}

// (p.bm and p.bq must be 64 and 16: the items counted for this kernel.)
void launch_simt_scan_lists(const ListPlan &p, uint64_t rbegin, uint64_t rend, const ScanArgs &a, int sms,
                            cudaStream_t st) {
  const dim3 grid((unsigned)sms * 8);
  switch (a.s.dtype) {
    case DT_F32: simt_scan_lists<DT_F32><<<grid, 256, 0, st>>>(p, rbegin, rend, a); break;
    case DT_F16: simt_scan_lists<DT_F16><<<grid, 256, 0, st>>>(p, rbegin, rend, a); break;
    case DT_E4M3: simt_scan_lists<DT_E4M3><<<grid, 256, 0, st>>>(p, rbegin, rend, a); break;
    case DT_NVFP4: simt_scan_lists<DT_NVFP4><<<grid, 256, 0, st>>>(p, rbegin, rend, a); break;
    default: break;
  }
}

uint32_t list_plan_scan_launches(uint32_t nlists) {
  const uint32_t nb = (nlists + SCAN_BLOCK - 1) / SCAN_BLOCK;
  return (nb > 0) + 1 + (nb > 1);
}

}  // namespace annb200
