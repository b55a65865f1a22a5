// scan_simt.cu - CUDA-core approximate scan (all formats, any dims, any batch).
//
// The reference's CUDA-core gather kernels score one row per warp with
// lane-strided dimensions (gather_f32/gather_f16, ann/server/cuvs.c:3597-3623;
// score_nvfp4, ann/server/blackwell.c:106-129). Here a 256-thread block owns
// a 64-row x BN-query tile instead: rows are gathered by id once per tile,
// decoded to FP32 in shared memory (FP16 exactly; FP8 and NVFP4 with the
// same FP32 multiplies as the exact rescoring), and reused by every query of
// the tile, so HBM reads a gathered row once per BN queries.
#include "internal.cuh"

namespace annb200 {

namespace {

constexpr int BM = 64;
constexpr int BK = 32;

__device__ __forceinline__ void emit(const ScanArgs &a, float v, uint64_t vi, uint64_t pos, uint32_t q) {
  if (a.mode == MODE_MATRIX) a.mat[(uint64_t)q * a.mat_ld + vi] = v;
  else if (v <= __ldg(a.thr + q)) append_candidate(a, v, pos, q);
}

template <int DT, int BN>
__global__ void __launch_bounds__(256) simt_scan(const ScanArgs a) {
  constexpr int TN = BN / 16;
  __shared__ __align__(16) float xs[BK][BM + 4];
  __shared__ float qs[BK][BN + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const uint64_t vbase = (uint64_t)blockIdx.x * BM;
  const uint32_t qbase = blockIdx.y * BN;

  const int lr = tid / 4, lc = (tid % 4) * 8;
  const uint64_t lvi = vbase + lr;
  const bool lvalid = lvi < a.count;
  const uint64_t lpos = a.base + lvi * a.stride;
  const uint64_t lid = lvalid ? cand_row(a.ids, lpos, a.s.rows) : 0;
  const uint32_t dims = a.s.dims;

  float acc[4][TN];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;

  for (uint32_t k0 = 0; k0 < dims; k0 += BK) {
    float v[8];
    if (lvalid) decode8<DT>(a.s, lid, k0 + lc, v);
    else {
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) xs[lc + j][lr] = v[j];
    // queries: BN x BK values, BN*BK/256 a thread
    constexpr int QPER = BN * BK / 256;
#pragma unroll
    for (int j = 0; j < QPER; j++) {
      int e = tid * QPER + j;
      int qi = e / BK, kk = e % BK;
      uint32_t q = qbase + qi, d = k0 + kk;
      qs[kk][qi] = (q < a.nq && d < dims) ? __ldg(a.queries + (uint64_t)q * dims + d) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < BK; kk++) {
      float4 x = *reinterpret_cast<const float4 *>(&xs[kk][ty * 4]);
      float b[TN];
#pragma unroll
      for (int j = 0; j < TN; j++) b[j] = qs[kk][tx * TN + j];
#pragma unroll
      for (int j = 0; j < TN; j++) {
        acc[0][j] = fmaf(x.x, b[j], acc[0][j]);
        acc[1][j] = fmaf(x.y, b[j], acc[1][j]);
        acc[2][j] = fmaf(x.z, b[j], acc[2][j]);
        acc[3][j] = fmaf(x.w, b[j], acc[3][j]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint64_t vi = vbase + ty * 4 + i;
    if (vi >= a.count) continue;
    uint64_t pos = a.base + vi * a.stride;
    uint64_t id = cand_row(a.ids, pos, a.s.rows);
    float al, be;
    row_affine(a.s, id, a.metric, 0, al, be);
#pragma unroll
    for (int j = 0; j < TN; j++) {
      uint32_t q = qbase + tx * TN + j;
      if (q < a.nq) emit(a, fmaf(acc[i][j], al, be), vi, pos, q);
    }
  }
}

// Hamming: rows and queries are packed bits; K runs over 32-bit words and the
// score is the exact popcount of XOR.
template <int BN>
__global__ void __launch_bounds__(256) simt_hamming(const ScanArgs a) {
  constexpr int TN = BN / 16;
  __shared__ __align__(16) uint32_t xs[BK][BM + 4];
  __shared__ uint32_t qs[BK][BN + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const uint64_t vbase = (uint64_t)blockIdx.x * BM;
  const uint32_t qbase = blockIdx.y * BN;
  const uint64_t rb = a.s.row_bytes;
  const uint32_t words = (uint32_t)((rb + 3) / 4);

  const int lr = tid / 4, lc = (tid % 4) * 8;
  const uint64_t lvi = vbase + lr;
  const bool lvalid = lvi < a.count;
  const uint64_t lpos = a.base + lvi * a.stride;
  const uint64_t lid = lvalid ? cand_row(a.ids, lpos, a.s.rows) : 0;
  const uint8_t *lrow = a.s.codes + lid * rb;
  const uint8_t *qbytes = reinterpret_cast<const uint8_t *>(a.queries);

  uint32_t acc[4][TN];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0;

  for (uint32_t k0 = 0; k0 < words; k0 += BK) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      uint32_t w = k0 + lc + j, val = 0;
      if (lvalid && w < words) {
        uint64_t b0 = (uint64_t)w * 4;
        if ((rb & 3) == 0) val = __ldg(reinterpret_cast<const uint32_t *>(lrow + b0));
        else
          for (int t = 0; t < 4; t++)
            if (b0 + t < rb) val |= (uint32_t)__ldg(lrow + b0 + t) << (8 * t);
      }
      xs[lc + j][lr] = val;
    }
    constexpr int QPER = BN * BK / 256;
#pragma unroll
    for (int j = 0; j < QPER; j++) {
      int e = tid * QPER + j;
      int qi = e / BK, kk = e % BK;
      uint32_t q = qbase + qi, w = k0 + kk, val = 0;
      if (q < a.nq && w < words) {
        const uint8_t *qr = qbytes + (uint64_t)q * rb;
        uint64_t b0 = (uint64_t)w * 4;
        if ((rb & 3) == 0) val = __ldg(reinterpret_cast<const uint32_t *>(qr + b0));
        else
          for (int t = 0; t < 4; t++)
            if (b0 + t < rb) val |= (uint32_t)__ldg(qr + b0 + t) << (8 * t);
      }
      qs[kk][qi] = val;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < BK; kk++) {
      uint4 x = *reinterpret_cast<const uint4 *>(&xs[kk][ty * 4]);
#pragma unroll
      for (int j = 0; j < TN; j++) {
        uint32_t b = qs[kk][tx * TN + j];
        acc[0][j] += __popc(x.x ^ b);
        acc[1][j] += __popc(x.y ^ b);
        acc[2][j] += __popc(x.z ^ b);
        acc[3][j] += __popc(x.w ^ b);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint64_t vi = vbase + ty * 4 + i;
    if (vi >= a.count) continue;
    uint64_t pos = a.base + vi * a.stride;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      uint32_t q = qbase + tx * TN + j;
      if (q < a.nq) emit(a, (float)acc[i][j], vi, pos, q);
    }
  }
}

template <int BN>
void launch_bn(const ScanArgs &a, cudaStream_t st) {
  dim3 grid((unsigned)((a.count + BM - 1) / BM), (a.nq + BN - 1) / BN);
  switch (a.s.dtype) {
    case DT_F32: simt_scan<DT_F32, BN><<<grid, 256, 0, st>>>(a); break;
    case DT_F16: simt_scan<DT_F16, BN><<<grid, 256, 0, st>>>(a); break;
    case DT_E4M3: simt_scan<DT_E4M3, BN><<<grid, 256, 0, st>>>(a); break;
    case DT_NVFP4: simt_scan<DT_NVFP4, BN><<<grid, 256, 0, st>>>(a); break;
    case DT_BIT: simt_hamming<BN><<<grid, 256, 0, st>>>(a); break;
  }
}

}  // namespace

// Scan a.count virtual rows against a.nq queries on CUDA cores.
void launch_simt_scan(const ScanArgs &a, cudaStream_t st) {
  if (a.count == 0 || a.nq == 0) return;
  if (a.nq > 16) launch_bn<64>(a, st);
  else launch_bn<16>(a, st);
}

}  // namespace annb200
