// scan_tc.cu - tcgen05 tensor-core approximate scan of FP16 rows.
//
// Replaces the reference's grouped score-matrix scan, which stages up to 64
// queries in shared memory and issues legacy warp-level mma.sync.m16n8k16
// per 8-query tile (score_mma_half, ann/server/blackwell.c:289-525). Here one
// persistent CTA per SM walks (128-row, BN-query) tiles, BN <= 256:
//
//   warp 0     TMA producer: per 64-dimension k-block (one pipeline stage of
//              4), one thread issues two tiled cp.async.bulk.tensor loads --
//              the 128 x 64 block of candidate rows and the BN x 64 block of
//              FP16 queries -- which land in the 128-byte-swizzled K-major
//              layout tcgen05 reads and complete on the stage's mbarrier.
//              Contiguous candidate rows (a whole shard, a staged copy) come
//              this way.
//   warps 6-9  (FP16 row lists and strided samples) gather: 16-byte
//              cp.async copies of the named rows straight from the shard into
//              the swizzled A tiles (8 lanes a row), completing on the stage
//              barrier through cp.async.mbarrier.arrive.noinc, with the next
//              tile's rows prefetched into L2; A and B then have separate
//              rings (6 x 16 KB of rows, 3 x 32 KB of queries). TMA's per-row
//              tile::gather4 was measured request-rate bound at about 13 GB/s
//              an SM; these copies sustain ~920 TFLOP/s of scan.
//   warps 6-9  (E4M3 / NVFP4 rows) converters: the raw codes arrive by TMA
//              in a ring of their own and are converted to FP16 A tiles.
//   warp 1     one thread issues tcgen05.mma.cta_group::1.kind::f16
//              (M=128, N=BN, K=16) into an FP32 accumulator in tensor memory,
//              and tcgen05.commit frees each stage and publishes each tile.
//   warps 2-5  epilogue: tcgen05.ld moves each row's BN scores to registers
//              (warp w reads TMEM lanes 32*(w%4)..+31), applies the per-row
//              affine map to the v-domain score and either stores it (sample
//              matrix) or appends (v, row) when v passes the query's
//              threshold: the 32 compares of a column chunk form a bitmask
//              first, and only a chunk with a passing score in the warp takes
//              the staging path. Two accumulators (2 x 256 columns) let the
//              epilogue of tile t overlap the MMAs of tile t+1.
//
// Every wait is bounded (4 s of %globaltimer; the pipeline waits of the flat
// scan by ANN_B200_PIPELINE_WAIT_NS when a test sets it); a wait that runs
// out sets FLAG_TIMEOUT, all roles leave their loops, in-flight MMAs are
// drained, bulk copies still in flight are waited for and tensor memory is
// freed before the kernel returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdlib>

#include "internal.cuh"

namespace annb200 {

namespace {

constexpr int BM = 128;
constexpr int MAXBN = 256;
constexpr int A_BYTES = BM * 128;
constexpr int B_BYTES = MAXBN * 128;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_BUF = 256;      // staged appends a warp buffers before a flush
constexpr int TMEM_COLS = 512;
constexpr unsigned long long kWaitNs = 4000000000ull;
// E4M3 rows on FP8 tensor cores (see TcCfg<QF8>)
constexpr int QF8 = 0x20 | DT_E4M3;

struct TcArgs {
  ScanArgs a;
  int64_t a_row0;      // row of the A tensor map holding virtual row 0
  uint32_t kpad;       // elements per query row: halves (multiple of 64) or, bit vectors, int8 (of 128)
  uint32_t kblocks;    // 128-byte k-blocks a row: kpad / 64, or kpad / 128 for bit vectors
  uint32_t bn;         // queries per tile, multiple of 32, <= 256
  uint32_t qtiles;
  uint64_t rtiles;
  uint64_t wait_ns;    // limit of each pipeline wait (the drains keep kWaitNs)
  int32_t q_lo_row;    // FP8 scan: row of the query map holding the low terms' first query
  uint32_t pf_tiles;   // gathered FP16 rows: L2 prefetch this many of the CTA's tiles ahead
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of `parity` to complete; false once `limit_ns` passes
// or another role has aborted.
__device__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort, uint32_t *flags,
                          uint64_t limit_ns = kWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    for (int i = 0; i < 32; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort = 1;
      atomicOr(flags, FLAG_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// A (box rows) x 64 tile at (x, y) of a 2-D tensor into dst; completes on bar.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// E4M3 A and B (the instruction descriptor's format fields are 0 for E4M3,
// as for FP16 under kind::f16), FP32 accumulator, K = 32.
__device__ __forceinline__ void tc_mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Signed 8-bit A and B, 32-bit integer accumulator (the +-1 expansion of bit vectors).
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle layout: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked
// along M/N (stride byte offset 1024), start address advanced 32 bytes per
// 16-element K step inside the atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3fffu)   // start address
         | ((uint64_t)1 << 16)                 // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)       // stride byte offset
         | ((uint64_t)1 << 46)                 // descriptor version (sm100)
         | ((uint64_t)2 << 61);                // 128-byte swizzle
}

// Instruction descriptor: FP16 A and B, FP32 accumulator, both K-major.
__device__ __forceinline__ uint32_t f16_idesc(uint32_t n) {
  return (1u << 4)                  // D format F32
         | ((n >> 3) << 17)         // N / 8
         | ((uint32_t)(BM >> 4) << 24);  // M / 16
}
// BF16 A and B (both the same type), FP32 accumulator, both K-major: the
// split FP32 scan.
__device__ __forceinline__ uint32_t bf16_idesc(uint32_t n) {
  return (1u << 4)                  // D format F32
         | (1u << 7) | (1u << 10)   // A, B BF16
         | ((n >> 3) << 17)         // N / 8
         | ((uint32_t)(BM >> 4) << 24);  // M / 16
}
// kind::i8: signed 8-bit A and B (both the same type), S32 accumulator, both K-major.
__device__ __forceinline__ uint32_t i8_idesc(uint32_t n) {
  return (2u << 4)                  // D format S32
         | (1u << 7) | (1u << 10)   // A, B signed 8-bit
         | ((n >> 3) << 17)         // N / 8
         | ((uint32_t)(BM >> 4) << 24);  // M / 16
}

#define TMEM_LD32(taddr, r)                                                                          \
  asm volatile(                                                                                      \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15," \
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                     \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),        \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),    \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), \
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), \
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                                         \
      : "r"(taddr))

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Passing (query, v, position) triples staged in a warp's shared buffer
// (warp-uniform slot arithmetic, no atomics) and flushed to the global
// candidate lists with every lane's atomics issued back to back, so a flush
// costs one memory round trip rather than one per passing score.
struct Appender {
  const ScanArgs &a;
  uint4 *buf;
  uint32_t n;
  int lane;
  __device__ void flush() {
    __syncwarp();
    uint32_t slot[EPI_BUF / 32];
#pragma unroll
    for (int u = 0; u < EPI_BUF / 32; u++) {
      const uint32_t i = u * 32 + lane;
      if (i < n) slot[u] = atomicAdd(a.cnt + buf[i].x, 1u);
    }
#pragma unroll
    for (int u = 0; u < EPI_BUF / 32; u++) {
      const uint32_t i = u * 32 + lane;
      if (i < n) {
        const uint4 e = buf[i];
        if (slot[u] < a.cap) a.cand[(uint64_t)e.x * a.cap + slot[u]] = make_uint2(e.y, e.z);
        else {
          atomicOr(a.flags, FLAG_OVERFLOW);
          atomicMax(a.flags + 1, slot[u] + 1);
        }
      }
    }
    __syncwarp();
    n = 0;
  }
};

// Score of an accumulator word: the FP32 dot product, or for bit vectors
// (nbits bits a row, +-1 expansion, S32 dot product d) the Hamming distance
// (nbits - d) / 2, exact in FP32.
template <int Q>
__device__ __forceinline__ float acc_score(uint32_t r, int32_t nbits) {
  if (Q == DT_BIT) return (float)(nbits - (int32_t)r) * 0.5f;
  return __uint_as_float(r);
}

// One warp's 32 accumulator rows (TMEM lanes at taddr; this lane's virtual
// row vi) against queries q_base .. q_base+bn-1: the score matrix, or the
// threshold filter -- the 32 compares of a column chunk form a bitmask first
// and only a chunk with a passing score in the warp takes the staging path.
template <int Q>
__device__ __forceinline__ void epilogue_rows(const ScanArgs &a, uint32_t taddr, uint64_t vi, uint32_t q_base,
                                              uint32_t bn, const float *thr_s, const float *qsc_s, Appender &app) {
  const int32_t nbits = (int32_t)(a.s.row_bytes * 8);
  const bool valid = vi < a.count;
  const uint64_t pos = a.base + vi * a.stride;
  float al = 0.0f, be = __int_as_float(0x7fc00000);  // invalid rows score NaN: never pass
  if (valid) {
    const uint64_t id = cand_row(a.ids, pos, a.s.rows);
    row_affine(a.s, id, a.metric, a.raw_scale, al, be);
  }
  for (uint32_t c0 = 0; c0 < bn; c0 += 32) {
    uint32_t r[32];
    TMEM_LD32(taddr + c0, r);
    tmem_ld_wait();
    const uint32_t q0 = q_base + c0;
    if (Q == QF8) {   // the FP8 scan's sums are in units of each query's term scale (a power of two)
#pragma unroll
      for (int j = 0; j < 32; j++) r[j] = __float_as_uint(__uint_as_float(r[j]) * qsc_s[q0 + j]);
    }
    if (a.mode == MODE_MATRIX) {
      if (valid) {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (q0 + j < a.nq) a.mat[(uint64_t)(q0 + j) * a.mat_ld + vi] = fmaf(acc_score<Q>(r[j], nbits), al, be);
      }
    } else {
      const float4 *tq = reinterpret_cast<const float4 *>(thr_s + q0);
      uint32_t m = 0;
#pragma unroll
      for (int j4 = 0; j4 < 8; j4++) {
        const float4 t4 = tq[j4];
        const float th[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
        for (int jj = 0; jj < 4; jj++)
          m |= (uint32_t)(fmaf(acc_score<Q>(r[j4 * 4 + jj], nbits), al, be) <= th[jj]) << (j4 * 4 + jj);
      }
      // rare path: each round every lane stages its lowest passing column
      while (__any_sync(0xffffffffu, m != 0)) {
        const bool has = m != 0;
        const int j = has ? __ffs(m) - 1 : 0;
        m &= m - 1;
        float v = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 32; jj++) v = (jj == j) ? acc_score<Q>(r[jj], nbits) : v;
        v = fmaf(v, al, be);
        const uint32_t ballot = __ballot_sync(0xffffffffu, has);
        if (app.n + 32 > (uint32_t)EPI_BUF) app.flush();
        if (has)
          app.buf[app.n + __popc(ballot & ((1u << app.lane) - 1u))] =
              make_uint4(q0 + j, __float_as_uint(v), (uint32_t)pos, 0u);
        app.n += __popc(ballot);
      }
    }
  }
}

// Per storage format: pipeline stages, raw-code ring (quantized formats stage
// their codes and convert them to FP16 -- bit vectors to int8 -- in shared
// memory), threads. Quantized formats run CONV_WARPS converter warps: with 4,
// a k-block's conversion (about 770 cycles) nearly matched its MMAs (about
// 850 at the sustained rate) and the MMAs waited on it 30% of the time.
constexpr int CONV_WARPS = 8;
constexpr int CONV_THREADS = 32 * CONV_WARPS;
// STG stages hold an A tile and a B tile each; the gathered-FP16 kernel
// instead keeps STG A tiles and BSTG B tiles in separate rings.
template <int Q> struct TcCfg;
template <> struct TcCfg<DT_F16> {
  static constexpr int STG = 4, BSTG = 4, RSTG = 0, RAWB = 0, RAW_X = 0, NT = 192;
  static constexpr int RING = STG * STAGE_BYTES;
};
template <> struct TcCfg<DT_E4M3> {   // 64 one-byte codes a row a k-block
  static constexpr int STG = 3, BSTG = 3, RSTG = 4, RAWB = BM * 64, RAW_X = 64, NT = 192 + 32 * CONV_WARPS;
  static constexpr int RING = STG * STAGE_BYTES;
};
template <> struct TcCfg<DT_NVFP4> {  // 64 nibbles (32 bytes) a row a k-block
  static constexpr int STG = 3, BSTG = 3, RSTG = 4, RAWB = BM * 32, RAW_X = 32, NT = 192 + 32 * CONV_WARPS;
  static constexpr int RING = STG * STAGE_BYTES;
};
template <> struct TcCfg<DT_BIT> {    // 128 bits (16 bytes) a row a k-block -> 128 int8
  static constexpr int STG = 3, BSTG = 3, RSTG = 4, RAWB = BM * 16, RAW_X = 16, NT = 192 + 32 * CONV_WARPS;
  static constexpr int RING = STG * STAGE_BYTES;
};
// FP32 rows: 64 floats (256 bytes) a row a k-block, split into two BF16
// tiles (hi = RN(x), lo = RN(x - hi)) against the query's two BF16 halves;
// a stage holds A hi, A lo, B hi, B lo with at most 128 queries a tile.
constexpr int F32_BN = 128;
constexpr int F32_STAGE = 2 * A_BYTES + 2 * F32_BN * 128;
template <> struct TcCfg<DT_F32> {
  static constexpr int STG = 2, BSTG = 2, RSTG = 2, RAWB = BM * 256, RAW_X = 64, NT = 192 + 32 * CONV_WARPS;
  static constexpr int RING = STG * F32_STAGE;
};
// E4M3 rows on FP8 tensor cores: TMA brings 128 codes of each of 128 rows a
// k-block in the 128-byte swizzle straight to the A tile, and kind::f8f6f4
// MMAs (K = 32) run them against the queries as two E4M3 terms -- hi and lo
// with one power-of-two scale a query, s * (hi + lo) within about 2^-8 of
// each query element -- both into one accumulator. No conversion: a stage
// holds the A tile and the two query terms' tiles (at most 256 queries).
constexpr int F8_BN = 256;
constexpr int F8_STAGE = A_BYTES + 2 * F8_BN * 128;
template <> struct TcCfg<QF8> {
  static constexpr int STG = 2, BSTG = 2, RSTG = 0, RAWB = 0, RAW_X = 0, NT = 192;
  static constexpr int RING = STG * F8_STAGE;
};
// FP16 rows named by a candidate list (or a strided sample): 4 gather warps
// copy them from the shard into the A tiles, TMA loads only the queries.
// Gathered rows come from random HBM locations and take far longer to land
// than the L2-resident query block, so the A ring is twice as deep (6 x 16 KB)
// as the B ring (3 x 32 KB).
constexpr int GF16 = 0x10 | DT_F16;
template <> struct TcCfg<GF16> {
  static constexpr int STG = 6, BSTG = 3, RSTG = 0, RAWB = 0, RAW_X = 0, NT = 320;
  static constexpr int RING = STG * A_BYTES + BSTG * B_BYTES;
};

// 16 bytes global -> shared, bypassing L1; n = 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t n) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

// Four E4M3 codes -> two FP16 pairs (exact: every E4M3 value is an FP16 value).
__device__ __forceinline__ void e4m3x4_to_f16(uint32_t w, uint32_t &o0, uint32_t &o1) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(o0), "=r"(o1)
      : "r"(w));
}
// Eight E2M1 codes (low nibble first) -> four FP16 pairs, each times the
// FP16 pair s: an E2M1 value (2 significant bits) times an E4M3 block scale
// (4 bits) is exact in FP16, whose range holds 2^-10 .. 2688.
__device__ __forceinline__ void e2m1x8_to_f16(uint32_t w, uint32_t s, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t.reg .b32 h0, h1, h2, h3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 h0, b0;\n\tcvt.rn.f16x2.e2m1x2 h1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 h2, b2;\n\tcvt.rn.f16x2.e2m1x2 h3, b3;\n\t"
      "mul.rn.f16x2 %0, h0, %5;\n\tmul.rn.f16x2 %1, h1, %5;\n\t"
      "mul.rn.f16x2 %2, h2, %5;\n\tmul.rn.f16x2 %3, h3, %5;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w), "r"(s));
}

// Byte offset of 16-byte chunk c (0..7) of row r in a 128-row x 128-byte
// K-major tile with the 128-byte swizzle (the layout TMA writes and the
// tcgen05 descriptor reads): chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Convert one stage's raw codes (BM rows of RAW_X bytes, dense) into the
// FP16 A tile (raw values: the row scale is applied in the epilogue). 128
// converter threads (CONV_THREADS); ct = converter thread, vrow0 = virtual row of tile row 0.
template <int Q>
__device__ __forceinline__ void convert_stage(const ScanArgs &a, const uint8_t *raw, uint8_t *atile, uint32_t ct,
                                              uint64_t vrow0, uint32_t kb) {
  if (Q == DT_E4M3) {
#pragma unroll
    for (int u = 0; u < 512 / CONV_THREADS; u++) {
      const uint32_t i = ct + CONV_THREADS * u, r = i >> 2, c = i & 3;  // 16 codes: dims 16c .. 16c+15
      const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 64 + c * 16);
      uint4 lo, hi;
      e4m3x4_to_f16(w.x, lo.x, lo.y);
      e4m3x4_to_f16(w.y, lo.z, lo.w);
      e4m3x4_to_f16(w.z, hi.x, hi.y);
      e4m3x4_to_f16(w.w, hi.z, hi.w);
      *reinterpret_cast<uint4 *>(atile + sw128_offset(r, 2 * c)) = lo;
      *reinterpret_cast<uint4 *>(atile + sw128_offset(r, 2 * c + 1)) = hi;
    }
  } else if (Q == DT_NVFP4) {
#pragma unroll
    for (int u = 0; u < 256 / CONV_THREADS; u++) {
      const uint32_t i = ct + CONV_THREADS * u, r = i >> 1, h = i & 1;  // 32 nibbles: dims 32h .. 32h+31
      const uint4 w = *reinterpret_cast<const uint4 *>(raw + r * 32 + h * 16);
      const uint64_t vi = vrow0 + r;
      uint32_t sc[2] = {0u, 0u};
      if (vi < a.count) {
        const uint64_t id = cand_row(a.ids, a.base + vi * a.stride, a.s.rows);
        const uint32_t b0 = kb * 4 + h * 2;
#pragma unroll
        for (int j = 0; j < 2; j++) {
          if (b0 + j < a.s.bblocks) {
            const uint32_t code = __ldg(a.s.bscales + id * a.s.bblocks + b0 + j);
            uint32_t pair, unused;
            e4m3x4_to_f16(code | (code << 8), pair, unused);
            sc[j] = pair;
          }
        }
      }
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint32_t o[4];
        e2m1x8_to_f16(ws[j], sc[j >> 1], o);
        *reinterpret_cast<uint4 *>(atile + sw128_offset(r, 4 * h + j)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  } else if (Q == DT_F32) {
    // 64 floats a row -> a BF16 tile of hi = RN(x) and, A_BYTES further, one
    // of lo = RN(x - hi) (x - hi is exact in FP32). Unit i: 8 floats of row
    // r (16-byte chunk c of both tiles).
#pragma unroll
    for (int u = 0; u < 1024 / CONV_THREADS; u++) {
      const uint32_t i = ct + CONV_THREADS * u, r = i >> 3, c = i & 7;
      const float4 p0 = *reinterpret_cast<const float4 *>(raw + r * 256 + c * 32);
      const float4 p1 = *reinterpret_cast<const float4 *>(raw + r * 256 + c * 32 + 16);
      const float x[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(x[2 * j]), h1 = __float2bfloat16_rn(x[2 * j + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(x[2 * j] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(x[2 * j + 1] - __bfloat162float(h1));
        hw[j] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        lw[j] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
      }
      *reinterpret_cast<uint4 *>(atile + sw128_offset(r, c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4 *>(atile + A_BYTES + sw128_offset(r, c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  } else if (Q == DT_BIT) {
    // 128 bits a row -> 128 int8: bit b of the k-block's 16 bytes (byte b/8,
    // bit b%8 from the least significant) is element b, +1 if clear, -1 if
    // set. A nibble times 0x00204081 puts its bit i at bit 8i (the other
    // products land at positions that are not multiples of 8, with no
    // carries), so each nibble becomes four bytes of 0 / 1, then of 1 / -1.
#pragma unroll
    for (int u = 0; u < 512 / CONV_THREADS; u++) {
      const uint32_t i = ct + CONV_THREADS * u, r = i >> 2, w = i & 3;  // bits 32w .. 32w+31
      const uint32_t x = *reinterpret_cast<const uint32_t *>(raw + r * 16 + w * 4);
      uint32_t o[8];
#pragma unroll
      for (int n = 0; n < 8; n++) {
        const uint32_t m = (((x >> (4 * n)) & 0xfu) * 0x00204081u) & 0x01010101u;
        o[n] = (m * 0xffu) | 0x01010101u;
      }
      *reinterpret_cast<uint4 *>(atile + sw128_offset(r, 2 * w)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4 *>(atile + sw128_offset(r, 2 * w + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// Wait (bounded) for the last load issued into each of n ring slots: no
// bulk copy may still be writing this CTA's shared memory when it exits.
__device__ void drain_ring(uint64_t *bars, int n, uint64_t issued) {
  for (int s = 0; s < n; s++) {
    if ((uint64_t)s >= issued) break;
    const uint64_t last = issued - 1 - ((issued - 1 - s) % n);  // last iteration that used slot s
    const uint32_t ph = (uint32_t)((last / n) & 1);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bars + s, ph) && globaltimer() - t0 < kWaitNs) {
    }
  }
}

template <int Q>
__global__ void __launch_bounds__(TcCfg<Q>::NT, 1)
    tc_scan(const __grid_constant__ CUtensorMap rows_map, const __grid_constant__ CUtensorMap query_map,
            const __grid_constant__ CUtensorMap query_lo_map, const TcArgs t) {
  using C = TcCfg<Q>;
  constexpr int STG = C::STG, BSTG = C::BSTG, RSTG = C::RSTG, RAWB = C::RAWB;
  constexpr int RSTG1 = RSTG > 0 ? RSTG : 1;  // (the FP16 kernels have no raw ring)
  constexpr bool SPLIT = Q == DT_F32;         // two BF16 halves of rows and queries, three MMAs a K step
  constexpr bool QUANT = Q == DT_E4M3 || Q == DT_NVFP4 || Q == DT_BIT || SPLIT;
  constexpr bool F8 = Q == QF8;
  constexpr int STAGE = SPLIT ? F32_STAGE : (F8 ? F8_STAGE : STAGE_BYTES);
  constexpr bool GATHER = Q == GF16;
  constexpr int32_t QX = (Q == DT_BIT || F8) ? 128 : 64;   // query elements a k-block (128 bytes)
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // A and B tiles of stage s (separate rings for the gathered kernel)
  // (split FP32: A hi, A lo, B hi, B lo; the lo tiles follow their hi tiles)
  auto a_tile = [&](uint32_t s) { return smem + (GATHER ? s * A_BYTES : s * STAGE); };
  auto b_tile = [&](uint32_t s) {
    return GATHER ? smem + STG * A_BYTES + s * B_BYTES : smem + s * STAGE + (SPLIT ? 2 : 1) * A_BYTES;
  };
  uint8_t *raw = smem + C::RING;
  uint64_t *full = reinterpret_cast<uint64_t *>(raw + RSTG * RAWB);  // A (and B for FP16) ready
  uint64_t *empty = full + STG;                                      // A stage consumed by the MMAs
  uint64_t *bfull = empty + STG;                                     // B ready (quantized, gathered)
  uint64_t *bempty = bfull + STG;                                    // B stage consumed (gathered)
  uint64_t *rawfull = bempty + STG;
  uint64_t *rawempty = rawfull + RSTG;
  uint64_t *tfull = rawempty + RSTG;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile uint32_t *abort = tmem_slot + 1;
  uint4 *stage_buf = reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(full) + 256);  // 4 warps x EPI_BUF
  float *thr_s = reinterpret_cast<float *>(stage_buf + 4 * EPI_BUF);
  float *qsc_s = thr_s + (t.a.nq + 255) / 256 * 256;          // FP8 scan: per-query term scales

  const ScanArgs &a = t.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t ntiles = t.rtiles * t.qtiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; s++) {
      mbar_init(full + s, QUANT ? CONV_WARPS : (GATHER ? 128 : 1));
      mbar_init(empty + s, 1);
      mbar_init(bfull + s, 1);
      mbar_init(bempty + s, 1);
    }
    for (int r = 0; r < RSTG; r++) {
      mbar_init(rawfull + r, 1);
      mbar_init(rawempty + r, CONV_WARPS);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // query slots past nq (padding of the last query tile) get NaN: never pass
  if (a.mode == MODE_FILTER)
    for (uint32_t i = threadIdx.x; i < (a.nq + 255) / 256 * 256; i += C::NT)
      thr_s[i] = i < a.nq ? a.thr[i] : __int_as_float(0x7fc00000);
  if (F8)
    for (uint32_t i = threadIdx.x; i < (a.nq + 255) / 256 * 256; i += C::NT) qsc_s[i] = i < a.nq ? a.qscale[i] : 0.0f;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // FP16: rows and queries into the stage (gathered FP16: the queries
    // only). Quantized: raw codes into the raw ring (the converters load the
    // queries).
    if (lane == 0) {
      constexpr int RING = QUANT ? RSTG1 : (GATHER ? BSTG : STG);
      uint64_t *ring_full = QUANT ? rawfull : (GATHER ? bfull : full);
      uint64_t *ring_empty = QUANT ? rawempty : (GATHER ? bempty : empty);
      const uint32_t tx_bytes =
          QUANT ? (uint32_t)RAWB : (GATHER ? 0u : (uint32_t)A_BYTES) + (F8 ? 2u : 1u) * t.bn * 128u;
      uint64_t it = 0;
      bool ok = true;
      for (uint64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const uint64_t rt = tile / t.qtiles;
        const uint32_t qt = (uint32_t)(tile % t.qtiles);
        const int32_t arow = (int32_t)(t.a_row0 + (int64_t)rt * BM);
        for (uint32_t kb = 0; kb < t.kblocks; kb++) {
          const uint32_t s = (uint32_t)(it % RING);
          const uint32_t ph = (uint32_t)((it / RING) & 1);
          if (!mbar_wait(ring_empty + s, ph ^ 1, abort, a.flags, t.wait_ns)) {
            ok = false;
            break;
          }
          mbar_expect_tx(ring_full + s, tx_bytes);
          if (QUANT) {
            tma_load_2d(smem_u32(raw + s * RAWB), &rows_map, (int32_t)(kb * C::RAW_X), arow, ring_full + s);
          } else {
            if (!GATHER)
              tma_load_2d(smem_u32(a_tile(s)), &rows_map, (int32_t)(kb * (F8 ? 128 : 64)), arow, ring_full + s);
            tma_load_2d(smem_u32(b_tile(s)), &query_map, (int32_t)(kb * QX), (int32_t)(qt * t.bn), ring_full + s);
            if (F8)   // the low terms, F8_BN rows of the stage further
              tma_load_2d(smem_u32(b_tile(s) + F8_BN * 128), &query_map, (int32_t)(kb * QX),
                          t.q_lo_row + (int32_t)(qt * t.bn), ring_full + s);
          }
          it++;
        }
      }
      drain_ring(ring_full, RING, it);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = Q == DT_BIT ? i8_idesc(t.bn) : (SPLIT ? bf16_idesc(t.bn) : f16_idesc(t.bn));
      uint64_t it = 0, tc = 0;
      bool ok = true;
      for (uint64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, tc++) {
        const uint32_t ab = (uint32_t)(tc & 1), use = (uint32_t)(tc >> 1);
        if (!mbar_wait(tempty + ab, (use & 1) ^ 1, abort, a.flags, t.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * 256;
        for (uint32_t kb = 0; kb < t.kblocks; kb++, it++) {
          const uint32_t s = (uint32_t)(it % STG);
          const uint32_t ph = (uint32_t)((it / STG) & 1);
          // the B tile: same stage index, or its own ring (gathered kernel)
          const uint32_t s_b = GATHER ? (uint32_t)(it % BSTG) : s;
          const uint32_t ph_b = GATHER ? (uint32_t)((it / BSTG) & 1) : ph;
          if (!mbar_wait(full + s, ph, abort, a.flags, t.wait_ns) ||
              ((QUANT || GATHER) && !mbar_wait(bfull + s_b, ph_b, abort, a.flags, t.wait_ns))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(a_tile(s));
          const uint32_t sb = smem_u32(b_tile(s_b));
#pragma unroll
          for (uint32_t kk = 0; kk < 4; kk++) {   // K = 16 halves or 32 int8: 32 bytes an MMA
            if (Q == DT_BIT) {
              tc_mma_i8(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
            } else if (F8) {   // 32 codes an MMA: x . hi, then x . lo into the same sums
              tc_mma_f8(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
              tc_mma_f8(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + F8_BN * 128 + kk * 32), idesc, 1u);
            } else if (SPLIT) {   // hi.hi + hi.lo + lo.hi (lo.lo is left to the error bound)
              const uint32_t sal = sa + A_BYTES, sbl = sb + F32_BN * 128;
              tc_mma_f16(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
              tc_mma_f16(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sbl + kk * 32), idesc, 1u);
              tc_mma_f16(d_tmem, sw128_desc(sal + kk * 32), sw128_desc(sb + kk * 32), idesc, 1u);
            } else {
              tc_mma_f16(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
            }
          }
          tc_commit(empty + s);
          if (GATHER) tc_commit(bempty + s_b);
        }
        if (ok) tc_commit(tfull + ab);
      }
      // every MMA this thread issued has completed before tensor memory is freed
      tc_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitNs) {
      }
    }
    __syncwarp();
  } else if (QUANT && warp >= 6) {
    // ------------------------------------------------------------ converters
    // raw codes -> FP16 A tile; converter thread 0 also loads the stage's
    // query block (B) once the MMAs have released the stage.
    const uint32_t ct = threadIdx.x - 192;
    uint64_t it = 0, bissued = 0;
    bool ok = true;
    for (uint64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const uint64_t rt = tile / t.qtiles;
      const uint32_t qt = (uint32_t)(tile % t.qtiles);
      for (uint32_t kb = 0; kb < t.kblocks; kb++, it++) {
        const uint32_t s = (uint32_t)(it % STG), ph = (uint32_t)((it / STG) & 1);
        const uint32_t r = (uint32_t)(it % RSTG1), rph = (uint32_t)((it / RSTG1) & 1);
        bool got = mbar_wait(empty + s, ph ^ 1, abort, a.flags, t.wait_ns);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (ct == 0) {
          mbar_expect_tx(bfull + s, (SPLIT ? 2u : 1u) * t.bn * 128u);
          tma_load_2d(smem_u32(b_tile(s)), &query_map, (int32_t)(kb * QX), (int32_t)(qt * t.bn), bfull + s);
          if (SPLIT)
            tma_load_2d(smem_u32(b_tile(s) + F32_BN * 128), &query_lo_map, (int32_t)(kb * QX), (int32_t)(qt * t.bn),
                        bfull + s);
          bissued = it + 1;
        }
        got = mbar_wait(rawfull + r, rph, abort, a.flags, t.wait_ns);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        convert_stage<Q>(a, raw + r * RAWB, a_tile(s), ct, rt * BM, kb);
        // generic-proxy stores -> visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(rawempty + r);
          mbar_arrive(full + s);
        }
      }
    }
    if (ct == 0) drain_ring(bfull, STG, bissued);
    __syncwarp();
  } else if (GATHER && warp >= 6) {
    // ------------------------------------------------------------ row gather
    // The tile's candidate rows straight from the shard into the swizzled A
    // tile: 8 lanes a row (its 128 bytes of the k-block), 16 rows a pass,
    // 16-byte cp.async each; each thread's copies arrive on the stage barrier
    // when they land (cp.async.mbarrier.arrive.noinc). Rows past the
    // candidates are zero-filled. Each thread also asks L2 for one whole row
    // of this CTA's next tile (cp.async.bulk.prefetch.L2), so that tile's
    // copies are served from L2 instead of random HBM accesses.
    const uint32_t gt = threadIdx.x - 192;
    const uint32_t c = gt & 7, r0 = gt >> 3;
    const uint64_t rb = a.s.row_bytes;
    uint64_t it = 0;
    bool ok = true;
    for (uint64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const uint64_t rt = tile / t.qtiles;
      const uint8_t *src[8];
      bool val[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint64_t vi = rt * BM + r0 + 16 * j;
        val[j] = vi < a.count;
        const uint64_t id = val[j] ? cand_row(a.ids, a.base + vi * a.stride, a.s.rows) : 0;
        src[j] = a.s.codes + id * rb;
      }
      // the tile pf_tiles ahead (at this CTA's first tile, every tile up to it)
      for (uint32_t d = tile == blockIdx.x ? 1 : t.pf_tiles; d <= t.pf_tiles; d++) {
        const uint64_t next = tile + (uint64_t)d * gridDim.x;
        if (next >= ntiles) break;
        const uint64_t vn = (next / t.qtiles) * BM + gt;
        if (vn < a.count) {
          const uint8_t *row = a.s.codes + cand_row(a.ids, a.base + vn * a.stride, a.s.rows) * rb;
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row), "r"((uint32_t)rb) : "memory");
        }
      }
      for (uint32_t kb = 0; kb < t.kblocks; kb++, it++) {
        const uint32_t s = (uint32_t)(it % STG), ph = (uint32_t)((it / STG) & 1);
        const bool got = mbar_wait(empty + s, ph ^ 1, abort, a.flags, t.wait_ns);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t sa = smem_u32(a_tile(s));
        const uint64_t off = (uint64_t)kb * 128 + c * 16;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const uint32_t n = (val[j] && off < rb) ? 16u : 0u;
          cp_async16(sa + sw128_offset(r0 + 16 * j, c), n ? src[j] + off : src[j], n);
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(full + s)) : "memory");
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    Appender app{a, stage_buf + (warp - 2) * EPI_BUF, 0, lane};
    const int quad = warp & 3;
    uint64_t tc = 0;
    for (uint64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, tc++) {
      const uint64_t rt = tile / t.qtiles;
      const uint32_t qt = (uint32_t)(tile % t.qtiles);
      const uint32_t ab = (uint32_t)(tc & 1), use = (uint32_t)(tc >> 1);
      bool got = mbar_wait(tfull + ab, use & 1, abort, a.flags, t.wait_ns);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      epilogue_rows<Q>(a, tmem_base + ab * 256 + ((uint32_t)(quad * 32) << 16), rt * BM + quad * 32 + lane,
                       qt * t.bn, t.bn, thr_s, qsc_s, app);
      tc_fence_before();
      mbar_arrive(tempty + ab);
    }
    __syncwarp();
    if (a.mode == MODE_FILTER && app.n) app.flush();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------- IVF list scan on tensor cores
//
// The list gather of ivf.cu on tcgen05. A work item is a 256-row tile of a
// probed list x up to 64 of the queries that probe the list (ListPlan with
// bm = 256, bq = 64). Rows are the MMA's N operand and queries its M
// operand (M = 64, N = 256, K = 16): an IVF list has few queries (about 4 in
// config 4), and a tcgen05.mma costs some 70-80 cycles to issue whatever its
// shape, so 256 rows an instruction (about 100 cycles of math at M = 64)
// keep the tensor core ahead of HBM where 128 rows x 32 queries did not.
// The rows of a list are contiguous in the shard: FP16 rows come by TMA
// straight into the row (B) tile, E4M3 / NVFP4 codes 128 bytes of each row
// at a time (and NVFP4's block scales for those bytes) into a raw ring the
// converter warps turn into FP16. The group's queries are gathered from the
// FP16 query copy by cp.async into the query (A) tile; rows of the tile past
// the group are left as they are (their accumulator rows are never read).
// The accumulator is 64 x 256 FP32, double buffered (all 512 TMEM
// columns); query m of the group sits in TMEM lane (m % 16) + 32 (m / 16),
// so epilogue warp w reads queries 16 (w % 4) .. +15 in its lanes 0-15.
// Each CTA walks a contiguous run of items and decodes them incrementally,
// so list metadata, query numbers and thresholds are read once a list.
constexpr int LQ = 64;                       // queries an item (MMA M)
constexpr int LR = 256;                      // rows an item (MMA N)
constexpr int LA_BYTES = LQ * 128;           // query tile a k-block: 64 x 64 halves
constexpr int LB_BYTES = LR * 128;           // row tile a k-block: 256 x 64 halves
constexpr int L_CW = 8;                      // converter warps (6 .. 13)
constexpr int L_QW = 6 + L_CW;               // the query-gather warp
constexpr int L_NT = 32 * (L_QW + 1);
constexpr int L_TMEM = 512;                  // 2 accumulators x 256 columns
constexpr int L_BAR = 1024;                  // barrier region bytes

// BSTG row (B) stages of converted (or TMA-loaded FP16) rows; ASTG query (A)
// stages, gathered up to ASTG k-blocks ahead so their L2 latency stays
// hidden; RSTG raw segments of codes in flight from HBM (quantized formats).
// A raw segment is 128 bytes of each of the tile's 256 rows (two TMA boxes
// of 128 rows, 128-byte swizzle) and covers SEGK k-blocks; NVFP4 adds the 16
// block-scale bytes of those k-blocks (SCB). Whole 128-byte row pieces keep
// the TMA request count per byte low.
template <int Q> struct LCfg;
template <> struct LCfg<DT_F16> {
  static constexpr int BSTG = 4, ASTG = 6, RSTG = 0, RAWB = 0, SEGK = 1, SCB = 0;
};
template <> struct LCfg<DT_E4M3> {
  static constexpr int BSTG = 3, ASTG = 6, RSTG = 2, RAWB = LR * 128, SEGK = 2, SCB = 0;
};
template <> struct LCfg<DT_NVFP4> {
  static constexpr int BSTG = 3, ASTG = 6, RSTG = 2, RAWB = LR * 128, SEGK = 4, SCB = LR * 16;
};

// Accumulator rows of a group of g queries: the group fills nqq = ceil(g/16)
// TMEM lane quarters (query j in row j), and groups of up to 32 queries are
// repeated rep = 4 / nqq times (copy c of query j in row j + 16 nqq c), so
// that every epilogue warp has queries to score and each copy's warps share
// the item's 256 rows: the MMA's cost is the same for any M-row content.
__device__ __forceinline__ void group_layout(uint32_t g, uint32_t &nqq, uint32_t &rep) {
  nqq = (g + 15) / 16;
  rep = nqq == 1 ? 4u : (nqq == 2 ? 2u : 1u);
}

struct ListTcArgs {
  ScanArgs a;
  ListPlan p;
  uint64_t rbegin, rend;   // the window of each list's rows this launch scans
  const __half *q16;       // FP16 queries [.][kpad]
  uint32_t kpad, kblocks;
};

// Instruction descriptor: FP16 A and B, FP32 accumulator, both K-major, M x N.
__device__ __forceinline__ uint32_t f16_idesc_mn(uint32_t m, uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Walks this CTA's run of items in order: list l, item t within it (row tile
// t / groups, query group t % groups), with the list's window and queries.
// Lists come from the compact list of lists with items (p.nzl), and the next
// list's metadata is requested while the current list is worked on, so a
// list change costs no memory round trip.
struct ItemCursor {
  const ListPlan *p;
  uint64_t rbegin, rend;
  uint64_t item, end, ci, nci;
  uint32_t l, nql;
  uint64_t t, tiles, groups, lo, hi, qoff;
  // the next list (loads in flight)
  uint32_t nl;
  unsigned long long ntiles, nlcount, noff0, noff1, nqoff;
  __device__ void set_list(uint32_t list, unsigned long long tl, unsigned long long lc, unsigned long long o0,
                           unsigned long long o1, unsigned long long qo) {
    l = list;
    tiles = tl;
    nql = (uint32_t)lc;
    groups = (nql + LQ - 1) / LQ;
    uint64_t h = o1 < p->rows ? o1 : p->rows;   // list_range's clamping
    uint64_t b = o0 < h ? o0 : h;
    const uint64_t len = h - b;
    lo = b + (rbegin < len ? rbegin : len);
    hi = b + (rend < len ? rend : len);
    qoff = qo;
  }
  __device__ void fetch_next() {
    if (ci + 1 < nci) {
      nl = p->nzl[ci + 1];
      ntiles = p->tiles[nl];
      nlcount = p->lcount[nl];
      noff0 = p->offsets[nl];
      noff1 = p->offsets[nl + 1];
      nqoff = p->qoff[nl];
    }
  }
  __device__ void start(uint64_t first, uint64_t last) {
    item = first;
    end = last;
    nci = p->nzoff[p->nlists];
    if (item < end) {
      uint64_t a = 0, b = nci;   // toff[nzl[a]] <= item < toff[nzl[b]] (or b = nci)
      while (b - a > 1) {
        const uint64_t mid = (a + b) >> 1;
        if (p->toff[p->nzl[mid]] <= item) a = mid;
        else b = mid;
      }
      ci = a;
      const uint32_t list = p->nzl[ci];
      set_list(list, p->tiles[list], p->lcount[list], p->offsets[list], p->offsets[list + 1], p->qoff[list]);
      t = item - p->toff[list];
      fetch_next();
    }
  }
  __device__ bool valid() const { return item < end; }
  __device__ void next() {
    ++item;
    if (item >= end) return;
    if (++t >= tiles) {
      t = 0;
      ++ci;
      set_list(nl, ntiles, nlcount, noff0, noff1, nqoff);
      fetch_next();
    }
  }
  __device__ uint64_t row0() const { return lo + (t / groups) * LR; }
  __device__ uint32_t group() const { return (uint32_t)(t % groups); }
  __device__ uint32_t nq_item() const {
    const uint32_t g0 = group() * LQ;
    return nql - g0 < (uint32_t)LQ ? nql - g0 : (uint32_t)LQ;
  }
  __device__ uint64_t qbase() const { return qoff + (uint64_t)group() * LQ; }
  // The query group of the next item: false if this is the run's last item.
  __device__ bool peek_group(uint64_t &qb, uint32_t &nqt) const {
    if (item + 1 >= end) return false;
    if (t + 1 < tiles) {
      const uint32_t g = (uint32_t)((t + 1) % groups);
      qb = qoff + (uint64_t)g * LQ;
      nqt = nql - g * LQ < (uint32_t)LQ ? nql - g * LQ : (uint32_t)LQ;
    } else {
      qb = nqoff;
      nqt = nlcount < (unsigned long long)LQ ? (uint32_t)nlcount : (uint32_t)LQ;
    }
    return true;
  }
};

// NVFP4 k-block q of a raw segment: codes (256 rows x 128 bytes, 128-byte
// swizzle; the k-block is 16-byte chunks 2q and 2q+1 of each row) and the
// rows' block scales (16 bytes a row, the k-block's four at byte 4q) -> FP16
// row tile of raw values (row scale in the epilogue). nth converter threads,
// ct the thread's index. Unit i is row r, half h with the eight lanes of a
// quarter warp on eight consecutive rows, so the swizzle spreads their 16-byte
// reads over all banks.
template <int NTH>
__device__ __forceinline__ void convert_nvfp4_seg(const uint8_t *raw, const uint8_t *sbox, uint8_t *btile,
                                                  uint32_t ct, uint32_t q) {
#pragma unroll
  for (int u = 0; u < 2 * LR / NTH; u++) {
    const uint32_t i = ct + NTH * u, h = (i >> 3) & 1, r = (i & 7) | ((i >> 4) << 3);  // dims 32h .. 32h+31
    const uint4 w = *reinterpret_cast<const uint4 *>(raw + sw128_offset(r, 2 * q + h));
    uint32_t sc[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const uint32_t code = sbox[r * 16 + q * 4 + h * 2 + j];
      uint32_t pair, unused;
      e4m3x4_to_f16(code | (code << 8), pair, unused);
      sc[j] = pair;
    }
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint32_t o[4];
      e2m1x8_to_f16(ws[j], sc[j >> 1], o);
      *reinterpret_cast<uint4 *>(btile + sw128_offset(r, 4 * h + j)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// E4M3 k-block q of a raw segment (256 rows x 128 codes, 128-byte swizzle;
// the k-block is chunks 4q .. 4q+3) -> FP16 row tile of raw values. Unit i
// is row r, chunk c, a quarter warp on eight consecutive rows.
template <int NTH>
__device__ __forceinline__ void convert_e4m3_seg(const uint8_t *raw, uint8_t *btile, uint32_t ct, uint32_t q) {
#pragma unroll
  for (int u = 0; u < 4 * LR / NTH; u++) {
    const uint32_t i = ct + NTH * u, c = (i >> 3) & 3, r = (i & 7) | ((i >> 5) << 3);  // dims 16c .. 16c+15
    const uint4 w = *reinterpret_cast<const uint4 *>(raw + sw128_offset(r, 4 * q + c));
    uint4 lo, hi;
    e4m3x4_to_f16(w.x, lo.x, lo.y);
    e4m3x4_to_f16(w.y, lo.z, lo.w);
    e4m3x4_to_f16(w.z, hi.x, hi.y);
    e4m3x4_to_f16(w.w, hi.z, hi.w);
    *reinterpret_cast<uint4 *>(btile + sw128_offset(r, 2 * c)) = lo;
    *reinterpret_cast<uint4 *>(btile + sw128_offset(r, 2 * c + 1)) = hi;
  }
}

template <int Q>
__global__ void __launch_bounds__(L_NT, 1)
    tc_scan_lists(const __grid_constant__ CUtensorMap rows_map, const __grid_constant__ CUtensorMap scales_map,
                  const ListTcArgs L) {
  using C = LCfg<Q>;
  constexpr bool QUANT = Q != DT_F16;
  constexpr int RAWS = C::RAWB + C::SCB;     // raw codes + (NVFP4) scale box a raw segment
  constexpr int BSTG = C::BSTG, ASTG = C::ASTG, RSTG = C::RSTG, RSTG1 = RSTG > 0 ? RSTG : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *qtiles = smem + BSTG * LB_BYTES;
  uint8_t *raw = qtiles + ASTG * LA_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(raw + RSTG * RAWS);   // row tile ready
  uint64_t *empty = full + BSTG;                                       // row stage consumed
  uint64_t *afull = empty + BSTG;                                      // query tile landed
  uint64_t *aempty = afull + ASTG;                                     // query stage consumed
  uint64_t *rawfull = aempty + ASTG;
  uint64_t *rawempty = rawfull + RSTG1;
  uint64_t *tfull = rawempty + RSTG1;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile uint32_t *abort = tmem_slot + 1;
  float2 *affine = reinterpret_cast<float2 *>(reinterpret_cast<uint8_t *>(full) + L_BAR);  // [2][LR] (alpha, beta)
  volatile uint32_t *epi_ok = reinterpret_cast<volatile uint32_t *>(affine + 2 * LR);     // [2][4 warps]

  const ScanArgs &a = L.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t items = L.p.toff[L.p.nlists];
  const uint64_t per = (items + gridDim.x - 1) / gridDim.x;
  const uint64_t first = blockIdx.x * per < items ? blockIdx.x * per : items;
  const uint64_t last = first + per < items ? first + per : items;
  ItemCursor cur{&L.p, L.rbegin, L.rend};
  cur.start(first, last);

  if (threadIdx.x == 0) {
    for (int s = 0; s < BSTG; s++) {
      mbar_init(full + s, QUANT ? L_CW : 1);   // converter warps | the row tile's TMA
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < ASTG; s++) {
      mbar_init(afull + s, 32);                // the gather warp's copies
      mbar_init(aempty + s, 1);
    }
    for (int r = 0; r < RSTG; r++) {
      mbar_init(rawfull + r, 1);
      mbar_init(rawempty + r, L_CW);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L_TMEM)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // FP16: a k-block of the tile's 256 rows (two 128-row boxes) into the row
    // stage. Quantized: a raw segment (128 bytes of every row, SEGK k-blocks,
    // + NVFP4 scale boxes) into the raw ring.
    if (lane == 0) {
      constexpr int RING = QUANT ? RSTG1 : BSTG;
      constexpr int HALF = 128 * 128;   // bytes of a 128-row box (codes or FP16 rows)
      uint64_t *ring_full = QUANT ? rawfull : full;
      uint64_t *ring_empty = QUANT ? rawempty : empty;
      const uint32_t steps = QUANT ? (L.kblocks + C::SEGK - 1) / C::SEGK : L.kblocks;
      uint64_t it = 0;
      bool ok = true;
      for (; cur.valid() && ok; cur.next()) {
        const int32_t row = (int32_t)cur.row0();
        for (uint32_t kb = 0; kb < steps; kb++, it++) {
          const uint32_t s = (uint32_t)(it % RING), ph = (uint32_t)((it / RING) & 1);
          if (!mbar_wait(ring_empty + s, ph ^ 1, abort, a.flags)) {
            ok = false;
            break;
          }
          if (QUANT) {
            mbar_expect_tx(ring_full + s, (uint32_t)RAWS);
            uint8_t *dst = raw + s * RAWS;
            for (int h = 0; h < 2; h++) {
              tma_load_2d(smem_u32(dst + h * HALF), &rows_map, (int32_t)(kb * 128), row + 128 * h, ring_full + s);
              if (C::SCB)
                tma_load_2d(smem_u32(dst + C::RAWB + h * 128 * 16), &scales_map, (int32_t)(kb * 16), row + 128 * h,
                            ring_full + s);
            }
          } else {
            mbar_expect_tx(ring_full + s, (uint32_t)LB_BYTES);
            uint8_t *dst = smem + s * LB_BYTES;
            for (int h = 0; h < 2; h++)
              tma_load_2d(smem_u32(dst + h * HALF), &rows_map, (int32_t)(kb * 64), row + 128 * h, ring_full + s);
          }
        }
      }
      drain_ring(ring_full, RING, it);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = f16_idesc_mn(LQ, LR);
      uint64_t it = 0, tc = 0;
      bool ok = true;
      for (uint64_t item = first; item < last && ok; item++, tc++) {
        const uint32_t ab = (uint32_t)(tc & 1), use = (uint32_t)(tc >> 1);
        if (!mbar_wait(tempty + ab, (use & 1) ^ 1, abort, a.flags)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * LR;
        for (uint32_t kb = 0; kb < L.kblocks; kb++, it++) {
          const uint32_t s = (uint32_t)(it % BSTG), ph = (uint32_t)((it / BSTG) & 1);
          const uint32_t sq = (uint32_t)(it % ASTG), phq = (uint32_t)((it / ASTG) & 1);
          if (!mbar_wait(full + s, ph, abort, a.flags) || !mbar_wait(afull + sq, phq, abort, a.flags)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(qtiles + sq * LA_BYTES);   // queries: A (M = 64)
          const uint32_t sb = smem_u32(smem + s * LB_BYTES);      // rows: B (N = 256)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; kk++)
            tc_mma_f16(d_tmem, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, (kb | kk) != 0);
          tc_commit(empty + s);
          tc_commit(aempty + sq);
        }
        if (ok) tc_commit(tfull + ab);
      }
      tc_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < kWaitNs) {
      }
    }
    __syncwarp();
  } else if (warp == L_QW) {
    // ------------------------------------------------------------ query gather
    // Lane j copies queries j and j + 32 of the item's group (their 128 bytes
    // of the k-block) into the query ring by cp.async, into the accumulator
    // rows group_layout gives, up to ASTG k-blocks ahead of the MMAs; rows
    // the group does not use are not written.
    uint64_t it = 0, pf_qb = ~0ull;
    uint32_t pf_q[2] = {0u, 0u};
    bool ok = true;
    for (; cur.valid() && ok; cur.next()) {
      const uint32_t nqt = cur.nq_item();
      const uint64_t qb = cur.qbase();
      uint32_t nqq, rep;
      group_layout(nqt, nqq, rep);
      const __half *src[2];
      uint32_t n[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const uint32_t j = (uint32_t)lane + 32u * h;
        const uint32_t qn = j < nqt ? (qb == pf_qb ? pf_q[h] : L.p.qlist[qb + j]) : 0u;
        n[h] = j < nqt ? 16u : 0u;
        src[h] = L.q16 + (uint64_t)qn * L.kpad;
      }
      {
        uint64_t nqb;
        uint32_t nnqt;
        if (cur.peek_group(nqb, nnqt) && nqb != qb) {
          pf_qb = nqb;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const uint32_t j = (uint32_t)lane + 32u * h;
            pf_q[h] = j < nnqt ? L.p.qlist[nqb + j] : 0u;
          }
        }
      }
      for (uint32_t kb = 0; kb < L.kblocks; kb++, it++) {
        const uint32_t sq = (uint32_t)(it % ASTG), ph = (uint32_t)((it / ASTG) & 1);
        const bool got = mbar_wait(aempty + sq, ph ^ 1, abort, a.flags);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t dst = smem_u32(qtiles + sq * LA_BYTES);
#pragma unroll
        for (int h = 0; h < 2; h++)
          if (n[h]) {
            const uint32_t j = (uint32_t)lane + 32u * h;
            for (uint32_t cp = 0; cp < rep; cp++) {
              const uint32_t m = j + 16u * nqq * cp;   // accumulator row of copy cp
#pragma unroll
              for (uint32_t c = 0; c < 8; c++) cp_async16(dst + sw128_offset(m, c), src[h] + kb * 64 + c * 8, 16u);
            }
          }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(afull + sq)) : "memory");
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------------------------------------ converters (quantized formats)
    if (QUANT) {
      const uint32_t ct = threadIdx.x - 192;
      uint64_t it = 0, seg = 0;   // row stages, raw segments
      bool ok = true;
      for (; cur.valid() && ok; cur.next()) {
        for (uint32_t kb = 0; kb < L.kblocks; kb++, it++) {
          const uint32_t s = (uint32_t)(it % BSTG), ph = (uint32_t)((it / BSTG) & 1);
          const uint32_t r = (uint32_t)(seg % RSTG1), rph = (uint32_t)((seg / RSTG1) & 1);
          const uint32_t q = kb % C::SEGK;
          const bool seg_end = q == C::SEGK - 1 || kb + 1 == L.kblocks;
          bool got = mbar_wait(empty + s, ph ^ 1, abort, a.flags);
          if (got) got = mbar_wait(rawfull + r, rph, abort, a.flags);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          const uint8_t *rs = raw + r * RAWS;
          uint8_t *btile = smem + s * LB_BYTES;
          if (Q == DT_NVFP4) convert_nvfp4_seg<32 * L_CW>(rs, rs + C::RAWB, btile, ct, q);
          else convert_e4m3_seg<32 * L_CW>(rs, btile, ct, q);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            if (seg_end) mbar_arrive(rawempty + r);
            mbar_arrive(full + s);
          }
          seg += seg_end;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Accumulator row m sits in TMEM lane (m % 16) + 32 (m / 16), so warp w
    // reads rows 16 (w % 4) .. +15: with group_layout's rows, copy
    // (w % 4) / nqq of queries 16 ((w % 4) % nqq) .. +15 of the group, and the
    // copy's share of the item's 256 rows. A lane scores its query against
    // those rows, 32 accumulator columns at a time, then reserves one block of candidate slots for all
    // its passing rows of the item (one atomicAdd, whose round trip would
    // otherwise be paid a chunk) and writes them in column order, re-reading
    // from TMEM only the chunks that have some. The rows'
    // alpha and beta (row scale, norm) are staged once an item in shared
    // memory by all 128 epilogue threads (two rows each, double buffered,
    // named barrier 1). The four warps also post whether their wait for the
    // accumulator ended in time before that barrier, so all of them leave the
    // loop at the same item and none is left at the barrier.
    const int quad = warp & 3;
    const uint32_t et = threadIdx.x - 64;                 // epilogue thread 0..127
    uint32_t qn = 0, c_lo = 0, c_hi = 0;   // this lane's query; this warp's 32-row chunks of the item
    float th = __int_as_float(0x7fc00000);
    uint64_t tc = 0, tab = ~0ull;
    for (; cur.valid(); cur.next(), tc++) {
      const uint32_t ab = (uint32_t)(tc & 1), use = (uint32_t)(tc >> 1);
      const uint32_t nqt = cur.nq_item();
      const uint64_t qb = cur.qbase();
      if (qb != tab) {          // a new query group: this lane's query, its threshold, the warp's rows
        uint32_t nqq, rep;
        group_layout(nqt, nqq, rep);
        const bool active = (uint32_t)quad < nqq * rep;
        const uint32_t jq = 16u * ((uint32_t)quad % nqq) + (uint32_t)lane;
        const bool mine = active && lane < 16 && jq < nqt;
        qn = mine ? L.p.qlist[qb + jq] : 0u;
        th = mine ? a.thr[qn] : __int_as_float(0x7fc00000);
        const uint32_t per = (uint32_t)(LR / 32) / rep;
        c_lo = active ? ((uint32_t)quad / nqq) * per : 0u;
        c_hi = active ? c_lo + per : 0u;
        tab = qb;
      }
      // the item's rows: alpha, beta into affine[tc & 1] (rows past the list never pass)
      const uint64_t row0 = cur.row0();
      float2 *aff = affine + (tc & 1) * LR;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const uint64_t row = row0 + et + 128u * h;
        float al = 0.0f, be = __int_as_float(0x7fc00000);
        if (row < cur.hi) row_affine(a.s, row, a.metric, a.raw_scale, al, be);
        aff[et + 128u * h] = make_float2(al, be);
      }
      const bool got = __all_sync(0xffffffffu, mbar_wait(tfull + ab, use & 1, abort, a.flags));
      if (lane == 0) epi_ok[(tc & 1) * 4 + (warp - 2)] = got ? 1u : 0u;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const volatile uint32_t *ok4 = epi_ok + (tc & 1) * 4;
      if (!(ok4[0] & ok4[1] & ok4[2] & ok4[3])) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + ab * LR + ((uint32_t)(quad * 32) << 16);
      // pass 1: the passing rows of each 32-column chunk, and their count
      uint32_t mk[LR / 32], total = 0;
#pragma unroll 1
      for (uint32_t c = c_lo; c < c_hi; c++) {
        uint32_t r[32];
        TMEM_LD32(acc + c * 32, r);
        tmem_ld_wait();
        uint32_t msk = 0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const float2 f = aff[c * 32 + j];
          msk |= (uint32_t)(fmaf(__uint_as_float(r[j]), f.x, f.y) <= th) << j;
        }
        mk[c] = msk;
        total += (uint32_t)__popc(msk);
      }
      // pass 2 (only where some row passed): one block of candidate slots a
      // lane, then the passing rows of each chunk, re-read from TMEM
      if (__any_sync(0xffffffffu, total != 0)) {
        const uint32_t base = total ? atomicAdd(a.cnt + qn, total) : 0u;
        uint2 *cand = a.cand + (uint64_t)qn * a.cap;
        uint32_t done = 0;
#pragma unroll 1
        for (uint32_t c = c_lo; c < c_hi; c++) {
          if (!__any_sync(0xffffffffu, mk[c] != 0)) continue;
          uint32_t r[32];
          TMEM_LD32(acc + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j++) {
            if ((mk[c] >> j) & 1u) {
              const uint32_t slot = base + done + (uint32_t)__popc(mk[c] & ((1u << j) - 1u));
              const float2 f = aff[c * 32 + j];
              if (slot < a.cap) {
                cand[slot] = make_uint2(__float_as_uint(fmaf(__uint_as_float(r[j]), f.x, f.y)),
                                        (uint32_t)(row0 + c * 32 + j));
              } else {
                atomicOr(a.flags, FLAG_OVERFLOW);
                atomicMax(a.flags + 1, slot + 1);
              }
            }
          }
          done += (uint32_t)__popc(mk[c]);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty + ab);        // every column read: the accumulator is free
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(L_TMEM)
                 : "memory");
  }
}

// Copy candidate rows (virtual row i = candidate position base + i*stride,
// row id ids[pos] or pos) to consecutive rows of out: one warp a row,
// 16-byte coalesced loads and stores (row_bytes a multiple of 16).
__global__ void __launch_bounds__(256) gather_rows(const uint8_t *codes, uint64_t row_bytes, uint64_t rows,
                                                   const uint32_t *ids, uint64_t base, uint64_t stride, uint64_t count,
                                                   uint8_t *out) {
  const uint64_t i = (uint64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= count) return;
  const uint64_t pos = base + i * stride;
  const uint64_t id = cand_row(ids, pos, rows);
  const uint4 *src = reinterpret_cast<const uint4 *>(codes + id * row_bytes);
  uint4 *dst = reinterpret_cast<uint4 *>(out + i * row_bytes);
  const uint32_t units = (uint32_t)(row_bytes / 16);
  uint4 v[4];
  for (uint32_t u0 = 0; u0 < units; u0 += 128) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t u = u0 + k * 32 + lane;
      if (u < units) v[k] = __ldg(src + u);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t u = u0 + k * 32 + lane;
      if (u < units) dst[u] = v[k];
    }
  }
}

}  // namespace

void launch_gather_rows(const uint8_t *codes, uint64_t row_bytes, uint64_t rows, const uint32_t *ids, uint64_t base,
                        uint64_t stride, uint64_t count, uint8_t *out, cudaStream_t st) {
  if (count)
    gather_rows<<<(unsigned)((count + 7) / 8), 256, 0, st>>>(codes, row_bytes, rows, ids, base, stride, count, out);
}

// Shared memory the tensor scan of storage format q needs for nq queries
// (thresholds included).
template <int Q>
size_t tc_scan_smem_t(uint32_t nq) {
  return 1024 + (size_t)TcCfg<Q>::RING + (size_t)TcCfg<Q>::RSTG * TcCfg<Q>::RAWB + 256 +
         4 * EPI_BUF * sizeof(uint4) + (size_t)((nq + 255) / 256 * 256) * sizeof(float) * (Q == QF8 ? 2 : 1);
}

// Largest query count one tensor-scan launch takes (thresholds in shared memory).
uint32_t tc_scan_max_queries() { return 4096; }

// How many of a CTA's tiles ahead the gathering FP16 scan asks L2 for:
// ANN_B200_PREFETCH_TILES (1-4), a tuning knob, else 1.
uint32_t prefetch_tiles() {
  static const uint32_t n = [] {
    const char *v = getenv("ANN_B200_PREFETCH_TILES");
    const int x = v && *v ? atoi(v) : 1;
    return (uint32_t)(x < 1 ? 1 : x > 4 ? 4 : x);
  }();
  return n;
}

// The limit of each pipeline wait in the flat tensor scan: 4 s, or, for
// tests of the time-out path, ANN_B200_PIPELINE_WAIT_NS (read at every
// launch). A wait that runs out sets FLAG_TIMEOUT and the search fails with
// ANN_BACKEND_ERROR; the drains that follow keep their 4 s.
uint64_t pipeline_wait_ns() {
  const char *v = getenv("ANN_B200_PIPELINE_WAIT_NS");
  if (v && *v) {
    const unsigned long long n = strtoull(v, nullptr, 10);
    if (n > 0) return n;
  }
  return kWaitNs;
}

template <int Q>
cudaError_t launch_tc_t(const CUtensorMap &rows_map, const CUtensorMap &query_map, const CUtensorMap &query_lo_map,
                        const TcArgs &t, int sms,
                        cudaStream_t st) {
  const size_t smem = tc_scan_smem_t<Q>(t.a.nq);
  cudaError_t e = cudaFuncSetAttribute(tc_scan<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const uint64_t ntiles = t.rtiles * t.qtiles;
  const unsigned grid = (unsigned)(ntiles < (uint64_t)sms ? ntiles : (uint64_t)sms);
  tc_scan<Q><<<grid, TcCfg<Q>::NT, smem, st>>>(rows_map, query_map, query_lo_map, t);
  return cudaGetLastError();
}

template <int Q>
size_t tc_scan_lists_smem() {
  using C = LCfg<Q>;
  return 1024 + (size_t)C::BSTG * LB_BYTES + (size_t)C::ASTG * LA_BYTES + (size_t)C::RSTG * (C::RAWB + C::SCB) +
         L_BAR + 2 * LR * sizeof(float2) + 2 * 4 * sizeof(uint32_t);
}

template <int Q>
cudaError_t launch_lists_t(const CUtensorMap &rows_map, const CUtensorMap &scales_map, const ListTcArgs &L, int sms,
                           cudaStream_t st) {
  const size_t smem = tc_scan_lists_smem<Q>();
  cudaError_t e = cudaFuncSetAttribute(tc_scan_lists<Q>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  tc_scan_lists<Q><<<sms, L_NT, smem, st>>>(rows_map, scales_map, L);
  return cudaGetLastError();
}

// Launch the tensor scan of a.count virtual rows against a.nq FP16 queries.
// FP16 rows named by a candidate list or a strided sample (a.ids set, or
// a.stride > 1) are gathered from the shard by the kernel itself (rows_map
// unused). Otherwise rows_map describes contiguous rows whose row a_row0 is
// virtual row 0 -- the shard itself or a staging copy of gathered
// candidates: FP16 ([rows][dims], box 64 x 128, 128-byte swizzle), or the raw codes of an
// E4M3 ([rows][dims] bytes, box 64 x 128) or NVFP4 shard ([rows][dims/2]
// bytes, box 32 x 128), converted to FP16 in shared memory (a.raw_scale
// must be set: scores are on the raw codes). query_map: the FP16 queries
// ([qtiles*bn][kpad], box 64 x bn). FP32 rows ([rows][dims] floats, box 64 x
// 128 unswizzled, dims a multiple of 4) are split on chip into two BF16
// tiles, hi = RN(x) and lo = RN(x - hi), and scored by three BF16 MMAs a K
// step (hi.hi + hi.lo + lo.hi) against query_map and *query_lo_map, the
// queries' two BF16 halves (bn <= 128). Bit vectors ([rows][row_bytes], box 16
// x 128, row_bytes a multiple of 16) are expanded to +-1 int8 on chip and
// scored by kind::i8 MMAs against query_map = the int8 query expansion
// ([qtiles*bn][kpad] bytes, box 128 x bn, 128-byte swizzle); their scores
// are exact Hamming distances. The epilogue reads per-row norms and
// scales through a.ids / a.base / a.stride. Returns a CUDA error from the
// launch.
cudaError_t launch_tc_scan(const ScanArgs &a, const CUtensorMap &rows_map, int64_t a_row0,
                           const CUtensorMap &query_map, const CUtensorMap *query_lo_map, uint32_t kpad, uint32_t bn,
                           int sms, cudaStream_t st) {
  const CUtensorMap &qlo = query_lo_map ? *query_lo_map : query_map;
  TcArgs t;
  t.a = a;
  t.a_row0 = a_row0;
  t.kpad = kpad;
  t.kblocks = a.s.dtype == DT_BIT ? kpad / 128 : kpad / 64;
  t.bn = bn;
  t.qtiles = (a.nq + bn - 1) / bn;
  t.rtiles = (a.count + BM - 1) / BM;
  t.wait_ns = pipeline_wait_ns();
  t.pf_tiles = prefetch_tiles();
  t.q_lo_row = (int32_t)(t.qtiles * bn);
  if (a.count == 0 || a.nq == 0) return cudaSuccess;
  if (a.f8) {
    // kpad: the query terms' bytes a row (a multiple of 128); rows_map: 128-byte
    // swizzled boxes of 128 codes x 128 rows; query_map: the terms as bytes
    // [2 * qtiles * bn][kpad], boxes of 128 bytes x bn rows, 128-byte swizzle
    if (a.s.dtype != DT_E4M3 || bn > (uint32_t)F8_BN || kpad % 128) return cudaErrorInvalidValue;
    t.kblocks = kpad / 128;
    return launch_tc_t<QF8>(rows_map, query_map, query_map, t, sms, st);
  }
  switch (a.s.dtype) {
    case DT_F16:
      return (a.ids || a.stride != 1) ? launch_tc_t<GF16>(rows_map, query_map, qlo, t, sms, st)
                                      : launch_tc_t<DT_F16>(rows_map, query_map, qlo, t, sms, st);
    case DT_E4M3: return launch_tc_t<DT_E4M3>(rows_map, query_map, qlo, t, sms, st);
    case DT_NVFP4: return launch_tc_t<DT_NVFP4>(rows_map, query_map, qlo, t, sms, st);
    case DT_BIT: return launch_tc_t<DT_BIT>(rows_map, query_map, qlo, t, sms, st);
    case DT_F32:
      if (!query_lo_map || bn > (uint32_t)F32_BN) return cudaErrorInvalidValue;
      return launch_tc_t<DT_F32>(rows_map, query_map, qlo, t, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

// The IVF list scan on tensor cores over the items launch_list_items counted
// with p.bm = 256 and p.bq = 64 (rows [rbegin, rend) of every probed list).
// rows_map: FP16 rows as launch_tc_scan reads contiguous runs of them
// (box 64 x 128, 128-byte swizzle), or the E4M3 / NVFP4 codes as bytes in
// boxes of 128 x 128 with the 128-byte swizzle; scales_map (NVFP4 only): the
// block scales [rows][bblocks] as bytes, box 16 x 128. q16: the FP16 queries [.][kpad] prep_queries wrote.
cudaError_t launch_tc_scan_lists(const ScanArgs &a, const ListPlan &p, uint64_t rbegin, uint64_t rend,
                                 const CUtensorMap &rows_map, const CUtensorMap &scales_map, const __half *q16,
                                 uint32_t kpad, int sms, cudaStream_t st) {
  ListTcArgs L;
  L.a = a;
  L.p = p;
  L.rbegin = rbegin;
  L.rend = rend;
  L.q16 = q16;
  L.kpad = kpad;
  L.kblocks = kpad / 64;
  switch (a.s.dtype) {
    case DT_F16: return launch_lists_t<DT_F16>(rows_map, scales_map, L, sms, st);
    case DT_E4M3: return launch_lists_t<DT_E4M3>(rows_map, scales_map, L, sms, st);
    case DT_NVFP4: return launch_lists_t<DT_NVFP4>(rows_map, scales_map, L, sms, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace annb200
