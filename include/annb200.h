/*
 * annb200.h - C ABI of libannb200.so, the B200 exact gather-scan.
 *
 * Plain pointers and sizes only. Device pointers are CUDA device addresses on
 * the shard's device; streams are cudaStream_t passed as void * (NULL = the
 * legacy default stream). Every entry point returns an AnnStatus value
 * (0 = ANN_OK, 1 = ANN_INVALID, 2 = ANN_UNSUPPORTED, 4 = ANN_NOMEM,
 * 5 = ANN_BACKEND_ERROR; ann/server/backend.h:12-28 in the reference) and
 * leaves a message for AnnB200LastError() when it fails.
 *
 * Which reference interface each entry point replaces (reference paths are
 * relative to the chenqin/pgvector project root):
 *
 *   AnnB200Backend()        the AnnBackend vtable constructor a worker selects
 *                           with --backend (ann/server/backend.h:114-164,
 *                           ann/server/worker.c:267-279); declared in
 *                           annb200_backend.h.
 *   AnnB200ShardCreate()    device upload of one index shard's rows plus the
 *                           per-row norms the scan needs: the loaded-index
 *                           shard upload of ann/server/cuvs.c:2677-2915 and
 *                           AnnBlackwellUpload, ann/server/blackwell.c:961-1064.
 *   AnnB200Search()         one exact gather-scan of a query batch over a
 *                           shard and a candidate row list: SearchGather,
 *                           ann/server/cuvs.c:4585-4930 (gather_f32/f16,
 *                           cuvsSelectK, host re-score), the grouped
 *                           tensor-core scan AnnBlackwellCandidates,
 *                           ann/server/blackwell.c:1452-1548, and the CPU
 *                           exact search it must equal, ann/server/cpu.c:82-276.
 *   AnnB200MergeTopk()      the per-shard top-k merge AnnIndexTreeMerge,
 *                           ann/server/indexfile.c:3235-3258 and MergeJob,
 *                           ann/server/cuvs.c:3446-3455, on the device.
 *   AnnB200BitmapRows()     filter bitmap to eligible row list, the expand_*
 *                           kernels of ann/server/cuvs.c:1910-1968.
 *   AnnB200IndexCreate/Search  a loaded index's exact search (the worker's
 *                           load_index / search_index, cpu.c:286-407);
 *                           AnnB200IndexCreateQuant the same from the
 *                           directory's quantized copy (the quantized scan
 *                           route, ann/server/cuvs.c:4585-4930), with
 *                           AnnB200RescoreRows its FP32 re-score
 *                           (ExactDistance, cuvs.c:2930-2942).
 */
#ifndef ANNB200_H
#define ANNB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C"
{
#endif

/* Row storage formats (ann/common/INDEX_FORMAT.md:38,54-57, plus bit rows). */
#define ANNB200_F32 0			/* FP32, dims x 4 bytes a row */
#define ANNB200_F16 1			/* IEEE half (halfvec), dims x 2 bytes */
#define ANNB200_E4M3 2			/* FP8 codes, dims rounded up to 16 bytes, +
								 * one FP32 row scale */
#define ANNB200_NVFP4 3			/* E2M1 pairs, ceil(dims/16) x 8 bytes, + one
								 * E4M3 scale per 16 dims + one FP32 row scale */
#define ANNB200_BIT 4			/* packed bits, ceil(dims/8) bytes */

/* Metrics: the worker's 0..2 (ann/server/cpu.c:139-142) plus Hamming. */
#define ANNB200_L2 0			/* Euclidean distance */
#define ANNB200_IP 1			/* negative inner product */
#define ANNB200_COSINE 2		/* 1 - cosine similarity; zero-norm rows skipped */
#define ANNB200_HAMMING 3		/* bit rows only */

/* AnnB200ShardCreate flags */
#define ANNB200_SHARD_HOST 1u	/* inputs are host pointers: copy them into
								 * device memory the shard owns */
#define ANNB200_SHARD_F32_TO_F16 2u	/* with ANNB200_SHARD_HOST and ANNB200_F16:
									 * codes are host FP32 rows, kept on the
									 * device as FP16 (round to nearest) */

/* AnnB200Search / AnnB200MergeTopk flags */
#define ANNB200_WINDOW 1u		/* gathered-job results: every row within
								 * d_k + 1e-3*|d_k| + 1e-6 of the k-th
								 * distance (ann/server/backend.h:45-50) */
#define ANNB200_FORCE_SIMT 2u	/* score on CUDA cores even where the tcgen05
								 * tensor-core scan applies */
#define ANNB200_FORCE_F16 8u	/* E4M3 rows: convert the codes to FP16 on
								 * chip for kind::f16 MMAs instead of the
								 * FP8 tensor scan (same results) */
#define ANNB200_BOUNDS_EXCHANGE 32u	/* sharded searches: exchange the ranks'
									 * bounds of the k-th distance before the
									 * exact re-score (a second all-gather) */
#define ANNB200_INDEX_L2 4u		/* L2 in the loaded-index form: the FP32
								 * sqrtf of tail + (left + right) lane sums
								 * (Distance, ann/server/indexfile.c:3133-3151)
								 * instead of the gathered jobs' FP64 sqrt */

typedef struct AnnB200Shard AnnB200Shard;

/* The message of the calling thread's last failed call ("" if none). */
const char *AnnB200LastError(void);

/* Number of CUDA devices the library can use (0 without a GPU). */
int			AnnB200DeviceCount(void);

/*
 * Make a shard of rows [0, rows) stored in one of the formats above, whose
 * global row ids start at first_id. codes: rows x row-bytes; block_scales:
 * NVFP4 only, rows x ceil(dims/16) E4M3 codes; row_scales: E4M3 and NVFP4,
 * rows FP32. Without ANNB200_SHARD_HOST the pointers are device memory that
 * the caller keeps alive until AnnB200ShardDestroy. The call computes each
 * row's squared norm on the device and returns once the shard is usable.
 */
int			AnnB200ShardCreate(int device, uint32_t dtype, uint32_t dims, uint64_t rows,
							   const void *codes, const void *block_scales,
							   const float *row_scales, int64_t first_id,
							   uint32_t flags, void *stream, AnnB200Shard **shard);
void		AnnB200ShardDestroy(AnnB200Shard *shard);

/*
 * Re-point an existing shard at other rows already in device memory (same
 * meaning as AnnB200ShardCreate without ANNB200_SHARD_HOST), reusing its
 * buffers: for callers that search a new row set per request, such as the
 * worker's gathered jobs (ann/server/backend.h:45-62).
 */
int			AnnB200ShardAssign(AnnB200Shard *shard, uint32_t dtype, uint32_t dims, uint64_t rows,
							   const void *codes, const void *block_scales,
							   const float *row_scales, int64_t first_id, void *stream);

/*
 * Exact k-nearest search of nq queries over the shard's candidate rows.
 *
 * queries  device, FP32 [nq][dims]; for Hamming, packed bits
 *          [nq][ceil(dims/8)].
 * rows     device u32 list of candidate row numbers within the shard,
 *          strictly increasing, nrows long; NULL scans every row.
 * Results  device [nq][out_cap] FP64 distances and int64 global row ids
 *          (first_id + row), sorted by (distance, id), counts [nq]. Without
 *          ANNB200_WINDOW each query gets min(k, eligible rows) results and
 *          out_cap must be >= k; with it, every row within the gathered
 *          tolerance of the k-th distance (out_cap >= nrows guarantees room).
 * status   optional device int32 [nq]: ANN_INVALID for a query with a
 *          non-finite value, or a zero norm under cosine.
 *
 * Distances equal, bit for bit, the reference CPU worker's on the rows
 * decoded to FP32 (ann/server/cpu.c:82-276): L2 as sqrt of the eight-lane
 * FP32 sum, inner product and cosine in FP64. The call is synchronous with
 * respect to stream (it waits for its own kernels).
 */
int			AnnB200Search(AnnB200Shard *shard, const void *queries, uint32_t nq,
						  const uint32_t *rows, uint64_t nrows, uint32_t k,
						  uint32_t metric, uint32_t flags, uint32_t out_cap,
						  double *out_dist, int64_t *out_id, uint32_t *out_count,
						  int32_t *status, void *stream);

/*
 * A batch of independent searches, each over its own FP32 rows in device
 * memory, with one synchronisation for the whole batch: the reference's
 * "one call = one device submission" for a lane's gathered jobs
 * (search_gathered, ann/server/backend.h:129-130, called per lane batch at
 * ann/server/server.c:1541). Per job: AnnB200Search of queries (nq <=
 * 4096) over rows [0, nrows) (ids = row numbers) with its k, metric (L2,
 * IP, cosine), flags and out_cap, results into its device arrays, its
 * AnnStatus in result. With ANNB200_REJECT_NONFINITE a job whose rows hold
 * a non-finite value fails with ANN_INVALID (the gathered job's rule). The
 * shard is the reusable context the jobs are bound to in turn (its rows
 * are replaced). A job whose candidate lists overflow runs again,
 * synchronously. Returns ANN_OK when the batch ran (see each result).
 */
#define ANNB200_REJECT_NONFINITE 16u
typedef struct AnnB200BatchJob
{
	const float *rows;			/* device [nrows][dims] */
	uint32_t	nrows;
	uint32_t	dims;
	const float *queries;		/* device [nq][dims] */
	uint32_t	nq;
	uint32_t	k;
	uint32_t	metric;
	uint32_t	flags;			/* ANNB200_WINDOW, ANNB200_REJECT_NONFINITE, ... */
	uint32_t	out_cap;
	uint32_t	reserved;
	double	   *out_dist;		/* device [nq][out_cap] */
	int64_t    *out_id;
	uint32_t   *out_count;		/* device [nq] */
	int32_t    *status;			/* device [nq], or NULL */
	int			result;			/* AnnStatus */
	int			reserved2;
} AnnB200BatchJob;
int			AnnB200SearchBatch(AnnB200Shard *shard, AnnB200BatchJob *jobs, uint32_t n, void *stream);

/*
 * Row-sharded search across GPUs (one rank a GPU). The reference spreads a
 * loaded index over the GPUs as row-range shards (placement
 * ann/server/cuvs.c:2845-2862) and merges the per-shard top-k lists on the
 * host (AnnIndexTreeMerge, ann/server/indexfile.c:3235-3258; MergeJob,
 * ann/server/cuvs.c:3446-3455). Here the ranks exchange their lists with one
 * NCCL all-gather and merge them on the device.
 *
 * Communicators: NCCL's C API, loaded at run time (libnccl.so.2; the copy
 * the process already has, if any; ANN_B200_NCCL_LIBRARY names another).
 * Several processes: one calls AnnB200CommId and hands the 128 bytes to the
 * others, then each calls AnnB200CommCreate with its device and rank. One
 * process over several devices (a worker with every GPU): AnnB200CommCreateAll
 * fills comms[i] for devices[i]; each is then driven by its own thread.
 * AnnB200CommDestroy releases one rank once every rank is done with the
 * group; AnnB200CommAbort ends this rank's part at once (for a rank whose
 * peers died or left: nothing of the group is waited for) and every later
 * call on it fails. ANN_UNSUPPORTED without NCCL.
 */
#define ANNB200_COMM_ID_BYTES 128
typedef struct AnnB200Comm AnnB200Comm;
int			AnnB200CommId(void *id);
int			AnnB200CommCreate(int device, int nranks, int rank, const void *id, AnnB200Comm **comm);
int			AnnB200CommCreateAll(int ndev, const int *devices, AnnB200Comm **comms);
void		AnnB200CommDestroy(AnnB200Comm *comm);
void		AnnB200CommAbort(AnnB200Comm *comm);
int			AnnB200CommRank(const AnnB200Comm *comm);
int			AnnB200CommSize(const AnnB200Comm *comm);

/*
 * One rank of a row-sharded search: every rank of comm calls this at the same
 * time with its own shard (its global ids first_id + row, disjoint from the
 * other ranks'), its own candidate rows, and the same queries, nq, k, metric
 * and flags. Arguments as AnnB200Search (strict top k only: ANNB200_WINDOW
 * is unsupported); out_* receive, on every rank, the k best of all ranks'
 * rows by (distance, id) -- the answer of one search over the union of the
 * shards, bit for bit. comm NULL: AnnB200Search. nranks * k <= 4096, nq <=
 * 32768.
 *
 * Each rank's search is enqueued on stream without a host round trip; one
 * all-gather (per rank: a header with its status and flags, then its
 * counts, distances and ids) and the device merge follow, then the one
 * synchronisation. With ANNB200_BOUNDS_EXCHANGE (every rank passes it or
 * none does) a second all-gather runs between the filter pass and the
 * exact re-score: each rank's bound of every query's k-th exact distance
 * (8 bytes a query), so that a rank re-scores and sends only the survivors
 * that can reach the merged top k. Every rank reads every rank's header, so all ranks
 * succeed or fail together, and when a rank's candidate list overflowed
 * they all search again synchronously and exchange once more; no rank
 * leaves a collective the others enter. If the exchange does not finish
 * within ANN_B200_COMM_TIMEOUT_MS (default 60,000: a peer that died or
 * never called), the communicator is aborted and every later call on it
 * fails with ANN_BACKEND_ERROR. Synchronous.
 */
int			AnnB200SearchSharded(AnnB200Shard *shard, AnnB200Comm *comm, const void *queries, uint32_t nq,
								 const uint32_t *rows, uint64_t nrows, uint32_t k, uint32_t metric,
								 uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
								 uint32_t *out_count, int32_t *status, void *stream);

/*
 * AnnB200SearchSharded (comm NULL: AnnB200Search) over the shard rows whose
 * bits are set in a device bitmap -- bit r of word r / 32, nbits <= the
 * shard's rows -- in one call: the bitmap's expansion to ascending rows (as
 * AnnB200BitmapRows; the reference's expand_* kernels before a bitmap
 * search, ann/server/cuvs.c:1910-1968) into a buffer of the shard, then the
 * search. *nrows (optional) receives the rows the bitmap selected. A bad
 * bitmap is this rank's status: with comm it still joins the exchange.
 * Arguments otherwise as AnnB200SearchSharded. Synchronous.
 */
int			AnnB200SearchBitmap(AnnB200Shard *shard, AnnB200Comm *comm, const void *queries, uint32_t nq,
								const uint32_t *words, uint64_t nbits, uint32_t k, uint32_t metric,
								uint32_t flags, uint32_t out_cap, double *out_dist, int64_t *out_id,
								uint32_t *out_count, int32_t *status, uint64_t *nrows, void *stream);

/*
 * IVF list gather: exact k-nearest search of each query over the rows of the
 * lists it probes -- the list scan of the reference's IVFFlat index
 * (src/ivfscan.c:124-186: visit the probed lists, score every entry, order
 * them), for a batch of queries at once.
 *
 * The shard holds its rows list-major: list l is rows
 * list_offsets[l] .. list_offsets[l+1]-1 (device u64 [nlists+1],
 * non-decreasing, last <= the shard's rows). probes is device u32
 * [nq][nprobe]: each query's list numbers, distinct and < nlists (a query
 * that breaks this gets status ANN_INVALID and no results); entries equal
 * to UINT32_MAX are padding, for queries with fewer lists on this shard
 * when the lists are sharded across GPUs. row_ids
 * (optional, device int64 [rows]) gives each stored row's global id;
 * without it the id is first_id + row. Results as AnnB200Search without
 * ANNB200_WINDOW: min(k, rows in the probed lists) per query, sorted by
 * (distance, id), distances bit-identical to the reference CPU worker's
 * (L2 as sqrt of the eight-lane FP32 sum, inner product and cosine in
 * FP64). Metrics L2, IP, cosine; every vector storage format. nlists <=
 * 2^24, nprobe <= 4096. Synchronous.
 */
int			AnnB200SearchLists(AnnB200Shard *shard, const float *queries, uint32_t nq,
							   const uint64_t *list_offsets, uint32_t nlists,
							   const uint32_t *probes, uint32_t nprobe, const int64_t *row_ids,
							   uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap,
							   double *out_dist, int64_t *out_id, uint32_t *out_count,
							   int32_t *status, void *stream);

/*
 * One rank of a sharded IVF list search: AnnB200SearchLists over this
 * rank's share of the list-major rows (each list it holds clipped to its
 * rows, list numbers and probes in its own numbering, UINT32_MAX for lists
 * it does not hold, global ids through row_ids or first_id), then the
 * all-gather and device merge of AnnB200SearchSharded: every rank receives
 * the k best over every rank's share of each query's probed lists. Same
 * conditions as AnnB200SearchSharded.
 */
int			AnnB200SearchListsSharded(AnnB200Shard *shard, AnnB200Comm *comm, const float *queries,
									  uint32_t nq, const uint64_t *list_offsets, uint32_t nlists,
									  const uint32_t *probes, uint32_t nprobe, const int64_t *row_ids,
									  uint32_t k, uint32_t metric, uint32_t flags, uint32_t out_cap,
									  double *out_dist, int64_t *out_id, uint32_t *out_count,
									  int32_t *status, void *stream);

/*
 * IVF coarse probe: each query's nprobe nearest list centroids -- the list
 * selection of the reference's IVFFlat scan (GetScanLists,
 * src/ivfscan.c:48-122: score every centroid, keep the nprobe nearest). The
 * centroids are a shard (row l = list l's centre; FP32 as the index stores
 * them, or any vector format); probes (device u32 [nq][nprobe]) receives the
 * list numbers (row - first_id) ordered by (exact distance, list number),
 * UINT32_MAX past the number of lists -- the probe table AnnB200SearchLists
 * takes. Where the reference's heap leaves the choice among lists at an
 * exactly equal distance open, the lower list number is kept. Metrics L2,
 * IP, cosine; nprobe <= 4096. Synchronous.
 */
int			AnnB200ProbeLists(AnnB200Shard *centroids, const float *queries, uint32_t nq,
							  uint32_t nprobe, uint32_t metric, uint32_t *probes, int32_t *status,
							  void *stream);

/*
 * The approximate score matrix the scan prunes with (the reference's
 * score-matrix route, score_mma_* / AnnBlackwellScore,
 * ann/server/blackwell.c:289-525,1066-1110): out [nq][n] FP32 approximate
 * distances of every candidate row to every query -- Euclidean distance
 * squared for L2, -dot for IP, 1 - cosine, Hamming -- n = nrows, or the
 * shard's rows when rows is NULL; nq <= 4096. err (optional, device FP64
 * [nq]) receives each query's bound on |approximate - exact| in the same
 * domain. Synchronous.
 */
int			AnnB200ScoreMatrix(AnnB200Shard *shard, const void *queries, uint32_t nq,
							   const uint32_t *rows, uint64_t nrows, uint32_t metric,
							   uint32_t flags, float *out, double *err, void *stream);

/*
 * Merge nlists per-shard result sets into one per query, on the device.
 * Inputs: device [nlists][nq][list_cap] distances/ids and [nlists][nq]
 * counts, each list sorted by (distance, id) with disjoint ids (the layout an
 * all-gather of AnnB200Search outputs produces). Output as AnnB200Search:
 * the k best by (distance, id), or with ANNB200_WINDOW every entry within
 * the gathered tolerance of the merged k-th distance. nlists * list_cap must
 * not exceed 4096. Without ANNB200_WINDOW the merge is only enqueued on
 * stream (results are ready when the stream reaches it); with it the call
 * waits for the merge, to report a window larger than out_cap.
 */
int			AnnB200MergeTopk(const double *dist, const int64_t *ids, const uint32_t *counts,
							 uint32_t nlists, uint32_t nq, uint32_t list_cap, uint32_t k,
							 uint32_t flags, uint32_t out_cap, double *out_dist,
							 int64_t *out_id, uint32_t *out_count, void *stream);

/*
 * Expand a filter bitmap (bit r of word r/32, least significant bit first)
 * into the strictly increasing list of set row numbers. rows must hold
 * nbits entries; *count (host) receives how many were written. Synchronous.
 */
int			AnnB200BitmapRows(const uint32_t *words, uint64_t nbits, uint32_t *rows,
							  uint64_t *count, void *stream);

/*
 * AnnB200BitmapRows with every row number offset by first_row: one shard's
 * bitset (ann/server/indexfile.h:117-144, the per-shard bitsets of a cached
 * filter) expanded into global row numbers (first_row + bit). first_row +
 * nbits <= 2^32. Synchronous.
 */
int			AnnB200BitmapRowsFrom(const uint32_t *words, uint64_t nbits, uint32_t first_row, uint32_t *rows,
								  uint64_t *count, void *stream);

/*
 * AnnB200BitmapRows for callers that must not allocate device memory on their
 * call path -- a worker serving from a device-memory budget it reserved at
 * start-up, or a latency-critical caller that cannot afford the device
 * synchronisation cudaMalloc / cudaFree bring. No counterpart in the
 * reference. Same arguments and result as AnnB200BitmapRows, but its scratch
 * (one offset per 32,768 bitmap bits and the row count) lives in a fixed
 * 256 KB array in device memory that every GPU loading this library holds
 * until exit, so it allocates nothing. Limit: nbits <= 2^31; larger bitmaps
 * fail with ANN_INVALID. The first call on a device looks the array's
 * address up on that device (make it before any stream capture). All calls
 * share the array: calls running on a device at the same time (other
 * streams or threads) race and must be serialised by the caller.
 */
int			AnnB200BitmapRowsStatic(const uint32_t *words, uint64_t nbits, uint32_t *rows,
									uint64_t *count, void *stream);

/*
 * Loaded on-disk indexes (the worker's load_index / search_index,
 * ann/server/backend.h:133-135). An AnnB200Index holds an index directory's
 * FP32 rows (vectors.f32, ann/common/INDEX_FORMAT.md, row i = the i-th
 * smallest key) resident on one device; AnnB200IndexSearch is the exact
 * route of the reference's loaded-index search (AnnIndexExact + Offer +
 * AnnIndexTreeMerge, ann/server/indexfile.c:3134-3258): per query the k
 * rows of smallest FP32 L2 distance (Distance's own arithmetic, bit for
 * bit), sorted by (distance, ordinal) -- key order is ordinal order, so this
 * is the reference's (distance, key) order.
 *
 * AnnB200IndexCreate copies rows x dims host floats (an mmap of vectors.f32
 * is fine) to `device` (-1: the next device round robin) and returns once
 * the index is searchable.
 *
 * AnnB200IndexSearch takes host memory throughout: queries [nq][dims];
 * ordinals (NULL: every row) a strictly increasing list of eligible rows,
 * nordinals long; results [nq][k] distances and ordinals and counts [nq].
 * Synchronous; safe to call from many threads at once (each thread stages
 * through its own buffers). ANN_INVALID for a non-finite query or an
 * ordinal list that is not increasing or runs past the rows.
 */
typedef struct AnnB200Index AnnB200Index;
int			AnnB200IndexCreate(int device, uint32_t dims, uint64_t rows, const float *vectors,
							   AnnB200Index **index);

/*
 * The same index with its FP32 rows row-sharded over ndev devices, as the
 * reference spreads an index's shards over its GPUs (placement
 * ann/server/cuvs.c:2845-2862): part p holds rows [rows*p/ndev,
 * rows*(p+1)/ndev) on devices[p] (distinct devices). AnnB200IndexSearch on
 * it searches every part at once (one host thread a part), joins the
 * parts' lists with one NCCL all-gather (AnnB200CommCreateAll,
 * AnnB200SearchSharded) and a device merge, and returns the same answer as
 * the unsharded index, bit for bit. Searches of one such index run one at a
 * time (every part must enter the exchanges in the same order). ndev == 1
 * is AnnB200IndexCreate. ANN_UNSUPPORTED without NCCL.
 */
int			AnnB200IndexCreateSharded(int ndev, const int *devices, uint32_t dims, uint64_t rows,
									  const float *vectors, AnnB200Index **index);
void		AnnB200IndexDestroy(AnnB200Index *index);
int			AnnB200IndexSearch(AnnB200Index *index, const float *queries, uint32_t nq,
							   const uint64_t *ordinals, uint64_t nordinals, uint32_t k,
							   float *out_dist, uint64_t *out_ordinal, uint32_t *out_count);

/*
 * AnnB200IndexSearch with the eligible rows as per-shard bitsets: the cached
 * filter forms the reference's server hands its backends (AnnIndexJob
 * bitsets / deviceBitsets, ann/server/backend.h:85-96; AnnIndexBitmap,
 * ann/server/indexfile.h:117-144). Shard s covers rows shard_first[s] ..
 * shard_first[s] + shard_rows[s] - 1 (increasing, disjoint); bit r of
 * bitsets[s] (word r/32, least significant bit first) marks row
 * shard_first[s] + r eligible; a NULL bitset marks none. With
 * ANNB200_BITSETS_DEVICE the bitsets are device memory on
 * AnnB200IndexDevice(index) (kept there between searches); else host
 * memory. Results as AnnB200IndexSearch. On an index with its FP32 rows on
 * one device the bitsets are expanded on the device, with no ordinal list;
 * other indexes take the rows as ordinals (device bitsets:
 * ANN_UNSUPPORTED).
 */
#define ANNB200_BITSETS_DEVICE 1u
int			AnnB200IndexSearchBitsets(AnnB200Index *index, const float *queries, uint32_t nq,
									  uint32_t nshards, const uint32_t *const *bitsets,
									  const uint64_t *shard_first, const uint64_t *shard_rows,
									  uint32_t flags, uint32_t k, float *out_dist,
									  uint64_t *out_ordinal, uint32_t *out_count);
/* 1 for an index served from a copy of its rows (quantized or FP16) with
 * the FP32 re-score of each shard's candidates, else 0. */
int			AnnB200IndexCopyRoute(const AnnB200Index *index);
/* The device holding an index's FP32 rows, or -1 (row-sharded, quantized copy). */
int			AnnB200IndexDevice(const AnnB200Index *index);
/*
 * Keep per-shard bitsets on that device (device[s]: shard s's copy, NULL
 * for a NULL bitset) -- the reference's cached-bitmap upload hook
 * (AnnIndexBitmapDevice.upload, ann/server/indexfile.h:147-165) -- and free
 * them (its release hook). ANN_UNSUPPORTED where AnnB200IndexDevice is -1.
 */
int			AnnB200IndexKeepBitsets(AnnB200Index *index, uint32_t nshards, const uint32_t *const *bitsets,
									const uint64_t *shard_rows, void **device);
void		AnnB200IndexDropBitsets(AnnB200Index *index, uint32_t nshards, void **device);

/*
 * A loaded index served from its quantized copy (manifest line
 * "quant fp8|nvfp4": vectors.e4m3 or vectors.nvfp4 + scales.e4m3, and
 * rowscale.f32, ann/common/INDEX_FORMAT.md; mapped by AnnIndexFileOpen,
 * ann/server/indexfile.c:2492-2507), for indexes whose FP32 rows do not fit
 * on the device. The codes and scales of each index shard go to the device
 * as one shard (AnnBlackwellUpload, ann/server/blackwell.c:961-1064, with
 * no repacking: the tensor-core scan reads the file's layout); the FP32 rows
 * (vectors.f32) stay in host memory, borrowed until AnnB200IndexDestroy.
 *
 * dtype ANNB200_E4M3 or ANNB200_NVFP4; block_scales NVFP4 only; nshards
 * index shards of shard_rows[s] consecutive rows (nshards 0: one shard).
 * dtype ANNB200_F16 is the same route over an FP16 copy: the manifest's
 * "dtype float16" (ann/common/INDEX_FORMAT.md; the reference keeps its
 * CAGRA dataset in FP16 and re-scores in FP32, --fp16-exact): codes are
 * host FP16 rows, or NULL to make the copy from `vectors` on the device
 * (round to nearest); no scales.
 * AnnB200IndexSearch on such an index is the reference's quantized scan
 * route (SearchGather, ann/server/cuvs.c:4585-4930): in each index shard
 * the min(k + slack, eligible) rows nearest to the query by the exact L2
 * distance of the decoded rows (ties by ordinal), slack = max(quant_slack,
 * k * slack_ratio / 100) (GatherSlack, ann/server/cuvs.c:4286-4296); their
 * FP32 rows re-scored on the device as the reference re-scores them
 * (ExactDistance, ann/server/cuvs.c:2930-2942); the best k of all shards by
 * (distance, ordinal). Like the reference's, the answer is the exact one
 * whenever the true k nearest are among each shard's candidates.
 * The FP32 rows' pages are registered for the device to read the
 * candidates' rows in place (ANN_B200_QUANT_MAPPED=0 turns this off) when
 * they take at most ANN_B200_QUANT_MAP_MAX_MB megabytes (default: a quarter
 * of physical memory, since registered pages stay locked for the index's
 * life); above that, or where registration fails, the candidates' rows are
 * copied through pinned staging.
 */
int			AnnB200IndexCreateQuant(int device, uint32_t dims, uint64_t rows, uint32_t dtype,
									const void *codes, const void *block_scales,
									const float *row_scales, const float *vectors,
									uint32_t nshards, const uint64_t *shard_rows,
									uint32_t quant_slack, uint32_t slack_ratio,
									AnnB200Index **index);

/*
 * The FP32 re-score of gathered candidate rows (device memory, current
 * device): out[q][j] = ExactDistance of rows[q][j] to queries[q]
 * (ann/server/cuvs.c:2930-2942: differences and squares in FP64 summed in
 * dimension order, the square root rounded to FP32) for j < counts[q]
 * (counts NULL: all stride). queries [nq][dims], rows [nq][stride][dims],
 * out [nq][stride] FP32. Asynchronous on stream.
 */
int			AnnB200RescoreRows(const float *queries, uint32_t nq, uint32_t dims,
							   const float *rows, uint32_t stride, const uint32_t *counts,
							   float *out, void *stream);

/*
 * The same re-score with the rows fetched by ordinal: out[q][j] =
 * ExactDistance of rows[ords[q][j]] to queries[q]. rows is any array the
 * device can read: device memory, or host memory registered and mapped for
 * the device (the quantized index route reads vectors.f32 this way where
 * the mapping can be registered). ords [nq][stride] u64, device.
 */
int			AnnB200RescoreGather(const float *queries, uint32_t nq, uint32_t dims,
								 const float *rows, const uint64_t *ords, uint32_t stride,
								 const uint32_t *counts, float *out, void *stream);

/*
 * Typed gathered jobs: the worker's gathered job (ops 7/10, AnnGatheredJob
 * and AnnGatheredExact semantics, ann/server/backend.h:45-62,
 * ann/server/cpu.c:218-276) for rows in any storage format above and a batch
 * of queries, the additive typed op the reference's protocol leaves room for
 * ("new operations get new numbers", ann/server/PROTOCOL.md:118-120): PG
 * callers with halfvec, FP8, NVFP4 or bit rows send them as they are instead
 * of converting them to FP32.
 *
 * Host memory throughout. Per job: rows x row-bytes codes (and scales) in
 * `dtype`'s format; queries FP32 [nq][dims], or packed bits
 * [nq][ceil(dims/8)] for Hamming (bit rows and Hamming go together). Each
 * query's results are every row within d_k + 1e-3*|d_k| + 1e-6 of its k-th
 * distance, sorted by (distance, row): distances[q*cap + i], ids[q*cap + i],
 * nresults[q]. status: ANN_INVALID for a bad combination, a missing scale
 * array, a non-finite query or row value (NaN codes included), a zero query
 * under cosine, or a window larger than cap (cap >= rows always has room);
 * k = 0 or rows = 0 give no results and ANN_OK. Synchronous; thread-safe
 * like search_gathered (each thread stages through its own buffers).
 */
typedef struct AnnB200TypedJob
{
	uint32_t	dtype;			/* ANNB200_F32 .. ANNB200_BIT */
	uint32_t	metric;			/* ANNB200_L2 .. ANNB200_HAMMING */
	uint32_t	dimensions;
	uint32_t	rows;
	uint32_t	nq;				/* queries in the batch */
	uint32_t	k;
	uint32_t	cap;			/* result room a query */
	uint32_t	reserved;		/* 0 */
	const void *queries;
	const void *codes;
	const void *block_scales;	/* NVFP4 only */
	const float *row_scales;	/* E4M3 and NVFP4 */
	double	   *distances;		/* [nq][cap] */
	uint32_t   *ids;			/* [nq][cap] row numbers */
	uint32_t   *nresults;		/* [nq] */
	int			status;			/* AnnStatus */
} AnnB200TypedJob;
int			AnnB200SearchTyped(AnnB200TypedJob *jobs, uint32_t n);

/*
 * Kernels this library has launched in this process (all devices). A caller
 * that times a region reads it before and after to count its launches.
 */
unsigned long long AnnB200LaunchCount(void);

/*
 * Per-stage device time, accumulated over calls when the environment sets
 * ANN_B200_KERNEL_TIMING=1 (CUDA events on each call's stream; the
 * reference's ANN_KERNEL_TIMING, ann/server/cuvs.c:6999-7060). Stages, in
 * order: 0 query preparation, 1 sample scan, 2 sample bound, 3 filter scan,
 * 4 tighten, 5 finalize (exact rescoring and ordering), 6 bitmap expansion,
 * 7 merge, 8 candidate-row gather (copies rows for the tensor scan; its time
 * is also inside stages 1 and 3), 9 coarse probe (AnnB200ProbeLists: its
 * centroid search's stages are all counted here). Fills up to n entries of
 * ms (milliseconds) and calls; reset clears the totals. Returns the number
 * of stages, or 0 when timing is off.
 */
#define ANNB200_STAGES 10
int			AnnB200StageTimes(double *ms, unsigned long long *calls, uint32_t n, int reset);

/*
 * Switch the stage timing on (1) or off (0) for later calls, whatever
 * ANN_B200_KERNEL_TIMING said; -1 only asks. Returns the previous state.
 * Timing records two CUDA events around each stage and reads them back in
 * later calls, which costs host time on the request path: a caller that
 * times its requests end to end keeps it off and samples stages apart.
 */
int			AnnB200StageTiming(int on);

#ifdef __cplusplus
}
#endif

#endif							/* ANNB200_H */
