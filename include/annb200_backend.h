/*
 * annb200_backend.h - the worker backend ABI that AnnB200Backend() fills.
 *
 * The ANN worker of the reference selects a backend as a const AnnBackend *
 * (ann/server/backend.h:114-151 in chenqin/pgvector) and calls it from its
 * lane threads. libannb200.so must be binary compatible with that header, so
 * the types below repeat its layout field for field (same order, same C
 * types); nothing else of the reference is reused. When the worker's own
 * backend.h is included first (it defines ANN_BACKEND_H), its definitions
 * are used instead and only the constructor below is added.
 *
 * Integration: declare AnnB200Backend() (or AnnB200WorkerBackend(), which
 * also serves loaded indexes) in backend.h beside AnnCpuBackend(), add
 * "--backend b200" to worker.c's selection (ann/server/worker.c:267-279) and
 * link -lannb200.
 */
#ifndef ANNB200_BACKEND_H
#define ANNB200_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifndef ANN_BACKEND_H
#define ANN_BACKEND_H

struct AnnIndexFile;

#define ANN_MAX_BYTES (64U * 1024U * 1024U)
#define ANN_MAX_DIM 16000U

/* Status codes, in the reference's order (backend.h:12-28). */
typedef enum AnnStatus
{
	ANN_OK,
	ANN_INVALID,
	ANN_UNSUPPORTED,
	ANN_STALE,
	ANN_NOMEM,
	ANN_BACKEND_ERROR,
	ANN_PENDING,
	ANN_OVERLOADED,
	ANN_TIMED_OUT,
	ANN_CANCELLED,
	ANN_CLOSED,
	ANN_MISSING,
	ANN_GENERATION
} AnnStatus;

/* An in-memory FP32 index built by op 0 (backend.h:30-37). */
typedef struct AnnIndex
{
	uint64_t	generation;
	uint32_t	rows;
	uint32_t	dimensions;
	float	   *vectors;
	void	   *backend_state;
} AnnIndex;

/* One result row: its position and distance (backend.h:39-43). */
typedef struct AnnCandidate
{
	uint32_t	id;
	double		distance;
} AnnCandidate;

/*
 * One gathered job (backend.h:45-62): a query scored against caller-supplied
 * FP32 rows; results, capacity >= rows, hold every row within the gathered
 * tolerance of the k-th distance, sorted.
 */
typedef struct AnnGatheredJob
{
	uint32_t	rows;
	uint32_t	dimensions;
	uint32_t	k;
	uint32_t	metric;
	const float *query;
	const float *vectors;
	AnnCandidate *results;
	uint32_t	nresults;
	AnnStatus	status;
} AnnGatheredJob;

/* A loaded-index hit (backend.h:64-70). */
typedef struct AnnIndexHit
{
	int64_t		key;
	float		distance;
	uint64_t	ordinal;
} AnnIndexHit;

#define ANN_ROUTE_ANN 0
#define ANN_ROUTE_FILTERED 1
#define ANN_ROUTE_EXACT 2

/* One query against a loaded index (backend.h:76-111). */
typedef struct AnnIndexJob
{
	char		name[64];
	uint32_t	dimensions;
	uint32_t	k;
	const float *query;
	const int64_t *filter;
	uint32_t	nfilter;
	int			filtered;
	const uint64_t *ordinals;
	uint32_t   *const *bitsets;
	void	   *const *deviceBitsets;
	void	   *const *deviceRows;
	AnnIndexHit *results;
	uint32_t	nresults;
	uint32_t	route;
	AnnStatus	status;
	const uint64_t *exclude;
	uint32_t	nexclude;
	uint64_t   *ownedOrdinals;
} AnnIndexJob;

/* The backend vtable, in the reference's positional order (backend.h:114-151). */
/*
 * A typed gathered job (the typed search operation, number 32, that a worker
 * built with it dispatches): host rows in a storage format (0 FP32, 1 FP16,
 * 2 FP8-E4M3 + row scales, 3 NVFP4 + block and row scales, 4 bits) and a
 * batch of queries, answered with each query's gathered-job window. The
 * layout is AnnB200TypedJob's (annb200.h).
 */
typedef struct AnnTypedJob
{
	uint32_t	dtype;
	uint32_t	metric;			/* 0 L2, 1 negative inner product, 2 cosine, 3 Hamming */
	uint32_t	dimensions;
	uint32_t	rows;
	uint32_t	nq;
	uint32_t	k;
	uint32_t	cap;			/* result room a query */
	uint32_t	reserved;
	const void *queries;		/* FP32 [nq][dimensions]; Hamming: [nq][ceil(dimensions / 8)] bytes */
	const void *codes;
	const void *block_scales;
	const float *row_scales;
	double	   *distances;		/* [nq][cap] */
	uint32_t   *ids;			/* [nq][cap] */
	uint32_t   *nresults;		/* [nq] */
	int			status;
} AnnTypedJob;

typedef struct AnnBackend
{
	const char *name;
	uint32_t	metrics;
	uint32_t	filters;
	const char *algorithm;
	const char *storage;
	int			exact;
	uint32_t	min_rows;
	uint32_t	max_k;
	AnnStatus	(*build) (AnnIndex *, uint64_t, uint32_t, uint32_t, const float *);
	AnnStatus	(*search) (const AnnIndex *, const float *, uint32_t,
						   const uint32_t *, uint32_t, uint32_t,
						   AnnCandidate *, uint32_t *);
	void		(*destroy) (AnnIndex *);
	void		(*search_gathered) (AnnGatheredJob *, uint32_t);
	uint64_t	(*device_jobs) (void);
	AnnStatus	(*load_index) (const char *, const char *);
	void		(*search_index) (AnnIndexJob *, uint32_t);
	const char *(*lost) (void);
	int			(*scan_preferred) (const struct AnnIndexFile *file, uint32_t k);
	/*
	 * An addition after the reference's last slot: typed gathered jobs for
	 * the typed search operation; sets each job's status. A worker built
	 * without the operation never reads it.
	 */
	void		(*search_typed) (AnnTypedJob *, uint32_t);
} AnnBackend;

#define ANN_EXIT_DEVICE_LOST 70
#define ANN_GATHERED_TOLERANCE 1e-3

#endif							/* ANN_BACKEND_H */

#ifdef __cplusplus
extern "C"
{
#endif

/*
 * The B200 backend: "b200", metrics L2/IP/cosine (mask 7), exact. Gathered
 * jobs and in-memory index searches run on the calling thread's CUDA device
 * through AnnB200Search. Loaded on-disk indexes live in the worker's own
 * registry, so this vtable leaves load_index and search_index NULL;
 * AnnB200WorkerBackend(), compiled inside the worker's build
 * (pgvector_b200/csrc/worker_index.c), is this vtable with them filled.
 */
const AnnBackend *AnnB200Backend(void);

#ifdef __cplusplus
}
#endif

#endif							/* ANNB200_BACKEND_H */
