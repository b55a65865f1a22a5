/*
 * backend.c - AnnB200Backend(): the worker backend vtable over libannb200.
 *
 * Drop-in for the reference worker's backend slot (ann/server/backend.h:
 * 114-151): gathered jobs (ops 7/10; the cpu backend's SearchGathered,
 * ann/server/cpu.c:218-283) and in-memory index build/search/destroy (ops
 * 0-6; cpu.c:10-154) run on a CUDA device through AnnB200Search, which
 * returns the CPU worker's exact results. Loaded on-disk indexes live in the
 * worker's own registry, so their load_index / search_index are filled by
 * AnnB200WorkerBackend() (worker_index.c, compiled inside the worker's
 * build); this vtable leaves them NULL.
 *
 * Threading: the worker calls search_gathered from many lane threads at once
 * (ann/server/server.c:1541). Each thread keeps its own device context (a
 * stream, a reusable shard and staging buffers, like the reference's
 * _Thread_local lane state in ann/server/cuvs.c:103-124); lanes spread over
 * the visible devices round robin.
 *
 * Host-side fault injection for tests, in the manner of the reference's mock
 * GPU backend (ann/server/mockgpu.c:148-200): ANN_B200_LOST_AFTER=N makes
 * every device job after the first N fail with ANN_BACKEND_ERROR, and lost()
 * then names a simulated lost context, so the worker's exit-70 path can be
 * exercised without faulting a GPU.
 */
#define _GNU_SOURCE
#include "../../include/annb200.h"
#include "../../include/annb200_backend.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

static atomic_ullong DeviceJobs;
static atomic_uint NextLane;
static atomic_int LostSimulated;
static char LostReason[256];
static pthread_mutex_t LostLock = PTHREAD_MUTEX_INITIALIZER;

/* Staging of one chunk of a quantized index search's candidate rows. */
typedef struct QuantSlot
{
	float	   *stage;			/* device: gathered candidate rows */
	size_t		stageBytes;
	float	   *hostStage;		/* pinned */
	size_t		hostStageBytes;
	float	   *rescored;		/* device: their FP32 distances */
	size_t		rescoredBytes;
	float	   *hostRescored;	/* pinned */
	size_t		hostRescoredBytes;
	uint32_t   *candCounts;		/* device: candidates a query */
	size_t		candCountsBytes;
	uint32_t   *hostCandCounts; /* pinned */
	size_t		hostCandCountsBytes;
	uint64_t   *ords;			/* device: candidate ordinals (mapped rows) */
	size_t		ordsBytes;
} QuantSlot;

typedef struct Lane
{
	int			ready;
	int			device;
	cudaStream_t stream;
	AnnB200Shard *shard;
	void	   *rows;			/* device: the job's FP32 rows */
	size_t		rowsBytes;
	float	   *query;			/* device */
	size_t		queryBytes;
	uint32_t   *ids;			/* device: candidate ids of an index search */
	size_t		idsBytes;
	double	   *dist;			/* device results */
	int64_t    *id;
	uint32_t   *count;
	size_t		resultCap;
	uint32_t   *counts;			/* device: per-query counts of a batch */
	size_t		countsBytes;
	uint8_t    *scales;			/* device: a typed job's NVFP4 block scales */
	size_t		scalesBytes;
	float	   *rowScales;		/* device: a typed job's row scales */
	size_t		rowScalesBytes;
	double	   *hostDist;		/* pinned result staging */
	int64_t    *hostId;
	size_t		hostCap;
	/* a batch of gathered jobs: their rows and queries staged in pinned memory */
	float	   *hostIn;
	size_t		hostInBytes;
	uint32_t   *hostCounts;		/* pinned */
	size_t		hostCountsBytes;
	int32_t    *statuses;		/* device: a status a job */
	size_t		statusesBytes;
	/* a quantized index's FP32 re-score: two chunks of queries in flight */
	int			rescoreReady;
	cudaStream_t rescoreStream;
	cudaEvent_t rescoreDone[2];
	QuantSlot	slot[2];
} Lane;

static _Thread_local Lane LaneState;

/* Per in-memory index: its rows on the device of the lane that built it. */
typedef struct IndexState
{
	int			device;
	AnnB200Shard *shard;
	void	   *rows;
} IndexState;

static long
EnvLong(const char *name, long fallback)
{
	const char *v = getenv(name);

	return v && *v ? strtol(v, NULL, 10) : fallback;
}

/* Whether a simulated device loss has been reached; counts this job. */
static int
InjectLost(void)
{
	long		after = EnvLong("ANN_B200_LOST_AFTER", -1);

	if (after < 0)
		return 0;
	if ((long) atomic_load(&DeviceJobs) >= after)
	{
		pthread_mutex_lock(&LostLock);
		if (!atomic_load(&LostSimulated))
		{
			snprintf(LostReason, sizeof(LostReason),
					 "GPU context lost (simulated after %ld device jobs)", after);
			atomic_store(&LostSimulated, 1);
		}
		pthread_mutex_unlock(&LostLock);
		return 1;
	}
	return 0;
}

static int
Grow(void **p, size_t *have, size_t want)
{
	if (want <= *have)
		return 1;
	if (*p)
		cudaFree(*p);
	*p = NULL;
	*have = 0;
	if (cudaMalloc(p, want) != cudaSuccess)
		return 0;
	*have = want;
	return 1;
}

static int
GrowHost(void **p, size_t *have, size_t want)
{
	if (want <= *have)
		return 1;
	if (*p)
		cudaFreeHost(*p);
	*p = NULL;
	*have = 0;
	if (cudaMallocHost(p, want) != cudaSuccess)
		return 0;
	*have = want;
	return 1;
}

static Lane *
LaneGet(void)
{
	Lane	   *lane = &LaneState;
	int			devices;

	if (lane->ready)
	{
		cudaSetDevice(lane->device);
		return lane;
	}
	devices = AnnB200DeviceCount();
	if (devices <= 0)
		return NULL;
	lane->device = (int) (atomic_fetch_add(&NextLane, 1) % (unsigned) devices);
	if (cudaSetDevice(lane->device) != cudaSuccess ||
		cudaStreamCreateWithFlags(&lane->stream, cudaStreamNonBlocking) != cudaSuccess)
		return NULL;
	lane->ready = 1;
	return lane;
}

/* Room for n results of one query on the device and in pinned memory. */
static int
LaneResults(Lane *lane, size_t n)
{
	size_t		dcap = lane->resultCap * sizeof(double);
	size_t		icap = lane->resultCap * sizeof(int64_t);
	size_t		hcap = lane->hostCap * sizeof(double);
	size_t		hicap = lane->hostCap * sizeof(int64_t);
	size_t		ccap = lane->resultCap ? 16 : 0;

	if (n == 0)
		n = 1;
	if (n > lane->resultCap)
	{
		if (!Grow((void **) &lane->dist, &dcap, n * sizeof(double)) ||
			!Grow((void **) &lane->id, &icap, n * sizeof(int64_t)) ||
			!Grow((void **) &lane->count, &ccap, 16))
			return 0;
		lane->resultCap = n;
	}
	if (n > lane->hostCap)
	{
		if (!GrowHost((void **) &lane->hostDist, &hcap, n * sizeof(double)) ||
			!GrowHost((void **) &lane->hostId, &hicap, n * sizeof(int64_t)))
			return 0;
		lane->hostCap = n;
	}
	return 1;
}

static int
AllFinite(const float *v, size_t n)
{
	for (size_t i = 0; i < n; i++)
		if (!isfinite(v[i]))
			return 0;
	return 1;
}

/*
 * A gathered job with no rows to search or k = 0 still answers as the
 * reference does (AnnGatheredExact, ann/server/cpu.c:218-276): ANN_INVALID
 * for a non-finite query or row value (cpu.c:97-99, 246-251) or a zero
 * query under cosine, else no results.
 */
#define GATHER_MAX_THREADS 32

/* One share of a gathered batch's staging copies: jobs [begin, end). */
typedef struct StageTask
{
	AnnGatheredJob *jobs;
	const uint32_t *slot;
	const size_t *at;			/* each job's start in the staging area (floats) */
	float	   *dst;
	uint32_t	begin;
	uint32_t	end;
} StageTask;

static size_t Align16(size_t floats);

static void *
StageJobs(void *arg)
{
	StageTask  *t = arg;

	for (uint32_t b = t->begin; b < t->end; b++)
	{
		const AnnGatheredJob *job = &t->jobs[t->slot[b]];
		size_t		rv = (size_t) job->rows * job->dimensions;

		memcpy(t->dst + t->at[b], job->vectors, rv * sizeof(float));
		memcpy(t->dst + t->at[b] + Align16(rv), job->query, job->dimensions * sizeof(float));
	}
	return NULL;
}

/*
 * Copy the batch's rows and queries into pinned staging on up to
 * ANN_B200_GATHER_THREADS host threads (default the online CPUs, at most
 * 16; about 8 MB a thread at least): a lane's batch of op-10 chunks is
 * hundreds of MB, which one thread copies at a fraction of the memory
 * bandwidth.
 */
static void
StageAll(AnnGatheredJob *jobs, const uint32_t *slot, const size_t *at, uint32_t m, float *dst, size_t bytes)
{
	StageTask	task[GATHER_MAX_THREADS];
	pthread_t	tid[GATHER_MAX_THREADS];
	int			started[GATHER_MAX_THREADS] = {0};
	long		threads = EnvLong("ANN_B200_GATHER_THREADS", 0);

	if (threads <= 0)
	{
		threads = sysconf(_SC_NPROCESSORS_ONLN);
		if (threads > 16)
			threads = 16;
	}
	if (threads > GATHER_MAX_THREADS)
		threads = GATHER_MAX_THREADS;
	if ((size_t) threads > bytes / (8u << 20) + 1)
		threads = (long) (bytes / (8u << 20) + 1);
	if (threads > (long) m)
		threads = m;
	if (threads < 1)
		threads = 1;
	for (long t = 0; t < threads; t++)
	{
		task[t] = (StageTask) {jobs, slot, at, dst, (uint32_t) ((uint64_t) m * t / threads),
			(uint32_t) ((uint64_t) m * (t + 1) / threads)};
		if (t > 0)
			started[t] = pthread_create(&tid[t], NULL, StageJobs, &task[t]) == 0;
	}
	StageJobs(&task[0]);
	for (long t = 1; t < threads; t++)
	{
		if (started[t])
			pthread_join(tid[t], NULL);
		else
			StageJobs(&task[t]);
	}
}

/* floats rounded up to 64 bytes: each staged job's rows and query start aligned */
static size_t
Align16(size_t floats)
{
	return (floats + 15) & ~(size_t) 15;
}

/* A finite query, with a nonzero norm under cosine (cpu.c:97-99, 139-142). */
static int
QueryValid(const AnnGatheredJob *job)
{
	double		qnorm = 0;

	if (!AllFinite(job->query, job->dimensions))
		return 0;
	for (uint32_t d = 0; d < job->dimensions; d++)
		qnorm += (double) job->query[d] * job->query[d];
	return job->metric != 2 || qnorm != 0;
}

static AnnStatus
TrivialStatus(const AnnGatheredJob *job)
{
	double		qnorm = 0;

	if (!AllFinite(job->query, job->dimensions) ||
		!AllFinite(job->vectors, (size_t) job->rows * job->dimensions))
		return ANN_INVALID;
	for (uint32_t d = 0; d < job->dimensions; d++)
		qnorm += (double) job->query[d] * job->query[d];
	return job->metric == 2 && qnorm == 0 ? ANN_INVALID : ANN_OK;
}

/* ---------------------------------------------------------------- loaded indexes */

#define INDEX_MAX_DEVICES 64

struct AnnB200Index
{
	int			device;
	uint32_t	dims;
	uint64_t	rows;
	AnnB200Shard *shard;		/* owns the device copy of the FP32 rows
								 * (NULL for an index served from its
								 * quantized copy) */
	/* an index served from its quantized copy */
	uint32_t	nshards;
	AnnB200Shard **shards;		/* per index shard: its codes on the device */
	uint64_t   *bounds;			/* nshards + 1 row bounds */
	const float *vectors;		/* host FP32 rows (borrowed) */
	const float *mapped;		/* the same rows as the device reads them, when
								 * their pages could be registered; else NULL */
	void	   *registered;		/* start of the registered pages */
	uint32_t	quantSlack;
	uint32_t	slackRatio;
	/* an index whose FP32 rows are row-sharded over several devices */
	uint32_t	nparts;
	AnnB200Shard **parts;		/* part p: rows partBounds[p] .. [p+1] */
	uint64_t   *partBounds;
	int		   *partDevices;
	AnnB200Comm **comms;		/* one NCCL rank a part */
	Lane	   *partLanes;		/* staging a part, used under searchLock */
	pthread_mutex_t searchLock; /* one search at a time: every part enters
								 * the same exchanges in the same order */
};

/* Per thread and device: staging for index searches on that device. */
static _Thread_local Lane IndexLanes[INDEX_MAX_DEVICES];

static Lane *
LaneOn(int device)
{
	Lane	   *lane;

	if (device < 0 || device >= INDEX_MAX_DEVICES)
		return NULL;
	lane = &IndexLanes[device];
	if (cudaSetDevice(device) != cudaSuccess)
		return NULL;
	if (!lane->ready)
	{
		lane->device = device;
		if (cudaStreamCreateWithFlags(&lane->stream, cudaStreamNonBlocking) != cudaSuccess)
			return NULL;
		lane->ready = 1;
	}
	return lane;
}

/* Free a lane's stream and buffers (a part's lane, owned by its index). */
static void
LaneRelease(Lane *lane)
{
	if (!lane->ready)
		return;
	cudaSetDevice(lane->device);
	cudaStreamSynchronize(lane->stream);
	cudaStreamDestroy(lane->stream);
	cudaFree(lane->query);
	cudaFree(lane->ids);
	cudaFree(lane->dist);
	cudaFree(lane->id);
	cudaFree(lane->count);
	cudaFree(lane->counts);
	cudaFreeHost(lane->hostDist);
	cudaFreeHost(lane->hostId);
	memset(lane, 0, sizeof(*lane));
}

int
AnnB200IndexCreate(int device, uint32_t dims, uint64_t rows, const float *vectors, AnnB200Index **out)
{
	AnnB200Index *ix;
	int			devices = AnnB200DeviceCount();
	int			prev = 0;
	int			status;

	if (out == NULL)
		return ANN_INVALID;
	*out = NULL;
	if (dims == 0 || rows == 0 || rows > UINT32_MAX || vectors == NULL)
		return ANN_INVALID;
	if (devices <= 0)
		return ANN_BACKEND_ERROR;
	if (device < 0)
		device = (int) (atomic_fetch_add(&NextLane, 1) % (unsigned) devices);
	if (device >= devices || device >= INDEX_MAX_DEVICES)
		return ANN_INVALID;
	ix = calloc(1, sizeof(*ix));
	if (ix == NULL)
		return ANN_NOMEM;
	ix->device = device;
	ix->dims = dims;
	ix->rows = rows;
	cudaGetDevice(&prev);
	status = AnnB200ShardCreate(device, ANNB200_F32, dims, rows, vectors, NULL, NULL, 0, ANNB200_SHARD_HOST,
								NULL, &ix->shard);
	cudaSetDevice(prev);
	if (status != ANN_OK)
	{
		free(ix);
		return status;
	}
	*out = ix;
	return ANN_OK;
}

/*
 * An index whose FP32 rows are row-sharded over several devices, as the
 * reference spreads an index's shards over its GPUs (placement
 * ann/server/cuvs.c:2845-2862): part p holds an equal share of the rows
 * (global ordinals as its ids) on devices[p], and one NCCL rank a part
 * (AnnB200CommCreateAll) joins the parts' lists in AnnB200IndexSearch.
 * ndev == 1 is AnnB200IndexCreate on that device.
 */
int
AnnB200IndexCreateSharded(int ndev, const int *devices, uint32_t dims, uint64_t rows, const float *vectors,
						  AnnB200Index **out)
{
	AnnB200Index *ix;
	int			prev = 0;
	int			status = ANN_OK;

	if (out == NULL)
		return ANN_INVALID;
	*out = NULL;
	if (ndev < 1 || devices == NULL || dims == 0 || rows == 0 || vectors == NULL || (uint64_t) ndev > rows)
		return ANN_INVALID;
	if (ndev == 1)
		return AnnB200IndexCreate(devices[0], dims, rows, vectors, out);
	for (int i = 0; i < ndev; i++)
		if (devices[i] < 0 || devices[i] >= AnnB200DeviceCount() || devices[i] >= INDEX_MAX_DEVICES)
			return ANN_INVALID;
	ix = calloc(1, sizeof(*ix));
	if (ix == NULL)
		return ANN_NOMEM;
	ix->device = devices[0];
	ix->dims = dims;
	ix->rows = rows;
	ix->nparts = (uint32_t) ndev;
	pthread_mutex_init(&ix->searchLock, NULL);
	ix->parts = calloc(ndev, sizeof(*ix->parts));
	ix->partBounds = calloc(ndev + 1, sizeof(*ix->partBounds));
	ix->partDevices = calloc(ndev, sizeof(*ix->partDevices));
	ix->comms = calloc(ndev, sizeof(*ix->comms));
	ix->partLanes = calloc(ndev, sizeof(*ix->partLanes));
	if (!ix->parts || !ix->partBounds || !ix->partDevices || !ix->comms || !ix->partLanes)
	{
		AnnB200IndexDestroy(ix);
		return ANN_NOMEM;
	}
	for (int p = 0; p < ndev; p++)
	{
		ix->partDevices[p] = devices[p];
		ix->partBounds[p + 1] = rows * (uint64_t) (p + 1) / (uint64_t) ndev;
	}
	cudaGetDevice(&prev);
	for (int p = 0; status == ANN_OK && p < ndev; p++)
	{
		uint64_t	lo = ix->partBounds[p];

		status = AnnB200ShardCreate(devices[p], ANNB200_F32, dims, ix->partBounds[p + 1] - lo,
									vectors + lo * dims, NULL, NULL, (int64_t) lo, ANNB200_SHARD_HOST, NULL,
									&ix->parts[p]);
	}
	if (status == ANN_OK)
		status = AnnB200CommCreateAll(ndev, devices, ix->comms);
	cudaSetDevice(prev);
	if (status != ANN_OK)
	{
		AnnB200IndexDestroy(ix);
		return status;
	}
	*out = ix;
	return ANN_OK;
}

void
AnnB200IndexDestroy(AnnB200Index *ix)
{
	if (ix == NULL)
		return;
	AnnB200ShardDestroy(ix->shard);
	for (uint32_t s = 0; ix->shards && s < ix->nshards; s++)
		AnnB200ShardDestroy(ix->shards[s]);
	for (uint32_t p = 0; p < ix->nparts; p++)
	{
		if (ix->parts)
			AnnB200ShardDestroy(ix->parts[p]);
		if (ix->comms)
			AnnB200CommDestroy(ix->comms[p]);
		if (ix->partLanes)
			LaneRelease(&ix->partLanes[p]);
	}
	if (ix->nparts)
		pthread_mutex_destroy(&ix->searchLock);
	free(ix->parts);
	free(ix->partBounds);
	free(ix->partDevices);
	free(ix->comms);
	free(ix->partLanes);
	if (ix->registered)
	{
		int			prev = 0;

		cudaGetDevice(&prev);
		cudaSetDevice(ix->device);
		cudaHostUnregister(ix->registered);
		cudaSetDevice(prev);
	}
	free(ix->shards);
	free(ix->bounds);
	free(ix);
}

/*
 * The most bytes of FP32 rows MapRows registers: ANN_B200_QUANT_MAP_MAX_MB,
 * else a quarter of the machine's physical memory. Registering pins the
 * pages for the index's whole life, so an index whose rows are larger (a
 * mapped vectors.f32 of hundreds of GB) keeps the copy path instead of
 * reading in and locking that much of the page cache.
 */
static uint64_t
MapCapBytes(void)
{
	long		mb = EnvLong("ANN_B200_QUANT_MAP_MAX_MB", -1);
	long		pages = sysconf(_SC_PHYS_PAGES);
	long		page = sysconf(_SC_PAGESIZE);

	if (mb >= 0)
		return (uint64_t) mb << 20;
	if (pages <= 0 || page <= 0)
		return 0;
	return (uint64_t) pages * (uint64_t) page / 4;
}

/*
 * Register the pages of a quantized index's FP32 rows for the device to read
 * them in place (read-only where the driver supports it, as a read-only file
 * mapping needs), when they are within MapCapBytes(). Where they are larger
 * or registration fails the rows are copied through pinned staging instead;
 * nothing else changes.
 */
static void
MapRows(AnnB200Index *ix)
{
	/*
	 * Exactly the rows' bytes: a range rounded out to whole pages could take
	 * in the ends of neighbouring allocations (heap arrays sit side by side),
	 * and a later copy from one of them would then start inside a
	 * registered range and run past it, which the runtime refuses.
	 */
	uintptr_t	start = (uintptr_t) ix->vectors;
	uintptr_t	base = start;
	size_t		len = (size_t) ix->rows * ix->dims * sizeof(float);
	unsigned	flags = cudaHostRegisterMapped | cudaHostRegisterPortable;
	void	   *dev = NULL;
	int			debug = EnvLong("ANN_B200_DEBUG", 0) > 0;
	uint64_t	cap = MapCapBytes();

	if ((uint64_t) len > cap)
	{
		if (debug)
			fprintf(stderr, "annb200 quantized index: FP32 rows copied through pinned staging "
					"(%zu bytes, above the %llu-byte registration cap)\n", len, (unsigned long long) cap);
		return;
	}
	if (cudaSetDevice(ix->device) != cudaSuccess)
		return;
	if (cudaHostRegister((void *) base, len, flags | cudaHostRegisterReadOnly) != cudaSuccess)
	{
		(void) cudaGetLastError();
		if (cudaHostRegister((void *) base, len, flags) != cudaSuccess)
		{
			(void) cudaGetLastError();
			if (debug)
				fprintf(stderr, "annb200 quantized index: FP32 rows copied through pinned staging "
						"(registration failed)\n");
			return;
		}
	}
	if (cudaHostGetDevicePointer(&dev, (void *) base, 0) != cudaSuccess || dev == NULL)
	{
		(void) cudaGetLastError();
		cudaHostUnregister((void *) base);
		if (debug)
			fprintf(stderr, "annb200 quantized index: FP32 rows copied through pinned staging "
					"(no device address)\n");
		return;
	}
	ix->registered = (void *) base;
	ix->mapped = (const float *) ((const char *) dev + (start - base));
	if (debug)
		fprintf(stderr, "annb200 quantized index: FP32 rows read in place (%zu bytes registered)\n", len);
}

int
AnnB200IndexCreateQuant(int device, uint32_t dims, uint64_t rows, uint32_t dtype, const void *codes,
						const void *block_scales, const float *row_scales, const float *vectors, uint32_t nshards,
						const uint64_t *shard_rows, uint32_t quant_slack, uint32_t slack_ratio, AnnB200Index **out)
{
	AnnB200Index *ix;
	int			devices = AnnB200DeviceCount();
	int			prev = 0;
	int			status = ANN_OK;
	uint64_t	blocks = (dims + 15) / 16;
	uint64_t	rowBytes = dtype == ANNB200_F16 ? (uint64_t) dims * 2 : blocks * (dtype == ANNB200_NVFP4 ? 8 : 16);
	uint64_t	total = 0;
	int			half = dtype == ANNB200_F16;

	if (out == NULL)
		return ANN_INVALID;
	*out = NULL;
	if (dims == 0 || rows == 0 || rows > UINT32_MAX || vectors == NULL ||
		(dtype != ANNB200_E4M3 && dtype != ANNB200_NVFP4 && !half) ||
		(!half && (codes == NULL || row_scales == NULL)) || (dtype == ANNB200_NVFP4 && block_scales == NULL) ||
		(nshards && shard_rows == NULL))
		return ANN_INVALID;
	for (uint32_t s = 0; s < nshards; s++)
	{
		if (shard_rows[s] == 0)
			return ANN_INVALID;
		total += shard_rows[s];
	}
	if (nshards && total != rows)
		return ANN_INVALID;
	if (devices <= 0)
		return ANN_BACKEND_ERROR;
	if (device < 0)
		device = (int) (atomic_fetch_add(&NextLane, 1) % (unsigned) devices);
	if (device >= devices || device >= INDEX_MAX_DEVICES)
		return ANN_INVALID;
	ix = calloc(1, sizeof(*ix));
	if (ix == NULL)
		return ANN_NOMEM;
	ix->device = device;
	ix->dims = dims;
	ix->rows = rows;
	ix->vectors = vectors;
	ix->quantSlack = quant_slack;
	ix->slackRatio = slack_ratio;
	ix->nshards = nshards ? nshards : 1;
	ix->shards = calloc(ix->nshards, sizeof(*ix->shards));
	ix->bounds = calloc(ix->nshards + 1, sizeof(*ix->bounds));
	if (ix->shards == NULL || ix->bounds == NULL)
	{
		AnnB200IndexDestroy(ix);
		return ANN_NOMEM;
	}
	for (uint32_t s = 0; s < ix->nshards; s++)
		ix->bounds[s + 1] = ix->bounds[s] + (nshards ? shard_rows[s] : rows);
	cudaGetDevice(&prev);
	for (uint32_t s = 0; status == ANN_OK && s < ix->nshards; s++)
	{
		uint64_t	first = ix->bounds[s];

		if (half && codes == NULL)	/* the FP32 rows kept as FP16 on the device */
			status = AnnB200ShardCreate(device, ANNB200_F16, dims, ix->bounds[s + 1] - first, vectors + first * dims,
										NULL, NULL, (int64_t) first, ANNB200_SHARD_HOST | ANNB200_SHARD_F32_TO_F16,
										NULL, &ix->shards[s]);
		else
			status = AnnB200ShardCreate(device, dtype, dims, ix->bounds[s + 1] - first,
										(const uint8_t *) codes + first * rowBytes,
										block_scales ? (const uint8_t *) block_scales + first * blocks : NULL,
										row_scales ? row_scales + first : NULL, (int64_t) first, ANNB200_SHARD_HOST,
										NULL, &ix->shards[s]);
	}
	if (status == ANN_OK && EnvLong("ANN_B200_QUANT_MAPPED", 1) != 0)
		MapRows(ix);
	cudaSetDevice(prev);
	if (status != ANN_OK)
	{
		AnnB200IndexDestroy(ix);
		return status;
	}
	*out = ix;
	return ANN_OK;
}

/* The slice of sorted `ordinals` in [lo, hi). */
static void
Slice(const uint64_t *ordinals, uint64_t n, uint64_t lo, uint64_t hi, uint64_t *start, uint64_t *len)
{
	uint64_t	a = 0,
				b = n;

	while (a < b)
	{
		uint64_t	m = a + (b - a) / 2;

		if (ordinals[m] < lo)
			a = m + 1;
		else
			b = m;
	}
	*start = a;
	b = n;
	while (a < b)
	{
		uint64_t	m = a + (b - a) / 2;

		if (ordinals[m] < hi)
			a = m + 1;
		else
			b = m;
	}
	*len = a - *start;
}

/* Reorder a[0..n) so that a[0..r) holds its r smallest keys (any order): quickselect. */
static void
SelectSmallest(uint64_t *a, uint32_t n, uint32_t r)
{
	uint32_t	lo = 0,
				hi = n;

	if (r == 0 || r >= n)
		return;
	while (hi - lo > 1)
	{
		uint64_t	x = a[lo],
					y = a[lo + (hi - lo) / 2],
					z = a[hi - 1];
		uint64_t	pivot = x < y ? (y < z ? y : (x < z ? z : x)) : (x < z ? x : (y < z ? z : y));
		uint32_t	i = lo,
					j = lo,
					e = hi;

		/* three-way partition: [lo, i) < pivot, [i, e) == pivot, [e, hi) > pivot */
		while (j < e)
		{
			uint64_t	v = a[j];

			if (v < pivot)
			{
				a[j] = a[i];
				a[i++] = v;
				j++;
			}
			else if (v > pivot)
			{
				a[j] = a[--e];
				a[e] = v;
			}
			else
				j++;
		}
		if (r <= i)
			hi = i;
		else if (r <= e)
			return;
		else
			lo = e;
	}
}

static int
KeyCompare(const void *a, const void *b)
{
	uint64_t	x = *(const uint64_t *) a,
				y = *(const uint64_t *) b;

	return x < y ? -1 : x > y;
}

static double
NowMs(void)
{
	struct timespec ts;

	clock_gettime(CLOCK_MONOTONIC, &ts);
	return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

/* One share of a chunk's candidate-row copies (queries [begin, end)). */
typedef struct GatherTask
{
	const AnnB200Index *ix;
	Lane	   *lane;
	QuantSlot  *slot;			/* where the rows go */
	const uint32_t *counts;		/* per shard and query: candidates found */
	uint64_t   *cand;			/* out: each query's candidate ordinals */
	const uint64_t *want;
	const uint64_t *off;
	size_t		m;
	uint64_t	C;
	uint32_t	begin;
	uint32_t	end;
} GatherTask;

static void *
GatherRows(void *arg)
{
	GatherTask *t = arg;
	const AnnB200Index *ix = t->ix;
	Lane	   *lane = t->lane;
	QuantSlot  *slot = t->slot;
	uint32_t	dims = ix->dims;

	for (uint32_t i = t->begin; i < t->end; i++)
	{
		uint32_t	pos = 0;

		for (uint32_t s = 0; s < ix->nshards; s++)
			for (uint32_t j = 0; t->want[s] && j < t->counts[(size_t) s * t->m + i]; j++)
			{
				uint64_t	ord = (uint64_t) lane->hostId[t->m * t->off[s] + (size_t) i * t->want[s] + j];

				memcpy(slot->hostStage + ((size_t) i * t->C + pos) * dims, ix->vectors + ord * dims,
					   sizeof(float) * dims);
				t->cand[(size_t) i * t->C + pos++] = ord;
			}
		slot->hostCandCounts[i] = pos;
	}
	return NULL;
}

/* Each query's candidate ordinals, shard after shard, without their rows. */
static void
ListCandidates(const AnnB200Index *ix, Lane *lane, QuantSlot *slot, const uint32_t *counts, uint64_t *cand,
			   const uint64_t *want, const uint64_t *off, size_t m, uint64_t C, uint32_t mm)
{
	for (uint32_t i = 0; i < mm; i++)
	{
		uint32_t	pos = 0;

		for (uint32_t s = 0; s < ix->nshards; s++)
			for (uint32_t j = 0; want[s] && j < counts[(size_t) s * m + i]; j++)
				cand[(size_t) i * C + pos++] = (uint64_t) lane->hostId[m * off[s] + (size_t) i * want[s] + j];
		slot->hostCandCounts[i] = pos;
	}
}


/*
 * Copy the candidates' FP32 rows of queries [0, mm) into pinned staging:
 * scattered row reads from host memory, split over threads by query
 * (ANN_B200_GATHER_THREADS, default the online CPUs up to 16).
 */
static void
GatherAll(const AnnB200Index *ix, Lane *lane, QuantSlot *slot, const uint32_t *counts, uint64_t *cand,
		  const uint64_t *want, const uint64_t *off, size_t m, uint64_t C, uint32_t mm)
{
	GatherTask	task[GATHER_MAX_THREADS];
	pthread_t	tid[GATHER_MAX_THREADS];
	int			started[GATHER_MAX_THREADS] = {0};
	long		threads = EnvLong("ANN_B200_GATHER_THREADS", 0);
	uint64_t	bytes = (uint64_t) mm * C * ix->dims * sizeof(float);

	if (threads <= 0)
	{
		threads = sysconf(_SC_NPROCESSORS_ONLN);
		if (threads > 16)
			threads = 16;
	}
	if (threads > GATHER_MAX_THREADS)
		threads = GATHER_MAX_THREADS;
	/* about 4 MB of rows a thread at least */
	if ((uint64_t) threads > bytes / (4u << 20) + 1)
		threads = (long) (bytes / (4u << 20) + 1);
	if (threads > (long) mm)
		threads = mm;
	if (threads < 1)
		threads = 1;
	for (long t = 0; t < threads; t++)
	{
		task[t] = (GatherTask) {ix, lane, slot, counts, cand, want, off, m, C,
			(uint32_t) ((uint64_t) mm * t / threads), (uint32_t) ((uint64_t) mm * (t + 1) / threads)};
		if (t > 0)
			started[t] = pthread_create(&tid[t], NULL, GatherRows, &task[t]) == 0;
	}
	GatherRows(&task[0]);
	for (long t = 1; t < threads; t++)
	{
		if (started[t])
			pthread_join(tid[t], NULL);
		else
			GatherRows(&task[t]);	/* no thread: copy this share here */
	}
}


/*
 * AnnB200IndexSearch on an index served from its quantized copy: the
 * reference's quantized scan route (SearchGather, ann/server/cuvs.c:
 * 4585-4930). Per index shard, the exact search of the codes picks the
 * min(k + slack, eligible) candidates (slack as GatherSlack, cuvs.c:
 * 4286-4296); their FP32 rows are copied from host memory into pinned
 * staging and re-scored on the device (ExactDistance, cuvs.c:2930-2942);
 * the k best of all shards' candidates by (distance, ordinal) -- the
 * reference's per-shard (distance, key) sort, cut at k, and tree merge
 * (cuvs.c:4919-4930) keep the same k, key order being ordinal order.
 * Queries are on the device (lane->query); results go to host memory.
 * Queries run in chunks whose candidate rows fill one staging slot
 * (ANN_B200_QUANT_STAGE_MB, default 256 MB); the host copies one chunk's
 * rows while the device re-scores the previous chunk's.
 */
static int
QuantSearch(AnnB200Index *ix, Lane *lane, uint32_t nq, const uint64_t *ordinals, uint64_t nordinals, uint32_t k,
			float *out_dist, uint64_t *out_ordinal, uint32_t *out_count)
{
	uint32_t	S = ix->nshards;
	uint32_t	dims = ix->dims;
	uint64_t	ratio = (uint64_t) k * ix->slackRatio / 100;
	uint64_t	want = (uint64_t) k + (ratio > ix->quantSlack ? ratio : ix->quantSlack);
	uint64_t   *start = calloc(S, sizeof(uint64_t));
	uint64_t   *elig = calloc(S, sizeof(uint64_t));
	uint64_t   *want_s = calloc(S, sizeof(uint64_t));
	uint64_t   *off = calloc(S, sizeof(uint64_t));
	uint32_t   *local = NULL;
	uint32_t   *counts = NULL;
	uint64_t   *cand[2] = {NULL, NULL};
	uint64_t   *keys = NULL;
	uint64_t	C = 0;
	size_t		m;
	uint32_t	chunks;
	int			status = ANN_OK;
	int			debug = EnvLong("ANN_B200_DEBUG", 0) > 0;
	size_t		stage = (size_t) EnvLong("ANN_B200_QUANT_STAGE_MB", 256) << 20;

	if (start == NULL || elig == NULL || want_s == NULL || off == NULL)
		status = ANN_NOMEM;
	for (uint32_t s = 0; status == ANN_OK && s < S; s++)
	{
		if (ordinals)
			Slice(ordinals, nordinals, ix->bounds[s], ix->bounds[s + 1], &start[s], &elig[s]);
		else
			elig[s] = ix->bounds[s + 1] - ix->bounds[s];
		want_s[s] = want < elig[s] ? want : elig[s];
		off[s] = C;
		C += want_s[s];
	}
	if (status == ANN_OK && C == 0)
		goto done;
	if (status == ANN_OK && C > UINT32_MAX / 2)
		status = ANN_UNSUPPORTED;
	m = stage / ((size_t) C * dims * sizeof(float) + 1);
	if (m == 0)
		m = 1;
	if (m > nq)
		m = nq;

	/* eligible rows of each shard, as shard-local row numbers */
	if (status == ANN_OK && ordinals)
	{
		local = malloc(sizeof(*local) * nordinals);
		if (local == NULL ||
			!Grow((void **) &lane->ids, &lane->idsBytes, nordinals * sizeof(uint32_t)))
			status = ANN_NOMEM;
		for (uint32_t s = 0; status == ANN_OK && s < S; s++)
			for (uint64_t i = start[s]; i < start[s] + elig[s]; i++)
				local[i] = (uint32_t) (ordinals[i] - ix->bounds[s]);
		if (status == ANN_OK &&
			cudaMemcpyAsync(lane->ids, local, nordinals * sizeof(uint32_t), cudaMemcpyHostToDevice,
							lane->stream) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
	}
	if (status == ANN_OK && !lane->rescoreReady)
	{
		if (cudaStreamCreateWithFlags(&lane->rescoreStream, cudaStreamNonBlocking) != cudaSuccess ||
			cudaEventCreateWithFlags(&lane->rescoreDone[0], cudaEventDisableTiming) != cudaSuccess ||
			cudaEventCreateWithFlags(&lane->rescoreDone[1], cudaEventDisableTiming) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
		else
			lane->rescoreReady = 1;
	}
	if (status == ANN_OK)
	{
		counts = malloc(sizeof(*counts) * S * m);
		cand[0] = malloc(sizeof(uint64_t) * m * C);
		cand[1] = malloc(sizeof(uint64_t) * m * C);
		keys = malloc(sizeof(*keys) * C);
		if (counts == NULL || cand[0] == NULL || cand[1] == NULL || keys == NULL || !LaneResults(lane, m * C) ||
			!Grow((void **) &lane->counts, &lane->countsBytes, S * m * sizeof(uint32_t)))
			status = ANN_NOMEM;
		for (int h = 0; status == ANN_OK && h < 2; h++)
		{
			QuantSlot  *sl = &lane->slot[h];

			if ((ix->mapped ? !Grow((void **) &sl->ords, &sl->ordsBytes, m * C * sizeof(uint64_t)) :
				 (!Grow((void **) &sl->stage, &sl->stageBytes, m * C * dims * sizeof(float)) ||
				  !GrowHost((void **) &sl->hostStage, &sl->hostStageBytes, m * C * dims * sizeof(float)))) ||
				!Grow((void **) &sl->rescored, &sl->rescoredBytes, m * C * sizeof(float)) ||
				!GrowHost((void **) &sl->hostRescored, &sl->hostRescoredBytes, m * C * sizeof(float)) ||
				!Grow((void **) &sl->candCounts, &sl->candCountsBytes, m * sizeof(uint32_t)) ||
				!GrowHost((void **) &sl->hostCandCounts, &sl->hostCandCountsBytes, m * sizeof(uint32_t)))
				status = ANN_NOMEM;
		}
	}

	/*
	 * Chunk c: its candidates (the codes' search) and their row copies on
	 * this thread while the device copies in and re-scores chunk c - 1 on
	 * the re-score stream; then chunk c - 1's best k, then chunk c's
	 * re-score queued. The slots alternate.
	 */
	chunks = (uint32_t) ((nq + m - 1) / m);
	for (uint32_t c = 0; status == ANN_OK && c <= chunks; c++)
	{
		double		t0 = NowMs(),
					t1 = t0,
					t2 = t0,
					t3;

		if (c < chunks)
		{
			uint32_t	q0 = (uint32_t) (c * m);
			uint32_t	mm = nq - q0 < m ? nq - q0 : (uint32_t) m;
			const float *q = lane->query + (size_t) q0 * dims;

			/* candidates: each shard's nearest by the codes' exact distance */
			for (uint32_t s = 0; status == ANN_OK && s < S; s++)
				if (want_s[s])
					status = AnnB200Search(ix->shards[s], q, mm, ordinals ? lane->ids + start[s] : NULL,
										   ordinals ? elig[s] : 0, (uint32_t) want_s[s], ANNB200_L2, 0,
										   (uint32_t) want_s[s], lane->dist + m * off[s], lane->id + m * off[s],
										   lane->counts + (size_t) s * m, NULL, lane->stream);
			if (status == ANN_OK &&
				(cudaMemcpyAsync(lane->hostId, lane->id, m * C * sizeof(int64_t), cudaMemcpyDeviceToHost,
								 lane->stream) != cudaSuccess ||
				 cudaMemcpyAsync(counts, lane->counts, S * m * sizeof(uint32_t), cudaMemcpyDeviceToHost,
								 lane->stream) != cudaSuccess ||
				 cudaStreamSynchronize(lane->stream) != cudaSuccess))
				status = ANN_BACKEND_ERROR;
			if (status != ANN_OK)
				break;

			/* their FP32 rows, from host memory (or only their ordinals, when
			 * the device reads the rows in place) */
			t1 = NowMs();
			if (ix->mapped)
				ListCandidates(ix, lane, &lane->slot[c & 1], counts, cand[c & 1], want_s, off, m, C, mm);
			else
				GatherAll(ix, lane, &lane->slot[c & 1], counts, cand[c & 1], want_s, off, m, C, mm);
			t2 = NowMs();
		}
		if (c > 0)
		{
			uint32_t	p0 = (uint32_t) ((c - 1) * m);
			uint32_t	pm = nq - p0 < m ? nq - p0 : (uint32_t) m;
			QuantSlot  *sl = &lane->slot[(c - 1) & 1];
			const uint64_t *cd = cand[(c - 1) & 1];

			if (cudaEventSynchronize(lane->rescoreDone[(c - 1) & 1]) != cudaSuccess)
			{
				status = ANN_BACKEND_ERROR;
				break;
			}

			/* the best k by (distance, ordinal): distances are >= 0, so their bits order them */
			for (uint32_t i = 0; i < pm; i++)
			{
				uint32_t	n = sl->hostCandCounts[i];
				uint32_t	r = n < k ? n : k;

				for (uint32_t j = 0; j < n; j++)
				{
					uint32_t	bits;

					memcpy(&bits, &sl->hostRescored[(size_t) i * C + j], sizeof(bits));
					keys[j] = (uint64_t) bits << 32 | cd[(size_t) i * C + j];
				}
				SelectSmallest(keys, n, r);
				qsort(keys, r, sizeof(*keys), KeyCompare);
				for (uint32_t j = 0; j < r; j++)
				{
					uint32_t	bits = (uint32_t) (keys[j] >> 32);

					memcpy(&out_dist[(size_t) (p0 + i) * k + j], &bits, sizeof(bits));
					out_ordinal[(size_t) (p0 + i) * k + j] = keys[j] & 0xffffffffu;
				}
				out_count[p0 + i] = r;
			}
		}
		t3 = NowMs();
		if (c < chunks)
		{
			uint32_t	q0 = (uint32_t) (c * m);
			uint32_t	mm = nq - q0 < m ? nq - q0 : (uint32_t) m;
			QuantSlot  *sl = &lane->slot[c & 1];
			cudaStream_t rs = lane->rescoreStream;

			if ((ix->mapped ?
				 cudaMemcpyAsync(sl->ords, cand[c & 1], (size_t) mm * C * sizeof(uint64_t), cudaMemcpyHostToDevice,
								 rs) :
				 cudaMemcpyAsync(sl->stage, sl->hostStage, (size_t) mm * C * dims * sizeof(float),
								 cudaMemcpyHostToDevice, rs)) != cudaSuccess ||
				cudaMemcpyAsync(sl->candCounts, sl->hostCandCounts, mm * sizeof(uint32_t), cudaMemcpyHostToDevice,
								rs) != cudaSuccess)
				status = ANN_BACKEND_ERROR;
			if (status == ANN_OK && ix->mapped)
				status = AnnB200RescoreGather(lane->query + (size_t) q0 * dims, mm, dims, ix->mapped, sl->ords,
											  (uint32_t) C, sl->candCounts, sl->rescored, rs);
			else if (status == ANN_OK)
				status = AnnB200RescoreRows(lane->query + (size_t) q0 * dims, mm, dims, sl->stage, (uint32_t) C,
											sl->candCounts, sl->rescored, rs);
			if (status == ANN_OK &&
				(cudaMemcpyAsync(sl->hostRescored, sl->rescored, (size_t) mm * C * sizeof(float),
								 cudaMemcpyDeviceToHost, rs) != cudaSuccess ||
				 cudaEventRecord(lane->rescoreDone[c & 1], rs) != cudaSuccess))
				status = ANN_BACKEND_ERROR;
		}
		if (debug)
			fprintf(stderr, "annb200 quantized index: chunk %u of %u, %llu candidates a query: search %.2f ms, "
					"row copies %.2f ms, re-score wait and best k %.2f ms\n", c, chunks, (unsigned long long) C,
					t1 - t0, t2 - t1, t3 - t2);
	}
	/* nothing of this call stays queued on the lane's buffers */
	if (lane->rescoreReady && cudaStreamSynchronize(lane->rescoreStream) != cudaSuccess && status == ANN_OK)
		status = ANN_BACKEND_ERROR;
done:
	free(start);
	free(elig);
	free(want_s);
	free(off);
	free(local);
	free(counts);
	free(cand[0]);
	free(cand[1]);
	free(keys);
	return status;
}

/* One part's share of a search on a row-sharded index. */
typedef struct PartTask
{
	AnnB200Index *ix;
	uint32_t	p;
	const float *queries;
	uint32_t	nq;
	const uint64_t *ordinals;	/* the whole list (NULL: every row) */
	uint64_t	start;			/* this part's slice of it */
	uint64_t	n;
	uint32_t	k;
	int			status;
} PartTask;

/*
 * Part p: its queries and eligible rows to its device, then its rank of
 * the sharded search (AnnB200SearchSharded: local search, all-gather of
 * the parts' lists, device merge). A part whose staging fails still joins
 * the exchange (with NULL buffers, which it reports as its status), so
 * the other parts never wait for it.
 */
static void *
PartSearch(void *arg)
{
	PartTask   *t = arg;
	AnnB200Index *ix = t->ix;
	Lane	   *lane = &ix->partLanes[t->p];
	size_t		values = (size_t) t->nq * ix->dims;
	size_t		results = (size_t) t->nq * t->k;
	int			ok;

	cudaSetDevice(ix->partDevices[t->p]);
	if (!lane->ready)
	{
		lane->device = ix->partDevices[t->p];
		if (cudaStreamCreateWithFlags(&lane->stream, cudaStreamNonBlocking) != cudaSuccess)
		{
			t->status = ANN_BACKEND_ERROR;
			return NULL;		/* no stream: cannot even join; the others time out */
		}
		lane->ready = 1;
	}
	ok = Grow((void **) &lane->query, &lane->queryBytes, values * sizeof(float)) &&
		Grow((void **) &lane->ids, &lane->idsBytes, (t->n ? t->n : 1) * sizeof(uint32_t)) &&
		LaneResults(lane, results) &&
		Grow((void **) &lane->counts, &lane->countsBytes, t->nq * sizeof(uint32_t));
	if (ok && cudaMemcpyAsync(lane->query, t->queries, values * sizeof(float), cudaMemcpyHostToDevice,
							  lane->stream) != cudaSuccess)
		ok = 0;
	if (ok && t->ordinals && t->n)
	{
		uint32_t   *rows = malloc(sizeof(*rows) * t->n);
		uint64_t	lo = ix->partBounds[t->p];

		if (rows == NULL)
			ok = 0;
		for (uint64_t i = 0; ok && i < t->n; i++)
			rows[i] = (uint32_t) (t->ordinals[t->start + i] - lo);
		if (ok && (cudaMemcpyAsync(lane->ids, rows, t->n * sizeof(uint32_t), cudaMemcpyHostToDevice,
								   lane->stream) != cudaSuccess ||
				   cudaStreamSynchronize(lane->stream) != cudaSuccess))
			ok = 0;
		free(rows);
	}
	t->status = AnnB200SearchSharded(ix->parts[t->p], ix->comms[t->p], ok ? lane->query : NULL, t->nq,
									 t->ordinals ? lane->ids : NULL, t->ordinals ? t->n : 0, t->k, ANNB200_L2,
									 ANNB200_INDEX_L2, t->k, ok ? lane->dist : NULL, lane->id, lane->counts, NULL,
									 lane->stream);
	if (!ok && t->status == ANN_OK)
		t->status = ANN_NOMEM;
	return NULL;
}

/* AnnB200IndexSearch on a row-sharded index: every part at once, one thread a part. */
static int
PartedSearch(AnnB200Index *ix, const float *queries, uint32_t nq, const uint64_t *ordinals, uint64_t nordinals,
			 uint32_t k, float *out_dist, uint64_t *out_ordinal, uint32_t *out_count)
{
	uint32_t	P = ix->nparts;
	PartTask   *task = calloc(P, sizeof(*task));
	pthread_t  *tid = calloc(P, sizeof(*tid));
	char	   *started = calloc(P, 1);
	uint32_t   *counts = malloc(sizeof(*counts) * nq);
	size_t		results = (size_t) nq * k;
	int			status = ANN_OK;
	int			prev = 0;

	if (!task || !tid || !started || !counts)
	{
		free(task);
		free(tid);
		free(started);
		free(counts);
		return ANN_NOMEM;
	}
	cudaGetDevice(&prev);
	pthread_mutex_lock(&ix->searchLock);
	for (uint32_t p = 0; p < P; p++)
	{
		task[p] = (PartTask) {ix, p, queries, nq, ordinals, 0, 0, k, ANN_OK};
		if (ordinals)
			Slice(ordinals, nordinals, ix->partBounds[p], ix->partBounds[p + 1], &task[p].start, &task[p].n);
	}
	/* every part must enter the exchange: a part without a thread runs here, after the others started */
	for (uint32_t p = 1; p < P; p++)
		started[p] = pthread_create(&tid[p], NULL, PartSearch, &task[p]) == 0;
	if (P > 1)
	{
		uint32_t	missing = 0;

		for (uint32_t p = 1; p < P; p++)
			missing += !started[p];
		if (missing)
		{
			/* cannot run the parts together: abort the group rather than wait */
			for (uint32_t p = 0; p < P; p++)
				AnnB200CommAbort(ix->comms[p]);
		}
	}
	PartSearch(&task[0]);
	for (uint32_t p = 1; p < P; p++)
		if (started[p])
			pthread_join(tid[p], NULL);
	for (uint32_t p = 0; p < P; p++)
		if (task[p].status != ANN_OK && status == ANN_OK)
			status = task[p].status;
	if (status == ANN_OK)
	{
		Lane	   *lane = &ix->partLanes[0];

		cudaSetDevice(ix->partDevices[0]);
		if (cudaMemcpyAsync(counts, lane->counts, nq * sizeof(uint32_t), cudaMemcpyDeviceToHost,
							lane->stream) != cudaSuccess ||
			cudaMemcpyAsync(lane->hostDist, lane->dist, results * sizeof(double), cudaMemcpyDeviceToHost,
							lane->stream) != cudaSuccess ||
			cudaMemcpyAsync(lane->hostId, lane->id, results * sizeof(int64_t), cudaMemcpyDeviceToHost,
							lane->stream) != cudaSuccess ||
			cudaStreamSynchronize(lane->stream) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
		for (uint32_t q = 0; status == ANN_OK && q < nq; q++)
		{
			out_count[q] = counts[q];
			for (uint32_t i = 0; i < counts[q]; i++)
			{
				out_dist[(size_t) q * k + i] = (float) lane->hostDist[(size_t) q * k + i];
				out_ordinal[(size_t) q * k + i] = (uint64_t) lane->hostId[(size_t) q * k + i];
			}
		}
	}
	pthread_mutex_unlock(&ix->searchLock);
	cudaSetDevice(prev);
	free(task);
	free(tid);
	free(started);
	free(counts);
	if (status == ANN_OK)
		atomic_fetch_add(&DeviceJobs, 1);
	return status;
}

int
AnnB200IndexSearch(AnnB200Index *ix, const float *queries, uint32_t nq, const uint64_t *ordinals,
				   uint64_t nordinals, uint32_t k, float *out_dist, uint64_t *out_ordinal, uint32_t *out_count)
{
	Lane	   *lane;
	uint32_t   *rows = NULL;
	uint32_t   *counts = NULL;
	size_t		values,
				results;
	int			prev = 0;
	int			status = ANN_OK;

	if (ix == NULL || (nq && (queries == NULL || out_count == NULL)))
		return ANN_INVALID;
	if (nq == 0)
		return ANN_OK;
	if (k && (out_dist == NULL || out_ordinal == NULL))
		return ANN_INVALID;
	values = (size_t) nq * ix->dims;
	if (!AllFinite(queries, values))
		return ANN_INVALID;
	for (uint64_t i = 0; ordinals && i < nordinals; i++)
		if (ordinals[i] >= ix->rows || (i && ordinals[i] <= ordinals[i - 1]))
			return ANN_INVALID;
	memset(out_count, 0, sizeof(*out_count) * nq);
	if (k == 0 || (ordinals && nordinals == 0))
		return ANN_OK;
	if (InjectLost())
		return ANN_BACKEND_ERROR;
	if (ix->nparts > 1)
		return PartedSearch(ix, queries, nq, ordinals, nordinals, k, out_dist, out_ordinal, out_count);
	results = (size_t) nq * k;
	cudaGetDevice(&prev);
	lane = LaneOn(ix->device);
	if (lane == NULL)
	{
		cudaSetDevice(prev);
		return ANN_BACKEND_ERROR;
	}
	if (ix->shard == NULL)
	{
		/* served from the quantized copy */
		if (!Grow((void **) &lane->query, &lane->queryBytes, values * sizeof(float)))
			status = ANN_NOMEM;
		else if (cudaMemcpyAsync(lane->query, queries, values * sizeof(float), cudaMemcpyHostToDevice,
								 lane->stream) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
		if (status == ANN_OK)
			status = QuantSearch(ix, lane, nq, ordinals, nordinals, k, out_dist, out_ordinal, out_count);
		if (status == ANN_OK)
			atomic_fetch_add(&DeviceJobs, 1);
		cudaSetDevice(prev);
		return status;
	}
	counts = malloc(sizeof(*counts) * nq);
	if (ordinals)
		rows = malloc(sizeof(*rows) * nordinals);
	if (counts == NULL || (ordinals && rows == NULL) ||
		!Grow((void **) &lane->query, &lane->queryBytes, values * sizeof(float)) ||
		(ordinals && !Grow((void **) &lane->ids, &lane->idsBytes, nordinals * sizeof(uint32_t))) ||
		!LaneResults(lane, results) ||
		!Grow((void **) &lane->counts, &lane->countsBytes, nq * sizeof(uint32_t)))
		status = ANN_NOMEM;
	for (uint64_t i = 0; status == ANN_OK && ordinals && i < nordinals; i++)
		rows[i] = (uint32_t) ordinals[i];
	if (status == ANN_OK &&
		(cudaMemcpyAsync(lane->query, queries, values * sizeof(float), cudaMemcpyHostToDevice,
						 lane->stream) != cudaSuccess ||
		 (ordinals && cudaMemcpyAsync(lane->ids, rows, nordinals * sizeof(uint32_t), cudaMemcpyHostToDevice,
									  lane->stream) != cudaSuccess)))
		status = ANN_BACKEND_ERROR;
	if (status == ANN_OK)
		status = AnnB200Search(ix->shard, lane->query, nq, ordinals ? lane->ids : NULL, ordinals ? nordinals : 0,
							   k, ANNB200_L2, ANNB200_INDEX_L2, k, lane->dist, lane->id, lane->counts, NULL,
							   lane->stream);
	if (status == ANN_OK &&
		(cudaMemcpyAsync(counts, lane->counts, nq * sizeof(uint32_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostDist, lane->dist, results * sizeof(double), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostId, lane->id, results * sizeof(int64_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	if (status == ANN_OK)
	{
		for (uint32_t q = 0; q < nq; q++)
		{
			out_count[q] = counts[q];
			for (uint32_t i = 0; i < counts[q]; i++)
			{
				out_dist[(size_t) q * k + i] = (float) lane->hostDist[(size_t) q * k + i];
				out_ordinal[(size_t) q * k + i] = (uint64_t) lane->hostId[(size_t) q * k + i];
			}
		}
		atomic_fetch_add(&DeviceJobs, 1);
	}
	free(rows);
	free(counts);
	cudaSetDevice(prev);
	return status;
}

/*
 * The eligible rows of per-shard bitsets as sorted global ordinals, on the
 * host (the forms whose search takes ordinals: a row-sharded index and one
 * served from its quantized copy). Returns the count, or -1 without memory.
 */
static int64_t
BitsetOrdinals(uint32_t nshards, const uint32_t *const *bitsets, const uint64_t *first, const uint64_t *rows,
			   uint64_t **out)
{
	uint64_t	total = 0,
				n = 0;

	for (uint32_t s = 0; s < nshards; s++)
		total += rows[s];
	*out = malloc(sizeof(uint64_t) * (total ? total : 1));
	if (*out == NULL)
		return -1;
	for (uint32_t s = 0; s < nshards; s++)
		for (uint64_t w = 0; bitsets[s] && w < (rows[s] + 31) / 32; w++)
		{
			uint32_t	x = bitsets[s][w];

			if ((w + 1) * 32 > rows[s])
				x &= (uint32_t) ((1ull << (rows[s] - w * 32)) - 1);
			while (x)
			{
				(*out)[n++] = first[s] + w * 32 + (uint64_t) __builtin_ctz(x);
				x &= x - 1;
			}
		}
	return (int64_t) n;
}

/*
 * A loaded-index search whose eligible rows come as per-shard bitsets (the
 * cached filter forms the reference's server hands its backends:
 * AnnIndexJob.bitsets / deviceBitsets, ann/server/backend.h:85-96). On an
 * index with its FP32 rows on one device the bitsets are expanded there
 * (AnnB200BitmapRowsFrom: shard s's set bits become global row numbers
 * first[s] + bit) and searched like an ordinal list; other indexes take
 * the same rows as ordinals.
 */
int
AnnB200IndexSearchBitsets(AnnB200Index *ix, const float *queries, uint32_t nq, uint32_t nshards,
						  const uint32_t *const *bitsets, const uint64_t *shard_first, const uint64_t *shard_rows,
						  uint32_t flags, uint32_t k, float *out_dist, uint64_t *out_ordinal, uint32_t *out_count)
{
	Lane	   *lane;
	uint32_t   *counts = NULL;
	size_t		values,
				results;
	uint64_t	total = 0,
				maxWords = 0,
				n = 0;
	int			prev = 0;
	int			status = ANN_OK;
	int			onDevice = (flags & ANNB200_BITSETS_DEVICE) != 0;

	if (ix == NULL || (nq && (queries == NULL || out_count == NULL)) || (nshards && (bitsets == NULL ||
																		   shard_first == NULL ||
																		   shard_rows == NULL)))
		return ANN_INVALID;
	if (nq == 0)
		return ANN_OK;
	if (k && (out_dist == NULL || out_ordinal == NULL))
		return ANN_INVALID;
	for (uint32_t s = 0; s < nshards; s++)
	{
		if (shard_first[s] + shard_rows[s] > ix->rows || (s && shard_first[s] < shard_first[s - 1] + shard_rows[s - 1]))
			return ANN_INVALID;
		total += shard_rows[s];
		if ((shard_rows[s] + 31) / 32 > maxWords)
			maxWords = (shard_rows[s] + 31) / 32;
	}
	values = (size_t) nq * ix->dims;
	if (!AllFinite(queries, values))
		return ANN_INVALID;
	if (ix->shard == NULL || ix->nparts > 1)
	{
		uint64_t   *ords = NULL;
		int64_t		m;

		if (onDevice)
			return ANN_UNSUPPORTED;
		m = BitsetOrdinals(nshards, bitsets, shard_first, shard_rows, &ords);
		if (m < 0)
			return ANN_NOMEM;
		status = AnnB200IndexSearch(ix, queries, nq, ords, (uint64_t) m, k, out_dist, out_ordinal, out_count);
		free(ords);
		return status;
	}
	memset(out_count, 0, sizeof(*out_count) * nq);
	if (k == 0 || total == 0)
		return ANN_OK;
	if (InjectLost())
		return ANN_BACKEND_ERROR;
	results = (size_t) nq * k;
	cudaGetDevice(&prev);
	lane = LaneOn(ix->device);
	if (lane == NULL)
	{
		cudaSetDevice(prev);
		return ANN_BACKEND_ERROR;
	}
	counts = malloc(sizeof(*counts) * nq);
	if (counts == NULL ||
		!Grow((void **) &lane->query, &lane->queryBytes, values * sizeof(float)) ||
		!Grow((void **) &lane->ids, &lane->idsBytes, total * sizeof(uint32_t)) ||
		(!onDevice && !Grow((void **) &lane->rows, &lane->rowsBytes, maxWords * sizeof(uint32_t))) ||
		!LaneResults(lane, results) ||
		!Grow((void **) &lane->counts, &lane->countsBytes, nq * sizeof(uint32_t)))
		status = ANN_NOMEM;
	if (status == ANN_OK &&
		cudaMemcpyAsync(lane->query, queries, values * sizeof(float), cudaMemcpyHostToDevice, lane->stream) !=
		cudaSuccess)
		status = ANN_BACKEND_ERROR;
	for (uint32_t s = 0; status == ANN_OK && s < nshards; s++)
	{
		const uint32_t *words = bitsets[s];
		uint64_t	found = 0;

		if (words == NULL || shard_rows[s] == 0)
			continue;
		if (!onDevice)
		{
			if (cudaMemcpyAsync(lane->rows, words, (shard_rows[s] + 31) / 32 * sizeof(uint32_t),
								cudaMemcpyHostToDevice, lane->stream) != cudaSuccess)
			{
				status = ANN_BACKEND_ERROR;
				break;
			}
			words = lane->rows;
		}
		status = AnnB200BitmapRowsFrom(words, shard_rows[s], (uint32_t) shard_first[s], lane->ids + n, &found,
									   lane->stream);
		n += found;
	}
	if (status == ANN_OK && n)
		status = AnnB200Search(ix->shard, lane->query, nq, lane->ids, n, k, ANNB200_L2, ANNB200_INDEX_L2, k,
							   lane->dist, lane->id, lane->counts, NULL, lane->stream);
	if (status == ANN_OK && n &&
		(cudaMemcpyAsync(counts, lane->counts, nq * sizeof(uint32_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostDist, lane->dist, results * sizeof(double), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostId, lane->id, results * sizeof(int64_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	if (status == ANN_OK && n)
	{
		for (uint32_t q = 0; q < nq; q++)
		{
			out_count[q] = counts[q];
			for (uint32_t i = 0; i < counts[q]; i++)
			{
				out_dist[(size_t) q * k + i] = (float) lane->hostDist[(size_t) q * k + i];
				out_ordinal[(size_t) q * k + i] = (uint64_t) lane->hostId[(size_t) q * k + i];
			}
		}
	}
	if (status == ANN_OK)
		atomic_fetch_add(&DeviceJobs, 1);
	free(counts);
	cudaSetDevice(prev);
	return status;
}

/*
 * Copy per-shard bitsets to the device of an index's FP32 rows, for
 * AnnB200IndexSearchBitsets with ANNB200_BITSETS_DEVICE: device[s] receives
 * shard s's copy (NULL for a NULL bitset). On failure nothing stays
 * allocated.
 */
int
AnnB200IndexKeepBitsets(AnnB200Index *ix, uint32_t nshards, const uint32_t *const *bitsets,
						const uint64_t *shard_rows, void **device)
{
	int			prev = 0;
	int			status = ANN_OK;

	if (ix == NULL || device == NULL || (nshards && (bitsets == NULL || shard_rows == NULL)))
		return ANN_INVALID;
	if (AnnB200IndexDevice(ix) < 0)
		return ANN_UNSUPPORTED;
	cudaGetDevice(&prev);
	cudaSetDevice(ix->device);
	for (uint32_t s = 0; s < nshards; s++)
		device[s] = NULL;
	for (uint32_t s = 0; status == ANN_OK && s < nshards; s++)
	{
		size_t		bytes = (shard_rows[s] + 31) / 32 * sizeof(uint32_t);

		if (bitsets[s] == NULL || bytes == 0)
			continue;
		if (cudaMalloc(&device[s], bytes) != cudaSuccess)
		{
			device[s] = NULL;
			status = ANN_NOMEM;
		}
		else if (cudaMemcpy(device[s], bitsets[s], bytes, cudaMemcpyHostToDevice) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
	}
	if (status != ANN_OK)
	{
		(void) cudaGetLastError();
		AnnB200IndexDropBitsets(ix, nshards, device);
	}
	cudaSetDevice(prev);
	return status;
}

/* Free what AnnB200IndexKeepBitsets kept. */
void
AnnB200IndexDropBitsets(AnnB200Index *ix, uint32_t nshards, void **device)
{
	int			prev = 0;

	if (ix == NULL || device == NULL)
		return;
	cudaGetDevice(&prev);
	cudaSetDevice(ix->device);
	for (uint32_t s = 0; s < nshards; s++)
	{
		if (device[s])
			cudaFree(device[s]);
		device[s] = NULL;
	}
	cudaSetDevice(prev);
}

/*
 * The device an index's FP32 rows live on, or -1 for an index that keeps
 * them elsewhere (a row-sharded index, one served from its quantized copy):
 * where a cached filter's bitsets may be kept for AnnB200IndexSearchBitsets.
 */
int
AnnB200IndexCopyRoute(const AnnB200Index *ix)
{
	return ix != NULL && ix->shard == NULL && ix->nparts <= 1;
}

int
AnnB200IndexDevice(const AnnB200Index *ix)
{
	return ix != NULL && ix->shard != NULL && ix->nparts <= 1 ? ix->device : -1;
}

/* Bytes a row takes in a storage format. */
static size_t
TypedRowBytes(uint32_t dtype, uint32_t dims)
{
	switch (dtype)
	{
		case ANNB200_F32:
			return (size_t) dims * 4;
		case ANNB200_F16:
			return (size_t) dims * 2;
		case ANNB200_E4M3:
			return (size_t) (dims + 15) / 16 * 16;
		case ANNB200_NVFP4:
			return (size_t) (dims + 15) / 16 * 8;
		default:
			return (size_t) (dims + 7) / 8;
	}
}

/*
 * Whether a typed job's queries and rows hold only values the reference's
 * arithmetic scores: finite FP32 / FP16 values, no E4M3 NaN code (E4M3 has
 * no infinity; E2M1 has neither), finite row scales, and a query of nonzero
 * norm under cosine.
 */
static int
TypedValid(const AnnB200TypedJob *job)
{
	uint32_t	dims = job->dimensions;
	size_t		rb = TypedRowBytes(job->dtype, dims);

	if (job->metric != ANNB200_HAMMING)
		for (uint32_t q = 0; q < job->nq; q++)
		{
			const float *v = (const float *) job->queries + (size_t) q * dims;
			double		norm = 0;

			if (!AllFinite(v, dims))
				return 0;
			for (uint32_t d = 0; d < dims; d++)
				norm += (double) v[d] * v[d];
			if (job->metric == ANNB200_COSINE && norm == 0)
				return 0;
		}
	for (uint32_t r = 0; r < job->rows; r++)
	{
		const uint8_t *row = (const uint8_t *) job->codes + (size_t) r * rb;

		switch (job->dtype)
		{
			case ANNB200_F32:
				if (!AllFinite((const float *) row, dims))
					return 0;
				break;
			case ANNB200_F16:
				for (uint32_t d = 0; d < dims; d++)
				{
					uint16_t	h;

					memcpy(&h, row + 2 * (size_t) d, 2);
					if ((h & 0x7c00) == 0x7c00)
						return 0;
				}
				break;
			case ANNB200_E4M3:
				for (uint32_t d = 0; d < dims; d++)
					if ((row[d] & 0x7f) == 0x7f)
						return 0;
				break;
			case ANNB200_NVFP4:
				for (uint32_t b = 0; b < (dims + 15) / 16; b++)
					if ((((const uint8_t *) job->block_scales)[(size_t) r * ((dims + 15) / 16) + b] & 0x7f) == 0x7f)
						return 0;
				break;
			default:
				break;
		}
		if ((job->dtype == ANNB200_E4M3 || job->dtype == ANNB200_NVFP4) && !isfinite(job->row_scales[r]))
			return 0;
	}
	return 1;
}

/*
 * One typed gathered job: rows of any storage format and a batch of
 * queries, each query with the gathered job's results (AnnGatheredExact
 * semantics, ann/server/cpu.c:218-276, over the rows decoded as the
 * shard search decodes them).
 */
static int
TypedJob(AnnB200TypedJob *job)
{
	Lane	   *lane;
	uint32_t	dims = job->dimensions;
	int			hamming = job->metric == ANNB200_HAMMING;
	size_t		rb,
				qb,
				blocks,
				results;
	int			status;

	for (uint32_t q = 0; job->nresults && q < job->nq; q++)
		job->nresults[q] = 0;
	if (job->dtype > ANNB200_BIT || job->metric > ANNB200_HAMMING || (job->dtype == ANNB200_BIT) != hamming ||
		dims == 0 || dims > (hamming ? 65536u : ANN_MAX_DIM) || job->reserved != 0)
		return ANN_INVALID;
	if (job->nq == 0 || job->k == 0 || job->rows == 0)
		return ANN_OK;
	if (job->queries == NULL || job->codes == NULL || job->nresults == NULL || job->distances == NULL ||
		job->ids == NULL || job->cap == 0 ||
		(job->dtype == ANNB200_NVFP4 && job->block_scales == NULL) ||
		((job->dtype == ANNB200_E4M3 || job->dtype == ANNB200_NVFP4) && job->row_scales == NULL))
		return ANN_INVALID;
	if (!TypedValid(job))
		return ANN_INVALID;
	if (InjectLost())
		return ANN_BACKEND_ERROR;
	lane = LaneGet();
	if (lane == NULL)
		return ANN_BACKEND_ERROR;
	rb = TypedRowBytes(job->dtype, dims);
	qb = hamming ? (size_t) (dims + 7) / 8 : (size_t) dims * 4;
	blocks = (dims + 15) / 16;
	results = (size_t) job->nq * job->cap;
	if (!Grow(&lane->rows, &lane->rowsBytes, (size_t) job->rows * rb) ||
		!Grow((void **) &lane->query, &lane->queryBytes, (size_t) job->nq * qb) ||
		(job->dtype == ANNB200_NVFP4 &&
		 !Grow((void **) &lane->scales, &lane->scalesBytes, (size_t) job->rows * blocks)) ||
		((job->dtype == ANNB200_E4M3 || job->dtype == ANNB200_NVFP4) &&
		 !Grow((void **) &lane->rowScales, &lane->rowScalesBytes, (size_t) job->rows * sizeof(float))) ||
		!Grow((void **) &lane->counts, &lane->countsBytes, (size_t) job->nq * sizeof(uint32_t)) ||
		!LaneResults(lane, results))
		return ANN_NOMEM;
	if (cudaMemcpyAsync(lane->rows, job->codes, (size_t) job->rows * rb, cudaMemcpyHostToDevice,
						lane->stream) != cudaSuccess ||
		cudaMemcpyAsync(lane->query, job->queries, (size_t) job->nq * qb, cudaMemcpyHostToDevice,
						lane->stream) != cudaSuccess ||
		(job->dtype == ANNB200_NVFP4 &&
		 cudaMemcpyAsync(lane->scales, job->block_scales, (size_t) job->rows * blocks, cudaMemcpyHostToDevice,
						 lane->stream) != cudaSuccess) ||
		((job->dtype == ANNB200_E4M3 || job->dtype == ANNB200_NVFP4) &&
		 cudaMemcpyAsync(lane->rowScales, job->row_scales, (size_t) job->rows * sizeof(float),
						 cudaMemcpyHostToDevice, lane->stream) != cudaSuccess))
		return ANN_BACKEND_ERROR;
	{
		const void *bs = job->dtype == ANNB200_NVFP4 ? lane->scales : NULL;
		const float *rs = job->dtype == ANNB200_E4M3 || job->dtype == ANNB200_NVFP4 ? lane->rowScales : NULL;

		if (lane->shard == NULL)
			status = AnnB200ShardCreate(lane->device, job->dtype, dims, job->rows, lane->rows, bs, rs, 0, 0,
										lane->stream, &lane->shard);
		else
			status = AnnB200ShardAssign(lane->shard, job->dtype, dims, job->rows, lane->rows, bs, rs, 0,
										lane->stream);
	}
	if (status == ANN_OK)
		status = AnnB200Search(lane->shard, lane->query, job->nq, NULL, 0, job->k, job->metric, ANNB200_WINDOW,
							   job->cap, lane->dist, lane->id, lane->counts, NULL, lane->stream);
	if (status == ANN_OK &&
		(cudaMemcpyAsync(job->nresults, lane->counts, (size_t) job->nq * sizeof(uint32_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostDist, lane->dist, results * sizeof(double), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostId, lane->id, results * sizeof(int64_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	if (status != ANN_OK)
	{
		for (uint32_t q = 0; q < job->nq; q++)
			job->nresults[q] = 0;
		return status;
	}
	for (uint32_t q = 0; q < job->nq; q++)
		for (uint32_t i = 0; i < job->nresults[q]; i++)
		{
			job->distances[(size_t) q * job->cap + i] = lane->hostDist[(size_t) q * job->cap + i];
			job->ids[(size_t) q * job->cap + i] = (uint32_t) lane->hostId[(size_t) q * job->cap + i];
		}
	atomic_fetch_add(&DeviceJobs, 1);
	return ANN_OK;
}

int
AnnB200SearchTyped(AnnB200TypedJob *jobs, uint32_t n)
{
	if (n && jobs == NULL)
		return ANN_INVALID;
	for (uint32_t i = 0; i < n; i++)
		jobs[i].status = TypedJob(&jobs[i]);
	return ANN_OK;
}

/*
 * A lane's batch of gathered jobs as one device submission (the reference's
 * contract for search_gathered, ann/server/backend.h:129-130): every job's
 * rows and query are staged into pinned memory and cross in one copy, the
 * searches run as one AnnB200SearchBatch (the rows' finiteness checked on
 * the device), and the results come back in one copy. Jobs the host can
 * settle (bad dimensions or metric, no rows, k = 0) are answered first.
 */
static void
SearchGathered(AnnGatheredJob *jobs, uint32_t count)
{
	Lane	   *lane;
	AnnB200BatchJob *batch = NULL;
	uint32_t   *slot = NULL;
	size_t	   *starts = NULL;
	size_t		values = 0,
				results = 0;
	uint32_t	m = 0;
	int			status = ANN_OK;

	for (uint32_t i = 0; i < count; i++)
	{
		AnnGatheredJob *job = &jobs[i];

		job->nresults = 0;
		job->status = ANN_OK;
		if (job->dimensions == 0 || job->dimensions > ANN_MAX_DIM || job->metric > 2)
			job->status = ANN_INVALID;
		else if (job->rows == 0 || job->k == 0)
			job->status = TrivialStatus(job);
		else if (!QueryValid(job))
			job->status = ANN_INVALID;
		else if (InjectLost())
			job->status = ANN_BACKEND_ERROR;
		else
		{
			values += Align16((size_t) job->rows * job->dimensions) + Align16(job->dimensions);
			results += job->rows;
			m++;
		}
	}
	if (m == 0)
		return;
	batch = calloc(m, sizeof(*batch));
	slot = calloc(m, sizeof(*slot));
	if (batch == NULL || slot == NULL)
	{
		for (uint32_t i = 0; i < count; i++)
			if (jobs[i].status == ANN_OK && jobs[i].rows && jobs[i].k)
				jobs[i].status = ANN_NOMEM;
		free(batch);
		free(slot);
		return;
	}
	for (uint32_t i = 0, b = 0; i < count; i++)
		if (jobs[i].status == ANN_OK && jobs[i].rows && jobs[i].k)
			slot[b++] = i;
	lane = LaneGet();
	if (lane == NULL)
		status = ANN_BACKEND_ERROR;
	if (status == ANN_OK &&
		(!GrowHost((void **) &lane->hostIn, &lane->hostInBytes, values * sizeof(float)) ||
		 !Grow(&lane->rows, &lane->rowsBytes, values * sizeof(float)) ||
		 !LaneResults(lane, results) ||
		 !Grow((void **) &lane->counts, &lane->countsBytes, m * sizeof(uint32_t)) ||
		 !Grow((void **) &lane->statuses, &lane->statusesBytes, m * sizeof(int32_t)) ||
		 !GrowHost((void **) &lane->hostCounts, &lane->hostCountsBytes, m * sizeof(uint32_t))))
		status = ANN_NOMEM;
	if (status == ANN_OK && (starts = malloc(sizeof(*starts) * m)) == NULL)
		status = ANN_NOMEM;
	if (status == ANN_OK)
	{
		size_t		at = 0,
					res = 0;
		uint32_t	b = 0;

		for (uint32_t i = 0; i < count; i++)
		{
			AnnGatheredJob *job = &jobs[i];
			size_t		rv = (size_t) job->rows * job->dimensions;

			if (job->status != ANN_OK || job->rows == 0 || job->k == 0)
				continue;
			starts[b] = at;
			batch[b] = (AnnB200BatchJob) {
				.rows = (const float *) lane->rows + at, .nrows = job->rows, .dims = job->dimensions,
				.queries = (const float *) lane->rows + at + Align16(rv), .nq = 1, .k = job->k,
				.metric = job->metric,
				.flags = ANNB200_WINDOW | ANNB200_REJECT_NONFINITE, .out_cap = job->rows,
				.out_dist = lane->dist + res, .out_id = lane->id + res, .out_count = lane->counts + b,
				.status = lane->statuses + b};
			b++;
			at += Align16(rv) + Align16(job->dimensions);
			res += job->rows;
		}
		StageAll(jobs, slot, starts, m, lane->hostIn, values * sizeof(float));
		if (cudaMemcpyAsync(lane->rows, lane->hostIn, values * sizeof(float), cudaMemcpyHostToDevice,
							lane->stream) != cudaSuccess)
			status = ANN_BACKEND_ERROR;
	}
	/* the lane's reusable context: a shard bound to each job in turn */
	if (status == ANN_OK && lane->shard == NULL)
		status = AnnB200ShardCreate(lane->device, ANNB200_F32, batch[0].dims, batch[0].nrows, batch[0].rows,
									NULL, NULL, 0, 0, lane->stream, &lane->shard);
	if (status == ANN_OK)
		status = AnnB200SearchBatch(lane->shard, batch, m, lane->stream);
	if (status == ANN_OK &&
		(cudaMemcpyAsync(lane->hostCounts, lane->counts, m * sizeof(uint32_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostDist, lane->dist, results * sizeof(double), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostId, lane->id, results * sizeof(int64_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	for (uint32_t b = 0, res = 0; b < m; b++)
	{
		AnnGatheredJob *job = &jobs[slot[b]];

		if (status != ANN_OK || batch[b].result != ANN_OK)
		{
			job->status = (AnnStatus) (status != ANN_OK ? status : batch[b].result);
			res += job->rows;
			continue;
		}
		for (uint32_t i = 0; i < lane->hostCounts[b]; i++)
		{
			job->results[i].id = (uint32_t) lane->hostId[res + i];
			job->results[i].distance = lane->hostDist[res + i];
		}
		job->nresults = lane->hostCounts[b];
		job->status = ANN_OK;
		atomic_fetch_add(&DeviceJobs, 1);
		res += job->rows;
	}
	free(batch);
	free(slot);
	free(starts);
}

static uint64_t
DeviceJobCount(void)
{
	return (uint64_t) atomic_load(&DeviceJobs);
}

static void
Destroy(AnnIndex *index)
{
	IndexState *state = index->backend_state;

	if (state)
	{
		int			prev = 0;

		cudaGetDevice(&prev);
		cudaSetDevice(state->device);
		AnnB200ShardDestroy(state->shard);
		if (state->rows)
			cudaFree(state->rows);
		cudaSetDevice(prev);
		free(state);
	}
	free(index->vectors);
	memset(index, 0, sizeof(*index));
}

/* In-memory FP32 index, validated like the cpu backend's Build (cpu.c:19-44). */
static AnnStatus
Build(AnnIndex *index, uint64_t generation, uint32_t rows, uint32_t dimensions, const float *vectors)
{
	uint64_t	wide = (uint64_t) rows * dimensions;
	size_t		count;
	float	   *copy;
	IndexState *state;
	Lane	   *lane;

	if (generation == 0 || dimensions == 0 || dimensions > ANN_MAX_DIM ||
		wide > ANN_MAX_BYTES / sizeof(float) || (wide && vectors == NULL))
		return ANN_INVALID;
	count = (size_t) wide;
	if (!AllFinite(vectors, count))
		return ANN_INVALID;
	lane = LaneGet();
	if (lane == NULL)
		return ANN_BACKEND_ERROR;
	copy = malloc(count ? count * sizeof(float) : 1);
	state = calloc(1, sizeof(*state));
	if (copy == NULL || state == NULL)
	{
		free(copy);
		free(state);
		return ANN_NOMEM;
	}
	if (count)
		memcpy(copy, vectors, count * sizeof(float));
	state->device = lane->device;
	if (count && (cudaMalloc(&state->rows, count * sizeof(float)) != cudaSuccess ||
				  cudaMemcpy(state->rows, vectors, count * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess))
	{
		if (state->rows)
			cudaFree(state->rows);
		free(copy);
		free(state);
		return ANN_NOMEM;
	}
	if (rows && AnnB200ShardCreate(state->device, ANNB200_F32, dimensions, rows, state->rows, NULL, NULL, 0, 0,
								   lane->stream, &state->shard) != ANN_OK)
	{
		cudaFree(state->rows);
		free(copy);
		free(state);
		return ANN_BACKEND_ERROR;
	}
	Destroy(index);
	index->vectors = copy;
	index->rows = rows;
	index->dimensions = dimensions;
	index->generation = generation;
	index->backend_state = state;
	return ANN_OK;
}

/*
 * The k best rows of an in-memory index by (distance, id), optionally among
 * sorted unique ids (the cpu backend's Search, ann/server/cpu.c:82-154).
 */
static AnnStatus
Search(const AnnIndex *index, const float *query, uint32_t metric, const uint32_t *ids, uint32_t nids,
	   uint32_t k, AnnCandidate *results, uint32_t *nresults)
{
	IndexState *state = index->backend_state;
	Lane	   *lane;
	double		qnorm = 0;
	uint32_t	count = 0;
	int			status;

	*nresults = 0;
	if (metric > 2)
		return ANN_UNSUPPORTED;
	if (!AllFinite(query, index->dimensions))
		return ANN_INVALID;
	for (uint32_t d = 0; d < index->dimensions; d++)
		qnorm += (double) query[d] * query[d];
	if (metric == 2 && qnorm == 0)
		return ANN_INVALID;
	for (uint32_t i = 0; ids && i < nids; i++)
		if (ids[i] >= index->rows || (i && ids[i] <= ids[i - 1]))
			return ANN_INVALID;
	if (k == 0 || index->rows == 0 || (ids && nids == 0) || state == NULL)
		return ANN_OK;
	if (InjectLost())
		return ANN_BACKEND_ERROR;
	lane = LaneGet();
	if (lane == NULL)
		return ANN_BACKEND_ERROR;
	cudaSetDevice(state->device);
	if (!Grow((void **) &lane->query, &lane->queryBytes, index->dimensions * sizeof(float)) ||
		(ids && !Grow((void **) &lane->ids, &lane->idsBytes, (size_t) nids * sizeof(uint32_t))) ||
		!LaneResults(lane, k))
		return ANN_NOMEM;
	if (cudaMemcpyAsync(lane->query, query, index->dimensions * sizeof(float), cudaMemcpyHostToDevice,
						lane->stream) != cudaSuccess ||
		(ids && cudaMemcpyAsync(lane->ids, ids, (size_t) nids * sizeof(uint32_t), cudaMemcpyHostToDevice,
								lane->stream) != cudaSuccess))
		return ANN_BACKEND_ERROR;
	status = AnnB200Search(state->shard, lane->query, 1, ids ? lane->ids : NULL, ids ? nids : 0, k, metric, 0, k,
						   lane->dist, lane->id, lane->count, NULL, lane->stream);
	if (status == ANN_OK &&
		(cudaMemcpyAsync(&count, lane->count, sizeof(count), cudaMemcpyDeviceToHost, lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	if (status == ANN_OK && count &&
		(cudaMemcpyAsync(lane->hostDist, lane->dist, count * sizeof(double), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaMemcpyAsync(lane->hostId, lane->id, count * sizeof(int64_t), cudaMemcpyDeviceToHost,
						 lane->stream) != cudaSuccess ||
		 cudaStreamSynchronize(lane->stream) != cudaSuccess))
		status = ANN_BACKEND_ERROR;
	if (status != ANN_OK)
		return (AnnStatus) status;
	for (uint32_t i = 0; i < count; i++)
	{
		results[i].id = (uint32_t) lane->hostId[i];
		results[i].distance = lane->hostDist[i];
	}
	*nresults = count;
	atomic_fetch_add(&DeviceJobs, 1);
	return ANN_OK;
}

/*
 * Why the device context is unusable, or NULL: a simulated loss, or a sticky
 * CUDA error on this thread's device (the reference's cuVS check,
 * ann/server/cuvs.c:8047-8080).
 */
static const char *
Lost(void)
{
	static _Thread_local char reason[256];
	cudaError_t e;

	if (atomic_load(&LostSimulated))
		return LostReason;
	if (!LaneState.ready)
		return NULL;
	cudaSetDevice(LaneState.device);
	e = cudaStreamSynchronize(LaneState.stream);
	if (e == cudaSuccess || e == cudaErrorNotReady)
		return NULL;
	if (e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure || e == cudaErrorIllegalInstruction ||
		e == cudaErrorMisalignedAddress || e == cudaErrorHardwareStackError || e == cudaErrorInvalidPc ||
		e == cudaErrorECCUncorrectable || e == cudaErrorAssert || e == cudaErrorInvalidAddressSpace ||
		e == cudaErrorLaunchTimeout)
	{
		snprintf(reason, sizeof(reason), "GPU context lost: %s", cudaGetErrorString(e));
		return reason;
	}
	return NULL;
}

/*
 * The typed search operation's jobs: AnnTypedJob is AnnB200TypedJob's layout
 * (checked below), so the worker's jobs are searched in place.
 */
_Static_assert(sizeof(AnnTypedJob) == sizeof(AnnB200TypedJob), "typed job layout");
_Static_assert(offsetof(AnnTypedJob, queries) == offsetof(AnnB200TypedJob, queries), "typed job layout");
_Static_assert(offsetof(AnnTypedJob, status) == offsetof(AnnB200TypedJob, status), "typed job layout");

static void
SearchTypedJobs(AnnTypedJob *jobs, uint32_t count)
{
	(void) AnnB200SearchTyped((AnnB200TypedJob *) jobs, count);
}

const AnnBackend *
AnnB200Backend(void)
{
	static const AnnBackend backend = {
		"b200", 7, 7, "flat", "fp32", 1, 0, UINT32_MAX, Build, Search, Destroy,
		SearchGathered, DeviceJobCount, NULL, NULL, Lost, NULL, SearchTypedJobs
	};

	return &backend;
}
