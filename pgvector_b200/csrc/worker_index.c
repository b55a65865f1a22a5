/*
 * worker_index.c - loaded on-disk indexes for the b200 worker backend.
 *
 * The worker keeps loaded index directories in its own registry
 * (AnnIndexFileOpen / AnnIndexRegister / AnnIndexGet, ann/server/indexfile.h:
 * 402-403,586-595), which the server consults for every index operation, so
 * a backend's load_index and search_index must work through it (the cpu
 * backend does, ann/server/cpu.c:286-407). This file is therefore compiled
 * inside the worker's build, against the worker's own backend.h and
 * indexfile.h, and linked with libannb200.so; it adds nothing to the library
 * itself. AnnB200WorkerBackend() is AnnB200Backend() with the two index
 * entry points filled in.
 *
 *   load_index     registers the directory like the cpu backend and copies
 *                  its FP32 rows (vectors.f32) to a GPU (AnnB200IndexCreate,
 *                  round robin over the devices), or row-shards them over
 *                  several GPUs (AnnB200IndexCreateSharded: one GPU's share
 *                  each, lists joined by an NCCL all-gather and a device
 *                  merge) when ANN_B200_INDEX_DEVICES asks for it or one
 *                  GPU cannot hold them; where no GPU set holds them and
 *                  the directory has a quantized copy, that copy instead
 *                  (a "dtype float16" directory: an FP16 copy made on the
 *                  device from vectors.f32, served the same way)
 *                  (AnnB200IndexCreateQuant: the reference's quantized scan
 *                  route, file->quantActive set as the reference's backend
 *                  sets it). The device copy hangs off file->device and is
 *                  freed by the registry's AnnIndexDeviceDestroy hook when
 *                  the index is unloaded.
 *   search_index   per job: drop excluded rows (AnnIndexJobDropExcluded),
 *                  resolve the index (ANN_STALE if not loaded, ANN_INVALID on
 *                  a dimension mismatch), map a key filter to ordinals
 *                  (AnnIndexOrdinals, unless the server passed them), and run
 *                  the exact scan on the device. Jobs on one index with the
 *                  same filter arrays (or none) run as one batch (the
 *                  tensor-core scan applies from 16 queries), over the
 *                  cheapest filter form they carry: bitsets kept on the
 *                  device, host bitsets expanded there, ordinals, or keys
 *                  mapped to ordinals. Hits carry the key of their ordinal and the
 *                  reference's FP32 distance; route is set as the cpu backend
 *                  sets it (cpu.c:394), or as the quantized scan route sets
 *                  it (ANN_ROUTE_EXACT, cuvs.c:4927).
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "backend.h"
#include "indexfile.h"

#include "annb200.h"
#include "annb200_backend.h"

static void
DestroyDevice(void *device)
{
	AnnB200IndexDestroy((AnnB200Index *) device);
}

/*
 * The device copy of a directory with a quantized copy ("quant fp8|nvfp4")
 * while the worker scans quantized copies (--quantized-scan, on by
 * default): its codes, per index shard, with the FP32 rows left in the
 * mapped vectors.f32 for re-scoring (AnnB200IndexCreateQuant).
 */
static AnnStatus
CreateQuant(const AnnIndexFile *file, AnnB200Index **index)
{
	uint64_t	rows[ANN_INDEX_MAX_SHARDS];
	uint32_t	nshards = file->nshards;

	for (uint32_t s = 0; s < nshards; s++)
		rows[s] = file->shards[s].rows;
	return (AnnStatus) AnnB200IndexCreateQuant(-1, file->dimensions, file->rows,
											   file->quant == ANN_QUANT_NVFP4 ? ANNB200_NVFP4 : ANNB200_E4M3,
											   file->quantData, file->quantScales, file->rowScales, file->vectors,
											   nshards, nshards ? rows : NULL, AnnIndexConfig.quant_slack,
											   AnnIndexConfig.slack_ratio, index);
}

/*
 * The FP32 rows on the devices: row-sharded over ANN_B200_INDEX_DEVICES
 * devices when that is set above 1 (the reference spreads an index's shards
 * over its GPUs, ann/server/cuvs.c:2845-2862); else on one device (round
 * robin), and where they do not fit one device, over every visible device.
 */
static AnnStatus
CreateRows(AnnIndexFile *file, AnnB200Index **index)
{
	const char *env = getenv("ANN_B200_INDEX_DEVICES");
	int			devices = AnnB200DeviceCount();
	int			want = env && *env ? atoi(env) : 1;
	int			list[64];
	AnnStatus	status;

	if (want > devices)
		want = devices;
	if (want > 64)
		want = 64;
	if (want <= 1)
	{
		status = (AnnStatus) AnnB200IndexCreate(-1, file->dimensions, file->rows, file->vectors, index);
		if (status != ANN_NOMEM || devices <= 1 || (env && *env))
			return status;
		want = devices < 64 ? devices : 64;
	}
	if ((uint64_t) want > file->rows)
		want = (int) file->rows;
	for (int d = 0; d < want; d++)
		list[d] = d;
	return (AnnStatus) AnnB200IndexCreateSharded(want, list, file->dimensions, file->rows, file->vectors, index);
}

/*
 * Which copy a loaded index searches on the device: its FP32 rows (exact)
 * where they fit (CreateRows), else its quantized copy when it has one and
 * quantized scans are on. ANN_B200_INDEX_COPY=fp32 or =quant chooses
 * instead.
 */
static AnnStatus
CreateDevice(AnnIndexFile *file, AnnB200Index **index)
{
	const char *copy = getenv("ANN_B200_INDEX_COPY");
	int			quant = file->quant != ANN_QUANT_NONE && AnnIndexConfig.quantized_scan;
	AnnStatus	status;

	file->quantActive = 0;
	if (strcmp(file->dtype, "float16") == 0 && !(copy && strcmp(copy, "fp32") == 0) &&
		!(quant && copy && strcmp(copy, "quant") == 0))
	{
		/*
		 * "dtype float16": the device keeps the rows in FP16 (half the
		 * memory of FP32; the reference keeps its CAGRA dataset so, with
		 * --fp16-exact re-scoring in FP32): each shard's k + slack nearest by
		 * the FP16 rows, their FP32 rows re-scored, as the quantized route
		 */
		uint64_t	rows[ANN_INDEX_MAX_SHARDS];

		for (uint32_t s = 0; s < file->nshards; s++)
			rows[s] = file->shards[s].rows;
		status = (AnnStatus) AnnB200IndexCreateQuant(-1, file->dimensions, file->rows, ANNB200_F16, NULL, NULL, NULL,
													 file->vectors, file->nshards,
													 file->nshards ? rows : NULL, AnnIndexConfig.quant_slack,
													 AnnIndexConfig.slack_ratio, index);
		if (status != ANN_NOMEM || !quant)
			return status;
		status = CreateQuant(file, index);
		file->quantActive = status == ANN_OK;
		return status;
	}
	if (quant && copy && strcmp(copy, "quant") == 0)
		status = CreateQuant(file, index);
	else
	{
		status = CreateRows(file, index);
		if (status != ANN_NOMEM || !quant || (copy && strcmp(copy, "fp32") == 0))
			return status;
		status = CreateQuant(file, index);
	}
	file->quantActive = status == ANN_OK;
	return status;
}

static AnnStatus
LoadIndex(const char *name, const char *directory)
{
	AnnIndexFile *file;
	AnnB200Index *index = NULL;
	AnnStatus	status = AnnIndexFileOpen(name, directory, &file);

	if (status != ANN_OK)
		return status;
	AnnIndexDeviceDestroy = DestroyDevice;
	status = CreateDevice(file, &index);
	if (status != ANN_OK)
	{
		AnnIndexFileClose(file);
		return status;
	}
	file->device = index;
	if ((status = AnnIndexRegister(file)) != ANN_OK)
	{
		file->device = NULL;
		AnnB200IndexDestroy(index);
		AnnIndexFileClose(file);
	}
	return status;
}

static void
Finish(AnnIndexJob *job, const AnnIndexFile *file, const float *dist, const uint64_t *ordinal, uint32_t n)
{
	/* the quantized (or FP16) scan route answers as an exact scan (cuvs.c:4927) */
	int			quant = AnnB200IndexCopyRoute((const AnnB200Index *) file->device);

	if (n > job->k)
		n = job->k;
	for (uint32_t i = 0; i < n; i++)
	{
		job->results[i].key = file->keys[ordinal[i]];
		job->results[i].distance = dist[i];
		job->results[i].ordinal = ordinal[i];
	}
	job->nresults = n;
	job->route = job->filtered || quant ? ANN_ROUTE_EXACT : ANN_ROUTE_ANN;
	job->status = ANN_OK;
}

/*
 * Whether job i joins the group of job `first`: one search of the group's
 * queries at the largest k. Unfiltered jobs on one index group together;
 * filtered jobs group when they share the same filter arrays -- the test
 * the server uses for identical searches (SameSearch, ann/server/server.c:
 * 1216-1225), and the lane batches same-filter jobs for one gather
 * (ann/server/server.c:1311-1545; SearchGatherGroup, ann/server/cuvs.c:5407).
 * On an index served from its quantized copy the group also needs one k
 * (the candidates each query re-scores follow from its own k).
 */
static int
SameGroup(AnnIndexJob *jobs, AnnIndexFile **files, const char *done, uint32_t first, uint32_t i)
{
	const AnnIndexJob *a = &jobs[first],
			   *b = &jobs[i];

	if (done[i] || files[i] != files[first] || a->filtered != b->filtered)
		return 0;
	if (AnnB200IndexCopyRoute((const AnnB200Index *) files[first]->device) && a->k != b->k)
		return 0;
	if (!a->filtered)
		return 1;
	return a->filter == b->filter && a->nfilter == b->nfilter && a->ordinals == b->ordinals &&
		a->bitsets == b->bitsets && a->deviceBitsets == b->deviceBitsets && a->deviceRows == b->deviceRows;
}

/*
 * The group's eligible rows into the search, in the cheapest form the job
 * carries: bitsets kept on the device (nothing crosses), host bitsets (one
 * bit a row crosses, expanded on the device), ordinals, or the filter's keys
 * mapped to ordinals (AnnIndexOrdinals, as the cpu backend does).
 */
static int
GroupSearch(AnnIndexFile *file, const AnnIndexJob *job, const float *queries, uint32_t n, uint32_t k, float *dist,
			uint64_t *ordinal, uint32_t *counts)
{
	AnnB200Index *ix = (AnnB200Index *) file->device;
	int			onDevice = AnnB200IndexDevice(ix) >= 0;
	uint64_t	first[ANN_INDEX_MAX_SHARDS],
				rows[ANN_INDEX_MAX_SHARDS];
	uint64_t   *owned = NULL;
	uint64_t	nords = job->nfilter;
	int			status;

	if (!job->filtered)
		return AnnB200IndexSearch(ix, queries, n, NULL, 0, k, dist, ordinal, counts);
	for (uint32_t s = 0; s < file->nshards; s++)
	{
		first[s] = file->shards[s].first;
		rows[s] = file->shards[s].rows;
	}
	if (job->deviceBitsets && onDevice && file->nshards)
		return AnnB200IndexSearchBitsets(ix, queries, n, file->nshards, (const uint32_t *const *) job->deviceBitsets,
										 first, rows, ANNB200_BITSETS_DEVICE, k, dist, ordinal, counts);
	if (job->bitsets && file->nshards && (onDevice || job->ordinals == NULL))
		return AnnB200IndexSearchBitsets(ix, queries, n, file->nshards, (const uint32_t *const *) job->bitsets,
										 first, rows, 0, k, dist, ordinal, counts);
	if (job->ordinals)
		return AnnB200IndexSearch(ix, queries, n, job->ordinals, job->nfilter, k, dist, ordinal, counts);
	owned = malloc(sizeof(uint64_t) * (job->nfilter ? job->nfilter : 1));
	if (owned == NULL)
		return ANN_NOMEM;
	nords = AnnIndexOrdinals(file, job->filter, job->nfilter, owned);
	status = AnnB200IndexSearch(ix, queries, n, owned, nords, k, dist, ordinal, counts);
	free(owned);
	return status;
}

/* The jobs grouped with job `first`: one search of their queries at the largest k. */
static void
SearchGroupOf(AnnIndexJob *jobs, AnnIndexFile **files, uint32_t count, uint32_t first, char *done)
{
	AnnIndexFile *file = files[first];
	uint32_t	dims = file->dimensions;
	uint32_t	n = 0,
				kmax = 0,
				g = 0;
	float	   *queries,
			   *dist;
	uint64_t   *ordinal;
	uint32_t   *counts;
	int			status;

	for (uint32_t i = first; i < count; i++)
		if (SameGroup(jobs, files, done, first, i))
		{
			n++;
			if (jobs[i].k > kmax)
				kmax = jobs[i].k;
		}
	queries = malloc(sizeof(float) * (size_t) n * dims);
	dist = malloc(sizeof(float) * (size_t) n * (kmax ? kmax : 1));
	ordinal = malloc(sizeof(uint64_t) * (size_t) n * (kmax ? kmax : 1));
	counts = malloc(sizeof(uint32_t) * n);
	status = queries && dist && ordinal && counts ? ANN_OK : ANN_NOMEM;
	for (uint32_t i = first; status == ANN_OK && i < count; i++)
		if (SameGroup(jobs, files, done, first, i))
			memcpy(queries + (size_t) g++ * dims, jobs[i].query, sizeof(float) * dims);
	if (status == ANN_OK)
		status = GroupSearch(file, &jobs[first], queries, n, kmax, dist, ordinal, counts);
	g = 0;
	for (uint32_t i = first; i < count; i++)
		if (SameGroup(jobs, files, done, first, i))
		{
			done[i] = 1;
			if (status == ANN_OK)
				Finish(&jobs[i], file, dist + (size_t) g * kmax, ordinal + (size_t) g * kmax, counts[g]);
			else
				jobs[i].status = (AnnStatus) status;
			g++;
		}
	free(queries);
	free(dist);
	free(ordinal);
	free(counts);
}

static void
SearchIndex(AnnIndexJob *jobs, uint32_t count)
{
	AnnIndexFile **files = calloc(count ? count : 1, sizeof(*files));
	char	   *done = calloc(count ? count : 1, 1);

	if (files == NULL || done == NULL)
	{
		for (uint32_t i = 0; i < count; i++)
		{
			jobs[i].nresults = 0;
			jobs[i].status = ANN_NOMEM;
		}
		free(files);
		free(done);
		return;
	}
	for (uint32_t i = 0; i < count; i++)
	{
		AnnIndexJob *job = &jobs[i];
		AnnIndexFile *file;

		job->nresults = 0;
		done[i] = 1;
		if (!AnnIndexJobDropExcluded(job))
			continue;
		if ((file = AnnIndexGet(job->name)) == NULL)
		{
			job->status = ANN_STALE;
			continue;
		}
		if (job->dimensions != file->dimensions || file->device == NULL)
		{
			job->status = file->device == NULL ? ANN_BACKEND_ERROR : ANN_INVALID;
			AnnIndexPut(file);
			continue;
		}
		files[i] = file;
		done[i] = 0;
	}
	for (uint32_t i = 0; i < count; i++)
		if (!done[i])
			SearchGroupOf(jobs, files, count, i, done);
	for (uint32_t i = 0; i < count; i++)
		if (files[i])
			AnnIndexPut(files[i]);
	free(files);
	free(done);
}

/*
 * Cached filter bitmaps (AnnIndexBitmapDevice, ann/server/indexfile.h:
 * 147-165): keep each shard's bitset on the device of an index whose FP32
 * rows live on one device, so a search over a cached filter copies nothing
 * (AnnB200IndexSearchBitsets with ANNB200_BITSETS_DEVICE). Row lists are not
 * kept: the device expands the bitsets per search. A failure leaves the
 * bitmap on the per-query path, as the reference's hook does.
 */
static void
UploadBitmap(AnnIndexFile *file, AnnIndexBitmap *bitmap)
{
	AnnB200Index *ix = (AnnB200Index *) file->device;
	uint64_t	rows[ANN_INDEX_MAX_SHARDS];
	void	  **device;
	uint64_t	bytes = 0;

	if (ix == NULL || AnnB200IndexDevice(ix) < 0 || bitmap->words == NULL || file->nshards == 0)
		return;
	device = calloc(file->nshards, sizeof(void *));
	if (device == NULL)
		return;
	for (uint32_t s = 0; s < file->nshards; s++)
	{
		rows[s] = file->shards[s].rows;
		bytes += (rows[s] + 31) / 32 * sizeof(uint32_t);
	}
	if (AnnB200IndexKeepBitsets(ix, file->nshards, (const uint32_t *const *) bitmap->bitsets, rows, device) != ANN_OK)
	{
		free(device);
		return;
	}
	bitmap->device = device;
	bitmap->deviceBytes = bytes;
}

static void
ReleaseBitmap(AnnIndexFile *file, AnnIndexBitmap *bitmap)
{
	if (bitmap->device)
	{
		AnnB200IndexDropBitsets((AnnB200Index *) file->device, file->nshards, bitmap->device);
		free(bitmap->device);
	}
	bitmap->device = NULL;
	bitmap->deviceRows = NULL;
	bitmap->deviceBytes = 0;
}

/*
 * Whether a search for k results over every row should run as a scan of a
 * cached row list instead of the backend's plain search (the server then
 * turns a match-all predicate into a filtered search, ann/server/server.c:
 * 3213-3218). Here the plain search already is the exact scan of every row,
 * batched with the other unfiltered jobs, so building a row list only adds
 * work: never.
 */
static int
ScanPreferred(const struct AnnIndexFile *file, uint32_t k)
{
	(void) file;
	(void) k;
	return 0;
}

static AnnBackend WorkerBackend;
static pthread_once_t WorkerBackendOnce = PTHREAD_ONCE_INIT;

static void
WorkerBackendInit(void)
{
	WorkerBackend = *AnnB200Backend();
	WorkerBackend.load_index = LoadIndex;
	WorkerBackend.search_index = SearchIndex;
	WorkerBackend.scan_preferred = ScanPreferred;
	AnnIndexBitmapDevice.upload = UploadBitmap;
	AnnIndexBitmapDevice.release = ReleaseBitmap;
}

const AnnBackend *AnnB200WorkerBackend(void);

const AnnBackend *
AnnB200WorkerBackend(void)
{
	pthread_once(&WorkerBackendOnce, WorkerBackendInit);
	return &WorkerBackend;
}
