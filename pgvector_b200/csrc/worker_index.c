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
 *                  round robin over the devices); where they do not fit and
 *                  the directory has a quantized copy, that copy instead
 *                  (AnnB200IndexCreateQuant: the reference's quantized scan
 *                  route, file->quantActive set as the reference's backend
 *                  sets it). The device copy hangs off file->device and is
 *                  freed by the registry's AnnIndexDeviceDestroy hook when
 *                  the index is unloaded.
 *   search_index   per job: drop excluded rows (AnnIndexJobDropExcluded),
 *                  resolve the index (ANN_STALE if not loaded, ANN_INVALID on
 *                  a dimension mismatch), map a key filter to ordinals
 *                  (AnnIndexOrdinals, unless the server passed them), and run
 *                  the exact scan on the device. Unfiltered jobs on one index
 *                  run as one batch (the tensor-core scan applies from 16
 *                  queries); filtered jobs run one at a time over their
 *                  ordinals. Hits carry the key of their ordinal and the
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
 * Which copy a loaded index searches on the device: its FP32 rows (exact)
 * where they fit, else its quantized copy when it has one and quantized
 * scans are on. ANN_B200_INDEX_COPY=fp32 or =quant chooses instead.
 */
static AnnStatus
CreateDevice(AnnIndexFile *file, AnnB200Index **index)
{
	const char *copy = getenv("ANN_B200_INDEX_COPY");
	int			quant = file->quant != ANN_QUANT_NONE && AnnIndexConfig.quantized_scan;
	AnnStatus	status;

	file->quantActive = 0;
	if (quant && copy && strcmp(copy, "quant") == 0)
		status = CreateQuant(file, index);
	else
	{
		status = (AnnStatus) AnnB200IndexCreate(-1, file->dimensions, file->rows, file->vectors, index);
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
	/* the quantized scan route answers as an exact scan (cuvs.c:4927) */
	int			quant = file->quantActive;

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
 * Whether job i joins the batch of job `first`: unfiltered, on the same
 * index, and, on an index served from its quantized copy, with the same k
 * (the number of candidates each query re-scores follows from its own k).
 */
static int
SameBatch(AnnIndexJob *jobs, AnnIndexFile **files, const char *done, uint32_t first, uint32_t i)
{
	return files[i] == files[first] && !jobs[i].filtered && !done[i] &&
		(!files[first]->quantActive || jobs[i].k == jobs[first].k);
}

/* Unfiltered jobs [first..] on `file`: one batch of queries, k = the largest. */
static void
SearchBatch(AnnIndexJob *jobs, AnnIndexFile **files, uint32_t count, uint32_t first, char *done)
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
		if (SameBatch(jobs, files, done, first, i))
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
		if (SameBatch(jobs, files, done, first, i))
			memcpy(queries + (size_t) g++ * dims, jobs[i].query, sizeof(float) * dims);
	if (status == ANN_OK)
		status = AnnB200IndexSearch((AnnB200Index *) file->device, queries, n, NULL, 0, kmax, dist, ordinal,
									counts);
	g = 0;
	for (uint32_t i = first; i < count; i++)
		if (SameBatch(jobs, files, done, first, i))
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
SearchFiltered(AnnIndexJob *job, AnnIndexFile *file)
{
	const uint64_t *ordinals = job->ordinals;
	uint64_t	n = job->nfilter;
	uint64_t   *owned = NULL;
	float	   *dist = malloc(sizeof(float) * (job->k ? job->k : 1));
	uint64_t   *ordinal = malloc(sizeof(uint64_t) * (job->k ? job->k : 1));
	uint32_t	found = 0;
	int			status = dist && ordinal ? ANN_OK : ANN_NOMEM;

	if (status == ANN_OK && ordinals == NULL)
	{
		owned = malloc(sizeof(uint64_t) * (job->nfilter ? job->nfilter : 1));
		if (owned == NULL)
			status = ANN_NOMEM;
		else
			n = AnnIndexOrdinals(file, job->filter, job->nfilter, owned);
		ordinals = owned;
	}
	if (status == ANN_OK)
		status = AnnB200IndexSearch((AnnB200Index *) file->device, job->query, 1, ordinals, n, job->k, dist,
									ordinal, &found);
	if (status == ANN_OK)
		Finish(job, file, dist, ordinal, found);
	else
		job->status = (AnnStatus) status;
	free(owned);
	free(dist);
	free(ordinal);
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
		if (!done[i] && !jobs[i].filtered)
			SearchBatch(jobs, files, count, i, done);
	for (uint32_t i = 0; i < count; i++)
		if (!done[i])
		{
			SearchFiltered(&jobs[i], files[i]);
			done[i] = 1;
		}
	for (uint32_t i = 0; i < count; i++)
		if (files[i])
			AnnIndexPut(files[i]);
	free(files);
	free(done);
}

static AnnBackend WorkerBackend;
static pthread_once_t WorkerBackendOnce = PTHREAD_ONCE_INIT;

static void
WorkerBackendInit(void)
{
	WorkerBackend = *AnnB200Backend();
	WorkerBackend.load_index = LoadIndex;
	WorkerBackend.search_index = SearchIndex;
}

const AnnBackend *AnnB200WorkerBackend(void);

const AnnBackend *
AnnB200WorkerBackend(void)
{
	pthread_once(&WorkerBackendOnce, WorkerBackendInit);
	return &WorkerBackend;
}
