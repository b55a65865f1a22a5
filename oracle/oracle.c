/*
 * oracle.c - CPU oracle for the exact gather-scan.
 *
 * TEST INFRASTRUCTURE ONLY. tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this file's shared library as the checker. The
 * product library (pgvector_b200/libannb200.so) never links, loads or calls
 * it, and has no CPU fallback through it.
 *
 * Semantics restated from the reference (paths relative to the reference
 * project root):
 *
 *   distance  = the reference CPU worker's formula applied to rows decoded to
 *               FP32:
 *                 metric 0 (L2): sqrt((double) L2Squared) with eight FP32
 *                   partial sums            ann/server/cpu.c:158-175,218-276
 *                 metric 1 (negative inner product) and metric 2 (cosine
 *                   distance, zero-norm rows skipped): FP64 sums in dimension
 *                   order                   ann/server/cpu.c:82-154
 *                 metric 3 (Hamming): popcount of XOR over the packed bits
 *                                           src/bitutils.c:49-69
 *   ordering  = (distance, row id) ascending  ann/server/cpu.c:46-51
 *   window    = every row within d_k + 1e-3*|d_k| + 1e-6 of the k-th
 *               distance (gathered jobs)    ann/server/cpu.c:264-275,
 *                                           ann/server/backend.h:45-50,156
 *   decoding  = half: ann/server/indexfile.c:71-90;
 *               FP8: e4m3 x row scale, NVFP4: e2m1 x (e4m3 block scale x
 *               row scale), FP32 multiplies ann/common/INDEX_FORMAT.md:54-57,
 *               ann/server/blackwell.c:63-105 (score4's decode order)
 *   quantizers= ann/builder/build_cuvs_index.py:296-348 restated with the
 *               same FP32 rounding as its NumPy code.
 *
 * Parity is pinned in tests/ against the reference's own compiled cpu.c
 * (oracle/_ref, built by oracle/Makefile from the reference sources) and
 * against committed golden vectors made by the reference's builder.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_F32 0
#define ORC_F16 1
#define ORC_E4M3 2
#define ORC_NVFP4 3
#define ORC_BIT 4

#define ORC_OK 0
#define ORC_INVALID 1
#define ORC_UNSUPPORTED 2
#define ORC_NOMEM 4

#define ORC_TOLERANCE 1e-3		/* ANN_GATHERED_TOLERANCE, backend.h:156 */

/* ---------------------------------------------------------------- decoding */

/* IEEE half to float: ann/server/indexfile.c:71-90. */
float
orc_half_to_float(uint16_t half)
{
	uint32_t	sign = (uint32_t) (half & 0x8000) << 16;
	uint32_t	exponent = (half >> 10) & 0x1f;
	uint32_t	mantissa = half & 0x3ff;
	uint32_t	bits;
	float		value;

	if (exponent == 0)
	{
		value = (float) mantissa * 5.9604644775390625e-08f;	/* 2^-24 */
		return sign ? -value : value;
	}
	if (exponent == 31)
		bits = sign | 0x7f800000u | (mantissa << 13);
	else
		bits = sign | ((exponent + 112) << 23) | (mantissa << 13);
	memcpy(&value, &bits, sizeof(value));
	return value;
}

/* Float to IEEE half, round to nearest even: ann/server/indexfile.c:29-69. */
uint16_t
orc_float_to_half(float value)
{
	uint32_t	bits;
	uint32_t	sign;
	int32_t		exponent;
	uint32_t	mantissa;

	memcpy(&bits, &value, sizeof(bits));
	sign = (bits >> 16) & 0x8000u;
	exponent = (int32_t) ((bits >> 23) & 0xff) - 112;
	mantissa = bits & 0x7fffffu;
	if (exponent >= 31)
		return (uint16_t) (sign | 0x7c00u);
	if (exponent <= 0)
	{
		uint32_t	shift,
					half,
					rest,
					middle;

		if (exponent < -10)
			return (uint16_t) sign;
		mantissa |= 0x800000u;
		shift = (uint32_t) (14 - exponent);
		half = mantissa >> shift;
		rest = mantissa & ((1u << shift) - 1);
		middle = 1u << (shift - 1);
		if (rest > middle || (rest == middle && (half & 1)))
			half++;
		return (uint16_t) (sign | half);
	}
	{
		uint32_t	half = sign | ((uint32_t) exponent << 10) | (mantissa >> 13);
		uint32_t	rest = mantissa & 0x1fffu;

		if (rest > 0x1000u || (rest == 0x1000u && (half & 1)))
			half++;
		return (uint16_t) half;
	}
}

/*
 * Non-negative E4M3 magnitude of a 7-bit code: exponent bits 6..3, mantissa
 * bits 2..0, bias 7, subnormals at exponent 0; code 127 is NaN
 * (ann/builder/build_cuvs_index.py:296-301).
 */
static float
E4m3Magnitude(uint32_t code)
{
	uint32_t	exponent = code >> 3;
	uint32_t	mantissa = code & 7;

	if (code >= 127)
		return NAN;
	if (exponent == 0)
		return ldexpf((float) mantissa, -9);	/* m/8 * 2^-6 */
	return ldexpf((float) (8 + mantissa), (int) exponent - 10);	/* (1+m/8) 2^(e-7) */
}

float
orc_e4m3(uint8_t code)
{
	float		m = E4m3Magnitude(code & 0x7f);

	return (code & 0x80) ? -m : m;
}

/* E2M1 magnitudes (ann/builder/build_cuvs_index.py:304); bit 3 is the sign. */
static const float E2m1Table[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

float
orc_e2m1(uint8_t nibble)
{
	float		m = E2m1Table[nibble & 7];

	return (nibble & 8) ? -m : m;
}

/* Bytes a row takes in each storage format (ann/common/INDEX_FORMAT.md:54-57). */
uint64_t
orc_row_bytes(uint32_t dtype, uint32_t dims)
{
	switch (dtype)
	{
		case ORC_F32:
			return (uint64_t) dims * 4;
		case ORC_F16:
			return (uint64_t) dims * 2;
		case ORC_E4M3:
			return ((uint64_t) dims + 15) / 16 * 16;
		case ORC_NVFP4:
			return ((uint64_t) dims + 15) / 16 * 8;
		case ORC_BIT:
			return ((uint64_t) dims + 7) / 8;
	}
	return 0;
}

/*
 * Decode one stored row to FP32. FP8: e4m3 x row scale. NVFP4: the block
 * scale is e4m3 x row scale, then each value is e2m1 x block scale, each an
 * FP32 multiply (the order of score4 in ann/server/blackwell.c:81-95).
 */
void
orc_decode_row(uint32_t dtype, uint32_t dims, const uint8_t *row,
			   const uint8_t *blockScales, float rowScale, float *out)
{
	switch (dtype)
	{
		case ORC_F32:
			memcpy(out, row, sizeof(float) * dims);
			break;
		case ORC_F16:
			for (uint32_t d = 0; d < dims; d++)
			{
				uint16_t	h;

				memcpy(&h, row + 2 * (size_t) d, 2);
				out[d] = orc_half_to_float(h);
			}
			break;
		case ORC_E4M3:
			for (uint32_t d = 0; d < dims; d++)
			{
				volatile float v = orc_e4m3(row[d]) * rowScale;

				out[d] = v;
			}
			break;
		case ORC_NVFP4:
			for (uint32_t d = 0; d < dims; d++)
			{
				volatile float block = orc_e4m3(blockScales[d / 16]) * rowScale;
				uint8_t		byte = row[d / 2];
				uint8_t		nibble = (d & 1) ? (uint8_t) (byte >> 4) : (uint8_t) (byte & 15);
				volatile float v = orc_e2m1(nibble) * block;

				out[d] = v;
			}
			break;
		default:
			memset(out, 0, sizeof(float) * dims);
	}
}

/* ---------------------------------------------------------------- distances */

/* Eight FP32 partial sums, then a fixed pairwise combine: ann/server/cpu.c:158-175. */
float
orc_l2_squared(const float *a, const float *b, uint32_t dimensions)
{
	float		sums[8] = {0};
	float		sum = 0;
	uint32_t	d = 0;

	for (; d + 8 <= dimensions; d += 8)
		for (int j = 0; j < 8; j++)
		{
			float		diff = a[d + j] - b[d + j];
			float		sq = diff * diff;

			sums[j] += sq;
		}
	for (; d < dimensions; d++)
	{
		float		diff = a[d] - b[d];
		float		sq = diff * diff;

		sum += sq;
	}
	{
		float		left = (sums[0] + sums[1]) + (sums[2] + sums[3]);
		float		right = (sums[4] + sums[5]) + (sums[6] + sums[7]);
		float		total = sum + left;

		total += right;
		return total;
	}
}

static uint64_t
Hamming(const uint8_t *a, const uint8_t *b, uint64_t bytes)
{
	uint64_t	distance = 0;
	uint64_t	i = 0;

	for (; i + 8 <= bytes; i += 8)
	{
		uint64_t	x,
					y;

		memcpy(&x, a + i, 8);
		memcpy(&y, b + i, 8);
		distance += (uint64_t) __builtin_popcountll(x ^ y);
	}
	for (; i < bytes; i++)
		distance += (uint64_t) __builtin_popcount((unsigned) (a[i] ^ b[i]));
	return distance;
}

/* FP64 dot and squared norm in dimension order, as Search accumulates them. */
static void
DotNorm(const float *v, const float *q, uint32_t dims, double *dot, double *norm)
{
	double		s = 0,
				n = 0;

	for (uint32_t d = 0; d < dims; d++)
	{
		double		a = v[d];
		double		b = q[d];

		s += a * b;
		n += a * a;
	}
	*dot = s;
	*norm = n;
}

/*
 * Distance of one decoded row under metrics 0-2 (returns 0 and sets *skip for
 * a zero-norm row under cosine). qnorm is the query's FP64 squared norm.
 */
double
orc_distance(uint32_t metric, const float *v, const float *q, uint32_t dims,
			 double qnorm, int *skip)
{
	double		dot,
				norm;

	*skip = 0;
	if (metric == 0)
		return sqrt((double) orc_l2_squared(v, q, dims));
	DotNorm(v, q, dims, &dot, &norm);
	if (metric == 1)
		return -dot;
	if (norm == 0)
	{
		*skip = 1;
		return 0;
	}
	return 1 - fmax(-1, fmin(1, dot / sqrt(norm * qnorm)));
}

/* ---------------------------------------------------------------- selection */

typedef struct OrcHit
{
	double		distance;
	int64_t		id;
} OrcHit;

static int
HitCompare(const OrcHit *a, const OrcHit *b)
{
	if (a->distance != b->distance)
		return a->distance < b->distance ? -1 : 1;
	return a->id < b->id ? -1 : a->id > b->id;
}

static int
HitSortCompare(const void *a, const void *b)
{
	return HitCompare(a, b);
}

/* Bounded max-heap of the best k hits, worst at the root (cpu.c:121-148). */
static void
Offer(OrcHit *heap, uint64_t *count, uint64_t k, OrcHit hit)
{
	uint64_t	i;

	if (*count < k)
	{
		i = (*count)++;
		while (i && HitCompare(&heap[(i - 1) / 2], &hit) < 0)
		{
			heap[i] = heap[(i - 1) / 2];
			i = (i - 1) / 2;
		}
		heap[i] = hit;
		return;
	}
	if (HitCompare(&hit, &heap[0]) >= 0)
		return;
	i = 0;
	for (;;)
	{
		uint64_t	child = i * 2 + 1;

		if (child >= *count)
			break;
		if (child + 1 < *count && HitCompare(&heap[child], &heap[child + 1]) < 0)
			child++;
		if (HitCompare(&heap[child], &hit) <= 0)
			break;
		heap[i] = heap[child];
		i = child;
	}
	heap[i] = hit;
}

/* Partition so hits[n] holds the n-th smallest distance (cpu.c:179-215). */
static void
SelectNth(OrcHit *items, uint64_t count, uint64_t n)
{
	uint64_t	left = 0,
				right = count - 1;

	while (left < right)
	{
		double		pivot = items[left + (right - left) / 2].distance;
		uint64_t	i = left,
					j = right;

		while (i <= j)
		{
			while (items[i].distance < pivot)
				i++;
			while (items[j].distance > pivot)
				j--;
			if (i <= j)
			{
				OrcHit		tmp = items[i];

				items[i] = items[j];
				items[j] = tmp;
				i++;
				if (j == 0)
					break;
				j--;
			}
		}
		if (n <= j)
			right = j;
		else if (n >= i)
			left = i;
		else
			break;
	}
}

/* ---------------------------------------------------------------- threads */

typedef struct OrcPool
{
	void		(*fn) (void *ctx, uint64_t i);
	void	   *ctx;
	uint64_t	n;
	atomic_ullong next;
} OrcPool;

static void *
PoolWorker(void *arg)
{
	OrcPool    *pool = arg;

	for (;;)
	{
		uint64_t	i = atomic_fetch_add(&pool->next, 1);

		if (i >= pool->n)
			break;
		pool->fn(pool->ctx, i);
	}
	return NULL;
}

/* Run fn(ctx, i) for i in [0, n) on up to threads POSIX threads. */
static void
ParallelFor(uint64_t n, int threads, void (*fn) (void *, uint64_t), void *ctx)
{
	OrcPool		pool;
	pthread_t	tids[256];
	int			started = 0;

	pool.fn = fn;
	pool.ctx = ctx;
	pool.n = n;
	atomic_init(&pool.next, 0);
	if (threads > 256)
		threads = 256;
	for (int t = 1; t < threads && (uint64_t) t < n; t++)
		if (pthread_create(&tids[started], NULL, PoolWorker, &pool) == 0)
			started++;
	PoolWorker(&pool);
	for (int t = 0; t < started; t++)
		pthread_join(tids[t], NULL);
}

/* ---------------------------------------------------------------- search */

typedef struct OrcCorpus
{
	uint32_t	dtype;
	uint32_t	dims;
	uint64_t	rows;
	const uint8_t *codes;
	const uint8_t *blockScales;
	const float *rowScales;
	uint64_t	rowBytes;
} OrcCorpus;

static void
DecodeRow(const OrcCorpus *c, uint64_t row, float *out)
{
	uint64_t	blocks = ((uint64_t) c->dims + 15) / 16;

	orc_decode_row(c->dtype, c->dims, c->codes + row * c->rowBytes,
				   c->blockScales ? c->blockScales + row * blocks : NULL,
				   c->rowScales ? c->rowScales[row] : 1.0f, out);
}

/*
 * One query over the candidate rows ids[0..n) (all rows when ids is NULL).
 * Strict mode keeps the k best by (distance, id); window mode keeps every row
 * within the gathered tolerance of the k-th distance, sorted. Returns a
 * status; results go to out_dist/out_id (capacity cap) and *out_count.
 */
static int
SearchOne(const OrcCorpus *c, const void *query, const uint32_t *ids, uint64_t n,
		  uint32_t k, uint32_t metric, int window, uint64_t cap,
		  double *out_dist, int64_t *out_id, uint32_t *out_count)
{
	OrcHit	   *hits;
	uint64_t	count = 0;
	float	   *row = NULL;
	const float *q = (const float *) query;
	double		qnorm = 0;
	int			status = ORC_OK;

	*out_count = 0;
	if (metric == 3 ? c->dtype != ORC_BIT : (metric > 2 || c->dtype == ORC_BIT))
		return ORC_UNSUPPORTED;
	if (metric != 3)
	{
		for (uint32_t d = 0; d < c->dims; d++)
		{
			if (!isfinite(q[d]))
				return ORC_INVALID;
			qnorm += (double) q[d] * q[d];
		}
		if (metric == 2 && qnorm == 0)
			return ORC_INVALID;
	}
	if (k == 0 || n == 0)
		return ORC_OK;
	hits = malloc(sizeof(*hits) * (window ? n : (k < n ? k : n)));
	if (metric != 3)
		row = malloc(sizeof(float) * (c->dims ? c->dims : 1));
	if (hits == NULL || (metric != 3 && row == NULL))
	{
		free(hits);
		free(row);
		return ORC_NOMEM;
	}
	for (uint64_t i = 0; i < n; i++)
	{
		uint64_t	id = ids ? ids[i] : i;
		OrcHit		hit;
		int			skip = 0;

		if (metric == 3)
			hit.distance = (double) Hamming(c->codes + id * c->rowBytes, (const uint8_t *) query, c->rowBytes);
		else
		{
			DecodeRow(c, id, row);
			hit.distance = orc_distance(metric, row, q, c->dims, qnorm, &skip);
			if (skip)
				continue;
			if (metric == 0 && !isfinite(hit.distance))
			{
				status = ORC_INVALID;
				goto done;
			}
		}
		hit.id = (int64_t) id;
		if (window)
			hits[count++] = hit;
		else
			Offer(hits, &count, k, hit);
	}
	if (window && k < count)
	{
		double		threshold;
		uint64_t	kept = 0;

		SelectNth(hits, count, k - 1);
		threshold = hits[k - 1].distance;
		threshold += ORC_TOLERANCE * fabs(threshold) + 1e-6;
		for (uint64_t i = 0; i < count; i++)
			if (hits[i].distance <= threshold)
				hits[kept++] = hits[i];
		count = kept;
	}
	qsort(hits, count, sizeof(*hits), HitSortCompare);
	if (count > cap)
		count = cap;
	for (uint64_t i = 0; i < count; i++)
	{
		out_dist[i] = hits[i].distance;
		out_id[i] = hits[i].id;
	}
	*out_count = (uint32_t) count;
done:
	free(hits);
	free(row);
	return status;
}

typedef struct SearchTask
{
	const OrcCorpus *c;
	const void *queries;
	uint64_t	qbytes;
	const uint32_t *ids;
	uint64_t	n;
	uint32_t	k;
	uint32_t	metric;
	int			window;
	uint64_t	cap;
	double	   *out_dist;
	int64_t    *out_id;
	uint32_t   *out_count;
	int32_t    *out_status;
} SearchTask;

static void
SearchTaskRun(void *arg, uint64_t q)
{
	SearchTask *t = arg;

	t->out_status[q] = SearchOne(t->c, (const uint8_t *) t->queries + q * t->qbytes, t->ids, t->n,
								 t->k, t->metric, t->window, t->cap,
								 t->out_dist + q * t->cap, t->out_id + q * t->cap,
								 t->out_count + q);
}

/*
 * Exact search of nq queries over one corpus and one shared candidate list.
 * queries: FP32 [nq][dims], or packed bits [nq][row bytes] for Hamming.
 * Results: [nq][cap] distances and row ids (row ids, not list positions),
 * counts [nq], statuses [nq]. Returns the first non-OK status, else OK.
 */
int
orc_search(uint32_t dtype, uint32_t dims, uint64_t rows, const void *codes,
		   const uint8_t *blockScales, const float *rowScales,
		   const void *queries, uint32_t nq, const uint32_t *ids, uint64_t nids,
		   uint32_t k, uint32_t metric, int window, uint64_t cap,
		   double *out_dist, int64_t *out_id, uint32_t *out_count,
		   int32_t *out_status, int threads)
{
	OrcCorpus	c;
	uint64_t	n = ids ? nids : rows;
	uint64_t	qbytes = metric == 3 ? orc_row_bytes(ORC_BIT, dims) : (uint64_t) dims * 4;
	int			status = ORC_OK;

	c.dtype = dtype;
	c.dims = dims;
	c.rows = rows;
	c.codes = (const uint8_t *) codes;
	c.blockScales = blockScales;
	c.rowScales = rowScales;
	c.rowBytes = orc_row_bytes(dtype, dims);
	if (threads < 1)
		threads = 1;
	for (uint64_t i = 0; ids && i < nids; i++)
		if (ids[i] >= rows || (i && ids[i] <= ids[i - 1]))
			return ORC_INVALID;
	{
		SearchTask	task = {&c, queries, qbytes, ids, n, k, metric, window, cap,
		out_dist, out_id, out_count, out_status};

		ParallelFor(nq, threads, SearchTaskRun, &task);
	}
	for (uint32_t q = 0; q < nq; q++)
		if (out_status[q] != ORC_OK && status == ORC_OK)
			status = out_status[q];
	return status;
}

typedef struct ListTask
{
	const OrcCorpus *c;
	const int64_t *rowIds;
	const uint64_t *offsets;
	uint32_t	nlists;
	const uint32_t *probes;
	uint32_t	nprobe;
	const float *queries;
	uint32_t	k;
	uint32_t	metric;
	double	   *out_dist;
	int64_t    *out_id;
	uint32_t   *out_count;
} ListTask;

static void
ListTaskRun(void *arg, uint64_t q)
{
	ListTask   *t = arg;
	const OrcCorpus *c = t->c;
	uint32_t	dims = c->dims;
	uint32_t	k = t->k;
	const float *query = t->queries + q * dims;
	float	   *row = malloc(sizeof(float) * dims);
	OrcHit	   *heap = malloc(sizeof(OrcHit) * (k ? k : 1));
	uint64_t	count = 0;
	double		qnorm = 0;

	t->out_count[q] = 0;
	if (row == NULL || heap == NULL)
	{
		free(row);
		free(heap);
		return;
	}
	for (uint32_t d = 0; d < dims; d++)
		qnorm += (double) query[d] * query[d];
	for (uint32_t p = 0; p < t->nprobe && k; p++)
	{
		uint32_t	list = t->probes[q * t->nprobe + p];

		if (list >= t->nlists)
			continue;
		for (uint64_t r = t->offsets[list]; r < t->offsets[list + 1]; r++)
		{
			OrcHit		hit;
			int			skip;

			DecodeRow(c, r, row);
			hit.distance = orc_distance(t->metric, row, query, dims, qnorm, &skip);
			if (skip)
				continue;
			hit.id = t->rowIds ? t->rowIds[r] : (int64_t) r;
			Offer(heap, &count, k, hit);
		}
	}
	qsort(heap, count, sizeof(*heap), HitSortCompare);
	for (uint64_t i = 0; i < count; i++)
	{
		t->out_dist[q * k + i] = heap[i].distance;
		t->out_id[q * k + i] = heap[i].id;
	}
	t->out_count[q] = (uint32_t) count;
	free(row);
	free(heap);
}

/*
 * IVF list gather: query q scans the rows of its probed lists. Lists are
 * stored list-major: list l holds corpus rows offsets[l] .. offsets[l+1]-1
 * (already in list order), and rowIds maps a stored row to its global id.
 * probes: [nq][nprobe] list numbers. Semantics of scanning the probed lists
 * and ordering every entry by distance: src/ivfscan.c:124-186. Results carry
 * global ids; ties by id. Strict mode only.
 */
int
orc_search_lists(uint32_t dtype, uint32_t dims, uint64_t rows, const void *codes,
				 const uint8_t *blockScales, const float *rowScales,
				 const int64_t *rowIds, const uint64_t *offsets, uint32_t nlists,
				 const uint32_t *probes, uint32_t nprobe,
				 const float *queries, uint32_t nq, uint32_t k, uint32_t metric,
				 double *out_dist, int64_t *out_id, uint32_t *out_count, int threads)
{
	OrcCorpus	c;
	int			status = ORC_OK;

	c.dtype = dtype;
	c.dims = dims;
	c.rows = rows;
	c.codes = (const uint8_t *) codes;
	c.blockScales = blockScales;
	c.rowScales = rowScales;
	c.rowBytes = orc_row_bytes(dtype, dims);
	if (metric > 2 || dtype == ORC_BIT)
		return ORC_UNSUPPORTED;
	if (threads < 1)
		threads = 1;
	{
		ListTask	task = {&c, rowIds, offsets, nlists, probes, nprobe, queries, k, metric,
		out_dist, out_id, out_count};

		ParallelFor(nq, threads, ListTaskRun, &task);
	}
	return status;
}

/* ---------------------------------------------------------------- quantizers */

/* Non-negative E4M3 values for codes 0..126, increasing (builder :296-301). */
static void
E4m3Table(float *table)
{
	for (uint32_t c = 0; c < 127; c++)
		table[c] = E4m3Magnitude(c);
}

/* numpy.searchsorted(table, x, side='left'): first index with table[i] >= x. */
static uint32_t
SearchSorted(const float *table, uint32_t size, float x)
{
	uint32_t	lo = 0,
				hi = size;

	while (lo < hi)
	{
		uint32_t	mid = (lo + hi) / 2;

		if (table[mid] < x)
			lo = mid + 1;
		else
			hi = mid;
	}
	return lo;
}

/* _nearest (builder :307-311): ties go to the lower table entry. */
static uint32_t
Nearest(const float *table, uint32_t size, float x)
{
	uint32_t	index = SearchSorted(table, size, x);
	volatile float below,
				above,
				lowGap,
				highGap;

	if (index < 1)
		index = 1;
	if (index > size - 1)
		index = size - 1;
	below = table[index - 1];
	above = table[index];
	lowGap = x - below;
	highGap = above - x;
	return lowGap <= highGap ? index - 1 : index;
}

/*
 * quantize_fp8 (builder :314-323): per row, scale = absmax/448 (1 for an
 * all-zero row), code = nearest E4M3 magnitude of |v/scale| with the sign in
 * bit 7. codes: rows x dims rounded up to 16 (zero padded).
 */
void
orc_quantize_fp8(const float *vectors, uint64_t rows, uint32_t dims,
				 uint8_t *codes, float *scales)
{
	float		table[127];
	uint32_t	padded = (dims + 15) / 16 * 16;

	E4m3Table(table);
	for (uint64_t r = 0; r < rows; r++)
	{
		const float *v = vectors + r * dims;
		float		amax = 0;
		volatile float scale;

		for (uint32_t d = 0; d < dims; d++)
			if (fabsf(v[d]) > amax)
				amax = fabsf(v[d]);
		scale = amax > 0 ? amax / 448.0f : 1.0f;
		scales[r] = scale;
		for (uint32_t d = 0; d < padded; d++)
		{
			volatile float x = d < dims ? v[d] / scale : 0.0f;
			uint8_t		code = (uint8_t) Nearest(table, 127, fabsf(x));

			codes[r * padded + d] = (uint8_t) (code | (x < 0 ? 0x80 : 0));
		}
	}
}

/*
 * quantize_nvfp4 (builder :326-348): row = absmax/(6*448); each 16-value
 * block's E4M3 scale code is the smallest table entry >= blockmax/(6*row)
 * (clipped to 126); values are the nearest E2M1 magnitude of
 * min(|v/(table[code]*row)|, 6) with the sign in bit 3, two a byte, the even
 * dimension in the low nibble.
 */
void
orc_quantize_nvfp4(const float *vectors, uint64_t rows, uint32_t dims,
				   uint8_t *packed, uint8_t *scaleCodes, float *rowScales)
{
	float		table[127];
	uint32_t	blocks = (dims + 15) / 16;

	E4m3Table(table);
	for (uint64_t r = 0; r < rows; r++)
	{
		const float *v = vectors + r * dims;
		float		amax = 0;
		volatile float row,
					six;

		for (uint32_t d = 0; d < dims; d++)
			if (fabsf(v[d]) > amax)
				amax = fabsf(v[d]);
		row = amax > 0 ? amax / 2688.0f : 1.0f;
		rowScales[r] = row;
		six = 6.0f * row;
		for (uint32_t b = 0; b < blocks; b++)
		{
			float		bmax = 0;
			volatile float target,
						scale;
			uint32_t	code;
			uint8_t		nibbles[16];

			for (uint32_t j = 0; j < 16; j++)
			{
				uint32_t	d = b * 16 + j;

				if (d < dims && fabsf(v[d]) > bmax)
					bmax = fabsf(v[d]);
			}
			target = bmax / six;
			code = SearchSorted(table, 127, target);
			if (code > 126)
				code = 126;
			scaleCodes[r * blocks + b] = (uint8_t) code;
			scale = table[code] * row;
			for (uint32_t j = 0; j < 16; j++)
			{
				uint32_t	d = b * 16 + j;
				float		value = d < dims ? v[d] : 0.0f;
				volatile float x = scale > 0 ? value / scale : 0.0f;
				float		mag = fabsf(x) < 6.0f ? fabsf(x) : 6.0f;
				uint8_t		nib = (uint8_t) Nearest(E2m1Table, 8, mag);

				nibbles[j] = (uint8_t) (nib | (x < 0 ? 8 : 0));
			}
			for (uint32_t j = 0; j < 8; j++)
				packed[r * blocks * 8 + b * 8 + j] = (uint8_t) (nibbles[2 * j] | (nibbles[2 * j + 1] << 4));
		}
	}
}

typedef struct DecodeTask
{
	const OrcCorpus *c;
	uint64_t	first;
	float	   *out;
} DecodeTask;

static void
DecodeTaskRun(void *arg, uint64_t i)
{
	DecodeTask *t = arg;

	DecodeRow(t->c, t->first + i, t->out + i * t->c->dims);
}

/* Decode whole rows to FP32 (for feeding the reference worker's FP32 API). */
void
orc_decode_rows(uint32_t dtype, uint32_t dims, uint64_t first, uint64_t count,
				const void *codes, const uint8_t *blockScales, const float *rowScales,
				float *out, int threads)
{
	OrcCorpus	c;

	c.dtype = dtype;
	c.dims = dims;
	c.rows = first + count;
	c.codes = (const uint8_t *) codes;
	c.blockScales = blockScales;
	c.rowScales = rowScales;
	c.rowBytes = orc_row_bytes(dtype, dims);
	if (threads < 1)
		threads = 1;
	{
		DecodeTask	task = {&c, first, out};

		ParallelFor(count, threads, DecodeTaskRun, &task);
	}
}
