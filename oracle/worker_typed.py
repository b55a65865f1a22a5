"""Test infrastructure: the reference's ANN worker with the typed search op.

Copies the reference's ann/server and ann/common sources into a scratch
directory (oracle/_ref/worker_src, never committed), adds operation 32 --
typed gathered search, the server half of libannb200's typed jobs -- and
`--backend b200` there, then compiles two workers into oracle/_ref/:

  ann-worker-typed   the reference's own backends; their vtables leave the
                     new search_typed slot NULL, so operation 32 checks its
                     frame and answers "unsupported"
  ann-worker-b200    also libannb200's AnnB200WorkerBackend
                     (pgvector_b200/csrc/worker_index.c), which serves it

The C added below is this repository's own: the additions a maintainer
would make to ann/server/server.h, backend.h, server.c and worker.c. The
only text taken from the reference is the anchor lines that locate each
insertion; a missing anchor fails the build loudly instead of patching
blindly. Usage: python oracle/worker_typed.py [REF] (REF: the reference
checkout; default: ANN_REFERENCE, else a `reference` directory beside this
repository).
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, '_ref')

OP = '#define ANN_OP_TYPED_SEARCH 32\n'

TYPED_JOB = '''
/*
 * Typed gathered search (operation 32): host rows in a storage format -- 0
 * FP32, 1 FP16, 2 FP8-E4M3 with FP32 row scales, 3 NVFP4 with E4M3 block
 * scales (one a 16 dimensions) and FP32 row scales, 4 bits -- and a batch of
 * queries, answered with each query's gathered-job window (ANN_GATHERED_TOLERANCE).
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
	uint32_t   *ids;			/* [nq][cap] row numbers */
	uint32_t   *nresults;		/* [nq] */
	int			status;
} AnnTypedJob;

'''

SLOT = '''
	/* Typed gathered jobs (operation 32); sets each status. NULL: unsupported. */
	void		(*search_typed) (AnnTypedJob *, uint32_t);
'''

B200_DECL = '''#ifdef ANN_USE_B200
const AnnBackend *AnnB200WorkerBackend(void);
#endif
'''

HANDLER = r'''
/*
 * Operation 32, typed gathered search. Payload: u32 rows, dimensions, k,
 * metric (0 L2, 1 negative inner product, 2 cosine, 3 Hamming), dtype (0
 * FP32, 1 FP16, 2 FP8-E4M3, 3 NVFP4, 4 bits; Hamming goes with bits and
 * bits with Hamming), queries (1..4096); then the queries (FP32, or
 * ceil(dimensions / 8) bytes each for Hamming), the rows (row bytes 4d, 2d,
 * d rounded up to 16, d/2 rounded up to 8, ceil(d / 8)), the FP32 row
 * scales (FP8, NVFP4) and NVFP4's block scales (ceil(d / 16) bytes a row).
 * Reply: per query u32 count, then (u32 row, f64 distance) in order: the
 * gathered window of operation 7 for each query. Served on the reader
 * thread, outside the lanes.
 */
static AnnStatus
TypedSearch(Service *service, Connection *connection, uint64_t request,
			const unsigned char *payload, uint32_t size)
{
	AnnTypedJob job;
	uint64_t	rowBytes,
				queryBytes,
				need,
				cap,
				replySize = 0;
	uint32_t	rows,
				dimensions,
				metric,
				dtype,
				nq;
	const unsigned char *at;
	float	   *scales = NULL;
	double	   *distances;
	uint32_t   *ids,
			   *counts;
	unsigned char *reply,
			   *out;

	if (size < 24)
		return ANN_INVALID;
	rows = (uint32_t) Read(payload, 4);
	dimensions = (uint32_t) Read(payload + 4, 4);
	metric = (uint32_t) Read(payload + 12, 4);
	dtype = (uint32_t) Read(payload + 16, 4);
	nq = (uint32_t) Read(payload + 20, 4);
	if (dimensions == 0 || dimensions > ANN_MAX_DIM || metric > 3 || dtype > 4 ||
		(metric == 3) != (dtype == 4) || nq == 0 || nq > 4096)
		return ANN_INVALID;
	rowBytes = dtype == 0 ? 4ull * dimensions : dtype == 1 ? 2ull * dimensions :
		dtype == 2 ? (dimensions + 15ull) / 16 * 16 : dtype == 3 ? (dimensions + 15ull) / 16 * 8 :
		(dimensions + 7ull) / 8;
	queryBytes = metric == 3 ? (dimensions + 7ull) / 8 : 4ull * dimensions;
	need = 24 + nq * queryBytes + (uint64_t) rows * rowBytes;
	if (dtype == 2 || dtype == 3)
		need += 4ull * rows;
	if (dtype == 3)
		need += (uint64_t) rows * ((dimensions + 15) / 16);
	if (need != size)
		return ANN_INVALID;
	if (!LittleEndian())
		return ANN_UNSUPPORTED;
	if (service->backend->search_typed == NULL)
		return ANN_UNSUPPORTED;

	/* room for a whole window a query, within one frame's bytes */
	cap = rows ? rows : 1;
	if (nq * cap * 12 > ANN_MAX_BYTES)
		cap = ANN_MAX_BYTES / 12 / nq;
	distances = malloc(nq * cap * sizeof(double));
	ids = malloc(nq * cap * sizeof(uint32_t));
	counts = malloc(nq * sizeof(uint32_t));
	memset(&job, 0, sizeof(job));
	at = payload + 24;
	job.dtype = dtype;
	job.metric = metric;
	job.dimensions = dimensions;
	job.rows = rows;
	job.nq = nq;
	job.k = (uint32_t) Read(payload + 8, 4);
	job.cap = (uint32_t) cap;
	job.queries = at;
	at += nq * queryBytes;
	job.codes = at;
	at += (uint64_t) rows * rowBytes;
	if (dtype == 2 || dtype == 3)
	{
		/* the row scales at a 4-byte boundary (bit queries can leave them off one) */
		scales = malloc(rows ? 4ull * rows : 4);
		if (scales)
			memcpy(scales, at, 4ull * rows);
		job.row_scales = scales;
		at += 4ull * rows;
	}
	if (dtype == 3)
		job.block_scales = at;
	job.distances = distances;
	job.ids = ids;
	job.nresults = counts;
	if (distances == NULL || ids == NULL || counts == NULL || ((dtype == 2 || dtype == 3) && scales == NULL))
		job.status = ANN_NOMEM;
	else
		service->backend->search_typed(&job, 1);
	if (job.status == ANN_OK)
	{
		for (uint32_t q = 0; q < nq; q++)
			replySize += 4 + 12ull * counts[q];
		reply = malloc(replySize ? replySize : 1);
		if (reply == NULL)
			job.status = ANN_NOMEM;
		else
		{
			out = reply;
			for (uint32_t q = 0; q < nq; q++)
			{
				Write(out, counts[q], 4);
				out += 4;
				for (uint32_t r = 0; r < counts[q]; r++)
				{
					uint64_t	bits;

					memcpy(&bits, &distances[q * cap + r], sizeof(bits));
					Write(out, ids[q * cap + r], 4);
					Write(out + 4, bits, 8);
					out += 12;
				}
			}
			Reply(connection, ANN_OP_TYPED_SEARCH, request, ANN_OK, reply, (size_t) replySize);
			free(reply);
		}
	}
	free(distances);
	free(ids);
	free(counts);
	free(scales);
	return (AnnStatus) job.status;
}

'''

DISPATCH = '''	else if (operation == ANN_OP_TYPED_SEARCH)
	{
		status = TypedSearch(service, connection, request, payload, length);
		if (status != ANN_OK)
			Reply(connection, operation, request, status, NULL, 0);
	}
'''

SELECT = '''#ifdef ANN_USE_B200
			else if (strcmp(value, "b200") == 0)
				backend = AnnB200WorkerBackend();
#endif
'''


def insert(path, anchor, text, before=True):
    """Insert text before (or after) the one occurrence of anchor in path."""
    with open(path) as f:
        s = f.read()
    if s.count(anchor) != 1:
        raise SystemExit('%s: anchor found %d times: %r' % (path, s.count(anchor), anchor[:60]))
    i = s.index(anchor) if before else s.index(anchor) + len(anchor)
    with open(path, 'w') as f:
        f.write(s[:i] + text + s[i:])


def patch(src):
    server = os.path.join(src, 'server')
    insert(os.path.join(server, 'server.h'), '#define ANN_OP_INDEX_PREDICATE 23\n', OP, before=False)
    backend = os.path.join(server, 'backend.h')
    insert(backend, '/* Vendor-specific objects and precision/layout conversion stay behind this API. */',
           TYPED_JOB.lstrip('\n'))
    insert(backend, '\tint\t\t\t(*scan_preferred) (const struct AnnIndexFile *file, uint32_t k);\n', SLOT,
           before=False)
    insert(backend, 'const AnnBackend *AnnMockGpuBackend(void);\n', B200_DECL, before=False)
    server_c = os.path.join(server, 'server.c')
    insert(server_c, 'static int\nServeFrame(Service *service, Connection *connection)\n', HANDLER.lstrip('\n'))
    insert(server_c, '\telse if (operation == ANN_OP_ATTACH_SHARED)\n'
                     '\t\tReply(connection, operation, request, Attach(connection, payload, length), NULL, 0);\n',
           DISPATCH)
    insert(os.path.join(server, 'worker.c'),
           '\t\t\telse if (strcmp(value, "mock-gpu") == 0)\n\t\t\t\tbackend = AnnMockGpuBackend();\n', SELECT,
           before=False)


def build(ref, cc='gcc'):
    src = os.path.join(OUT, 'worker_src')
    if os.path.exists(src):
        shutil.rmtree(src)
    os.makedirs(src)
    for part in ('server', 'common'):
        shutil.copytree(os.path.join(ref, 'ann', part), os.path.join(src, part))
    patch(src)
    server = os.path.join(src, 'server')
    # the worker's sources and flags as its Makefile lists them (ann-worker),
    # without -Werror (a newer compiler's new warning must not fail the test
    # build); the reference's own backends initialise their vtables by
    # position and leave the new last slot to zero initialisation
    srcs = ['worker.c', 'cpu.c', 'mockgpu.c', 'batching.c', 'server.c', 'indexfile.c', '../common/filter.c',
            'canonical.c', 'udf.c', 'rdma.c']
    flags = ['-O2', '-g', '-std=c11', '-Wall', '-Wextra', '-Wno-missing-field-initializers', '-pedantic', '-I.',
             '-I../common', '-pthread']
    subprocess.run([cc] + flags + srcs + ['-lm', '-o', os.path.join(OUT, 'ann-worker-typed')], cwd=server,
                   check=True)
    lib_dir = os.path.join(ROOT, 'pgvector_b200')
    subprocess.run([cc] + flags + ['-DANN_USE_B200', '-I' + os.path.join(ROOT, 'include')] + srcs +
                   [os.path.join(ROOT, 'pgvector_b200', 'csrc', 'worker_index.c'), '-L' + lib_dir, '-lannb200',
                    '-Wl,-rpath,$ORIGIN/../../pgvector_b200', '-lm', '-o', os.path.join(OUT, 'ann-worker-b200')],
                   cwd=server, check=True)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        'ANN_REFERENCE', os.path.join(os.path.dirname(ROOT), 'reference'))
    if not os.path.isdir(os.path.join(ref, 'ann', 'server')):
        raise SystemExit('no reference tree at %s' % ref)
    build(ref)


if __name__ == '__main__':
    main()
