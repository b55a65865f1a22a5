"""The row-sharded search through libannb200's own NCCL communicator
(AnnB200SearchSharded / AnnB200SearchListsSharded): per-rank search, one
all-gather of the ranks' packets, device merge -- against the oracle over
the whole corpus, bit for bit.

One GPU: a one-rank communicator runs the whole exchange (packet, NCCL
all-gather, merge, header check), including the second round that follows a
candidate-list overflow. Two GPUs (skipped with fewer): two processes, one a
GPU, each holding half the rows; and a rank that never joins, whose peer's
exchange ends with ANN_BACKEND_ERROR at the communicator's time limit (the
communicator is aborted; no GPU faults). NVLS is off in these tests
(NCCL_NVLS_ENABLE=0)."""
import os
import socket

import numpy as np
import pytest

import oracle
from pgvector_b200 import sharded, synth

pytestmark = pytest.mark.gpu


def to_dev(a, dev):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    return torch.from_numpy(a).to(dev)


def one_rank_comm(device=0):
    import pgvector_b200 as pb
    return pb.Comm(device, 1, 0, pb.Comm.unique_id())


def same(got, want, nq):
    gd, gi, gc = (t.cpu().numpy() for t in got)
    od, oi, oc = want[:3]
    assert np.array_equal(gc, oc.astype(gc.dtype))
    for q in range(nq):
        c = int(oc[q])
        assert np.array_equal(gi[q, :c], oi[q, :c]), q
        assert np.array_equal(gd[q, :c], od[q, :c]), q


def test_one_rank_exchange_equals_oracle(cuda):
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    import pgvector_b200 as pb
    comm = one_rank_comm()
    try:
        # FP16 cosine over a filter row list (the headline workload's path)
        x = synth.mixture(50000, 256, 40, seed=11, normalize=True)
        h = synth.to_half_bits(x)
        q = synth.mixture_queries(300, 256, 40, seed=12, normalize=True).astype(np.float16).astype(np.float32)
        words, ids = synth.bitmap(50000, 0.5, seed=13)
        shard = pb.Shard(pb.F16, 256, to_dev(h, cuda), first_id=1000)
        got = shard.search_sharded(comm, to_dev(q, cuda), 50, pb.COSINE, rows=to_dev(ids, cuda))
        od, oi, oc, _ = oracle.search(oracle.F16, 256, h, q, 50, 2, ids=ids)
        want = (od, np.where(oi >= 0, oi + 1000, -1), oc)
        same(got, want, 300)
        # the same filter as a bitmap (AnnB200SearchBitmap), through the
        # communicator and without one
        for c, bx in ((comm, False), (comm, True), (None, False)):
            d, i, cnt, n = shard.search_bitmap(c, to_dev(q, cuda), 50, pb.COSINE, to_dev(words.view(np.int32), cuda),
                                               50000, bounds_exchange=bx)
            assert n == len(ids)
            same((d, i, cnt), want, 300)
        # an empty bitmap: no rows, no results; a bitmap longer than the shard: INVALID
        zero = np.zeros_like(words)
        d, i, cnt, n = shard.search_bitmap(comm, to_dev(q, cuda), 50, pb.COSINE, to_dev(zero.view(np.int32), cuda),
                                           50000)
        assert n == 0 and int(cnt.sum()) == 0
        with pytest.raises(pb.AnnB200Error) as err:
            shard.search_bitmap(comm, to_dev(q, cuda), 50, pb.COSINE, to_dev(words.view(np.int32), cuda), 50001)
        assert err.value.status == pb.INVALID
        # bit rows, Hamming, whole shard
        rows, proto = synth.bit_rows(40000, 512, 64, flip=0.05, seed=14)
        qs = rows[np.arange(0, 40000, 997)][:40] ^ 1
        bshard = pb.Shard(pb.BIT, 512, to_dev(rows, cuda))
        same(bshard.search_sharded(comm, to_dev(qs, cuda), 100, pb.HAMMING), oracle.search(oracle.BIT, 512, rows, qs,
                                                                                              100, 3), 40)
        # heavy ties: 30,000 identical rows overflow the candidate lists and
        # need the large sort -- the second, synchronous round
        t = synth.mixture(36000, 64, 8, seed=15)
        t[3000:33000] = t[7]
        q2 = np.repeat(t[7:8], 20, axis=0) + np.float32(1e-3)
        tshard = pb.Shard(pb.F32, 64, to_dev(t, cuda))
        same(tshard.search_sharded(comm, to_dev(q2, cuda), 40, pb.L2), oracle.search(oracle.F32, 64, t, q2, 40, 0), 20)
        # IVF lists
        xi, offsets, cent, row_ids = synth.ivf_corpus(30000, 96, 64, seed=16)
        qi = (cent[np.arange(48) % 64] + 0.05).astype(np.float32)
        probes = synth.ivf_probes(qi, cent, 6)
        hi_ = synth.to_half_bits(xi)
        lshard = pb.Shard(pb.F16, 96, to_dev(hi_, cuda))
        got = lshard.search_lists_sharded(comm, to_dev(qi, cuda), 20, pb.L2, to_dev(offsets, cuda),
                                          to_dev(probes, cuda), row_ids=to_dev(row_ids, cuda))
        same(got, oracle.search_lists(oracle.F16, 96, hi_, qi, offsets, probes, 20, 0, row_ids=row_ids), 48)
        for s in (shard, bshard, tshard, lshard):
            s.close()
    finally:
        comm.close()


def free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


ROWS, DIMS, NQ, K = 60000, 192, 200, 64
# two query blocks (the tensor scan takes 4,096 queries a launch), each with
# its own exchange of bounds between the ranks
MB_ROWS, MB_DIMS, MB_NQ, MB_K = 6000, 64, 4100, 16


def multi_block_case():
    x = synth.mixture(MB_ROWS, MB_DIMS, 20, seed=24)
    q = synth.mixture_queries(MB_NQ, MB_DIMS, 20, seed=25)
    return x, q


def two_gpu_case():
    x = synth.mixture(ROWS, DIMS, 30, seed=21, normalize=True)
    h = synth.to_half_bits(x)
    q = synth.mixture_queries(NQ, DIMS, 30, seed=22, normalize=True).astype(np.float16).astype(np.float32)
    words, ids = synth.bitmap(ROWS, 0.4, seed=23)
    return h, q, words, ids


def two_gpu_worker(rank, world, port, out, missing):
    import torch
    import torch.distributed as dist
    import pgvector_b200 as pb
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0',
                      ANN_B200_COMM_TIMEOUT_MS='3000')
    torch.cuda.set_device(rank)
    dev = torch.device('cuda', rank)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    comm = None
    try:
        comm = sharded.comm_from_process_group(rank)
        h, q, words, _ = two_gpu_case()
        b = sharded.shard_bounds(ROWS, world)
        lo, hi = b[rank], b[rank + 1]
        w, nbits = sharded.bitmap_slice(words, lo, hi)
        rows = pb.bitmap_rows(to_dev(w.view(np.int32), dev), nbits)
        shard = pb.Shard(pb.F16, DIMS, to_dev(h[lo:hi], dev), first_id=lo)
        qd = to_dev(q, dev)
        if missing:
            # rank 1 never joins the exchange (it stays idle, with nothing in
            # flight); rank 0's call must end with an error at the time limit
            if rank == 0:
                try:
                    shard.search_sharded(comm, qd, K, pb.COSINE, rows=rows)
                    out[rank] = 'no error'
                except pb.AnnB200Error as e:
                    out[rank] = (e.status, str(e))
            dist.barrier()
        else:
            d, i, c = shard.search_sharded(comm, qd, K, pb.COSINE, rows=rows)
            torch.cuda.synchronize()
            out[rank] = (d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy())
            d, i, c = shard.search_sharded(comm, qd, K, pb.COSINE, rows=rows, bounds_exchange=True)
            out[(rank, 'bounds')] = (d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy())
            # rank 1 has no candidate rows: its search ends before the bounds
            # exchange, which it still takes part in
            mine = rows if rank == 0 else rows[:0]
            d, i, c = shard.search_sharded(comm, qd, K, pb.COSINE, rows=mine, bounds_exchange=True)
            out[(rank, 'empty')] = (d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy())
            # two query blocks over an unfiltered FP32 shard
            x, q2 = multi_block_case()
            b2 = sharded.shard_bounds(MB_ROWS, world)
            s2 = pb.Shard(pb.F32, MB_DIMS, to_dev(x[b2[rank]:b2[rank + 1]], dev), first_id=b2[rank])
            d, i, c = s2.search_sharded(comm, to_dev(q2, dev), MB_K, pb.L2, bounds_exchange=True)
            out[(rank, 'blocks')] = (d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy())
            s2.close()
            dist.barrier()
        shard.close()
    finally:
        if comm is not None:
            if missing:
                comm.abort()           # the group is gone: wait for none of it
            comm.close()
        dist.destroy_process_group()


def run_two(missing):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    mp.start_processes(two_gpu_worker, args=(2, free_port(), out, missing), nprocs=2, join=True,
                       start_method='spawn')
    return out


def test_two_gpu_sharded_search_equals_whole(cuda):
    out = run_two(False)
    h, q, _, ids = two_gpu_case()
    od, oi, oc, _ = oracle.search(oracle.F16, DIMS, h, q, K, 2, ids=ids)
    half = sharded.shard_bounds(ROWS, 2)[1]
    ed, ei, ec, _ = oracle.search(oracle.F16, DIMS, h, q, K, 2, ids=ids[ids < half])
    x, q2 = multi_block_case()
    md, mi, mc, _ = oracle.search(oracle.F32, MB_DIMS, x, q2, MB_K, 0)
    for r in range(2):
        for (d, i, c), (wd, wi, wc) in ((out[r], (od, oi, oc)), (out[(r, 'bounds')], (od, oi, oc)),
                                        (out[(r, 'empty')], (ed, ei, ec)), (out[(r, 'blocks')], (md, mi, mc))):
            assert np.array_equal(c, wc.astype(c.dtype))
            assert np.array_equal(i, wi) and np.array_equal(d, wd)


def test_two_gpu_missing_rank_times_out(cuda):
    import pgvector_b200 as pb
    out = run_two(True)
    status, msg = out[0]
    assert status == pb.BACKEND_ERROR and 'did not finish' in msg


def test_two_gpu_loaded_index_parts_equal_one_device(cuda):
    # AnnB200IndexCreateSharded: a loaded index's FP32 rows row-sharded over
    # two GPUs answers exactly as the same index on one GPU (which equals the
    # reference's loaded-index search), unfiltered and over ordinal lists
    import ctypes
    import torch
    import pgvector_b200 as pb
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    lib = pb.load()
    n, d, nq = 50001, 96, 40
    x = synth.mixture(n, d, 25, seed=31)
    q = synth.mixture_queries(nq, d, 25, seed=32)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    one, two = ctypes.c_void_p(), ctypes.c_void_p()
    devs = (ctypes.c_int * 2)(0, 1)
    assert lib.AnnB200IndexCreate(0, d, n, P(x), ctypes.byref(one)) == 0
    assert lib.AnnB200IndexCreateSharded(2, devs, d, n, P(x), ctypes.byref(two)) == 0
    try:
        rng = np.random.default_rng(33)
        cases = [(None, 10), (None, 100), (np.sort(rng.choice(n, 7000, replace=False)).astype(np.uint64), 25),
                 (np.arange(24990, 25020, dtype=np.uint64), 12), (np.arange(5, 40, dtype=np.uint64), 50)]
        for ords, k in cases:
            out = []
            for ix in (one, two):
                dist = np.zeros((nq, k), np.float32)
                o = np.zeros((nq, k), np.uint64)
                cnt = np.zeros(nq, np.uint32)
                assert lib.AnnB200IndexSearch(ix, P(q), nq, None if ords is None else P(ords),
                                              0 if ords is None else len(ords), k, P(dist), P(o), P(cnt)) == 0
                out.append((dist.view(np.uint32).tolist(), o.tolist(), cnt.tolist()))
            assert out[0] == out[1], k
    finally:
        lib.AnnB200IndexDestroy(one)
        lib.AnnB200IndexDestroy(two)
