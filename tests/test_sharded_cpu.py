"""The multi-GPU path's host logic on CPU: two gloo ranks shard a corpus by
row range, search their shard (the CPU oracle stands in for the GPU scan),
all-gather the per-rank lists in the layout the device merge takes, merge,
and must equal one search over the whole corpus -- for the flat search over
a filter bitmap and for the IVF list search with lists cut at the rank
boundaries."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from pgvector_b200 import sharded, synth

ROWS, DIMS, NQ, K = 5000, 24, 6, 40


def free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


class OracleShard:
    """Stand-in for pgvector_b200.Shard on a CPU rank: same search contract
    (global ids = first_id + row, [nq][k] tensors)."""

    def __init__(self, x, first_id):
        self.x, self.first = x, first_id

    def search(self, queries, k, metric, rows=None):
        ids = None if rows is None else rows.numpy().view(np.uint32)
        d, i, c, s = oracle.search(oracle.F32, DIMS, self.x, queries.numpy(), k, metric, ids=ids, threads=1)
        i = np.where(i >= 0, i + self.first, -1)
        return torch.from_numpy(d), torch.from_numpy(i), torch.from_numpy(c.astype(np.int32))


def merge_host(gd, gi, gc, k):
    """Sorted union of the gathered lists by (distance, id): the device
    merge's contract, in numpy."""
    world, nq, cap = gd.shape
    od = np.full((nq, k), np.inf)
    oi = np.full((nq, k), -1, dtype=np.int64)
    oc = np.zeros(nq, dtype=np.int32)
    for q in range(nq):
        entries = sorted((float(gd[r, q, j]), int(gi[r, q, j])) for r in range(world) for j in range(int(gc[r, q])))
        entries = entries[:k]
        oc[q] = len(entries)
        for j, (d, i) in enumerate(entries):
            od[q, j], oi[q, j] = d, i
    return torch.from_numpy(od), torch.from_numpy(oi), torch.from_numpy(oc)


def worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world)
    try:
        x = synth.mixture(ROWS, DIMS, 10, seed=31)
        q = torch.from_numpy(synth.mixture_queries(NQ, DIMS, 10, seed=31))
        words, _ = synth.bitmap(ROWS, 0.3, seed=31)
        b = sharded.shard_bounds(ROWS, world)
        lo, hi = b[rank], b[rank + 1]
        w, nbits = sharded.bitmap_slice(words, lo, hi)
        bits = np.unpackbits(w.view(np.uint8), bitorder='little')[:nbits]
        rows = torch.from_numpy(np.nonzero(bits)[0].astype(np.uint32).view(np.int32))
        shard = OracleShard(x[lo:hi], lo)
        d, i, c = sharded.search_sharded(shard, q, K, 0, rows, merge=merge_host)
        out[rank] = (d.numpy(), i.numpy(), c.numpy())
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize('world', [2])
def test_two_rank_sharded_search_equals_whole(world):
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    mp.start_processes(worker, args=(world, free_port(), out), nprocs=world, join=True, start_method='spawn')
    x = synth.mixture(ROWS, DIMS, 10, seed=31)
    q = synth.mixture_queries(NQ, DIMS, 10, seed=31)
    _, ids = synth.bitmap(ROWS, 0.3, seed=31)
    od, oi, oc, _ = oracle.search(oracle.F32, DIMS, x, q, K, 0, ids=ids)
    for r in range(world):
        d, i, c = out[r]
        assert np.array_equal(c, oc.astype(np.int32))
        assert np.array_equal(i, oi) and np.array_equal(d, od)


IVF_ROWS, IVF_DIMS, IVF_LISTS, IVF_NQ, IVF_K, IVF_PROBE = 20000, 16, 24, 8, 30, 6


def ivf_case():
    # Zipf(1.6) list sizes: a few large lists, which the row split must cut
    x, offsets, cent, row_ids = synth.ivf_corpus(IVF_ROWS, IVF_DIMS, IVF_LISTS, zipf=1.6, seed=41)
    q = (cent[np.arange(IVF_NQ) % IVF_LISTS] + 0.05).astype(np.float32)
    probes = synth.ivf_probes(q, cent, IVF_PROBE)
    return x, offsets, row_ids, q, probes


def ivf_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world)
    try:
        x, offsets, row_ids, q, probes = ivf_case()
        lo, hi, l0, l1, loc = sharded.ivf_shard(offsets, world, rank)
        lp = sharded.local_probes(probes, l0, l1)
        d, i, c = oracle.search_lists(oracle.F32, IVF_DIMS, x[lo:hi], q, loc.astype(np.uint64), lp, IVF_K, 0,
                                      row_ids=row_ids[lo:hi], threads=1)
        gd, gi, gc = sharded.gather_lists(torch.from_numpy(d), torch.from_numpy(i),
                                          torch.from_numpy(c.astype(np.int32)))
        md, mi, mc = merge_host(gd.numpy(), gi.numpy(), gc.numpy(), IVF_K)
        out[rank] = (md.numpy(), mi.numpy(), mc.numpy(), hi - lo, l1 - l0)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize('world', [2])
def test_ivf_row_range_shards_equal_whole(world):
    # each rank holds equal rows of the list-major storage with lists cut at
    # the boundaries; its probes name only the lists it holds (the others are
    # padding); merging the ranks' lists gives the unsharded IVF search
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    mp.start_processes(ivf_worker, args=(world, free_port(), out), nprocs=world, join=True, start_method='spawn')
    x, offsets, row_ids, q, probes = ivf_case()
    od, oi, oc = oracle.search_lists(oracle.F32, IVF_DIMS, x, q, offsets, probes, IVF_K, 0, row_ids=row_ids)
    assert sum(out[r][3] for r in range(world)) == IVF_ROWS
    assert sum(out[r][4] for r in range(world)) > IVF_LISTS       # some list is cut
    for r in range(world):
        d, i, c = out[r][:3]
        assert np.array_equal(c, oc.astype(np.int32))
        for j in range(IVF_NQ):
            n = int(oc[j])
            assert np.array_equal(i[j, :n], oi[j, :n]) and np.array_equal(d[j, :n], od[j, :n])


def test_ivf_shard_tables():
    x, offsets, row_ids, q, probes = ivf_case()
    sizes = np.diff(offsets.astype(np.int64))
    for world in (1, 2, 3, 8):
        tot = np.zeros(IVF_LISTS, dtype=np.int64)
        for r in range(world):
            lo, hi, l0, l1, loc = sharded.ivf_shard(offsets, world, r)
            assert loc[0] == 0 and loc[-1] == hi - lo and (np.diff(loc) >= 0).all()
            tot[l0:l1] += np.diff(loc)
            lp = sharded.local_probes(probes, l0, l1)
            held = (probes >= l0) & (probes < l1)
            assert (lp[held] == probes[held] - l0).all() and (lp[~held] == 0xffffffff).all()
        assert (tot == sizes).all()


def test_shard_bounds_word_aligned():
    for rows in (1, 31, 32, 1000, 10_000_000):
        for world in (1, 2, 3, 4, 8):
            b = sharded.shard_bounds(rows, world)
            assert b[0] == 0 and b[-1] == rows and all(x % 32 == 0 for x in b[:-1])
            assert all(b0 <= b1 for b0, b1 in zip(b, b[1:]))


def check_worker(rank, world, port, out):
    # bench.py's multi-rank check: each rank answers with the oracle over its
    # own rows; rank 0 holds every rank's list and checks merged answers
    import bench
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.distributed.init_process_group('gloo', rank=rank, world_size=world)
    try:
        x = synth.mixture(ROWS, DIMS, 10, seed=37)
        q = synth.mixture_queries(NQ, DIMS, 10, seed=37)
        b = sharded.shard_bounds(ROWS, world)
        lo, hi = b[rank], b[rank + 1]
        d, i, c, _ = oracle.search(oracle.F32, DIMS, x[lo:hi], q, K, 0, threads=1)
        lists = bench.gather_objects((d, np.where(i >= 0, i + lo, -1), c), world)
        if rank == 0:
            out['lists'] = lists
    finally:
        torch.distributed.destroy_process_group()


def test_multi_rank_check_catches_bad_merges():
    import bench
    world = 2
    ctx = mp.get_context('spawn')
    mgr = ctx.Manager()
    out = mgr.dict()
    mp.start_processes(check_worker, args=(world, free_port(), out), nprocs=world, join=True, start_method='spawn')
    lists = out['lists']
    gd = np.stack([l[0] for l in lists])
    gi = np.stack([l[1] for l in lists])
    gc = np.stack([l[2].astype(np.int32) for l in lists])
    good = merge_host(gd, gi, gc, K)
    assert bench.check_global(good, lists, NQ, K)
    # and it is the whole corpus's answer
    x = synth.mixture(ROWS, DIMS, 10, seed=37)
    q = synth.mixture_queries(NQ, DIMS, 10, seed=37)
    od, oi, oc, _ = oracle.search(oracle.F32, DIMS, x, q, K, 0)
    assert np.array_equal(good[1].numpy(), oi) and np.array_equal(good[0].numpy(), od)
    # a merge that dropped rank 1's list
    dropped = merge_host(gd[:1], gi[:1], gc[:1], K)
    assert not bench.check_global(dropped, lists, NQ, K)
    # a merge that swapped two neighbours of one query's list
    d, i, c = (t.clone() for t in good)
    d[2, [3, 4]] = d[2, [4, 3]]
    i[2, [3, 4]] = i[2, [4, 3]]
    assert not bench.check_global((d, i, c), lists, NQ, K)
    # a merge that concatenated the ranks' lists without ordering them
    cat_d = np.concatenate([gd[1], gd[0]], axis=1)[:, :K]
    cat_i = np.concatenate([gi[1], gi[0]], axis=1)[:, :K]
    bad = (torch.from_numpy(cat_d), torch.from_numpy(cat_i), torch.full((NQ,), K, dtype=torch.int32))
    assert not bench.check_global(bad, lists, NQ, K)
    # the rank-0 rescoring check rejects a returned row whose distance is off
    part = [{'returned': {int(good[1][0, j]): float(good[0][0, j]) for j in range(K)},
             'sample': [(float(gd[1][0, j]), int(gi[1][0, j])) for j in range(K)]}]
    one = tuple(t[:1] for t in good)
    assert bench.check_rescored(one, [part], 1)
    off = tuple(t.clone() for t in one)
    off[0][0, 5] = np.nextafter(float(off[0][0, 5]), np.inf)
    assert not bench.check_rescored(off, [part], 1)


def test_bench_arms_share_the_workload_config(monkeypatch):
    # bench.py's two arms (ours, and --impl reference) print the same
    # `config`: the workload only; how each arm ran it sits beside it
    import sys
    import bench
    for config in (1, 2, 3, 4, 5):
        monkeypatch.setattr(sys, 'argv', ['bench.py', '--config', str(config)])
        args = bench.args_parse()
        cfg = bench.workload_config(args)
        assert cfg['workload'] == bench.WORKLOADS[config]
        assert {'global_batch', 'rows', 'dims', 'k', 'l2'} <= set(cfg)
        assert 'parallelism' not in cfg and 'candidate_rows' not in cfg
        assert ('selectivity' in cfg) == (config == 2)
