"""Index directories with a quantized copy, and the oracle of the quantized
scan route, without a GPU.

* The directory writer's quantized files are what the reference's own
  loader accepts (AnnIndexFileOpen maps vectors.e4m3 / vectors.nvfp4 +
  scales.e4m3 + rowscale.f32 at their documented sizes,
  ann/server/indexfile.c:2492-2507, and refuses a short file), loaded through
  the reference cpu backend compiled from its sources.
* The restated re-score (ExactDistance, ann/server/cuvs.c:2930-2942) equals
  a plain FP64 loop in dimension order, and the restated route equals the
  full ranking by that distance whenever k + slack covers every eligible row.
"""
import ctypes
import math
import os

import numpy as np
import pytest

import oracle
from pgvector_b200 import _abi, synth


def test_exact_distance_f64_is_the_sequential_fp64_loop():
    rng = np.random.default_rng(3)
    for d in (1, 7, 37, 96):
        rows = (rng.standard_normal((5, d)) * 10 ** rng.uniform(-3, 3, (5, 1))).astype(np.float32)
        q = rng.standard_normal(d).astype(np.float32)
        got = oracle.exact_distance_f64(rows, q)
        for r in range(5):
            s = 0.0
            for j in range(d):
                delta = float(rows[r, j]) - float(q[j])
                s += delta * delta
            assert got[r] == np.float32(math.sqrt(s))


@pytest.mark.parametrize('kind', ['fp8', 'nvfp4'])
def test_route_with_room_for_every_row_is_the_full_ranking(kind):
    rng = np.random.default_rng(5)
    n, d = 600, 40
    x = synth.mixture(n, d, 6, seed=5)
    q = synth.mixture_queries(3, d, 6, seed=6)
    if kind == 'fp8':
        codes, rs = oracle.quantize_fp8(x)
        bs, dt = None, oracle.E4M3
    else:
        codes, bs, rs = oracle.quantize_nvfp4(x)
        dt = oracle.NVFP4
    ords = np.sort(rng.choice(n, 300, replace=False))
    for o in (None, ords):
        got = oracle.quant_index_search(dt, x, codes, q, 12, [0, 200, 450, n], ordinals=o, block_scales=bs,
                                        row_scales=rs, quant_slack=n)
        elig = np.arange(n) if o is None else ords
        for qi in range(len(q)):
            dist = oracle.exact_distance_f64(x[elig], q[qi])
            order = np.lexsort((elig, dist))[:12]
            assert got[qi] == [(int(elig[i]), dist[i]) for i in order]


def test_route_keeps_at_most_k_plus_slack_candidates_a_shard():
    # slack 0: each shard offers its k nearest by the codes alone
    n, d = 400, 32
    x = synth.mixture(n, d, 4, seed=9)
    q = synth.mixture_queries(2, d, 4, seed=10)
    codes, bs, rs = oracle.quantize_nvfp4(x)
    got = oracle.quant_index_search(oracle.NVFP4, x, codes, q, 5, [0, n], block_scales=bs, row_scales=rs,
                                    quant_slack=0, slack_ratio=0)
    for qi in range(len(q)):
        _, ids, cnt, _ = oracle.search(oracle.NVFP4, d, codes, q[qi:qi + 1], 5, 0, block_scales=bs,
                                       row_scales=rs)
        cand = ids[0, :cnt[0]]
        assert sorted(o for o, _ in got[qi]) == sorted(int(c) for c in cand)


def _cpu_backend():
    if not os.path.exists(oracle.REF_SO):
        pytest.skip('reference library not built (make -C oracle ref)')
    ref = ctypes.CDLL(oracle.REF_SO, mode=ctypes.RTLD_GLOBAL)
    ref.AnnCpuBackend.restype = ctypes.POINTER(_abi.AnnBackend)
    return ref.AnnCpuBackend().contents


@pytest.mark.parametrize('kind,d', [('fp8', 40), ('nvfp4', 40), ('nvfp4', 96)])
def test_reference_loader_accepts_the_quantized_copy(tmp_path, kind, d):
    cpu = _cpu_backend()
    n = 1000
    x = synth.mixture(n, d, 5, seed=2)
    keys = np.arange(n, dtype=np.int64) * 5 - 77
    quant = ('fp8',) + oracle.quantize_fp8(x) if kind == 'fp8' else ('nvfp4',) + oracle.quantize_nvfp4(x)
    directory = str(tmp_path / ('ix_%s_%d' % (kind, d)))
    synth.write_index_dir(directory, keys, x, shards=2, quant=quant)
    name = ('q_%s_%d_%d' % (kind, d, os.getpid())).encode()
    assert _abi.LOAD_INDEX(cpu.load_index)(name, directory.encode()) == 0
    # one job through the reference cpu backend: the directory serves
    job = (_abi.AnnIndexJob * 1)()
    qv = np.ascontiguousarray(x[17], dtype=np.float32)
    res = (_abi.AnnIndexHit * 3)()
    job[0].name = name
    job[0].dimensions = d
    job[0].k = 3
    job[0].query = qv.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    job[0].results = res
    _abi.SEARCH_INDEX(cpu.search_index)(job, 1)
    assert job[0].status == 0 and job[0].nresults == 3
    assert res[0].ordinal == 17 and res[0].distance == 0.0

    # a short quantized file is refused
    bad = str(tmp_path / ('bad_%s_%d' % (kind, d)))
    synth.write_index_dir(bad, keys, x, shards=1, quant=quant)
    victim = os.path.join(bad, 'scales.e4m3' if kind == 'nvfp4' else 'vectors.e4m3')
    with open(victim, 'r+b') as f:
        f.truncate(os.path.getsize(victim) - 1)
    assert _abi.LOAD_INDEX(cpu.load_index)(('bad_' + name.decode()).encode(), bad.encode()) != 0
