"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

    python tests/golden/make_golden.py [--reference REFERENCE_TREE]   (default: $ANN_REFERENCE)

quant.npz     the reference builder's quantize_fp8 / quantize_nvfp4
              (ann/builder/build_cuvs_index.py:314-348), imported from the
              reference tree, on seeded vectors with edge rows.
gathered.npz  the reference worker's AnnGatheredExact (ann/server/cpu.c:
              218-276), compiled from the reference sources into
              oracle/_ref/libannref.so by oracle/Makefile, on seeded jobs.
merge.npz     the reference's AnnIndexTreeMerge (ann/server/indexfile.c:
              3235-3258) on seeded sorted lists.

Needs the reference tree (this machine only); the fixtures it writes are
what the CPU tests read elsewhere.
"""
import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def load_builder(reference):
    path = os.path.join(reference, 'ann', 'builder', 'build_cuvs_index.py')
    spec = importlib.util.spec_from_file_location('reference_builder', path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def quant_inputs():
    rng = np.random.default_rng(20261201)
    blocks = []
    for dims in (7, 16, 33, 128):
        v = rng.standard_normal((24, dims)).astype(np.float32)
        v[0] = 0                                              # all-zero row
        v[1] *= 1e-6                                          # tiny values
        v[2] *= 1e4                                           # large values
        v[3] = np.where(rng.random(dims) < 0.5, -v[3], v[3]) * 3
        v[4, :] = np.linspace(-1, 1, dims, dtype=np.float32)  # exact ties to table midpoints
        v[5] = np.round(v[5] * 4) / 4
        blocks.append(v)
    return blocks


def main():
    ap = argparse.ArgumentParser()
    beside = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))),
                          'reference')
    ap.add_argument('--reference', default=os.environ.get('ANN_REFERENCE') or beside,
                    help='the reference tree (default: $ANN_REFERENCE, else `reference` beside this repository)')
    args = ap.parse_args()
    import oracle
    oracle.build(args.reference)
    builder = load_builder(args.reference)

    out = {}
    for i, v in enumerate(quant_inputs()):
        codes, scale = builder.quantize_fp8(v)
        packed, sc, row = builder.quantize_nvfp4(v)
        out['v%d' % i] = v
        out['fp8_codes%d' % i] = np.asarray(codes)
        out['fp8_scale%d' % i] = np.asarray(scale, dtype=np.float32)
        out['nvfp4_packed%d' % i] = np.asarray(packed)
        out['nvfp4_scales%d' % i] = np.asarray(sc)
        out['nvfp4_row%d' % i] = np.asarray(row, dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, 'quant.npz'), **out)

    rng = np.random.default_rng(42)
    jobs = {}
    n = 0
    for metric in (0, 1, 2):
        for dims, rows, k in ((7, 80, 1), (7, 80, 7), (16, 300, 10), (33, 500, 100), (96, 257, 400),
                              (2, 5, 1), (3, 64, 0)):
            v = np.round(rng.uniform(-2, 2, (rows, dims)), 2).astype(np.float32)
            q = np.round(rng.uniform(-2, 2, dims), 2).astype(np.float32)
            if n % 5 == 4:
                v[rows // 2:] = v[0]      # ties
            if dims == 2:
                v = np.array([[1, 0], [0, 1], [-1, 0], [0, -1], [3, 3]], dtype=np.float32)
                q = np.zeros(2, dtype=np.float32)
            status, res = oracle.ref_gathered_exact(q, v, k, metric)
            jobs['q%d' % n] = q
            jobs['v%d' % n] = v
            jobs['meta%d' % n] = np.array([k, metric, status], dtype=np.int64)
            jobs['ids%d' % n] = np.array([r[0] for r in res], dtype=np.int64)
            jobs['dist%d' % n] = np.array([r[1] for r in res], dtype=np.float64)
            n += 1
    jobs['count'] = np.array([n])
    np.savez_compressed(os.path.join(HERE, 'gathered.npz'), **jobs)

    merges = {}
    for t, (nlists, k) in enumerate(((1, 5), (3, 10), (8, 100), (5, 700))):
        lists = []
        for l in range(nlists):
            m = int(rng.integers(0, k + 1))
            keys = np.sort(rng.choice(1 << 20, m, replace=False)) * nlists + l
            d = np.round(rng.uniform(0, 10, m), 1).astype(np.float32)
            order = np.lexsort((keys, d))
            lists.append([(int(keys[i]), float(d[i])) for i in order])
        merged = oracle.ref_tree_merge(lists, k)
        merges['k%d' % t] = np.array([k])
        merges['lists%d' % t] = np.array([[l, key, d] for l, lst in enumerate(lists) for key, d in lst],
                                         dtype=np.float64).reshape(-1, 3)
        merges['nlists%d' % t] = np.array([nlists])
        merges['merged%d' % t] = np.array([[key, d] for key, d in merged], dtype=np.float64).reshape(-1, 2)
    merges['count'] = np.array([4])
    np.savez_compressed(os.path.join(HERE, 'merge.npz'), **merges)
    print('wrote quant.npz gathered.npz merge.npz')


if __name__ == '__main__':
    main()
