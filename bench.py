#!/usr/bin/env python
"""Throughput of the exact gather-scan on BASELINE.json's config 2.

Workload: cosine kNN over halfvec (FP16) rows, d=768, N=10M
unit-normalised rows from a 1,000-centre Gaussian mixture, a uniform 10%
row-filter bitmap (the scan gathers the ~1M surviving rows), batch 1,024
queries, k=100. Data are seeded synthetic stand-ins generated on the GPU.

One step = one request: the filter bitmap is expanded to a row list on the
device, the batch is scanned (tcgen05 FP16 scan, bound, filter, exact FP64
rescoring), and with N GPUs the corpus is row-sharded: every rank scans its
rows, the per-rank top-k lists are all-gathered over NCCL and merged on the
device (strong scaling: the 10M-row corpus is fixed, N GPUs share it).

  value  queries/s with inputs resident in HBM (CUDA events, max over ranks)
  e2e    the same through the public API with pinned host buffers: queries
         and the bitmap copied in, results copied out, every step
  roofline  the filter scan (the dominant kernel), timed by the library's
         CUDA-event stage clock on its stream during the timed region

    python bench.py [--gpus N --steps K --warmup W]
    python bench.py --impl reference ...   the reference's CPU worker code
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'QPS at batch 1024, k=100 (1/2/4/8 B200); achieved HBM GB/s vs peak'
WORKLOAD = ('config 2: cosine kNN, halfvec (fp16) d=768, N=10M unit-normalised rows from a 1,000-centre '
            'Gaussian mixture, uniform 10% row-filter bitmap, batch 1,024, k=100')


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=40)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--rows', type=int, default=10_000_000)
    ap.add_argument('--dims', type=int, default=768)
    ap.add_argument('--batch', type=int, default=1024)
    ap.add_argument('--k', type=int, default=100)
    ap.add_argument('--selectivity', type=float, default=0.1)
    ap.add_argument('--centres', type=int, default=1000)
    ap.add_argument('--seed', type=int, default=20261201)
    ap.add_argument('--cpu-seconds', type=float, default=12.0, help='bound of the CPU-baseline sample')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--verify', type=int, default=2, help='queries checked against the CPU oracle (N=1)')
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, 'MEASURED_PEAKS.json')) as f:
            p = json.load(f)
        return p['hbm_gbs'], p['bf16_tflops'], p.get('bf16_tflops_sustained', p['bf16_tflops']), 'measured'
    except Exception:
        return 6650.0, 1590.0, 1400.0, 'fallback'


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '--query-gpu=' + self.FIELDS, '--format=csv,noheader,nounits',
                                          '-i', str(self.gpu), '-lms', '200'], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.thread.join(2)
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith('active'):
                    reasons.add(name)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ---------------------------------------------------------------- CPU baseline (reference worker code)

def cpu_sample(args, rows, queries):
    """A bounded sample of the workload on the host: `rows` candidate rows of
    the config-2 distribution (FP16 values decoded to FP32 exactly) and
    `queries` queries, numpy-generated from the same mixture."""
    import numpy as np
    from pgvector_b200 import synth
    x = synth.mixture(rows, args.dims, args.centres, seed=args.seed, normalize=True).astype(np.float16)
    q = synth.mixture_queries(queries, args.dims, args.centres, seed=args.seed, normalize=True)
    return x.astype(np.float32), q.astype(np.float16).astype(np.float32)


def cpu_run(x, q, k, threads, budget_s=None, count=None):
    """Gathered cosine jobs through the reference's AnnGatheredExact
    (oracle/_ref, ann/server/cpu.c:218-276) -- or the oracle's restatement
    when the reference library is absent -- on `threads` host threads, for
    budget_s seconds or exactly `count` queries; returns (queries done,
    seconds, kind)."""
    from concurrent.futures import ThreadPoolExecutor
    import oracle
    kind = 'reference' if oracle.ref_available() else 'port'

    def one(i):
        if kind == 'reference':
            st, res = oracle.ref_gathered_exact(q[i % len(q)], x, k, 2)
        else:
            oracle.search(oracle.F32, x.shape[1], x, q[i % len(q)][None], k, 2, window=True, threads=1)
        return 1

    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        if count is not None:
            done = sum(pool.map(one, range(count)))
        else:
            while time.perf_counter() - t0 < budget_s:
                done += sum(pool.map(one, range(done, done + threads)))
    return done, time.perf_counter() - t0, kind


def full_candidates(args):
    return int(round(args.rows * args.selectivity))


def reference_arm(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    sample_rows = 100_000
    x, q = cpu_sample(args, sample_rows, 64)
    per_step = max(threads, 8)
    scale = sample_rows / full_candidates(args)
    for _ in range(args.warmup):
        cpu_run(x, q, args.k, threads, count=per_step)
    total_q, total_s, kind = 0, 0.0, 'reference'
    for _ in range(args.steps):
        done, secs, kind = cpu_run(x, q, args.k, threads, count=per_step)
        total_q += done
        total_s += secs
    qps = total_q / total_s * scale
    line = {'metric': METRIC, 'value': qps, 'unit': 'queries/s', 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': args.batch / qps * 1e3,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
            'data': 'synthetic (seeded 1,000-centre Gaussian mixture, unit-normalised, FP16 values)',
            'config': {'workload': WORKLOAD, 'global_batch': args.batch, 'rows': args.rows, 'dims': args.dims,
                       'k': args.k, 'selectivity': args.selectivity, 'parallelism': 'host threads'},
            'impl': 'reference',
            'cpu_baseline': {'value': qps, 'unit': 'queries/s', 'cores': threads, 'kind': kind,
                             'sample': '%d queries a step x %d candidate rows (cosine, k=%d, gathered jobs via '
                                       'AnnGatheredExact), time scaled linearly to %d candidate rows'
                                       % (per_step, sample_rows, args.k, full_candidates(args))},
            'e2e': {'value': qps, 'unit': 'queries/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm

def main():
    args = args_parse()
    if args.impl == 'reference':
        return reference_arm(args)
    os.environ.setdefault('ANN_B200_KERNEL_TIMING', '1')
    import numpy as np
    import torch
    import torch.distributed as dist
    import pgvector_b200 as pb
    from pgvector_b200 import sharded, synth
    from datetime import timedelta

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=timedelta(seconds=180), device_id=dev)
    lib = pb.load()

    # ---- data: this rank's contiguous row range of the global corpus
    bounds = sharded.shard_bounds(args.rows, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    chunk = 1 << 20
    codes = torch.empty((hi - lo, args.dims), dtype=torch.float16, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    centres = torch.randn((args.centres, args.dims), generator=g, device=dev)
    for c0 in range(lo // chunk * chunk, hi, chunk):
        g.manual_seed(args.seed * 1000003 + c0 // chunk)
        m = min(chunk, args.rows - c0)
        lab = torch.randint(0, args.centres, (m,), generator=g, device=dev)
        v = centres[lab] + 0.1 * torch.randn((m, args.dims), generator=g, device=dev)
        v /= v.norm(dim=1, keepdim=True).clamp_min(1e-30)
        a, b = max(c0, lo), min(c0 + m, hi)
        codes[a - lo:b - lo] = v[a - c0:b - c0].to(torch.float16)
        del v, lab
    g.manual_seed(args.seed + 7919)
    lab = torch.randint(0, args.centres, (args.batch,), generator=g, device=dev)
    qv = centres[lab] + 0.1 * torch.randn((args.batch, args.dims), generator=g, device=dev)
    qv /= qv.norm(dim=1, keepdim=True)
    queries = qv.to(torch.float16).to(torch.float32).contiguous()       # halfvec query values
    words = synth.torch_bitmap(args.rows, args.selectivity, seed=args.seed + 1, device=dev)
    my_words, nbits = sharded.bitmap_slice(words, lo, hi)
    my_words = my_words.contiguous()
    del centres, qv, lab
    torch.cuda.synchronize()

    shard = pb.Shard(pb.F16, args.dims, codes, first_id=lo)
    k = args.k

    def step(q, w):
        rows = pb.bitmap_rows(w, nbits)
        d, i, c = sharded.search_sharded(shard, q, k, pb.COSINE, rows)
        return d, i, c, rows.numel()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident value (the clock sampler starts before warm-up so
    # its start-up stays outside the timed region)
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    for _ in range(args.warmup):
        step(queries, my_words)
    barrier()
    stage_ms = (ctypes.c_double * 9)()
    stage_calls = (ctypes.c_ulonglong * 9)()
    lib.AnnB200StageTimes(stage_ms, stage_calls, 9, 1)
    launches0 = lib.AnnB200LaunchCount()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    nrows_local = 0
    for _ in range(args.steps):
        out = step(queries, my_words)
        nrows_local = out[3]
    e1.record()
    barrier()
    clock_info = clocks.stop() if clocks else None
    launches = lib.AnnB200LaunchCount() - launches0
    lib.AnnB200StageTimes(stage_ms, stage_calls, 9, 0)
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = args.steps * args.batch / (ms / 1e3)
    result = out

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        hq = queries.cpu().pin_memory()
        hw = my_words.cpu().pin_memory()
        hd = torch.empty((args.batch, k), dtype=torch.float64).pin_memory()
        hi_ = torch.empty((args.batch, k), dtype=torch.int64).pin_memory()
        dq = torch.empty_like(queries)
        dw = torch.empty_like(my_words)
        for _ in range(args.warmup):
            dq.copy_(hq, non_blocking=True)
            dw.copy_(hw, non_blocking=True)
            d, i, c, _n = step(dq, dw)
            hd.copy_(d[:, :k], non_blocking=True)
            hi_.copy_(i[:, :k], non_blocking=True)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(args.steps):
            dq.copy_(hq, non_blocking=True)
            dw.copy_(hw, non_blocking=True)
            d, i, c, _n = step(dq, dw)
            hd.copy_(d[:, :k], non_blocking=True)
            hi_.copy_(i[:, :k], non_blocking=True)
        f1.record()
        barrier()
        ems = max_over_ranks(f0.elapsed_time(f1))
        e2e = {'value': args.steps * args.batch / (ems / 1e3), 'unit': 'queries/s',
               'h2d_bytes_per_step': int(hq.numel() * 4 + hw.numel() * 4),
               'd2h_bytes_per_step': int(hd.numel() * 8 + hi_.numel() * 8) if rank == 0 else 0,
               'ms_per_step': ems / args.steps}

    # ---- roofline of the filter pass (stage 3: every tcgen05 scan launch of
    # one step's filter pass, timed by the library's stage clock on its
    # stream). Algorithmic work per pass: 2 * batch * candidate rows * dims
    # FLOPs; algorithmic bytes: the candidate rows (dims * 2 B + 4 B row id)
    # plus the FP16 query block.
    hbm, tf_burst, tf_sust, kind = peaks()
    pass_ms = stage_ms[3] / args.steps
    flops = 2.0 * args.batch * nrows_local * args.dims
    achieved_tf = flops / (pass_ms * 1e-3) / 1e12
    bytes_alg = nrows_local * (args.dims * 2 + 4) + args.batch * args.dims * 2
    traffic = None
    tpath = os.path.join(ROOT, 'profiles', 'tc_scan_f16_config2.md')
    if os.path.exists(tpath):
        for line in open(tpath):
            if line.startswith('traffic_bytes_per_row:'):
                traffic = float(line.split(':', 1)[1]) * nrows_local
    roofline = {'bound': 'tensor', 'achieved': achieved_tf, 'peak': tf_sust, 'unit': 'TFLOP/s',
                'frac': achieved_tf / tf_sust, 'traffic': traffic,
                'kernel': 'tc_scan_f16, filter pass (%d launches a step)' % round(stage_calls[3] / args.steps),
                'peak_source': kind + ' bf16_tflops_sustained', 'pass_ms': pass_ms, 'flops_per_pass': flops,
                'algorithmic_bytes_per_pass': bytes_alg,
                'hbm_achieved_gbs': bytes_alg / (pass_ms * 1e-3) / 1e9, 'hbm_peak_gbs': hbm,
                'hbm_frac': bytes_alg / (pass_ms * 1e-3) / 1e9 / hbm,
                'stage_ms_per_step': {n: stage_ms[j] / args.steps for j, n in enumerate(
                    ['prep', 'sample_scan', 'bound', 'filter_scan', 'tighten', 'finalize', 'bitmap', 'merge',
                     'gather'])}}

    # ---- correctness spot check against the CPU oracle (single GPU)
    verified = None
    if world == 1 and args.verify > 0:
        import oracle
        rows_t = pb.bitmap_rows(my_words, nbits)
        rows_np = rows_t.cpu().numpy().view(np.uint32).astype(np.int64)
        h = codes[rows_t.long()].cpu().numpy().view(np.uint16)          # only the candidate rows
        qn = queries[:args.verify].cpu().numpy()
        od, oi, oc, _ = oracle.search(oracle.F16, args.dims, h, qn, k, 2)
        verified = bool(np.array_equal(result[1][:args.verify].cpu().numpy(), rows_np[oi] + lo) and
                        np.array_equal(result[0][:args.verify].cpu().numpy(), od))
        del h

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        x, q = cpu_sample(args, 50_000, 64)
        done, secs, ckind = cpu_run(x, q, k, threads, budget_s=args.cpu_seconds)
        scale = 50_000 / full_candidates(args)
        cpu = {'value': done / secs * scale, 'unit': 'queries/s', 'cores': threads, 'kind': ckind,
               'sample': '%d cosine gathered jobs (k=%d) over %d candidate rows of the config-2 distribution '
                         'in %.1f s on %d threads, scaled linearly to %d candidate rows'
                         % (done, k, 50_000, secs, threads, full_candidates(args))}

    if rank == 0:
        line = {'metric': METRIC, 'value': value, 'unit': 'queries/s', 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True,
                'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f16',
                'data': 'synthetic (seeded 1,000-centre Gaussian mixture, unit-normalised, generated on the GPU)',
                'config': {'workload': WORKLOAD, 'global_batch': args.batch, 'rows': args.rows, 'dims': args.dims,
                           'k': args.k, 'selectivity': args.selectivity,
                           'candidate_rows': int(nrows_local) * world,
                           'l2': 'inputs larger than L2 (%.2f GB of gathered rows a step)'
                                 % (nrows_local * world * args.dims * 2 / 1e9),
                           'parallelism': 'row-sharded x%d, NCCL all-gather of top-k + device merge' % world
                           if world > 1 else 'single GPU'},
                'e2e': e2e, 'gpu_launches': int(launches), 'roofline': roofline, 'cpu_baseline': cpu,
                'clocks': clock_info, 'verified_vs_oracle': verified}
        print(json.dumps(line), flush=True)
    shard.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == '__main__':
    sys.exit(main())
