#!/usr/bin/env python
"""Throughput of the exact gather-scan on BASELINE.json's config 2.

Workload (configs[1], the default): cosine kNN over halfvec (FP16) rows,
d=768, N=10M unit-normalised rows from a 1,000-centre Gaussian mixture, a
uniform 10% row-filter bitmap (the scan gathers the ~1M surviving rows),
batch 1,024 queries, k=100. Data are seeded synthetic stand-ins generated on
the GPU.

One step = one request: the filter bitmap is expanded to a row list on the
device, the batch is scanned (tcgen05 FP16 scan, bound, filter, exact FP64
rescoring), and with N GPUs the corpus is row-sharded: every rank scans its
rows, the per-rank top-k lists are all-gathered over NCCL and merged on the
device (strong scaling: the corpus is fixed, N GPUs share it).

--config 3 / 4 / 5 measure the other GPU-sized configurations the same way
(not the headline line): 3 = inner product over FP8-E4M3 rows with row
scales, d=1024, N=100M from a 4,096-centre mixture, batch 1,024, k=500, no
filter; 4 = IVF search over NVFP4 rows, d=768, N=200M in 65,536 lists
with Zipf(1.1) sizes, nprobe=64, batch 4,096, k=100, L2 (each step probes the
FP32 centres, then gathers the probed lists), rows sharded by rank with lists
cut at the boundaries; 5 = Hamming over 1,024-bit rows, N=1B (128 GB: one B200 holds it)
XOR-perturbed from 65,536 random prototypes at a 5% flip rate, batch 1,024,
k=100, row-sharded.

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
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'QPS at batch 1024, k=100 (1/2/4/8 B200); achieved HBM GB/s vs peak'
WORKLOADS = {
    1: 'config 1: exact L2 kNN, fp32, d=128, N=100,000 rows from a 100-centre Gaussian mixture (centres ~N(0,1), '
       'sigma 0.1), 1,000 queries drawn the same way, k=10, no filter (the reference worker\'s CPU-runnable case)',
    2: 'config 2: cosine kNN, halfvec (fp16) d=768, N=10M unit-normalised rows from a 1,000-centre '
       'Gaussian mixture, uniform 10% row-filter bitmap, batch 1,024, k=100',
    3: 'config 3: inner-product kNN, FP8-E4M3 codes + per-row scale (absmax/448), d=1024, N=100M from a '
       '4,096-centre Gaussian mixture, batch 1,024, k=500, row-sharded',
    4: 'config 4: IVF gather-scan, NVFP4 (e2m1 + E4M3 scale per 16 + row scale), d=768, N=200M in 65,536 '
       'lists with Zipf(1.1) sizes, nprobe=64, batch 4,096, k=100, L2, sharded by row range (lists cut at '
       'rank boundaries)',
    5: 'config 5: Hamming kNN on 1,024-bit vectors, N=1B rows XOR-perturbed from 65,536 Bernoulli(0.5) '
       'prototypes at a 5% flip rate, batch 1,024, k=100, row-sharded; integer distances, ties by row id',
    6: 'config 6 (loaded index from its quantized copy): L2 kNN through AnnB200IndexSearch with host buffers, '
       'd=768, N=2M FP32 rows from a 1,000-centre Gaussian mixture (sigma 0.3) with their NVFP4 copy on the '
       'device in 3 index shards, the FP32 rows in host memory; batch 1,024, k=100, quant_slack 256, '
       'slack_ratio 100',
}
DEFAULTS = {1: dict(rows=100_000, dims=128, batch=1000, k=10, centres=100),
            2: dict(rows=10_000_000, dims=768, batch=1024, k=100, centres=1000),
            3: dict(rows=100_000_000, dims=1024, batch=1024, k=500, centres=4096),
            4: dict(rows=200_000_000, dims=768, batch=4096, k=100, centres=65536),
            5: dict(rows=1_000_000_000, dims=1024, batch=1024, k=100, centres=65536),
            6: dict(rows=2_000_000, dims=768, batch=1024, k=100, centres=1000)}


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=None, help='timed steps (default 300; 10 for configs 3/4, 5 for 5)')
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--config', type=int, default=2, choices=[1, 2, 3, 4, 5, 6])
    ap.add_argument('--rows', type=int, default=None)
    ap.add_argument('--dims', type=int, default=None)
    ap.add_argument('--batch', type=int, default=None)
    ap.add_argument('--k', type=int, default=None)
    ap.add_argument('--selectivity', type=float, default=0.1, help='config 2 row-filter bitmap density')
    ap.add_argument('--centres', type=int, default=None, help='mixture centres (config 4: IVF lists)')
    ap.add_argument('--nprobe', type=int, default=64)
    ap.add_argument('--seed', type=int, default=20261201)
    ap.add_argument('--cpu-seconds', type=float, default=12.0, help='bound of the CPU-baseline sample')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--verify', type=int, default=2, help='queries checked against the CPU oracle')
    args = ap.parse_args()
    for key, val in DEFAULTS[args.config].items():
        if getattr(args, key) is None:
            setattr(args, key, val)
    if args.steps is None:
        args.steps = {1: 300, 2: 300, 5: 5}.get(args.config, 10)
    return args


def peaks():
    try:
        with open(os.path.join(ROOT, 'MEASURED_PEAKS.json')) as f:
            p = json.load(f)
        return p['hbm_gbs'], p['bf16_tflops'], p.get('bf16_tflops_sustained', p['bf16_tflops']), 'measured'
    except Exception:
        return 6650.0, 1590.0, 1400.0, 'fallback'


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and throttle reasons sampled every 10 ms during a region,
    read through NVML in a thread of this process (nvidia-smi's -lms loop
    where NVML's Python binding is missing). Reading only: no setting of the
    GPU is touched."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
    NAMES = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.nvml = None
        self.samples = []         # (sm MHz, max MHz, set of reasons)
        self.lines = []
        self.skip = 0
        self.running = False

    def start(self, wait_s=10.0):
        """Start sampling and wait (up to wait_s) for the first reading, so
        that the sampler's own start-up stays outside any timed region; that
        first reading is not counted."""
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = None
            try:      # the CUDA device's own NVML handle, by PCI address (indices may differ)
                import torch
                pr = torch.cuda.get_device_properties(self.gpu)
                bus = '%08x:%02x:%02x.0' % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                pass
            if self.handle is None:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.bits = [pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap]
            self.running = True
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:
            self.nvml = None
            try:
                self.proc = subprocess.Popen(['nvidia-smi', '--query-gpu=' + self.FIELDS,
                                              '--format=csv,noheader,nounits', '-i', str(self.gpu), '-lms', '20'],
                                             stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.thread = threading.Thread(target=self._read, daemon=True)
                self.thread.start()
            except Exception:
                self.proc = None
                return
        t0 = time.perf_counter()
        while not (self.samples or self.lines) and time.perf_counter() - t0 < wait_s:
            time.sleep(0.005)
        self.skip = max(len(self.samples), len(self.lines))

    def mark(self):
        """Count readings from here on (the measured region starts)."""
        self.skip = max(len(self.samples), len(self.lines))

    def _poll(self):
        n = self.nvml
        while self.running:
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                mx = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
                r = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((float(sm), float(mx), {nm for nm, b in zip(self.NAMES, self.bits) if r & b}))
            except Exception:
                pass
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.strip().split(',')]
            if len(parts) < 9:
                continue
            try:
                self.samples.append((float(parts[1]), float(parts[2]),
                                     {nm for nm, v in zip(self.NAMES, parts[5:9]) if v.lower().startswith('active')}))
            except ValueError:
                continue

    def stop(self):
        if self.nvml is not None:
            self.running = False
            self.thread.join(2)
        elif self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            self.thread.join(2)
        else:
            return None
        got = self.samples[self.skip:]
        if not got:
            return None
        reasons = set()
        for _, _, r in got:
            reasons |= r
        return {'sm_mhz': statistics.median(x[0] for x in got), 'sm_max_mhz': got[-1][1],
                'reasons': sorted(reasons), 'samples': len(got), 'window': 'warm-up and timed region, 10 ms apart'}


# ---------------------------------------------------------------- CPU baseline (reference worker code)

METRIC_CODE = {1: 0, 2: 2, 3: 1, 4: 0, 5: 3}   # L2, cosine, inner product, L2, Hamming


def cpu_sample_device(args, rows, queries):
    """Config 2's host sample made on the GPU (numpy takes minutes for a
    million 768-d rows): `rows` rows of the bench's own seeded mixture,
    unit-normalised and rounded to FP16 as the shard stores them, copied to
    host memory as FP32, and `queries` of its queries. Only the data is made
    on the device; the timed work runs on the host cores."""
    import numpy as np
    import torch
    dev = torch.device('cuda', torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    centres = torch.randn((args.centres, args.dims), generator=g, device=dev)
    x = np.empty((rows, args.dims), np.float32)

    def fill(a, b, v):
        x[a:b] = v.to(torch.float16).to(torch.float32).cpu().numpy()
    mixture_rows(args, dev, 0, rows, centres, fill, normalize=True)
    g.manual_seed(args.seed + 7919)
    lab = torch.randint(0, args.centres, (queries,), generator=g, device=dev)
    qv = centres[lab] + 0.1 * torch.randn((queries, args.dims), generator=g, device=dev)
    qv /= qv.norm(dim=1, keepdim=True)
    q = qv.to(torch.float16).to(torch.float32).cpu().numpy()
    del centres, qv
    torch.cuda.empty_cache()
    return x, q


def cpu_sample(args, rows, queries):
    """A bounded host sample of the workload's distribution: `rows` rows
    decoded to FP32 exactly as the device format stores them (config 5: the
    bit rows themselves), and `queries` queries (numpy, same mixture)."""
    import numpy as np
    import oracle
    from pgvector_b200 import synth
    if args.config == 2 and rows > 100_000:
        try:
            import torch
            if torch.cuda.is_available():
                return cpu_sample_device(args, rows, queries)
        except ImportError:
            pass
    if args.config == 5:
        x, proto = synth.bit_rows(rows, args.dims, args.centres, flip=0.05, seed=args.seed)
        rng = np.random.default_rng(args.seed + 7919)
        flips = np.packbits(rng.random((queries, args.dims)) < 0.05, axis=1, bitorder='little')
        return x, proto[rng.integers(0, args.centres, queries)] ^ flips
    if args.config == 1:
        return (synth.mixture(rows, args.dims, args.centres, seed=args.seed),
                synth.mixture_queries(queries, args.dims, args.centres, seed=args.seed))
    if args.config == 2:
        x = synth.mixture(rows, args.dims, args.centres, seed=args.seed, normalize=True).astype(np.float16)
        q = synth.mixture_queries(queries, args.dims, args.centres, seed=args.seed, normalize=True)
        return x.astype(np.float32), q.astype(np.float16).astype(np.float32)
    x = synth.mixture(rows, args.dims, args.centres, seed=args.seed)
    q = synth.mixture_queries(queries, args.dims, args.centres, seed=args.seed)
    codes, scale = oracle.quantize_fp8(x)
    return oracle.decode_rows(oracle.E4M3, args.dims, codes, row_scales=scale), q


def cpu_run(x, q, k, threads, metric, budget_s=None, count=None):
    """Gathered jobs through the reference's AnnGatheredExact (oracle/_ref,
    ann/server/cpu.c:218-276) -- or the oracle's restatement when the
    reference library is absent -- on `threads` host threads, for budget_s
    seconds or exactly `count` queries; returns (queries done, seconds,
    kind)."""
    from concurrent.futures import ThreadPoolExecutor
    import oracle
    kind = 'reference' if oracle.ref_available() else 'port'

    if metric == 3:       # bit vectors: no worker entry point scores them; the oracle's restatement
        kind = 'port'

    def one(i):
        if metric == 3:
            oracle.search(oracle.BIT, x.shape[1] * 8, x, q[i % len(q)][None], k, metric, threads=1)
        elif kind == 'reference':
            oracle.ref_gathered_exact(q[i % len(q)], x, k, metric)
        else:
            oracle.search(oracle.F32, x.shape[1], x, q[i % len(q)][None], k, metric, window=True, threads=1)
        return 1

    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        if count is not None:
            done = sum(pool.map(one, range(count)))
        else:
            while time.perf_counter() - t0 < budget_s:
                done += sum(pool.map(one, range(done, done + threads)))
    return done, time.perf_counter() - t0, kind


def ivf_cpu_sample(args, rows):
    """Config 4 on the host: the oracle's IVF list gather (the reference's
    IVF scan is PostgreSQL code, src/ivfscan.c:124-186, with no worker entry
    point, so its C restatement is timed) over an NVFP4 corpus of `rows`
    rows with the full configuration's mean list size (N/nlist) and nprobe,
    so each query does the full-size amount of work."""
    import numpy as np
    import oracle
    from pgvector_b200 import synth
    nlists = max(args.nprobe, int(round(args.centres * rows / args.rows)))
    x, offsets, cent, _ = synth.ivf_corpus(rows, args.dims, nlists, seed=args.seed)
    codes, bs, rs = oracle.quantize_nvfp4(x)
    rng = np.random.default_rng(args.seed + 5)
    lab = rng.integers(0, nlists, 256)
    q = (cent[lab] + 0.1 * rng.standard_normal((256, args.dims))).astype(np.float32)
    probes = synth.ivf_probes(q, cent, args.nprobe)
    return codes, bs, rs, offsets, q, probes


def ivf_cpu_run(sample, args, threads, budget_s=None, count=None):
    import oracle
    codes, bs, rs, offsets, q, probes = sample
    done, t0, i = 0, time.perf_counter(), 0
    while (count is not None and done < count) or (count is None and time.perf_counter() - t0 < budget_s):
        m = threads if count is None else min(threads, count - done)
        sel = [(i + j) % len(q) for j in range(m)]
        oracle.search_lists(oracle.NVFP4, args.dims, codes, q[sel], offsets, probes[sel], args.k, 0,
                            block_scales=bs, row_scales=rs, threads=threads)
        done += m
        i += m
    return done, time.perf_counter() - t0, 'port'


_SAMPLES = {}


def cpu_measure(args, threads, budget_s=None, count=None, rows=None):
    """(queries/s at full size, sample description, kind) of the host path.
    `rows`: candidate rows a query of the sample scans (default: config 1's
    whole corpus, config 2's whole candidate set; a sample of the others,
    whose corpora do not fit host memory); the rate is scaled linearly to the
    full candidate count when they are fewer."""
    if args.config == 4:
        rows = 200_000
        if 4 not in _SAMPLES:
            _SAMPLES[4] = ivf_cpu_sample(args, rows)
        sample = _SAMPLES[4]
        done, secs, kind = ivf_cpu_run(sample, args, threads, budget_s=budget_s, count=count)
        desc = ('%d IVF queries (NVFP4 L2, k=%d, nprobe=%d over %d-row lists on average) in %.1f s on %d threads; '
                'the per-query work equals the full configuration\'s' %
                (done, args.k, args.nprobe, rows // max(1, len(sample[3]) - 1), secs, threads))
        return done / secs, desc, kind
    full = full_candidates(args)
    if rows is None:
        rows = {1: args.rows, 2: full, 5: 200_000}.get(args.config, 20_000)
    have = _SAMPLES.get(args.config)
    if have is None or have[0].shape[0] < rows:
        _SAMPLES[args.config] = cpu_sample(args, rows, 64)
    x, q = _SAMPLES[args.config]
    x = x[:rows]          # leading rows: a contiguous view
    done, secs, kind = cpu_run(x, q, args.k, threads, METRIC_CODE[args.config], budget_s=budget_s, count=count)
    desc = ('%d gathered jobs (metric %d, k=%d) over %d candidate rows of the config-%d distribution in %.1f s on '
            '%d threads' % (done, METRIC_CODE[args.config], args.k, rows, args.config, secs, threads))
    if rows != full:
        desc += ', scaled linearly to %d candidate rows (x%.2f)' % (full, full / rows)
    else:
        desc += ' (the full configuration\'s candidate set: no scaling)'
    return done / secs * rows / full, desc, kind


def full_candidates(args):
    return int(round(args.rows * args.selectivity)) if args.config == 2 else args.rows


def reference_arm(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return 0
    if args.config == 6:
        print(json.dumps({'impl': 'reference', 'unavailable': 'the reference serves quantized copies only from '
                          'its cuVS / Blackwell GPU backend, which does not build without cuVS'}), flush=True)
        return 0
    threads = os.cpu_count() or 1
    per_step = max(threads, 8)
    rows = None
    if args.config == 2:
        # each step: per_step queries over the whole candidate set when such a
        # step fits the run's budget (all steps within about two minutes),
        # else over the largest leading sample of it that does, scaled
        full = full_candidates(args)
        cpu_sample_cached(args, full)
        probe = min(full, 100_000)
        qps_p, _, _ = cpu_measure(args, threads, count=per_step, rows=probe)
        est_full = per_step / (qps_p * full / probe) * full / probe     # seconds a full-size step
        budget = min(4.0, 120.0 / max(1, args.steps + args.warmup))
        rows = full if est_full <= budget else max(probe, int(full * budget / est_full))
    for _ in range(args.warmup):
        cpu_measure(args, threads, count=per_step, rows=rows)
    rates, desc, kind, walls = [], '', 'reference', []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        qps, desc, kind = cpu_measure(args, threads, count=per_step, rows=rows)
        walls.append(time.perf_counter() - t0)
        rates.append(qps)
    qps = len(rates) / sum(1.0 / r for r in rates)
    line = {'metric': METRIC, 'value': qps, 'unit': 'queries/s', 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': 1e3 * sum(walls) / len(walls),
            'step': '%d queries a step on %d host threads (the CPU serves them one a thread)' % (per_step, threads),
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'f64',
            'data': 'synthetic (seeded Gaussian mixture of the configuration)',
            'config': workload_config(args), 'parallelism': '%d host threads' % threads,
            'impl': 'reference',
            'cpu_baseline': {'value': qps, 'unit': 'queries/s', 'cores': threads, 'kind': kind,
                             'sample': '%d queries a step: %s' % (per_step, desc)},
            'e2e': {'value': qps, 'unit': 'queries/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


def cpu_sample_cached(args, rows):
    if args.config not in _SAMPLES or _SAMPLES[args.config][0].shape[0] < rows:
        _SAMPLES[args.config] = cpu_sample(args, rows, 64)


def workload_config(args):
    """The `config` of both arms' lines: the workload, nothing of the
    implementation (that goes in `parallelism`)."""
    cfg = {'workload': WORKLOADS[args.config], 'global_batch': args.batch, 'rows': args.rows, 'dims': args.dims,
           'k': args.k}
    if args.config == 2:
        cfg['selectivity'] = args.selectivity
    if args.config == 4:
        cfg.update({'nlist': args.centres, 'nprobe': args.nprobe})
    row_bytes = {1: args.dims * 4, 2: args.dims * 2 + 4, 3: (args.dims + 15) // 16 * 16 + 4,
                 4: args.dims // 2 + args.dims // 16 + 4, 5: args.dims // 8}.get(args.config, args.dims * 4)
    gb = full_candidates(args) * row_bytes / 1e9
    cfg['l2'] = ('inputs larger than L2: about %.2f GB of candidate rows a step' % gb if gb > 0.126 else
                 'inputs fit in L2 (%.0f MB): the GPU arm writes a 256 MB buffer before every step, its time '
                 'included' % (gb * 1e3))
    return cfg


# ---------------------------------------------------------------- workloads

class Workload:
    """One configuration on this rank: the shard, the batch's device inputs
    (`inputs`: tensors copied from host memory each step in the end-to-end
    loop) and one step of the public API over them."""
    metric = 0
    dtype = 'f16'
    kernel = ''
    bound = 'tensor'
    ops = 'f16'         # tensor-core operand type of the dominant kernel

    def step(self, *inputs):
        raise NotImplementedError


def mixture_rows(args, dev, lo, hi, centres, fill, chunk=1 << 20, normalize=False, label_of=None):
    """Rows lo..hi of the seeded global mixture, generated chunk by chunk
    (per-chunk seeds: every rank draws the same global rows) and handed to
    fill(a, b, float32 rows) -- row a..b of the local range."""
    import torch
    g = torch.Generator(device=dev)
    for c0 in range(lo // chunk * chunk, hi, chunk):
        g.manual_seed(args.seed * 1000003 + c0 // chunk)
        m = min(chunk, args.rows - c0)
        lab = (torch.randint(0, centres.shape[0], (m,), generator=g, device=dev) if label_of is None
               else label_of(c0, m))
        v = centres[lab] + 0.1 * torch.randn((m, args.dims), generator=g, device=dev)
        if normalize:
            v /= v.norm(dim=1, keepdim=True).clamp_min(1e-30)
        a, b = max(c0, lo), min(c0 + m, hi)
        fill(a - lo, b - lo, v[a - c0:b - c0])
        del v, lab


def build_config1(args, rank, world, dev):
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import sharded, synth
    w = Workload()
    bounds = sharded.shard_bounds(args.rows, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    x = synth.mixture(args.rows, args.dims, args.centres, seed=args.seed)      # the CPU sample's rows
    codes = torch.from_numpy(x[lo:hi]).to(dev)
    queries = torch.from_numpy(synth.mixture_queries(args.batch, args.dims, args.centres, seed=args.seed)).to(dev)
    w.inputs = [queries]
    w.shard = pb.Shard(pb.F32, args.dims, codes, first_id=lo)
    w.metric, w.dtype, w.bound = pb.L2, 'f32 (BF16 hi/lo split, 3 MMAs a K step)', 'tensor'
    w.kernel = 'tc_scan<F32> (split BF16), filter pass'
    w.data = 'synthetic (seeded 100-centre Gaussian mixture, sigma 0.1, the same rows as the CPU baseline)'
    w.row_bytes = args.dims * 4
    w.profile = 'none'
    # the corpus (51 MB) fits in L2: every step first overwrites a buffer
    # twice L2's size, and that time is part of the step
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step(q):
        flush.fill_(1)
        d, i, c = w.shard.search_sharded(w.comm, q, args.k, pb.L2)
        return d, i, c, hi - lo
    w.step = step

    def local_oracle(nq):
        import oracle
        od, oi, oc, _ = oracle.search(oracle.F32, args.dims, x[lo:hi], queries[:nq].cpu().numpy(), args.k, 0)
        return od, oi + lo, oc
    w.local_oracle = local_oracle
    w.vtable = lambda: vtable_paths(args, x, synth.mixture_queries(args.batch, args.dims, args.centres,
                                                                    seed=args.seed))
    return w


def vtable_paths(args, x, q, seconds=3.0):
    """Config 1 through the worker's own entry points, host buffers in and
    out, timed by the host clock (the calls are synchronous):
      gathered  -- the backend vtable's search_gathered (ops 7/10): lane
                   batches of 64 gathered jobs, each one query against 8,192
                   of the corpus's rows (an op-10 chunk), k = 10, one call a
                   batch (rows staged, one device submission);
      index     -- a loaded index's search (AnnB200IndexSearch, the worker's
                   search_index): the 100,000-row corpus, all queries of the
                   batch in one call, k = 10."""
    import ctypes
    import pgvector_b200 as pb
    lib = pb.load()
    out = {}
    rows_per_job, jobs_per_call = 8192, 64
    jobs = [(q[j % len(q)], x[(j * 1531) % (len(x) - rows_per_job):][:rows_per_job], args.k, 0)
            for j in range(jobs_per_call)]
    pb.search_gathered(jobs)
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or calls < 3:
        res = pb.search_gathered(jobs)
        calls += 1
    secs = (time.perf_counter() - t0) / calls
    out['gathered'] = {'jobs_per_s': jobs_per_call / secs, 'ms_per_call': secs * 1e3, 'jobs_per_call': jobs_per_call,
                       'rows_per_job': rows_per_job, 'ok': all(st == 0 and len(r) >= args.k for st, r in res)}
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ix = ctypes.c_void_p()
    pb.check(lib.AnnB200IndexCreate(0, args.dims, len(x), P(x), ctypes.byref(ix)))
    nq = len(q)
    dist = np.zeros((nq, args.k), np.float32)
    ords = np.zeros((nq, args.k), np.uint64)
    cnt = np.zeros(nq, np.uint32)
    pb.check(lib.AnnB200IndexSearch(ix, P(q), nq, None, 0, args.k, P(dist), P(ords), P(cnt)))
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or calls < 3:
        pb.check(lib.AnnB200IndexSearch(ix, P(q), nq, None, 0, args.k, P(dist), P(ords), P(cnt)))
        calls += 1
    secs = (time.perf_counter() - t0) / calls
    lib.AnnB200IndexDestroy(ix)
    out['index'] = {'queries_per_s': nq / secs, 'ms_per_call': secs * 1e3, 'queries_per_call': nq}
    return out


def build_config2(args, rank, world, dev):
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import sharded, synth
    w = Workload()
    bounds = sharded.shard_bounds(args.rows, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    centres = torch.randn((args.centres, args.dims), generator=g, device=dev)
    codes = torch.empty((hi - lo, args.dims), dtype=torch.float16, device=dev)

    def fill(a, b, v):
        codes[a:b] = v.to(torch.float16)
    mixture_rows(args, dev, lo, hi, centres, fill, normalize=True)
    g.manual_seed(args.seed + 7919)
    lab = torch.randint(0, args.centres, (args.batch,), generator=g, device=dev)
    qv = centres[lab] + 0.1 * torch.randn((args.batch, args.dims), generator=g, device=dev)
    qv /= qv.norm(dim=1, keepdim=True)
    queries = qv.to(torch.float16).to(torch.float32).contiguous()       # halfvec query values
    words = synth.torch_bitmap(args.rows, args.selectivity, seed=args.seed + 1, device=dev)
    my_words, nbits = sharded.bitmap_slice(words, lo, hi)
    w.inputs = [queries, my_words.contiguous()]
    w.shard = pb.Shard(pb.F16, args.dims, codes, first_id=lo)
    w.codes, w.lo, w.metric, w.dtype = codes, lo, pb.COSINE, 'f16'
    w.kernel = 'tc_scan<F16>, filter pass'
    w.data = 'synthetic (seeded 1,000-centre Gaussian mixture, unit-normalised, generated on the GPU)'
    w.row_bytes = args.dims * 2 + 4                         # row + its id in the row list
    w.profile = 'tc_scan_f16_config2.md'

    def step(q, words_):
        # the bitmap's expansion and the search in one library call
        return w.shard.search_bitmap(w.comm, q, args.k, pb.COSINE, words_, nbits)
    w.step = step

    def local_oracle(nq):
        # the oracle over this rank's candidate rows only, with global ids
        import numpy as np
        import oracle
        rows_t = pb.bitmap_rows(w.inputs[1], nbits)
        rows_np = rows_t.cpu().numpy().view(np.uint32).astype(np.int64)
        h = codes[rows_t.long()].cpu().numpy().view(np.uint16)
        od, oi, oc, _ = oracle.search(oracle.F16, args.dims, h, queries[:nq].cpu().numpy(), args.k, 2)
        return od, np.where(oi >= 0, rows_np[np.maximum(oi, 0)] + lo, -1), oc
    w.local_oracle = local_oracle
    del centres, qv, lab
    return w


def build_config3(args, rank, world, dev):
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import sharded, synth
    w = Workload()
    bounds = sharded.shard_bounds(args.rows, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    centres = torch.randn((args.centres, args.dims), generator=g, device=dev)
    pad = (args.dims + 15) // 16 * 16
    codes = torch.empty((hi - lo, pad), dtype=torch.uint8, device=dev)
    scales = torch.empty((hi - lo,), dtype=torch.float32, device=dev)

    def fill(a, b, v):
        c, s = synth.torch_quantize_fp8(v)
        codes[a:b] = c
        scales[a:b] = s
    mixture_rows(args, dev, lo, hi, centres, fill)
    g.manual_seed(args.seed + 7919)
    lab = torch.randint(0, args.centres, (args.batch,), generator=g, device=dev)
    queries = (centres[lab] + 0.1 * torch.randn((args.batch, args.dims), generator=g, device=dev)).contiguous()
    w.inputs = [queries]
    w.shard = pb.Shard(pb.E4M3, args.dims, codes, None, scales, first_id=lo)
    w.metric, w.dtype = pb.IP, 'e4m3 (FP8 MMAs; queries as two E4M3 terms)'
    w.kernel = 'tc_scan<FP8 E4M3>, filter pass'
    w.ops = 'e4m3'
    w.data = 'synthetic (seeded 4,096-centre Gaussian mixture, FP8-quantised on the GPU with the builder\'s rules)'
    w.row_bytes = pad + 4                                   # codes + row scale
    w.profile = 'tc_scan_fp8_config3.md'

    def step(q):
        d, i, c = w.shard.search_sharded(w.comm, q, args.k, pb.IP)
        return d, i, c, hi - lo
    w.step = step

    def local_rescore(result, nq):
        return rescore_local(args, w, result, nq, codes, None, scales, oracle_dtype=2, lo=lo, hi=hi, world=world)
    w.local_rescore = local_rescore
    del centres
    return w


def build_config4(args, rank, world, dev):
    import numpy as np
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import sharded, synth
    w = Workload()
    nlists = args.centres
    rng = np.random.default_rng(args.seed + 3)
    weights = 1.0 / np.arange(1, nlists + 1, dtype=np.float64) ** 1.1
    weights = weights[rng.permutation(nlists)]
    sizes = np.floor(weights / weights.sum() * args.rows).astype(np.int64)
    sizes[np.argmax(sizes)] += args.rows - sizes.sum()
    offsets = np.zeros(nlists + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(sizes)
    # rows lo..hi of the list-major storage on this rank: equal shares of the
    # rows, lists cut at the boundaries (Zipf sizes put 27M of the 200M rows
    # in one list, so shares of whole lists cannot balance). The rank's lists
    # are l0..l1-1, each clipped to its rows; a list on two ranks is searched
    # on both and the device merge joins them.
    lo, hi, l0, l1, loc_np = sharded.ivf_shard(offsets, world, rank)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    cent = torch.randn((nlists, args.dims), generator=g, device=dev)
    doff = torch.from_numpy(offsets).to(dev)
    blocks = (args.dims + 15) // 16
    codes = torch.empty((hi - lo, blocks * 8), dtype=torch.uint8, device=dev)
    bscales = torch.empty((hi - lo, blocks), dtype=torch.uint8, device=dev)
    rscales = torch.empty((hi - lo,), dtype=torch.float32, device=dev)

    def label_of(c0, m):
        idx = torch.arange(c0, c0 + m, device=dev)
        return torch.searchsorted(doff[1:], idx, right=True)

    def fill(a, b, v):
        p, s, r = synth.torch_quantize_nvfp4(v)
        codes[a:b] = p
        bscales[a:b] = s
        rscales[a:b] = r
    mixture_rows(args, dev, lo, hi, cent, fill, label_of=label_of)
    # queries: the centre of a uniformly chosen list plus noise, so that a
    # probe touches a list of the mean size (N / nlist rows) on average, the
    # per-query gather the configuration's cost figures assume
    g.manual_seed(args.seed + 7919)
    qlab = torch.randint(0, nlists, (args.batch,), generator=g, device=dev)
    queries = (cent[qlab] + 0.1 * torch.randn((args.batch, args.dims), generator=g, device=dev)).contiguous()
    # coarse probe, part of every step: the nprobe nearest centres of each
    # query (an exact search of the FP32 centres, AnnB200ProbeLists), then
    # this rank's lists renumbered and the others padding (-1 = UINT32_MAX)
    centres = pb.Shard(pb.F32, args.dims, cent.contiguous())

    def rank_probes(q):
        pr = centres.probe_lists(q, args.nprobe, pb.L2)
        return torch.where((pr >= l0) & (pr < l1), pr - l0, torch.full_like(pr, -1)).contiguous()
    local = rank_probes(queries)
    loc_off = torch.from_numpy(loc_np).to(dev)
    w.inputs = [queries]
    w.shard = pb.Shard(pb.NVFP4, args.dims, codes, bscales, rscales, first_id=lo)
    w.metric, w.dtype, w.bound = pb.L2, 'nvfp4->f32', 'hbm'
    w.kernel = 'tc_scan_lists<NVFP4>, list pass'
    w.data = ('synthetic (seeded: %d list centres ~N(0,1), rows = centre + 0.1 noise, Zipf(1.1) list sizes, '
              'NVFP4-quantised on the GPU with the builder\'s rules)' % nlists)
    w.row_bytes = blocks * 8 + blocks + 4
    w.profile = 'tc_scan_lists_nvfp4_config4.md'
    # algorithmic bytes of a pass: every probed list's rows, read once
    hit = torch.zeros(l1 - l0, dtype=torch.bool, device=dev)
    lp = local[local >= 0].long()
    hit[lp] = True
    lsz = torch.from_numpy(np.diff(loc_np)).to(dev)
    w.pass_rows = int(lsz[hit].sum().item())
    pairs = int(lsz[lp].sum().item())
    w.pass_flops = 2.0 * pairs * args.dims

    def step(q):
        d, i, c = w.shard.search_lists_sharded(w.comm, q, args.k, pb.L2, loc_off, rank_probes(q))
        return d, i, c, w.pass_rows
    w.step = step

    def local_oracle(nq):
        # the oracle over the lists this rank holds (its share of each), with global ids
        import oracle
        qn = queries[:nq].cpu().numpy()
        pr = local[:nq].cpu().numpy().view(np.uint32)
        lists = sorted(set(int(x) for x in pr.ravel() if x != 0xffffffff))
        if not lists:
            return (np.full((nq, args.k), np.inf), np.full((nq, args.k), -1, dtype=np.int64),
                    np.zeros(nq, dtype=np.uint32))
        # the probed lists only, re-packed list-major with their global ids
        parts, new_off, ids = [], [0], []
        for l in lists:
            a, b = int(loc_np[l]), int(loc_np[l + 1])
            parts.append((a, b))
            new_off.append(new_off[-1] + b - a)
            ids.append(np.arange(a, b, dtype=np.int64) + lo)
        sel = torch.cat([torch.arange(a, b, device=dev) for a, b in parts])
        remap = {l: j for j, l in enumerate(lists)}
        pr2 = np.array([[remap.get(int(x), 0xffffffff) for x in row] for row in pr], dtype=np.uint32)
        od, oi, oc = oracle.search_lists(oracle.NVFP4, args.dims, codes[sel].cpu().numpy(), qn,
                                         np.array(new_off, dtype=np.uint64), pr2, args.k, 0,
                                         row_ids=np.concatenate(ids), block_scales=bscales[sel].cpu().numpy(),
                                         row_scales=rscales[sel].cpu().numpy())
        return od, oi, oc
    w.local_oracle = local_oracle
    del cent
    return w


def build_config5(args, rank, world, dev):
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import sharded
    w = Workload()
    bounds = sharded.shard_bounds(args.rows, world)
    lo, hi = bounds[rank], bounds[rank + 1]
    nb = args.dims // 8
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed)
    proto = torch.randint(0, 256, (args.centres, nb), generator=g, device=dev, dtype=torch.uint8)
    weights = torch.tensor([1, 2, 4, 8, 16, 32, 64, 128], dtype=torch.int32, device=dev)   # bit i of a byte

    def perturbed(m, gen):
        # prototype rows XOR Bernoulli(0.05) bits, packed least significant bit first
        lab = torch.randint(0, args.centres, (m,), generator=gen, device=dev)
        flips = torch.rand((m, nb, 8), generator=gen, device=dev) < 0.05
        return proto[lab] ^ (flips.to(torch.int32) * weights).sum(dim=2).to(torch.uint8)
    codes = torch.empty((hi - lo, nb), dtype=torch.uint8, device=dev)
    chunk = 1 << 18
    for c0 in range(lo // chunk * chunk, hi, chunk):      # per-chunk seeds: every rank draws the same rows
        g.manual_seed(args.seed * 1000003 + c0 // chunk)
        m = min(chunk, args.rows - c0)
        v = perturbed(m, g)
        a, b = max(c0, lo), min(c0 + m, hi)
        codes[a - lo:b - lo] = v[a - c0:b - c0]
        del v
    g.manual_seed(args.seed + 7919)
    queries = perturbed(args.batch, g).contiguous()
    w.inputs = [queries]
    w.shard = pb.Shard(pb.BIT, args.dims, codes, first_id=lo)
    w.metric, w.dtype = pb.HAMMING, 'bit->int8 (+-1), s32 accumulate'
    w.kernel = 'tc_scan<BIT> (kind::i8), filter pass'
    w.data = ('synthetic (seeded: 65,536 uniform random 1,024-bit prototypes, rows = prototype XOR Bernoulli(0.05) '
              'bits, generated on the GPU)')
    w.row_bytes = nb
    w.profile = 'tc_scan_bit_config5.md'
    w.ops = 'int8'

    def step(q):
        d, i, c = w.shard.search_sharded(w.comm, q, args.k, pb.HAMMING)
        return d, i, c, hi - lo
    w.step = step

    def local_rescore(result, nq):
        return rescore_local(args, w, result, nq, codes, None, None, oracle_dtype=4, lo=lo, hi=hi, world=world)
    w.local_rescore = local_rescore
    return w


def rescore_local(args, w, result, nq, codes, bscales, rscales, oracle_dtype, lo, hi, world):
    """This rank's half of the size-independent check for shards too large
    for the oracle (configs 3 and 5): per checked query, the oracle's exact
    distance of every returned row this rank holds, and of a random sample
    of this rank's rows (200,000 rows over all ranks). The check itself
    (check_rescored) runs on rank 0 over every rank's part."""
    import numpy as np
    import torch
    import oracle
    rng = np.random.default_rng(args.seed + 11 + lo)
    sample = np.unique(rng.integers(0, hi - lo, max(1, 200_000 // world)))
    parts = []
    for qi in range(nq):
        q = w.inputs[0][qi:qi + 1].cpu().numpy()
        n = int(result[2][qi].item())
        ids = result[1][qi, :n].cpu().numpy()
        mine = ids[(ids >= lo) & (ids < hi)] - lo
        rows = np.unique(np.concatenate([mine, sample])).astype(np.int64)
        rt = torch.from_numpy(rows).to(codes.device)
        sub = codes[rt].cpu().numpy()
        bs = None if bscales is None else bscales[rt].cpu().numpy()
        rs = None if rscales is None else rscales[rt].cpu().numpy()
        od, oi, oc, _ = oracle.search(oracle_dtype, args.dims, sub, q, len(rows), w.metric, block_scales=bs,
                                      row_scales=rs)
        exact = dict(zip((rows[oi[0][:oc[0]]] + lo).tolist(), od[0][:oc[0]].tolist()))
        mine_set = set((mine + lo).tolist())
        parts.append({'returned': {r: d for r, d in exact.items() if r in mine_set},
                      'sample': [(d, r) for r, d in exact.items()]})
    return parts


def check_rescored(result, parts, nq):
    """Rank 0: every returned row's distance equals the oracle's exact one
    (bit for bit), the rows are sorted by (distance, id), and no sampled row
    of any rank beats the k-th returned one."""
    import numpy as np
    ok = True
    for qi in range(nq):
        n = int(result[2][qi].item())
        ids = result[1][qi, :n].cpu().numpy().tolist()
        dist = result[0][qi, :n].cpu().numpy().tolist()
        exact, sample = {}, []
        for p in parts:
            exact.update(p[qi]['returned'])
            sample.extend(p[qi]['sample'])
        ok &= n > 0 and all(i in exact for i in ids)
        if not ok:
            return False
        ok &= bool(np.array_equal(np.array([exact[i] for i in ids]), np.array(dist)))
        ok &= all((dist[j], ids[j]) <= (dist[j + 1], ids[j + 1]) for j in range(n - 1))
        kth = (dist[-1], ids[-1])
        member = set(ids)
        ok &= all((d, r) >= kth for d, r in sample if r not in member)
    return bool(ok)


def merge_reference_lists(lists, k):
    """The oracle's answer for the whole corpus from every rank's oracle
    answer over its own rows: lists = [(dist [nq][cap], global id [nq][cap],
    count [nq])] per rank; per query the k smallest (distance, id) pairs of
    their union -- the host tree merge of per-shard lists the reference does
    (AnnIndexTreeMerge, ann/server/indexfile.c:3235-3258), written in numpy
    as the checker, independent of the device merge."""
    nq = len(lists[0][2])
    out = []
    for q in range(nq):
        entries = []
        for d, i, c in lists:
            n = int(c[q])
            entries.extend(zip(np.asarray(d)[q, :n].tolist(), np.asarray(i)[q, :n].tolist()))
        entries.sort()
        out.append(entries[:k])
    return out


def check_global(result, lists, nq, k):
    """Rank 0: the merged device answer (dist, id, count) equals, bit for
    bit, the merge of every rank's oracle list."""
    want = merge_reference_lists(lists, k)
    d = np.asarray(result[0][:nq].cpu())
    i = np.asarray(result[1][:nq].cpu())
    c = np.asarray(result[2][:nq].cpu())
    for q in range(nq):
        n = int(c[q])
        if n != len(want[q]) or list(zip(d[q, :n].tolist(), i[q, :n].tolist())) != want[q]:
            return False
    return True


def gather_objects(obj, world):
    """Every rank's `obj` on every rank (a collective all ranks enter)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def verify(w, result, nq, world, rank, k):
    """The multi-rank correctness check: each rank answers the checked
    queries with the CPU oracle over the rows it holds (or rescores the
    returned rows and a sample, for shards too large for the oracle); rank 0
    checks the merged device answer against all of them. None on the other
    ranks."""
    if hasattr(w, 'local_oracle'):
        lists = gather_objects(w.local_oracle(nq), world)
        return check_global(result, lists, nq, k) if rank == 0 else None
    parts = gather_objects(w.local_rescore(result, nq), world)
    return check_rescored(result, [p for p in parts], nq) if rank == 0 else None


# ---------------------------------------------------------------- our arm

def index_quant_bench(args):
    """Config 6: a loaded index served from its NVFP4 copy (the reference's
    quantized scan route) through the host-memory API, beside the same index
    served from its FP32 rows on the device. One step = one synchronous
    AnnB200IndexSearch of the batch, timed by the host clock around the call
    (its inputs and results are host memory, so this is the end-to-end
    figure); every copy and kernel of the route is inside it."""
    import ctypes
    import numpy as np
    import torch
    import pgvector_b200 as pb
    from pgvector_b200 import synth
    if int(os.environ.get('RANK', '0')) != 0:
        return 0
    torch.cuda.set_device(0)
    lib = pb.load()
    n, d, nq, k = args.rows, args.dims, args.batch, args.k
    blocks = (d + 15) // 16
    xh = np.empty((n, d), np.float32)
    codes = np.empty((n, blocks * 8), np.uint8)
    bs = np.empty((n, blocks), np.uint8)
    rs = np.empty(n, np.float32)
    chunk = 1 << 18
    x = synth.torch_mixture(n, d, args.centres, sigma=0.3, seed=args.seed, dtype=torch.float32)
    for lo in range(0, n, chunk):
        c, b, r = synth.torch_quantize_nvfp4(x[lo:lo + chunk])
        hi = lo + c.shape[0]
        codes[lo:hi], bs[lo:hi], rs[lo:hi] = c.cpu().numpy(), b.cpu().numpy(), r.cpu().numpy()
        xh[lo:hi] = x[lo:hi].cpu().numpy()
    del x
    torch.cuda.empty_cache()
    q = synth.torch_mixture_queries(nq, d, args.centres, sigma=0.3, seed=args.seed + 1).cpu().numpy()
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    quant, exact = ctypes.c_void_p(), ctypes.c_void_p()
    shards = (ctypes.c_uint64 * 3)(n // 3, n // 3, n - 2 * (n // 3))
    pb.check(lib.AnnB200IndexCreateQuant(0, d, n, pb.NVFP4, P(codes), P(bs), P(rs), P(xh), 3, shards, 256, 100,
                                         ctypes.byref(quant)))
    pb.check(lib.AnnB200IndexCreate(0, d, n, P(xh), ctypes.byref(exact)))
    out = {}
    for name, ix in (('quant', quant), ('fp32', exact)):
        dist = np.zeros((nq, k), np.float32)
        ords = np.zeros((nq, k), np.uint64)
        cnt = np.zeros(nq, np.uint32)
        for _ in range(args.warmup):
            pb.check(lib.AnnB200IndexSearch(ix, P(q), nq, None, 0, k, P(dist), P(ords), P(cnt)))
        clocks = ClockSampler(0)
        clocks.start()
        launches0 = lib.AnnB200LaunchCount()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            pb.check(lib.AnnB200IndexSearch(ix, P(q), nq, None, 0, k, P(dist), P(ords), P(cnt)))
        secs = time.perf_counter() - t0
        launches = lib.AnnB200LaunchCount() - launches0
        out[name] = (nq * args.steps / secs, secs / args.steps * 1e3, ords.copy(), launches, clocks.stop())
    lib.AnnB200IndexDestroy(quant)
    lib.AnnB200IndexDestroy(exact)
    qps, ms, ords, launches, clock_info = out['quant']

    # CPU baseline: the oracle's restatement of the route (the reference has
    # no CPU implementation of it) on a bounded sample of the batch, all host
    # threads; its answers checked against the device's
    cpu, verified = None, None
    if not args.no_cpu_baseline:
        import oracle
        threads = os.cpu_count() or 1
        bounds = [0, n // 3, 2 * (n // 3), n]
        done, t0, agree = 0, time.perf_counter(), True
        while done < nq and (done < 1 or time.perf_counter() - t0 < args.cpu_seconds):
            got = oracle.quant_index_search(oracle.NVFP4, xh, codes, q[done:done + 1], k, bounds, block_scales=bs,
                                            row_scales=rs, threads=threads)[0]
            agree = agree and [o for o, _ in got] == [int(o) for o in ords[done][:len(got)]]
            done += 1
        secs = time.perf_counter() - t0
        cpu = {'value': done / secs, 'unit': 'queries/s', 'cores': threads, 'kind': 'port',
               'sample': '%d queries of the batch through oracle.quant_index_search (3 shard searches of the '
                         'NVFP4 codes + FP64 re-score of the candidates) in %.1f s' % (done, secs)}
        verified = agree
    recall = float(np.mean([len(set(ords[i].tolist()) & set(out['fp32'][2][i].tolist())) / k for i in range(nq)]))
    cands = 3 * (k + max(256, k))                    # per query: k + slack in each of the 3 shards
    line = {'metric': 'QPS at batch %d, k=%d, loaded index served from its NVFP4 copy' % (nq, k),
            'value': qps, 'unit': 'queries/s', 'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
            'data': 'synthetic (seeded Gaussian mixture on the GPU, quantized there, held in host memory)',
            'config': {'workload': WORKLOADS[6], 'global_batch': nq, 'rows': n, 'dims': d, 'k': k,
                       'parallelism': 'single GPU + host copy threads',
                       'timing': 'host clock around the synchronous call (end to end)'},
            'e2e': {'value': qps, 'unit': 'queries/s', 'h2d_bytes_per_step': nq * d * 4 * (1 + cands),
                    'd2h_bytes_per_step': nq * (cands * 12 + k * 12)},
            'roofline': None,
            'roofline_note': 'bound by the candidates\' FP32 rows crossing from host memory '
                             '(%.0f MB a batch)' % (nq * cands * d * 4 / 1e6),
            'cpu_baseline': cpu, 'gpu_launches': launches, 'clocks': clock_info,
            'fp32_route_qps': out['fp32'][0], 'recall_vs_fp32_route': recall, 'verified_vs_oracle': verified}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = args_parse()
    if args.impl == 'reference':
        return reference_arm(args)
    if args.config == 6:
        return index_quant_bench(args)
    os.environ.setdefault('ANN_B200_KERNEL_TIMING', '1')
    import torch
    import torch.distributed as dist
    import pgvector_b200 as pb
    from datetime import timedelta

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=timedelta(seconds=180), device_id=dev)
    lib = pb.load()
    # the clock sampler starts before the workload is built, so that its
    # start-up (NVML's first calls) is long over when anything is timed; its
    # readings count from the warm-up on
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    w = {1: build_config1, 2: build_config2, 3: build_config3, 4: build_config4,
         5: build_config5}[args.config](args, rank, world, dev)
    # N > 1: the library's own NCCL communicator carries the per-rank lists
    # (AnnB200SearchSharded); torch.distributed only hands its id around
    from pgvector_b200 import sharded
    w.comm = sharded.comm_from_process_group(local) if world > 1 else None
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident value. Python's cyclic garbage collector runs at
    # moments of its own choosing and a full pass over this process's objects
    # takes tens of ms, during which the host launches nothing (a timed step
    # once took 48 ms instead of 2.2): collect now, and keep it off while
    # anything is timed.
    gc.collect()
    gc.disable()
    # the stage events (two a stage, read back in later calls) cost host time
    # inside the step: they are off while the headline is timed and on in a
    # second loop of the same steps that gives the per-stage split
    lib.AnnB200StageTiming(0)
    if clocks:
        clocks.mark()
    # warm-up steps keep their result alive while the next step runs, as the
    # timed loop does, so that the caching allocator has grown to that
    # pattern before the clock starts (else the second timed step paid for
    # a fresh device allocation)
    out = None
    for _ in range(args.warmup):
        out = w.step(*w.inputs)
    barrier()
    stage_ms = (ctypes.c_double * 10)()
    stage_calls = (ctypes.c_ulonglong * 10)()
    launches0 = lib.AnnB200LaunchCount()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    e0.record()
    nrows_local = 0
    for j in range(args.steps):
        out = w.step(*w.inputs)
        nrows_local = out[3]
        marks[j].record()
    e1.record()
    barrier()
    step_ms = [e0.elapsed_time(marks[0])] + [marks[j - 1].elapsed_time(marks[j]) for j in range(1, args.steps)]
    clock_info = clocks.stop() if clocks else None
    launches = lib.AnnB200LaunchCount() - launches0
    ms = max_over_ranks(e0.elapsed_time(e1))
    # ---- the per-stage split: the same steps once more, stage events on
    lib.AnnB200StageTiming(1)
    barrier()
    lib.AnnB200StageTimes(stage_ms, stage_calls, 10, 1)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(args.steps):
        w.step(*w.inputs)
    s1.record()
    barrier()
    stage_loop_ms = max_over_ranks(s0.elapsed_time(s1)) / args.steps
    lib.AnnB200StageTimes(stage_ms, stage_calls, 10, 0)
    lib.AnnB200StageTiming(0)
    value = args.steps * args.batch / (ms / 1e3)
    result = out

    # ---- end to end through the public API with host buffers
    e2e = None
    k = args.k
    if not args.no_e2e:
        hin = [x.cpu().pin_memory() for x in w.inputs]
        hd = torch.empty((args.batch, k), dtype=torch.float64).pin_memory()
        hi_ = torch.empty((args.batch, k), dtype=torch.int64).pin_memory()
        # The inputs cross on their own stream, overlapping the searches as a
        # server's would: step j+1's inputs go into the other of two device
        # buffer sets while step j searches. Every step still copies all of
        # its inputs in and its k best out inside the timed region.
        cs = torch.cuda.Stream()
        main = torch.cuda.current_stream()
        # the inputs packed in one pinned block, so a step's inputs cross in one copy
        offs, total = [], 0
        for h_ in hin:
            offs.append(total)
            total += (h_.numel() * h_.element_size() + 255) // 256 * 256
        hblock = torch.empty(total, dtype=torch.uint8).pin_memory()
        for o, h_ in zip(offs, hin):
            hblock[o:o + h_.numel() * h_.element_size()].copy_(h_.reshape(-1).view(torch.uint8))
        dblock = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(2)]
        din = [[b[o:o + h_.numel() * h_.element_size()].view(h_.dtype).view(h_.shape) for o, h_ in zip(offs, hin)]
               for b in dblock]
        copied = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]

        def h2d(slot):
            with torch.cuda.stream(cs):
                cs.wait_event(freed[slot])          # the step that last read these buffers has ended
                dblock[slot].copy_(hblock, non_blocking=True)
                copied[slot].record(cs)

        def e2e_run(n):
            for e in freed:
                e.record(main)
            h2d(0)
            for j in range(n):
                slot = j % 2
                main.wait_event(copied[slot])
                if j + 1 < n:
                    h2d(1 - slot)
                d, i, c, _n = w.step(*din[slot])
                freed[slot].record(main)
                # the k best come back on the search's own stream: on the copy
                # stream they queued ahead of the next search's small reads
                # (its row count, its exchange headers) on the same copy engine
                hd.copy_(d[:, :k], non_blocking=True)
                hi_.copy_(i[:, :k], non_blocking=True)
            main.wait_stream(cs)
        e2e_run(args.warmup)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        e2e_run(args.steps)
        f1.record()
        barrier()
        ems = max_over_ranks(f0.elapsed_time(f1))
        e2e = {'value': args.steps * args.batch / (ems / 1e3), 'unit': 'queries/s',
               'h2d_bytes_per_step': int(hblock.numel()),
               'd2h_bytes_per_step': int(hd.numel() * 8 + hi_.numel() * 8) if rank == 0 else 0,
               'ms_per_step': ems / args.steps,
               'copies': 'inputs on a second stream (step j+1 in while step j searches), results after each step'}

    gc.enable()

    # ---- roofline of the dominant pass (stage 3: every scan launch of one
    # step's filter / list pass, timed by the library's stage clock on its
    # stream). Algorithmic work per pass: 2 * batch * candidate rows * dims
    # FLOPs (IVF: 2 * dims per probed (row, query) pair); algorithmic bytes:
    # each candidate row once (codes, scales and its row id) plus the query
    # block.
    hbm, tf_burst, tf_sust, kind = peaks()
    pass_ms = stage_ms[3] / args.steps
    if args.config == 4:
        flops, bytes_alg = w.pass_flops, w.pass_rows * (w.row_bytes - 4) + args.batch * args.dims * 4
    else:
        flops = 2.0 * args.batch * nrows_local * args.dims
        bytes_alg = nrows_local * w.row_bytes + args.batch * args.dims * (1 if w.ops == 'int8' else 2)
    achieved_tf = flops / (pass_ms * 1e-3) / 1e12
    hbm_gbs = bytes_alg / (pass_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, 'profiles', w.profile)
    if os.path.exists(tpath):
        for line in open(tpath):
            if line.startswith('traffic_bytes_per_row:'):
                traffic = float(line.split(':', 1)[1]) * (w.pass_rows if args.config == 4 else nrows_local)
    stage_names = ['prep', 'sample_scan', 'bound', 'filter_scan', 'tighten', 'finalize', 'bitmap', 'merge', 'gather',
                   'probe']
    stages = {n: round(stage_ms[j] / args.steps, 4) for j, n in enumerate(stage_names) if stage_calls[j]}
    # The tensor denominator: the measured burst cuBLAS figure for a timed
    # region shorter than a second (clocks stay at their maximum), the
    # sustained one (under the power cap) for a longer region.
    region_s = ms / 1e3
    burst = region_s < 1.0
    tf_peak = tf_burst if burst else tf_sust
    tf_src = '%s bf16_tflops%s (timed region %.2f s)' % (kind, '' if burst else '_sustained', region_s)
    common = {'kernel': '%s (%d launches a step)' % (w.kernel, round(stage_calls[3] / args.steps)),
              'pass_ms': round(pass_ms, 4), 'flops_per_pass': flops, 'algorithmic_bytes_per_pass': bytes_alg}
    if w.bound == 'tensor' and w.ops == 'int8':
        # dense int8 runs at twice the bf16 rate on B200: the measured bf16
        # figure doubled is the denominator
        roofline = {'bound': 'tensor', 'achieved': achieved_tf, 'peak': 2 * tf_peak, 'unit': 'TOP/s (int8)',
                    'frac': achieved_tf / (2 * tf_peak), 'traffic': traffic,
                    'peak_source': tf_src + ' x 2 (int8 dense rate)',
                    'frac_of_sustained': achieved_tf / (2 * tf_sust), 'hbm_frac': hbm_gbs / hbm, **common}
    elif w.bound == 'tensor':
        roofline = {'bound': 'tensor', 'achieved': achieved_tf, 'peak': tf_peak, 'unit': 'TFLOP/s',
                    'frac': achieved_tf / tf_peak, 'traffic': traffic, 'peak_source': tf_src,
                    'frac_of_sustained': achieved_tf / tf_sust, 'hbm_frac': hbm_gbs / hbm, **common}
        if args.config == 1:   # achieved counts the algorithmic FLOPs; the split runs three MMAs for each
            roofline['mma_flops_per_algorithmic_flop'] = 3
        if w.ops == 'e4m3':
            # FP8 operands: the dense FP8 rate is twice bf16's; the two query
            # terms make the MMAs do twice the algorithmic FLOPs
            roofline['frac_of_fp8_dense'] = achieved_tf / (2 * tf_peak)
            roofline['mma_flops_per_algorithmic_flop'] = 2
    else:
        roofline = {'bound': 'hbm', 'achieved': hbm_gbs, 'peak': hbm, 'unit': 'GB/s', 'frac': hbm_gbs / hbm,
                    'traffic': traffic, 'peak_source': kind + ' hbm_gbs', 'achieved_tflops': achieved_tf,
                    **common}

    # ---- correctness spot check against the CPU oracle
    verified = verify(w, result, args.verify, world, rank, args.k) if args.verify > 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        qps, desc, ckind = cpu_measure(args, threads, budget_s=args.cpu_seconds)
        cpu = {'value': qps, 'unit': 'queries/s', 'cores': threads, 'kind': ckind, 'sample': desc}

    if rank == 0:
        cand = int(nrows_local) * world if args.config != 4 else None
        # the workload (the same dict the reference arm prints); what this
        # implementation does with it goes beside
        cfg = workload_config(args)
        impl = {'parallelism': ('%s x%d, NCCL all-gather of top-k + device merge' % (
            'row-sharded (IVF lists cut at rank boundaries)' if args.config == 4 else 'row-sharded', world)
            if world > 1 else 'single GPU')}
        if cand is not None:
            impl['candidate_rows'] = cand
        if getattr(w, 'vtable', None) and world == 1:
            impl['worker_entry_points'] = w.vtable()
        # the per-step stage times and the check close the line, so that a
        # reader keeping only its end still has them
        line = {'metric': METRIC, 'value': value, 'unit': 'queries/s', 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True,
                'scaling': 'strong', 'vs_baseline': None, 'dtype': w.dtype, 'data': w.data, 'config': cfg, **impl,
                'e2e': e2e, 'gpu_launches': int(launches), 'roofline': roofline, 'cpu_baseline': cpu,
                'clocks': clock_info, 'verified_vs_oracle': verified, 'timed_steps': args.steps,
                'step_ms': {'min': round(min(step_ms), 4), 'median': round(statistics.median(step_ms), 4),
                            'max': round(max(step_ms), 4), 'slowest_step': int(np.argmax(step_ms))},
                'stage_loop_ms_per_step': round(stage_loop_ms, 4), 'stage_ms_per_step': stages}
        print(json.dumps(line), flush=True)
    w.shard.close()
    if w.comm is not None:
        w.comm.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == '__main__':
    sys.exit(main())
