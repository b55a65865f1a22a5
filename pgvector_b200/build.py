"""Build libannb200.so in-tree: AOT sm_100a CUDA plus the C backend.

    python -m pgvector_b200.build        (or pgvector_b200.build.build())

Objects go to pgvector_b200/_build/, the library to pgvector_b200/libannb200.so.
"""
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, 'csrc')
INCLUDE = os.path.join(os.path.dirname(HERE), 'include')
OUT_DIR = os.path.join(HERE, '_build')
LIB = os.path.join(HERE, 'libannb200.so')

CUDA_HOME = os.environ.get('CUDA_HOME', '/usr/local/cuda')
NVCC = os.path.join(CUDA_HOME, 'bin', 'nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ARCH + ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '-I' + INCLUDE,
                     '--expt-relaxed-constexpr']
CU_SOURCES = ['scan_simt.cu', 'scan_tc.cu', 'select.cu', 'shard.cu', 'ivf.cu', 'bitmap_static.cu', 'comm.cu']
C_SOURCES = ['backend.c']


def _run(cmd):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError('command failed: %s\n%s' % (' '.join(cmd), proc.stdout))
    return proc.stdout


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build(verbose=False, force=False, ptxas_info=False):
    """Compile every source that changed and link libannb200.so."""
    os.makedirs(OUT_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(('.cuh', '.h'))]
    headers += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    jobs, objects = [], []
    for src in CU_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(OUT_DIR, src + '.o')
        objects.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [NVCC] + NVCC_FLAGS + (['-Xptxas', '-v'] if ptxas_info else []) + ['-c', path, '-o', obj]
            jobs.append(cmd)
    cc = shutil.which('gcc') or 'gcc'
    for src in C_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(OUT_DIR, src + '.o')
        objects.append(obj)
        if force or _stale(obj, [path] + headers):
            jobs.append([cc, '-std=c11', '-O2', '-fPIC', '-Wall', '-Wextra', '-I' + INCLUDE,
                         '-I' + os.path.join(CUDA_HOME, 'include'), '-c', path, '-o', obj])
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for out in pool.map(_run, jobs):
            if verbose and out.strip():
                print(out)
    if force or jobs or _stale(LIB, objects):
        _run([NVCC] + ARCH + ['-shared', '-o', LIB] + objects + ['-lpthread', '-ldl'])
    return LIB


if __name__ == '__main__':
    build(verbose=True, force='--force' in sys.argv, ptxas_info='--ptxas' in sys.argv)
    print(LIB)
