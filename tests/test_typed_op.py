"""The typed search operation (32) over the worker's socket protocol.

The reference worker built with the operation added (oracle/worker_typed.py,
into oracle/_ref/): frames of the protocol's own layout (32-byte header
`PVAN`, version 1, operation, request id, generation, payload bytes,
status) sent over its Unix socket. On CPU the reference's own backends have
no typed search: the worker checks each frame and answers "unsupported" or
"invalid", and its other operations are untouched. On a GPU the worker with
libannb200's backend (`--backend b200`) answers with every query's gathered
window, equal to the oracle's, for every storage format."""
import os
import socket
import struct
import subprocess
import tempfile
import time

import numpy as np
import pytest

import oracle
from pgvector_b200 import synth

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'oracle', '_ref')
OP_TYPED = 32
OK, INVALID, UNSUPPORTED = 0, 1, 2


def frame(op, request, payload):
    return b'PVAN' + struct.pack('<HHQQII', 1, op, request, 0, len(payload), 0) + payload


def read_exact(sock, n):
    buf = bytearray()
    while len(buf) < n:
        part = sock.recv(n - len(buf))
        if not part:
            raise ConnectionError('worker closed the connection')
        buf += part
    return bytes(buf)


def call(sock, op, payload, request=1):
    sock.sendall(frame(op, request, payload))
    head = read_exact(sock, 32)
    assert head[:4] == b'PVAN'
    _, rop, rreq, _, size, status = struct.unpack('<HHQQII', head[4:])
    assert rop == op and rreq == request
    return status, read_exact(sock, size)


class Worker:
    def __init__(self, binary, backend):
        self.dir = tempfile.mkdtemp(prefix='annw')
        self.path = os.path.join(self.dir, 'w.sock')
        self.proc = subprocess.Popen([binary, '--backend', backend, '--listen', self.path],
                                     stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
        t0 = time.time()
        while not os.path.exists(self.path):
            if self.proc.poll() is not None or time.time() - t0 > 30:
                self.close()
                raise RuntimeError('worker did not start: %s' % self.proc.stderr.read().decode()[-500:])
            time.sleep(0.05)
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.settimeout(120)
        self.sock.connect(self.path)

    def close(self):
        if getattr(self, 'sock', None):
            self.sock.close()
        if self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
        if os.path.exists(self.path):
            os.unlink(self.path)
        os.rmdir(self.dir)


def typed_payload(dtype, metric, dims, k, queries, codes, row_scales=None, block_scales=None, rows=None):
    q = np.ascontiguousarray(queries)
    c = np.ascontiguousarray(codes)
    n = c.shape[0] if rows is None else rows
    parts = [struct.pack('<6I', n, dims, k, metric, dtype, q.shape[0]), q.tobytes(), c.tobytes()]
    if row_scales is not None:
        parts.append(np.ascontiguousarray(row_scales, np.float32).tobytes())
    if block_scales is not None:
        parts.append(np.ascontiguousarray(block_scales, np.uint8).tobytes())
    return b''.join(parts)


def parse_windows(payload, nq):
    out, at = [], 0
    for _ in range(nq):
        (count,) = struct.unpack_from('<I', payload, at)
        at += 4
        hits = []
        for _ in range(count):
            row, dist = struct.unpack_from('<Id', payload, at)
            hits.append((row, dist))
            at += 12
        out.append(hits)
    assert at == len(payload)
    return out


def binary(name):
    path = os.path.join(REF, name)
    if not os.path.exists(path):
        pytest.skip('%s not built (oracle/worker_typed.py needs the reference sources)' % name)
    return path


def test_typed_op_frames_checked_by_reference_backends():
    w = Worker(binary('ann-worker-typed'), 'cpu-exact')
    try:
        d = 16
        x = synth.mixture(50, d, 4, seed=1)
        q = synth.mixture_queries(3, d, 4, seed=2)
        h = synth.to_half_bits(x)
        good = typed_payload(1, 2, d, 5, q, h)
        # a well-formed frame: this backend has no typed search
        assert call(w.sock, OP_TYPED, good)[0] == UNSUPPORTED
        bad = [good[:-2],                                              # payload shorter than its fields say
               typed_payload(5, 2, d, 5, q, h),                        # no such dtype
               typed_payload(1, 3, d, 5, q, h),                        # Hamming needs bit rows
               typed_payload(4, 0, d, 5, q, h),                        # bit rows need Hamming
               typed_payload(1, 4, d, 5, q, h),                        # no such metric
               typed_payload(1, 2, 0, 5, q[:, :0], h[:, :0]),          # no dimensions
               typed_payload(1, 2, d, 5, q[:0], h),                    # no queries
               struct.pack('<5I', 50, d, 5, 2, 1)]                     # header cut short
        for i, p in enumerate(bad):
            assert call(w.sock, OP_TYPED, p, request=10 + i)[0] == INVALID, i
        # the reference's own operations are unchanged: capabilities, and a
        # gathered search (op 7) equal to the oracle's window
        st, caps = call(w.sock, 0, b'', request=20)
        assert st == OK and b'"exact"' in caps
        st, body = call(w.sock, 7, struct.pack('<4I', 50, d, 5, 0) + q[0].tobytes() + x.tobytes(), request=21)
        od, oi, oc, _ = oracle.search(oracle.F32, d, x, q[:1], 5, 0, window=True, cap=50)
        assert st == OK
        assert parse_windows(body, 1)[0] == [(int(oi[0, r]), float(od[0, r])) for r in range(oc[0])]
    finally:
        w.close()


@pytest.mark.gpu
def test_typed_op_served_by_b200_backend(cuda):
    w = Worker(binary('ann-worker-b200'), 'b200')
    try:
        d = 96
        x = synth.mixture(3000, d, 30, seed=31)
        q = synth.mixture_queries(24, d, 30, seed=32)
        h = synth.to_half_bits(x)
        c8, r8 = oracle.quantize_fp8(x)
        c4, b4, r4 = oracle.quantize_nvfp4(x)
        bits, _ = synth.bit_rows(3000, 256, 16, flip=0.05, seed=33)
        qb = bits[np.random.default_rng(34).integers(0, 3000, 20)].copy()
        cases = [(oracle.F32, 0, x, q, None, None, 10, d),
                 (oracle.F16, 2, h, q, None, None, 100, d),            # halfvec cosine, a tensor-core batch
                 (oracle.E4M3, 1, c8, q, None, r8, 50, d),
                 (oracle.NVFP4, 0, c4, q[:5], b4, r4, 20, d),
                 (oracle.BIT, 3, bits, qb, None, None, 30, 256),       # Hamming: ties kept in the window
                 (oracle.F32, 2, x[:1], q[:1], None, None, 3, d)]      # k past the rows
        for i, (dt, m, codes, qs, bs, rs, k, dims) in enumerate(cases):
            st, body = call(w.sock, OP_TYPED, typed_payload(dt, m, dims, k, qs, codes, rs, bs), request=100 + i)
            assert st == OK, (dt, m)
            od, oi, oc, _ = oracle.search(dt, dims, codes, qs, k, m, block_scales=bs, row_scales=rs, window=True,
                                          cap=codes.shape[0])
            got = parse_windows(body, qs.shape[0])
            for qi in range(qs.shape[0]):
                assert got[qi] == [(int(oi[qi, r]), float(od[qi, r])) for r in range(oc[qi])], (dt, m, qi)
        # a zero query under cosine is the backend's INVALID, sent as the frame's status
        zq = np.zeros((1, d), np.float32)
        assert call(w.sock, OP_TYPED, typed_payload(oracle.F16, 2, d, 5, zq, h), request=200)[0] == INVALID
    finally:
        w.close()
