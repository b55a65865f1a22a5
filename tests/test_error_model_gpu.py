"""The scan's approximate scores against exact arithmetic.

Exactness of every search rests on one inequality: for each (row, query)
pair, |approximate - exact| <= the per-query bound the library computes
(scan_gamma and prep_queries). Pruning uses that bound as its margin, so a
row whose exact distance can still reach the answer is never dropped. This
test measures the inequality over millions of pairs on both scan paths,
and requires the observed error to stay below half of the bound.
"""
import numpy as np
import pytest

from pgvector_b200 import synth

pytestmark = pytest.mark.gpu


def exact(x64, q64, metric):
    dot = q64 @ x64.T
    if metric == 1:
        return -dot
    if metric == 2:
        nx = (x64 * x64).sum(1)
        nq = (q64 * q64).sum(1)
        return 1 - np.clip(dot / np.sqrt(np.outer(nq, nx)), -1, 1)
    return (q64 * q64).sum(1)[:, None] + (x64 * x64).sum(1)[None, :] - 2 * dot


@pytest.mark.parametrize('metric', [2, 1, 0])
@pytest.mark.parametrize('simt', [False, True])
def test_bound_holds_on_f16_rows(cuda, metric, simt):
    import torch
    import pgvector_b200 as pb
    n, d, nq = 20000, 768, 256
    x = synth.mixture(n, d, 50, seed=40, normalize=(metric == 2)).astype(np.float16)
    q = synth.mixture_queries(nq, d, 50, seed=40, normalize=(metric == 2))
    q[: nq // 2] = q[: nq // 2].astype(np.float16).astype(np.float32)   # half the queries FP16-exact
    shard = pb.Shard(pb.F16, d, torch.from_numpy(x.view(np.int16)).to(cuda))
    approx, err = shard.score_matrix(torch.from_numpy(q).to(cuda), metric, force_simt=simt)
    approx = approx.cpu().numpy().astype(np.float64)
    err = err.cpu().numpy()
    ex = exact(x.astype(np.float64), q.astype(np.float64), metric)
    diff = np.abs(approx - ex)
    ratio = (diff / err[:, None]).max()
    print('metric %d simt %s: max |approx - exact| = %.3g, max ratio to bound = %.4f'
          % (metric, simt, diff.max(), ratio))
    assert (diff <= err[:, None]).all()
    assert ratio < 0.5


@pytest.mark.parametrize('dtype,dims,f16', [(2, 1024, False), (2, 1024, True), (2, 200, False), (3, 768, False),
                                           (3, 224, False)])
@pytest.mark.parametrize('metric', [1, 0, 2])
@pytest.mark.parametrize('simt', [False, True])
def test_bound_holds_on_quantized_rows(cuda, dtype, dims, f16, metric, simt):
    # exact: FP64 arithmetic on the rows decoded to FP32 as the reference
    # decodes them (code x scale products rounded to FP32)
    import torch
    import oracle
    import pgvector_b200 as pb
    n, nq = 12000, 128
    x = synth.mixture(n, dims, 40, seed=42 + dims)
    q = synth.mixture_queries(nq, dims, 40, seed=42 + dims)
    if dtype == oracle.E4M3:
        codes, rs = oracle.quantize_fp8(x)
        bs = None
        shard = pb.Shard(pb.E4M3, dims, torch.from_numpy(codes).to(cuda), None, torch.from_numpy(rs).to(cuda))
    else:
        codes, bs, rs = oracle.quantize_nvfp4(x)
        shard = pb.Shard(pb.NVFP4, dims, torch.from_numpy(codes).to(cuda), torch.from_numpy(bs).to(cuda),
                         torch.from_numpy(rs).to(cuda))
    dec = oracle.decode_rows(dtype, dims, codes, block_scales=bs, row_scales=rs).astype(np.float64)
    # E4M3 rows: the FP8 tensor scan (queries as two E4M3 terms), or with
    # f16 the codes converted to FP16 for kind::f16 MMAs
    approx, err = shard.score_matrix(torch.from_numpy(q).to(cuda), metric, force_simt=simt, force_f16=f16)
    approx = approx.cpu().numpy().astype(np.float64)
    err = err.cpu().numpy()
    ex = exact(dec, q.astype(np.float64), metric)
    diff = np.abs(approx - ex)
    ratio = (diff / err[:, None]).max()
    print('dtype %d dims %d f16 %s metric %d simt %s: max |approx - exact| = %.3g, max ratio to bound = %.4f'
          % (dtype, dims, f16, metric, simt, diff.max(), ratio))
    assert (diff <= err[:, None]).all()
    assert ratio < 0.5


def test_hamming_scores_are_exact(cuda):
    import torch
    import pgvector_b200 as pb
    rows, proto = synth.bit_rows(5000, 1024, 64, seed=41)
    rng = np.random.default_rng(41)
    qs = rng.integers(0, 256, (64, 128), dtype=np.uint8)
    shard = pb.Shard(pb.BIT, 1024, torch.from_numpy(rows).to(cuda))
    approx, err = shard.score_matrix(torch.from_numpy(qs).to(cuda), pb.HAMMING)
    ex = np.unpackbits(qs[:, None, :] ^ rows[None, :, :], axis=2).sum(2)
    assert np.array_equal(approx.cpu().numpy(), ex.astype(np.float32))
    assert (err.cpu().numpy() == 0).all()


@pytest.mark.parametrize('dims', [128, 200])
@pytest.mark.parametrize('metric', [1, 0, 2])
@pytest.mark.parametrize('simt', [False, True])
def test_bound_holds_on_f32_rows(cuda, dims, metric, simt):
    # FP32 rows on tensor cores are split into two BF16 halves (L2 and inner
    # product; cosine scores on CUDA cores); columns scaled over many binades
    # and a few subnormal elements exercise the split's relative and absolute
    # terms
    import torch
    import pgvector_b200 as pb
    n, nq = 12000, 128
    x = synth.mixture(n, dims, 40, seed=44 + dims)
    q = synth.mixture_queries(nq, dims, 40, seed=44 + dims)
    scale = np.ones(dims, dtype=np.float32)
    scale[::7] = 1e-6
    scale[3::11] = 300.0
    x *= scale
    x[::97, 5] = np.float32(1e-40)
    shard = pb.Shard(pb.F32, dims, torch.from_numpy(x).to(cuda))
    approx, err = shard.score_matrix(torch.from_numpy(q).to(cuda), metric, force_simt=simt)
    approx = approx.cpu().numpy().astype(np.float64)
    err = err.cpu().numpy()
    ex = exact(x.astype(np.float64), q.astype(np.float64), metric)
    diff = np.abs(approx - ex)
    ratio = (diff / err[:, None]).max()
    print('f32 dims %d metric %d simt %s: max |approx - exact| = %.3g, max ratio to bound = %.4f'
          % (dims, metric, simt, diff.max(), ratio))
    assert (diff <= err[:, None]).all()
    assert ratio < 0.5


@pytest.mark.parametrize('dims', [1024, 4096])
def test_fp8_accumulation_error(cuda, dims):
    # The FP8 tensor scan's accumulation alone: queries that are exactly a
    # power of two times E4M3 values (their low terms are zero, nothing is
    # lost to their rounding), so |approx - exact| is what the tensor core's
    # sums of E4M3 products lose. Measured against sum |x_i q_i| it must stay
    # a quarter of the share of the bound scan_gamma allows for it.
    import torch
    import oracle
    import pgvector_b200 as pb
    n, nq = 8000, 64
    rng = np.random.default_rng(dims)
    x = (rng.standard_normal((n, dims)) * np.exp(rng.uniform(-3, 3, (1, dims)))).astype(np.float32)
    codes, rs = oracle.quantize_fp8(x)
    qc, _ = oracle.quantize_fp8(rng.standard_normal((nq, dims)).astype(np.float32) * 50)
    q = (oracle.decode_rows(oracle.E4M3, dims, qc) * np.float32(2.0 ** -3)).astype(np.float32)
    shard = pb.Shard(pb.E4M3, dims, torch.from_numpy(codes).to(cuda), None, torch.from_numpy(rs).to(cuda))
    approx, err = shard.score_matrix(torch.from_numpy(q).to(cuda), 1)
    dec = oracle.decode_rows(oracle.E4M3, dims, codes, row_scales=rs).astype(np.float64)
    q64 = q.astype(np.float64)
    ex = -(q64 @ dec.T)
    mag = np.abs(q64) @ np.abs(dec).T
    rel = np.abs(approx.cpu().numpy().astype(np.float64) - ex) / mag
    kpad = (dims + 127) // 128 * 128
    allowed = (2.0 * kpad / 32 + 2.0) * 2.0 ** -19
    print('dims %d: largest accumulation error %.3g of sum |x q| (2^%.1f); the bound allows %.3g'
          % (dims, rel.max(), np.log2(max(rel.max(), 1e-300)), allowed))
    assert rel.max() <= allowed / 4
    assert (np.abs(approx.cpu().numpy() - ex) <= err.cpu().numpy()[:, None]).all()
