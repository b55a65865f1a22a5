"""Seeded synthetic corpora with the shapes and distributions of the benchmark
configurations (no public dataset is named for this path, so generated data
stands in for real embeddings):

  config 1  fp32, d=128, 100-centre Gaussian mixture, centres ~N(0,1),
            per-point noise sigma 0.1
  config 2  halfvec, d=768, 1,000-centre mixture, unit-normalised, 10%
            uniform row-filter bitmap
  config 3  FP8-E4M3 + per-row scale absmax/448, d=1024, 4,096-centre mixture
  config 4  NVFP4 (E2M1 + E4M3 block scale per 16 + row scale), d=768
  config 5  1,024-bit rows: 65,536 Bernoulli(0.5) prototypes, 5% bit flips

numpy functions make small host arrays (tests); torch functions generate
full-size data directly on a GPU in chunks (bench).
"""
import numpy as np


# ---------------------------------------------------------------- numpy (small)

def mixture(n, d, centres, sigma=0.1, seed=0, normalize=False, dtype=np.float32):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((centres, d)).astype(np.float32)
    lab = rng.integers(0, centres, n)
    x = c[lab] + sigma * rng.standard_normal((n, d)).astype(np.float32)
    if normalize:
        x /= np.maximum(np.linalg.norm(x, axis=1, keepdims=True), 1e-30)
    return x.astype(dtype)


def mixture_queries(q, d, centres, sigma=0.1, seed=0, normalize=False):
    """Queries drawn the same way as the corpus (same centres: same seed)."""
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((centres, d)).astype(np.float32)
    rng2 = np.random.default_rng(seed + 7919)
    lab = rng2.integers(0, centres, q)
    x = c[lab] + sigma * rng2.standard_normal((q, d)).astype(np.float32)
    if normalize:
        x /= np.maximum(np.linalg.norm(x, axis=1, keepdims=True), 1e-30)
    return x.astype(np.float32)


def to_half_bits(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).astype(np.float16)).view(np.uint16)


def bit_rows(n, dims, prototypes, flip=0.05, seed=0):
    rng = np.random.default_rng(seed)
    nbytes = dims // 8
    proto = rng.integers(0, 256, (prototypes, nbytes), dtype=np.uint8)
    lab = rng.integers(0, prototypes, n)
    flips = np.packbits(rng.random((n, dims)) < flip, axis=1, bitorder='little')
    return proto[lab] ^ flips, proto


def bitmap(n, selectivity, seed=0):
    """u32 words, bit r of word r//32 set with probability selectivity."""
    rng = np.random.default_rng(seed)
    bits = rng.random(n) < selectivity
    padded = np.zeros((n + 31) // 32 * 32, dtype=bool)
    padded[:n] = bits
    return np.packbits(padded, bitorder='little').view(np.uint32), np.nonzero(bits)[0].astype(np.uint32)


def ivf_corpus(n, d, nlists, zipf=1.1, sigma=0.1, seed=0, normalize=False):
    """IVF-shaped corpus stored list-major: list sizes follow Zipf(zipf) over
    a random list order, list l's rows are its centroid plus noise. Returns
    (rows [n][d] f32, offsets u64 [nlists+1], centroids [nlists][d],
    row_ids i64 [n]: a random permutation of 0..n-1, the rows' global ids)."""
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((nlists, d)).astype(np.float32)
    w = 1.0 / np.arange(1, nlists + 1, dtype=np.float64) ** zipf
    w = w[rng.permutation(nlists)]
    sizes = np.floor(w / w.sum() * n).astype(np.int64)
    sizes[np.argmax(sizes)] += n - sizes.sum()
    lab = np.repeat(np.arange(nlists), sizes)
    x = cent[lab] + sigma * rng.standard_normal((n, d)).astype(np.float32)
    if normalize:
        x /= np.maximum(np.linalg.norm(x, axis=1, keepdims=True), 1e-30)
        cent = cent / np.maximum(np.linalg.norm(cent, axis=1, keepdims=True), 1e-30)
    offsets = np.zeros(nlists + 1, dtype=np.uint64)
    offsets[1:] = np.cumsum(sizes)
    return x.astype(np.float32), offsets, cent, rng.permutation(n).astype(np.int64)


def ivf_probes(queries, centroids, nprobe):
    """Each query's nprobe nearest centroids (squared L2), nearest first."""
    q = np.asarray(queries, dtype=np.float64)
    c = np.asarray(centroids, dtype=np.float64)
    d2 = (q * q).sum(1)[:, None] - 2.0 * q @ c.T + (c * c).sum(1)[None, :]
    return np.argsort(d2, axis=1, kind='stable')[:, :nprobe].astype(np.uint32)


def write_index_dir(directory, keys, vectors, shards=1, quant=None, dtype='float32'):
    """An index directory in the worker's documented format
    (ann/common/INDEX_FORMAT.md, version 1): rows sorted by key into
    keys.i64 and vectors.f32, and a manifest naming `shards` contiguous
    graphless shards. `quant` adds a quantized copy of the rows (given in
    the same order as `vectors`): ('fp8', codes, row_scales) writes
    vectors.e4m3, ('nvfp4', codes, block_scales, row_scales) vectors.nvfp4
    and scales.e4m3, both rowscale.f32 and the manifest's quant line;
    `dtype` is the manifest's dtype line (float32 or float16).
    Returns (sorted keys, rows in key order)."""
    import os
    order = np.argsort(np.asarray(keys, dtype=np.int64), kind='stable')
    k = np.ascontiguousarray(np.asarray(keys, dtype=np.int64)[order])
    v = np.ascontiguousarray(np.asarray(vectors, dtype=np.float32)[order])
    n, d = v.shape
    os.makedirs(directory, exist_ok=True)
    k.astype('<i8').tofile(os.path.join(directory, 'keys.i64'))
    v.astype('<f4').tofile(os.path.join(directory, 'vectors.f32'))
    bounds = [n * i // shards for i in range(shards + 1)]
    lines = ['pgvector-ann-index 1', 'dimensions %d' % d, 'rows %d' % n, 'metric l2', 'dtype %s' % dtype,
             'shards %d' % shards]
    lines += ['shard %d %d %d -' % (i, bounds[i], bounds[i + 1] - bounds[i]) for i in range(shards)]
    if quant is not None:
        kind = quant[0]
        if kind == 'fp8':
            np.ascontiguousarray(np.asarray(quant[1], dtype=np.uint8)[order]).tofile(
                os.path.join(directory, 'vectors.e4m3'))
        elif kind == 'nvfp4':
            np.ascontiguousarray(np.asarray(quant[1], dtype=np.uint8)[order]).tofile(
                os.path.join(directory, 'vectors.nvfp4'))
            np.ascontiguousarray(np.asarray(quant[2], dtype=np.uint8)[order]).tofile(
                os.path.join(directory, 'scales.e4m3'))
        else:
            raise ValueError('quant must be fp8 or nvfp4')
        np.ascontiguousarray(np.asarray(quant[-1], dtype=np.float32)[order]).astype('<f4').tofile(
            os.path.join(directory, 'rowscale.f32'))
        lines.append('quant %s' % kind)
    with open(os.path.join(directory, 'manifest.tmp'), 'w') as f:
        f.write('\n'.join(lines) + '\n')
    os.rename(os.path.join(directory, 'manifest.tmp'), os.path.join(directory, 'manifest'))
    return k, v


# ---------------------------------------------------------------- torch (full size, on the GPU)

def torch_mixture(n, d, centres, sigma=0.1, seed=0, normalize=False, dtype=None, device='cuda',
                  chunk=1 << 20, out=None):
    """Gaussian-mixture rows generated on the device in chunks; returns a
    [n, d] tensor of `dtype` (float16 by default)."""
    import torch
    dtype = dtype or torch.float16
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    c = torch.randn((centres, d), generator=g, device=device, dtype=torch.float32)
    x = out if out is not None else torch.empty((n, d), dtype=dtype, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        lab = torch.randint(0, centres, (m,), generator=g, device=device)
        v = c[lab] + sigma * torch.randn((m, d), generator=g, device=device, dtype=torch.float32)
        if normalize:
            v /= v.norm(dim=1, keepdim=True).clamp_min(1e-30)
        x[s:s + m] = v.to(dtype)
    return x


def torch_mixture_queries(q, d, centres, sigma=0.1, seed=0, normalize=False, device='cuda'):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    c = torch.randn((centres, d), generator=g, device=device, dtype=torch.float32)
    g2 = torch.Generator(device=device)
    g2.manual_seed(seed + 7919)
    lab = torch.randint(0, centres, (q,), generator=g2, device=device)
    v = c[lab] + sigma * torch.randn((q, d), generator=g2, device=device, dtype=torch.float32)
    if normalize:
        v /= v.norm(dim=1, keepdim=True).clamp_min(1e-30)
    return v


def torch_bitmap(n, selectivity, seed=0, device='cuda'):
    """u32 bitmap words with each row's bit set with probability selectivity."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nw = (n + 31) // 32
    bits = (torch.rand((nw * 32,), generator=g, device=device) < selectivity)
    bits[n:] = False
    w = (bits.view(nw, 32).to(torch.int64) << torch.arange(32, device=device, dtype=torch.int64)).sum(dim=1)
    # the same 32 bits as a signed int32 (two's complement)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


# ---------------------------------------------------------------- torch quantizers (builder semantics)
#
# The index builder's FP8 and NVFP4 quantizers (ann/builder/build_cuvs_index.py
# :296-348) restated over torch tensors, so full-size corpora can be encoded
# on the GPU; oracle.quantize_fp8 / quantize_nvfp4 are the C statements of
# the same steps, and tests/test_oracle.py checks that both agree bit for bit.

def _e4m3_table(device):
    """Non-negative E4M3 magnitudes of codes 0..126, increasing."""
    import torch
    c = torch.arange(127, device=device)
    e = (c >> 3).to(torch.float32)
    m = (c & 7).to(torch.float32)
    return torch.where(c < 8, m * 2.0 ** -9, (8.0 + m) * torch.exp2(e - 10.0)).to(torch.float32)


def _nearest(table, x):
    """Index of the nearest table entry (ties to the lower entry)."""
    import torch
    size = table.numel()
    i = torch.searchsorted(table, x.contiguous()).clamp_(1, size - 1)
    below, above = table[i - 1], table[i]
    return torch.where((x - below) <= (above - x), i - 1, i)


def torch_quantize_fp8(x):
    """[n, d] float32 -> (codes uint8 [n, ceil(d/16)*16], row scales float32
    [n]): scale = absmax/448, code = nearest E4M3 magnitude of |v/scale|
    with the sign in bit 7."""
    import torch
    n, d = x.shape
    pad = (d + 15) // 16 * 16
    amax = x.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    v = x / scale[:, None]
    code = _nearest(_e4m3_table(x.device), v.abs()).to(torch.uint8)
    code = code | torch.where(v < 0, 0x80, 0).to(torch.uint8)
    out = torch.zeros((n, pad), dtype=torch.uint8, device=x.device)
    out[:, :d] = code
    return out, scale


def torch_quantize_nvfp4(x):
    """[n, d] float32 -> (packed uint8 [n, blocks*8], block scale codes uint8
    [n, blocks], row scales float32 [n]), blocks = ceil(d/16): row =
    absmax/(6*448); a block's scale code is the smallest E4M3 entry >=
    blockmax/(6*row) (at most 126); values are the nearest E2M1 magnitude of
    min(|v/(table[code]*row)|, 6), sign in bit 3, even dimension low."""
    import torch
    n, d = x.shape
    blocks = (d + 15) // 16
    xp = torch.zeros((n, blocks * 16), dtype=torch.float32, device=x.device)
    xp[:, :d] = x
    amax = x.abs().amax(dim=1)
    row = torch.where(amax > 0, amax / 2688.0, torch.ones_like(amax))
    six = 6.0 * row
    xb = xp.view(n, blocks, 16)
    bmax = xb.abs().amax(dim=2)
    table = _e4m3_table(x.device)
    code = torch.searchsorted(table, (bmax / six[:, None]).contiguous()).clamp_(max=126)
    scale = table[code] * row[:, None]
    v = torch.where(scale[:, :, None] > 0, xb / scale[:, :, None], torch.zeros_like(xb))
    e2m1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32, device=x.device)
    nib = _nearest(e2m1, v.abs().clamp(max=6.0)).to(torch.uint8) | torch.where(v < 0, 8, 0).to(torch.uint8)
    nib = nib.view(n, blocks * 8, 2)
    packed = nib[:, :, 0] | (nib[:, :, 1] << 4)
    return packed.contiguous(), code.to(torch.uint8).contiguous(), row
