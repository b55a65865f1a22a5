"""The tensor scan's bounded waits: a pipeline wait that runs out makes the
search fail with ANN_BACKEND_ERROR (the kernel sets FLAG_TIMEOUT, leaves its
loops, drains its MMAs and bulk copies and frees tensor memory), and the
device stays usable: the next search is bit-exact with the oracle.

ANN_B200_PIPELINE_WAIT_NS shortens only the flat scan's pipeline waits (read
at every launch); the drains after an abort keep their 4 s limit. Nothing
here faults or hangs the GPU: the shortened limit makes the kernel return
early with an error status that the host reads."""
import numpy as np
import pytest

import oracle
from pgvector_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('dtype', ['f16_list', 'f16', 'e4m3'])
def test_pipeline_wait_runs_out_then_device_recovers(cuda, monkeypatch, dtype):
    import torch
    import pgvector_b200 as pb
    n, d, nq, k = 60000, 256, 64, 20
    x = synth.mixture(n, d, 32, seed=91)
    q = synth.mixture_queries(nq, d, 32, seed=92)
    rows = None
    if dtype == 'e4m3':
        codes, rs = oracle.quantize_fp8(x)
        shard = pb.Shard(pb.E4M3, d, torch.from_numpy(codes).to(cuda), None, torch.from_numpy(rs).to(cuda))
        want = oracle.search(oracle.E4M3, d, codes, q, k, 0, row_scales=rs)
    else:
        h = synth.to_half_bits(x)
        shard = pb.Shard(pb.F16, d, torch.from_numpy(h.view(np.int16)).to(cuda))
        ids = None
        if dtype == 'f16_list':                  # the row-gathering scan
            _, ids = synth.bitmap(n, 0.6, seed=93)
            rows = torch.from_numpy(ids.view(np.int32)).to(cuda)
        want = oracle.search(oracle.F16, d, h, q, k, 0, ids=ids)
    qd = torch.from_numpy(q).to(cuda)
    monkeypatch.setenv('ANN_B200_PIPELINE_WAIT_NS', '1')
    with pytest.raises(pb.AnnB200Error) as err:
        shard.search(qd, k, pb.L2, rows=rows)
    assert err.value.status == pb.BACKEND_ERROR and 'timed out' in str(err.value)
    monkeypatch.delenv('ANN_B200_PIPELINE_WAIT_NS')
    for _ in range(2):
        gd, gi, gc = shard.search(qd, k, pb.L2, rows=rows)
        torch.cuda.synchronize()
        assert np.array_equal(gc.cpu().numpy(), want[2].astype(np.int32))
        assert np.array_equal(gi.cpu().numpy(), want[1]) and np.array_equal(gd.cpu().numpy(), want[0])
    shard.close()
