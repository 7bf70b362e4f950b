"""strata_cuda_gemv_noalloc: the decode GEMV for callers that cannot allocate
device memory (for example while a stream is being captured into a CUDA
graph), with its scratch in a static device array of the library.

It must give the same result as the context-based entry point on the same
inputs, on consecutive calls (the shared scratch keeps the previous call's
contents), and must refuse sizes beyond its fixed scratch.
"""
import numpy as np
import pytest

import strata_cuda as sc
from conftest import rel_err
from synth import Q4_K, Q5_K, activations, quant_matrix

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _noalloc(w_dev, quant, rows, cols, x, y, batch, stream):
    return sc.lib().strata_cuda_gemv_noalloc(w_dev, quant, rows, cols, x, y, batch, stream)


def _status(stream, clear):
    return sc.lib().strata_cuda_gemv_noalloc_status(stream, clear)


# K = 2304 and 1280 are not whole 2048-weight chunks: those rows are staged by
# per-row bulk copies instead of the tensor map
@pytest.mark.parametrize("quant,rows,cols,batch", [(Q4_K, 4096, 4096, 1), (Q5_K, 1000, 2048, 3),
                                                   (Q4_K, 777, 8192, 8), (Q4_K, 300, 2304, 1),
                                                   (Q5_K, 64, 1280, 5)])
def test_noalloc_matches_context_entry_point(quant, rows, cols, batch):
    import torch
    data = quant_matrix(3000 + cols + batch, quant, rows, cols)
    w_dev = torch.from_numpy(data).cuda()
    with sc.Context(0) as ctx:
        w = ctx.upload(data, quant, rows, cols)
        s = torch.cuda.current_stream()
        for call in range(2):  # two calls in a row through the shared scratch
            x = torch.from_numpy(activations(3001 + call, batch, cols)).cuda()
            y_ref = torch.empty(batch, rows, device="cuda")
            y = torch.full((batch, rows), float("nan"), device="cuda")
            ctx.gemv_dev(w, x.data_ptr(), y_ref.data_ptr(), batch, s.cuda_stream)
            rc = _noalloc(w_dev.data_ptr(), quant, rows, cols, x.data_ptr(), y.data_ptr(), batch, s.cuda_stream)
            assert rc == sc.OK
            torch.cuda.synchronize()
            assert rel_err(y.cpu().numpy(), y_ref.cpu().numpy()) < TOL, (quant, call)
        # no kernel of these calls gave up a wait; reading the status clears nothing else
        assert _status(s.cuda_stream, 1) == sc.OK
        assert _status(s.cuda_stream, 0) == sc.OK
        w.free()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    rows, cols, batch = 16, 16384, 8           # cols * batch = 131,072 > 65,536
    w_dev = torch.zeros(rows * cols // 256 * 144, dtype=torch.uint8, device="cuda")
    x = torch.zeros(batch, cols, device="cuda")
    y = torch.zeros(batch, rows, device="cuda")
    rc = _noalloc(w_dev.data_ptr(), Q4_K, rows, cols, x.data_ptr(), y.data_ptr(), batch, None)
    assert rc == sc.ERR_SCRATCH_LIMIT
    rc = _noalloc(w_dev.data_ptr(), 14, rows, 256, x.data_ptr(), y.data_ptr(), 1, None)  # Q6_K
    assert rc == sc.ERR_UNSUPPORTED_QUANT
