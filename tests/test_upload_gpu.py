"""Large uploads go through the pinned double-buffered staging path (tensors of
64 MiB and more); the weights must arrive byte for byte: dequantized rows from
the start, the chunk boundaries and the end of a 300 MB tensor match the
oracle bit for bit."""
import time

import numpy as np
import pytest

import oracle
import strata_cuda as sc
from synth import Q4_K, quant_blocks, rng

pytestmark = pytest.mark.gpu


def test_large_upload_round_trips():
    rows, cols = 8192 * 16, 2048          # 151 MB of Q4_K
    rb = cols // 256 * 144
    g = rng(4242)
    data = quant_blocks(g, Q4_K, rows * cols // 256).reshape(-1)
    with sc.Context(0) as ctx:
        ctx.upload(data[:80 << 20], Q4_K, (80 << 20) // rb, cols).free()  # staging buffers allocated
        t0 = time.perf_counter()
        w = ctx.upload(data, Q4_K, rows, cols)
        dt = time.perf_counter() - t0
        import torch
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        plain = torch.from_numpy(data).cuda()  # one pageable copy, for comparison
        torch.cuda.synchronize()
        dp = time.perf_counter() - t1
        del plain
        print(f"upload {data.nbytes / 1e6:.0f} MB in {dt * 1e3:.1f} ms: {data.nbytes / dt / 1e9:.1f} GB/s "
              f"(one pageable copy: {data.nbytes / dp / 1e9:.1f} GB/s)")
        chunk_rows = (32 << 20) // rb
        for r0 in (0, chunk_rows - 1, chunk_rows, 3 * chunk_rows + 7, rows - 3):
            got = ctx.dequant(w, r0, 3 if r0 + 3 <= rows else rows - r0)
            want = oracle.dequantize(Q4_K, data[r0 * rb:(r0 + got.shape[0]) * rb], got.shape[0], cols)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), r0
        w.free()


def test_destroy_releases_weights_left_resident():
    """strata_cuda_destroy frees weights the caller did not free (a backend
    dropped with its cache full must not leak HBM)."""
    import torch
    torch.cuda.init()
    free0, _ = torch.cuda.mem_get_info(0)
    data = np.zeros(512 << 20, np.uint8)  # 512 MiB of Q8_0 blocks (zero scales)
    cols = 4096
    rows = data.nbytes // (cols // 32 * 34)
    ctx = sc.Context(0)
    kept = ctx.upload(data[:rows * (cols // 32 * 34)], sc.Q8_0, rows, cols)
    gone = ctx.upload(data[:1 << 20], sc.Q8_0, (1 << 20) // (cols // 32 * 34), cols)
    gone.free()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free0 - free1 > 400 << 20
    ctx.close()
    kept.free()  # a no-op once the context is gone
    free2, _ = torch.cuda.mem_get_info(0)
    assert free0 - free2 < 100 << 20, (free0 - free2) >> 20
