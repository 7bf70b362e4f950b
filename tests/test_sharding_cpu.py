"""The multi-GPU split, checked on the CPU with world-size-2 gloo groups.

Each rank runs ops::gemv (the oracle) on its row shard of a Q4_K matrix and
the shards are all-gathered: the result must equal the full product bit for
bit, which pins the byte ranges sharding.row_shard hands to each rank. The
expert split is checked the same way on expert_gemv.
"""
import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "strata-rs_b200"),
                        os.path.join(os.path.dirname(HERE), "oracle")]
        import torch
        import torch.distributed as dist
        import oracle
        import sharding
        from synth import Q4_K, activations, quant_matrix
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        N, K = 512, 1024
        data = quant_matrix(3000, Q4_K, N, K)
        x = activations(3001, 2, K)
        part = oracle.gemv(Q4_K, sharding.row_shard(data, Q4_K, N, K, world, rank), N // world, K, x)
        parts = [torch.empty((2, N // world), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(part)))
        got = torch.cat(parts, dim=1).numpy()
        want = oracle.gemv(Q4_K, data, N, K, x)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        # experts: this rank's slice of an [E][IN][OUT] tensor, expert by expert
        E, IN, OUT = 8, 256, 512
        ed = quant_matrix(3002, Q4_K, IN, OUT, E)
        sl = sharding.expert_shard(ed, E, world, rank)
        e0, e1 = sharding.expert_range(E, world, rank)
        xe = activations(3003, 1, IN)
        for e in range(e0, e1):
            a = oracle.expert_gemv(Q4_K, sl, e1 - e0, IN, OUT, e - e0, xe)
            b = oracle.expert_gemv(Q4_K, ed, E, IN, OUT, e, xe)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_row_and_expert_shards_gloo_world2():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(m == "ok" for m in res.values()), res


def test_ranges_cover_without_overlap():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "strata-rs_b200"))
    import sharding
    for n, g in [(4096, 1), (4096, 2), (28672, 8), (256, 4)]:
        rs = [sharding.row_range(n, g, r) for r in range(g)]
        assert rs[0][0] == 0 and rs[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    try:
        sharding.row_range(10, 3, 0)
    except ValueError:
        pass
    else:
        raise AssertionError("uneven split accepted")
