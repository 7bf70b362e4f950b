"""The multi-GPU split, checked on the CPU with world-size-2 gloo groups.

Each rank runs ops::gemv (the oracle) on its row shard of a Q4_K matrix and
the shards are all-gathered: the result must equal the full product bit for
bit, which pins the byte ranges sharding.row_shard hands to each rank. The
expert split is checked the same way on expert_gemv, and the expert-parallel
MoE layer end to end: each rank's weighted partial sum over its experts (the
shared expert on rank 0), all-reduced, equals the oracle's whole layer.
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


def _ep_worker(rank, world, port, q):
    """Expert parallelism on gloo ranks: each rank sums its experts' weighted
    outputs (the shared expert on rank 0 only), the partial sums are
    all-reduced, and the total must match the oracle's whole layer."""
    try:
        sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "strata-rs_b200"),
                        os.path.join(os.path.dirname(HERE), "oracle")]
        import datetime

        import torch
        import torch.distributed as dist

        import oracle
        import sharding
        from synth import Q4_K, activations, quant_matrix
        from test_moe_restatement_cpu import route, silu, sigmoid
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        n_embd, E, k, n_ff, n_ffs = 256, 8, 3, 256, 256
        t = {"router": (Q4_K, quant_matrix(6001, Q4_K, E, n_embd)),
             "gate_exps": (Q4_K, quant_matrix(6002, Q4_K, n_embd, n_ff, E)),
             "up_exps": (Q4_K, quant_matrix(6003, Q4_K, n_embd, n_ff, E)),
             "down_exps": (Q4_K, quant_matrix(6004, Q4_K, n_ff, n_embd, E)),
             "gate_shexp": (Q4_K, quant_matrix(6005, Q4_K, n_ffs, n_embd)),
             "up_shexp": (Q4_K, quant_matrix(6006, Q4_K, n_ffs, n_embd)),
             "down_shexp": (Q4_K, quant_matrix(6007, Q4_K, n_embd, n_ffs)),
             "gate_inp_shexp": (Q4_K, quant_matrix(6008, Q4_K, 1, n_embd))}
        x = activations(6009, 2, n_embd)
        logits = np.random.default_rng(6010).standard_normal((2, E)).astype(np.float32)
        e0, e1 = sharding.expert_range(E, world, rank)
        per = {nm: t[nm][1].size // E for nm in ("gate_exps", "up_exps", "down_exps")}
        mine = {nm: t[nm][1][e0 * per[nm]:e1 * per[nm]] for nm in per}  # this rank's bytes only
        part = np.zeros((2, n_embd), np.float32)
        for tok in range(2):
            ids, w = route(logits[tok], k)
            for e, we in zip(ids, w):
                if not e0 <= e < e1 or we == 0.0:
                    continue
                g = oracle.expert_gemv(Q4_K, mine["gate_exps"], e1 - e0, n_embd, n_ff, int(e) - e0, x[tok])
                u = oracle.expert_gemv(Q4_K, mine["up_exps"], e1 - e0, n_embd, n_ff, int(e) - e0, x[tok])
                h = (silu(g.reshape(-1)) * u.reshape(-1)).astype(np.float32)
                d = oracle.expert_gemv(Q4_K, mine["down_exps"], e1 - e0, n_ff, n_embd, int(e) - e0, h).reshape(-1)
                part[tok] = (part[tok] + np.float32(we) * d).astype(np.float32)
            if rank == 0:
                g = oracle.gemv(Q4_K, t["gate_shexp"][1], n_ffs, n_embd, x[tok]).reshape(-1)
                u = oracle.gemv(Q4_K, t["up_shexp"][1], n_ffs, n_embd, x[tok]).reshape(-1)
                h = (silu(g) * u).astype(np.float32)
                d = oracle.gemv(Q4_K, t["down_shexp"][1], n_embd, n_ffs, h).reshape(-1)
                sg = sigmoid(oracle.gemv(Q4_K, t["gate_inp_shexp"][1], 1, n_embd, x[tok]).reshape(-1))[0]
                part[tok] = (part[tok] + sg * d).astype(np.float32)
        total = torch.from_numpy(part.copy())
        dist.all_reduce(total)
        want, _, _ = oracle.moe_layer(t, n_embd, E, k, n_ff, n_ffs, x, logits)
        from conftest import rel_err
        for tok in range(2):
            assert rel_err(total.numpy()[tok], want[tok]) < 1e-5, (rank, tok)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_expert_parallel_partial_sums_gloo_world2():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(m == "ok" for m in res.values()), res
