"""Multi-GPU paths through the C ABI: one spawned process per GPU.

Row-sharded GEMV / GEMM + all-gather and expert-parallel MoE + all-reduce are
compared with the single-GPU results of the same context (themselves pinned
to the oracle by the other GPU tests). The communicator-timeout case needs
only one GPU: rank 0 of a world of 2 whose rank 1 never joins.
"""
import multiprocessing as mp
import os
import sys
import traceback

import numpy as np
import pytest

import strata_cuda as sc

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _ngpu():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank, world, uid, q):
    try:
        sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "strata-rs_b200"),
                        os.path.join(os.path.dirname(HERE), "oracle")]
        import torch
        import strata_cuda as sc
        import sharding
        from conftest import rel_err
        from synth import Q4_K, Q5_K, activations, bf16_bits, quant_matrix, rng
        torch.cuda.set_device(rank)
        ctx = sc.Context(rank)
        ctx.set_wait_timeout_ms(60000)
        ctx.comm_init(rank, world, uid)
        ctx.set_wait_timeout_ms(10000)  # bounds each peer-gather wait below
        assert ctx.comm_info() == (rank, world)
        st = torch.cuda.Stream()
        dev = f"cuda:{rank}"

        # row-sharded GEMV: bitwise the single-GPU GEMV, through both gathers
        # (NCCL all-gathers; the all-gather fused into the GEMV over peer
        # memory), several calls in a row so both exchange halves are used
        avail, cap = ctx.comm_peer_info()
        assert avail and cap >= 8 * 4096, (avail, cap)
        N, K = 4096, 2048
        data = quant_matrix(2000, Q4_K, N, K)
        full = ctx.upload(data, Q4_K, N, K)
        shard = ctx.upload(sharding.row_shard(data, Q4_K, N, K, world, rank), Q4_K, N // world, K)
        for mode in (ctx.GATHER_NCCL, ctx.GATHER_PEER, ctx.GATHER_AUTO):
            ctx.comm_set_gather(mode)
            for B in (1, 3, 8, 2, 5):
                x = torch.from_numpy(activations(2001 + B, B, K)).to(dev)
                y = torch.empty((B, N), dtype=torch.float32, device=dev)
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    ctx.gemv_sharded_dev(shard, x.data_ptr(), y.data_ptr(), B, st.cuda_stream)
                st.synchronize()
                want = ctx.gemv(full, x.cpu().numpy())
                assert np.array_equal(y.cpu().numpy().reshape(B, N).view(np.uint32),
                                      want.reshape(B, N).view(np.uint32)), ("gemv", mode, B)

        # the fused gather captured in a CUDA graph and replayed with new inputs
        # (its exchange half and arrival count live on the device)
        ctx.comm_set_gather(ctx.GATHER_PEER)
        xg = torch.zeros((2, K), dtype=torch.float32, device=dev)
        yg2 = torch.empty((2, N), dtype=torch.float32, device=dev)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            ctx.gemv_sharded_dev(shard, xg.data_ptr(), yg2.data_ptr(), 2, st.cuda_stream)
            ctx.gemv_sharded_dev(shard, xg.data_ptr(), yg2.data_ptr(), 2, st.cuda_stream)
        for rep in range(3):
            xa = activations(2050 + rep, 2, K)
            xg.copy_(torch.from_numpy(xa))
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                graph.replay()
            st.synchronize()
            want = ctx.gemv(full, xa)
            assert np.array_equal(yg2.cpu().numpy().view(np.uint32), want.reshape(2, N).view(np.uint32)), ("graph", rep)
        del graph
        ctx.comm_set_gather(ctx.GATHER_AUTO)

        # several sharded GEMVs in one collective group (one NCCL launch at group_end)
        x1 = torch.from_numpy(activations(2005, 1, K)).to(dev)
        x4 = torch.from_numpy(activations(2006, 4, K)).to(dev)
        y1 = torch.empty((1, N), dtype=torch.float32, device=dev)
        y4 = torch.empty((4, N), dtype=torch.float32, device=dev)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.comm_group_start()
            ctx.gemv_sharded_dev(shard, x1.data_ptr(), y1.data_ptr(), 1, st.cuda_stream)
            ctx.gemv_sharded_dev(shard, x4.data_ptr(), y4.data_ptr(), 4, st.cuda_stream)
            ctx.comm_group_end()
        st.synchronize()
        for xx, yy in ((x1, y1), (x4, y4)):
            want = ctx.gemv(full, xx.cpu().numpy())
            assert np.array_equal(yy.cpu().numpy().view(np.uint32), want.reshape(yy.shape).view(np.uint32)), "group"
        # more grouped calls than one all-gather kernel takes (it flushes midway)
        ys34 = [torch.empty((1, N), dtype=torch.float32, device=dev) for _ in range(34)]
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.comm_group_start()
            for i, yy in enumerate(ys34):
                ctx.gemv_sharded_dev(shard, (x1 if i % 2 else x4).data_ptr(), yy.data_ptr(), 1, st.cuda_stream)
            ctx.comm_group_end()
        st.synchronize()
        w1, w4 = ctx.gemv(full, x1.cpu().numpy()), ctx.gemv(full, x4.cpu().numpy()[:1])
        for i, yy in enumerate(ys34):
            want = w1 if i % 2 else w4
            assert np.array_equal(yy.cpu().numpy().view(np.uint32), want.reshape(1, N).view(np.uint32)), ("group34", i)
        # the same under the NCCL gather: one NCCL group for both calls
        ctx.comm_set_gather(ctx.GATHER_NCCL)
        y1.zero_()
        y4.zero_()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.comm_group_start()
            ctx.gemv_sharded_dev(shard, x1.data_ptr(), y1.data_ptr(), 1, st.cuda_stream)
            ctx.gemv_sharded_dev(shard, x4.data_ptr(), y4.data_ptr(), 4, st.cuda_stream)
            ctx.comm_group_end()
        st.synchronize()
        for xx, yy in ((x1, y1), (x4, y4)):
            want = ctx.gemv(full, xx.cpu().numpy())
            assert np.array_equal(yy.cpu().numpy().view(np.uint32), want.reshape(yy.shape).view(np.uint32)), "nccl group"
        ctx.comm_set_gather(ctx.GATHER_AUTO)

        # row-sharded GEMM (m = 70): the single-GPU GEMM within fp32 reassociation
        Kg, Ng, M = 2048, 1024, 70
        dg = quant_matrix(2010, Q5_K, Ng, Kg)
        fg = ctx.upload(dg, Q5_K, Ng, Kg)
        sgw = ctx.upload(sharding.row_shard(dg, Q5_K, Ng, Kg, world, rank), Q5_K, Ng // world, Kg)
        bits = bf16_bits(activations(2011, M, Kg))
        xb = torch.from_numpy(bits.view(np.int16)).to(dev)
        yg = torch.empty((M, Ng), dtype=torch.float32, device=dev)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.gemm_sharded_dev(sgw, xb.data_ptr(), yg.data_ptr(), M, st.cuda_stream)
        st.synchronize()
        wantg = ctx.gemm_bf16(fg, bits)
        got = yg.cpu().numpy()
        for t in range(M):
            assert rel_err(got[t], wantg[t]) < 1e-5, ("gemm", t)

        # expert-parallel MoE: the all-reduced partials equal the one-GPU layer
        n_embd, E, k, n_ff = 512, 16, 4, 256
        ge = quant_matrix(2020, Q4_K, n_embd, n_ff, E)
        ue = quant_matrix(2021, Q4_K, n_embd, n_ff, E)
        de = quant_matrix(2022, Q4_K, n_ff, n_embd, E)
        sh = {nm: ctx.upload(quant_matrix(2023 + i, Q4_K, r, c), Q4_K, r, c)
              for i, (nm, r, c) in enumerate([("gate_shexp", 256, n_embd), ("up_shexp", 256, n_embd),
                                              ("down_shexp", n_embd, 256), ("gate_inp_shexp", 1, n_embd)])}
        wf = dict(sh, gate_exps=ctx.upload(ge, Q4_K, n_embd, n_ff, n_expert=E),
                  up_exps=ctx.upload(ue, Q4_K, n_embd, n_ff, n_expert=E),
                  down_exps=ctx.upload(de, Q4_K, n_ff, n_embd, n_expert=E))
        lf = ctx.moe_create(wf, n_embd, E, k, n_ff, 256)
        e0, e1 = sharding.expert_range(E, world, rank)
        wr = dict(sh, gate_exps=ctx.upload(sharding.expert_shard(ge, E, world, rank), Q4_K, n_embd, n_ff,
                                           n_expert=e1 - e0),
                  up_exps=ctx.upload(sharding.expert_shard(ue, E, world, rank), Q4_K, n_embd, n_ff, n_expert=e1 - e0),
                  down_exps=ctx.upload(sharding.expert_shard(de, E, world, rank), Q4_K, n_ff, n_embd,
                                       n_expert=e1 - e0))
        lr = ctx.moe_create(wr, n_embd, E, k, n_ff, 256, expert_begin=e0, expert_end=e1, with_shared=(rank == 0))
        T = 9
        x = activations(2030, T, n_embd)
        lg = rng(2031).standard_normal((T, E)).astype(np.float32)
        want_m, _, _ = ctx.moe_ffn(lf, x, lg)
        xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
        od = torch.empty((T, n_embd), dtype=torch.float32, device=dev)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.moe_ffn_ep_dev(lr, xd.data_ptr(), ld.data_ptr(), T, od.data_ptr(), st.cuda_stream)
        st.synchronize()
        got_m = od.cpu().numpy()
        for t in range(T):  # fp32 sums in another order (see test_moe_expert_parallel_partials_sum)
            assert rel_err(got_m[t], want_m[t]) < 1e-3, ("moe", t)
        # the peer all-reduce (rank-ordered sum: the same bits every call) against NCCL's
        again = torch.empty_like(od)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.moe_ffn_ep_dev(lr, xd.data_ptr(), ld.data_ptr(), T, again.data_ptr(), st.cuda_stream)
        st.synchronize()
        assert np.array_equal(again.cpu().numpy().view(np.uint32), got_m.view(np.uint32)), "peer all-reduce repeat"
        ctx.comm_set_gather(ctx.GATHER_NCCL)
        on = torch.empty_like(od)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            ctx.moe_ffn_ep_dev(lr, xd.data_ptr(), ld.data_ptr(), T, on.data_ptr(), st.cuda_stream)
        st.synchronize()
        ctx.comm_set_gather(ctx.GATHER_AUTO)
        got_n = on.cpu().numpy()
        for t in range(T):
            assert rel_err(got_m[t], got_n[t]) < 1e-5, ("peer vs nccl all-reduce", t)
        ctx.close()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _config_worker(rank, world, uid, q):
    """The configuration shapes: row-sharded Q4_K 8192 -> 28672 and 28672 ->
    8192 GEMVs at batch 1 and 8 through the peer gather, their M = 1024 GEMMs
    (against the f64 product, the GEMM's 1e-2 bound), and the 256-expert layer
    (hidden 2048, expert width 512, top 8, shared expert 512) expert-parallel
    at T = 1 and 64 (within 1e-3 of the one-GPU layer).

    A shard's GEMV equals the one-GPU GEMV bit for bit when the shard's row
    count selects the same kernel shape; the consumer-warp count (four or
    eight, from the number of 16-row tiles) and the tall batch-1 kernel follow
    the row count, and a different shape adds the same per-block partial sums
    in another grouping. So the shard is held to 1e-5 of the one-GPU result
    (fp32 regrouping only; the parity bound is 1e-3) and to ops::gemv itself
    on a row range, and to the bits when the shapes agree (world 2 here)."""
    try:
        sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "strata-rs_b200"),
                        os.path.join(os.path.dirname(HERE), "oracle")]
        import torch
        import strata_cuda as sc
        import sharding
        from conftest import rel_err
        from synth import Q4_K, activations, bf16_bits, quant_matrix, rng
        torch.cuda.set_device(rank)
        ctx = sc.Context(rank)
        ctx.set_wait_timeout_ms(60000)
        ctx.comm_init(rank, world, uid)
        ctx.set_wait_timeout_ms(10000)
        st = torch.cuda.Stream()
        dev = f"cuda:{rank}"
        for (K, N) in ((8192, 28672), (28672, 8192)):
            data = quant_matrix(2100 + K, Q4_K, N, K)
            full = ctx.upload(data, Q4_K, N, K)
            shard = ctx.upload(sharding.row_shard(data, Q4_K, N, K, world, rank), Q4_K, N // world, K)
            for B in (1, 8):
                x = torch.from_numpy(activations(2101 + B, B, K)).to(dev)
                y = torch.empty((B, N), dtype=torch.float32, device=dev)
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    ctx.gemv_sharded_dev(shard, x.data_ptr(), y.data_ptr(), B, st.cuda_stream)
                st.synchronize()
                want = ctx.gemv(full, x.cpu().numpy()).reshape(B, N)
                got = y.cpu().numpy()
                assert rel_err(got, want) < 1e-5, ("config gemv", K, N, B, rel_err(got, want))
                if world == 2:
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), ("config gemv bits", K, N, B)
                r0 = (N // world) * rank
                import oracle
                ref = oracle.gemv_rows(Q4_K, data, N, K, x[0].cpu().numpy(), r0, r0 + 256, threads=4)
                assert rel_err(got[0, r0:r0 + 256], ref) < 1e-3, ("config gemv parity", K, N, B)
            M = 1024
            bits = bf16_bits(activations(2102, M, K))
            xb = torch.from_numpy(bits.view(np.int16)).to(dev)
            yg = torch.empty((M, N), dtype=torch.float32, device=dev)
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                ctx.gemm_sharded_dev(shard, xb.data_ptr(), yg.data_ptr(), M, st.cuda_stream)
            st.synchronize()
            # sampled tokens against the f64 product of the oracle's bit-exact
            # dequantized weights with the bf16 activations (the GEMM's 1e-2 bound;
            # the shard and the full matrix take other split-K factors, so the
            # sharded result is not the one-GPU GEMM's bits)
            import oracle
            got = yg.cpu().numpy()
            toks = list(range(0, M, 37))
            Wd = torch.from_numpy(oracle.dequantize(Q4_K, data, N, K)).to(dev).double()
            xr = (bits[toks].astype(np.uint32) << 16).view(np.float32)
            ref = (torch.from_numpy(xr).to(dev).double() @ Wd.T).cpu().numpy()
            del Wd
            worst = max(rel_err(got[t], ref[i]) for i, t in enumerate(toks))
            assert worst < 1e-2, ("config gemm", K, N, worst)
            full.free()
            shard.free()

        n_embd, E, k, n_ff, n_ff_s = 2048, 256, 8, 512, 512
        ge = quant_matrix(2120, Q4_K, n_embd, n_ff, E)
        ue = quant_matrix(2121, Q4_K, n_embd, n_ff, E)
        de = quant_matrix(2122, Q4_K, n_ff, n_embd, E)
        sh = {nm: ctx.upload(quant_matrix(2123 + i, Q4_K, r, c), Q4_K, r, c)
              for i, (nm, r, c) in enumerate([("gate_shexp", n_ff_s, n_embd), ("up_shexp", n_ff_s, n_embd),
                                              ("down_shexp", n_embd, n_ff_s), ("gate_inp_shexp", 1, n_embd)])}
        wf = dict(sh, gate_exps=ctx.upload(ge, Q4_K, n_embd, n_ff, n_expert=E),
                  up_exps=ctx.upload(ue, Q4_K, n_embd, n_ff, n_expert=E),
                  down_exps=ctx.upload(de, Q4_K, n_ff, n_embd, n_expert=E))
        lf = ctx.moe_create(wf, n_embd, E, k, n_ff, n_ff_s)
        e0, e1 = sharding.expert_range(E, world, rank)
        wr = dict(sh, gate_exps=ctx.upload(sharding.expert_shard(ge, E, world, rank), Q4_K, n_embd, n_ff,
                                           n_expert=e1 - e0),
                  up_exps=ctx.upload(sharding.expert_shard(ue, E, world, rank), Q4_K, n_embd, n_ff, n_expert=e1 - e0),
                  down_exps=ctx.upload(sharding.expert_shard(de, E, world, rank), Q4_K, n_ff, n_embd,
                                       n_expert=e1 - e0))
        lr = ctx.moe_create(wr, n_embd, E, k, n_ff, n_ff_s, expert_begin=e0, expert_end=e1, with_shared=(rank == 0))
        for T in (1, 64):
            x = activations(2130 + T, T, n_embd)
            lg = rng(2131 + T).standard_normal((T, E)).astype(np.float32)
            want_m, _, _ = ctx.moe_ffn(lf, x, lg)
            xd, ld = torch.from_numpy(x).to(dev), torch.from_numpy(lg).to(dev)
            od = torch.empty((T, n_embd), dtype=torch.float32, device=dev)
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                ctx.moe_ffn_ep_dev(lr, xd.data_ptr(), ld.data_ptr(), T, od.data_ptr(), st.cuda_stream)
            st.synchronize()
            got_m = od.cpu().numpy()
            for t in range(T):
                assert rel_err(got_m[t], want_m[t]) < 1e-3, ("config moe", T, t)
        ctx.close()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _peer_timeout_worker(rank, world, uid, q, bar):
    """Rank 1 skips a sharded GEMV: rank 0's wait for its arrivals expires
    (bounded), the call reports STRATA_ERR_TIMEOUT and the context stays
    usable; the ranks then meet on the host and close normally."""
    try:
        sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), "strata-rs_b200"),
                        os.path.join(os.path.dirname(HERE), "oracle")]
        import torch
        import strata_cuda as sc
        import sharding
        from synth import Q4_K, activations, quant_matrix
        torch.cuda.set_device(rank)
        ctx = sc.Context(rank)
        ctx.set_wait_timeout_ms(60000)
        ctx.comm_init(rank, world, uid)
        ctx.comm_set_gather(ctx.GATHER_PEER)
        N, K = 1024, 512
        data = quant_matrix(2060, Q4_K, N, K)
        shard = ctx.upload(sharding.row_shard(data, Q4_K, N, K, world, rank), Q4_K, N // world, K)
        if rank == 0:
            ctx.set_wait_timeout_ms(1000)
            st = torch.cuda.Stream()
            x = torch.from_numpy(activations(2061, 1, K)).to(f"cuda:{rank}")
            y = torch.empty((1, N), dtype=torch.float32, device=f"cuda:{rank}")
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                ctx.gemv_sharded_dev(shard, x.data_ptr(), y.data_ptr(), 1, st.cuda_stream)
            st.synchronize()
            try:
                ctx.synchronize()
                raise AssertionError("no timeout reported")
            except sc.BackendError as e:
                assert e.code == sc.ERR_TIMEOUT, e
            w = ctx.upload(data, Q4_K, N, K)
            assert np.isfinite(ctx.gemv(w, activations(2062, 1, K))).all()
            ctx.set_wait_timeout_ms(60000)
        bar.wait(timeout=300)
        ctx.close()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run_world(world, target=None, worker=None):
    uid = sc.comm_unique_id()
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    if target is None:
        procs = [ctxm.Process(target=worker or _worker, args=(r, world, uid, q)) for r in range(world)]
    else:
        bar = ctxm.Barrier(world)
        procs = [ctxm.Process(target=target, args=(r, world, uid, q, bar)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, msg = q.get(timeout=600)
        res[r] = msg
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_sharded_paths_world2():
    res = _run_world(2)
    assert all(m == "ok" for m in res.values()), res


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_peer_gather_times_out_when_a_rank_skips_the_call():
    res = _run_world(2, _peer_timeout_worker)
    assert all(m == "ok" for m in res.values()), res


@pytest.mark.skipif(_ngpu() < 4, reason="needs 4 GPUs")
def test_sharded_paths_world4():
    res = _run_world(4)
    assert all(m == "ok" for m in res.values()), res


@pytest.mark.skipif(_ngpu() < 8, reason="needs 8 GPUs")
def test_sharded_paths_world8():
    res = _run_world(8)
    assert all(m == "ok" for m in res.values()), res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config_shapes_sharded(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run_world(world, worker=_config_worker)
    assert all(m == "ok" for m in res.values()), res


def test_comm_init_times_out_when_a_rank_never_joins():
    ctx = sc.Context(0)
    ctx.set_wait_timeout_ms(3000)
    with pytest.raises(sc.BackendError) as e:
        ctx.comm_init(0, 2, sc.comm_unique_id())
    assert e.value.code in (sc.ERR_TIMEOUT, sc.ERR_NCCL)
    # the context is still usable afterwards
    from synth import Q4_K, activations, quant_matrix
    w = ctx.upload(quant_matrix(2040, Q4_K, 64, 256), Q4_K, 64, 256)
    assert np.isfinite(ctx.gemv(w, activations(2041, 1, 256))).all()
    w.free()
    ctx.close()
