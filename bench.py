#!/usr/bin/env python
"""Benchmark: Q4_K decode GEMV sweep on B200 (the reference's headline path).

Workload (the "Q4_K decode GEMV sweep" configuration): Q4_K weights of shapes
(K -> N) 4096->4096, 4096->12288, 12288->4096 and 2048->151936, activations
f32 N(0,1) at batch 1, 2, 4 and 8. One step = one pass over all 16
(shape, batch) GEMVs, batch-major, so no matrix is re-read before the ~241 MB
of the other matrices have streamed through L2 (126 MB). Each step also uses
its own copy of every matrix (copies rotated so each set exceeds 4x L2), so
every launch reads its weights from HBM.

value     = algorithmic bytes of all GEMVs (weights once + activations + outputs)
            / device time of the K timed steps (CUDA events on the launch stream,
            max over ranks), GB/s.
e2e       = the same metric through the public host-buffer C ABI call
            (strata_cuda_gemv: pinned host copy in, kernel, result copied out,
            bounded wait), timed on the host clock.
roofline  = that kernel against the measured HBM copy bandwidth.
cpu_baseline = the CPU oracle (the C restatement of ops::gemv, all host
            threads, row-parallel) on the same sweep.

The same line carries the other measured rows of the path:
  gemm      the mixed K-quant prefill configuration (Q5_K, Q6_K; K4096->N12288
            and K12288->N4096; M = 64, 512, 2048 bf16 tokens) on the tcgen05
            GEMM: TFLOP/s (2MNK per launch) against the measured bf16 peak;
  moe       the MoE FFN configuration (hidden 2048, 256 Q4_K experts of width
            512, top-8 from N(0,1) logits, shared expert) at 1 and 64 tokens:
            tokens/s, expert-parallel across the ranks;
  sharded   the large row-sharded projections (Q4_K 8192->28672, 28672->8192)
            as a batch-1 GEMV and an M=1024 GEMM, rows split across the ranks.

`--impl reference` times only the reference path on the CPU (the oracle port;
the Rust reference cannot be built on this image) and prints its own line.
Multi-GPU (torchrun): every projection is row-sharded across the ranks and
assembled by the library's all-gather (strata_cuda_gemv_sharded_dev: local
GEMV + NCCL all-gather inside the C ABI call), MoE is expert-parallel with
the library's all-reduce (strong scaling: the same total work at every N).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "strata-rs_b200"
sys.path.insert(0, str(PKG))

from synth import (Q4K_SWEEP, SWEEP_BATCHES, Q4_K, Q5_K, Q6_K, Q8_0, activations, bf16_bits,  # noqa: E402
                   quant_matrix, rng)
import sharding  # noqa: E402

METRIC = "Q4_K GEMV GB/s (% of HBM peak); MoE layer tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"


DTYPE = ("f32 activations (split into two fp16 limbs, 22 significant bits, with a power-of-two scale per "
         "256-block), Q4_K weights, fp32 accumulate")


def sweep_config(world: int) -> dict:
    """The workload keys both arms print (the reference arm and this one)."""
    return {"workload": "Q4_K decode GEMV sweep: K->N 4096->4096, 4096->12288, 12288->4096, 2048->151936 at "
                        "batch 1,2,4,8 (16 GEMVs per step, batch-major)",
            "l2": "inputs larger than L2: per step 964 MB of weights, rotated weight copies (>= 4x L2 per "
                  "matrix), no matrix re-read within 241 MB of traffic",
            "parallelism": "single GPU" if world == 1 else f"row-sharded x{world}: output rows split across "
                                                           f"ranks, gathered after every GEMV"}


def gemv_bytes(k: int, n: int, b: int) -> int:
    return n * (k // 256) * 144 + b * k * 4 + b * n * 4


def sweep_bytes(shapes, batches) -> int:
    return sum(gemv_bytes(k, n, b) for b in batches for (k, n) in shapes)


def profiled_traffic():
    """DRAM bytes per GEMV launch from the committed ncu summary
    (profiles/gemv_q4k_sweep_dram.md), or None when it is absent."""
    p = ROOT / "profiles" / "gemv_q4k_sweep_dram.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":")[1])
    return None


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Measured dense bf16 TFLOP/s (burst: each GEMM case is timed alone)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback (burst)"


def timed(torch, stream, fn, reps: int, warm: int = 3) -> float:
    """Average ms of fn() over reps launches on `stream` (CUDA events)."""
    with torch.cuda.stream(stream):
        for _ in range(warm):
            fn()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(reps):
            fn()
        a1.record(stream)
    a1.synchronize()
    return a0.elapsed_time(a1) / reps


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 100 ms while running."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(device), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU (oracle port)

class CpuSweep:
    """The CPU restatement of ops::gemv (oracle/, the checker, used here only as
    the CPU baseline) over the sweep, or a row sample of it sized to a time budget.
    Every (shape, batch) is one ops::gemv per activation column, as the
    reference's batch-1 trait does; rows are split across `threads` pthreads."""

    def __init__(self, shapes, batches, threads: int):
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle
        self.oracle = oracle
        self.shapes, self.batches, self.threads = shapes, batches, threads
        self.mats = {(k, n): quant_matrix(k + n, Q4_K, n, k) for (k, n) in shapes}
        self.xs = {b: activations(900 + b, b, max(k for k, _ in shapes)) for b in batches}
        k0, n0 = max(shapes, key=lambda s: s[0] * s[1])
        probe = max(threads * 16, 256)
        oracle.gemv_rows(Q4_K, self.mats[(k0, n0)], n0, k0, self.xs[1][0, :k0], 0, probe, threads)
        t = time.perf_counter()
        oracle.gemv_rows(Q4_K, self.mats[(k0, n0)], n0, k0, self.xs[1][0, :k0], 0, probe, threads)
        self.elem_rate = probe * k0 / max(time.perf_counter() - t, 1e-6)

    def run(self, budget_s: float):
        total_elems = sum(n * k * b for b in self.batches for (k, n) in self.shapes)
        frac = min(1.0, budget_s * self.elem_rate / total_elems)
        nbytes = 0
        t = time.perf_counter()
        for b in self.batches:
            for (k, n) in self.shapes:
                rows = max(1, int(n * frac))
                for j in range(b):
                    self.oracle.gemv_rows(Q4_K, self.mats[(k, n)], n, k, self.xs[b][j, :k], 0, rows, self.threads)
                nbytes += rows * (k // 256) * 144 + b * k * 4 + b * rows * 4
        dt = time.perf_counter() - t
        desc = (f"Q4_K sweep ({len(self.shapes)} shapes x batches {self.batches}), first {frac:.2%} of each "
                f"matrix's rows per step, one ops::gemv per activation column, {self.threads} threads")
        return nbytes / dt / 1e9, desc, dt


def serial_baseline(shapes, batches) -> dict:
    """The same sweep on one thread, as the reference runs ops::gemv (it is
    single-threaded): a bounded 3 s sample beside the all-cores figure."""
    v, desc, _ = CpuSweep(shapes, batches, 1).run(3.0)
    return {"value": round(v, 3), "unit": UNIT, "cores": 1, "sample": desc}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    shapes, batches = Q4K_SWEEP, SWEEP_BATCHES
    cpu = CpuSweep(shapes, batches, threads)
    per_step = max(0.02, 120.0 / max(1, args.steps + args.warmup))
    vals = []
    desc = ""
    for i in range(args.warmup + args.steps):
        v, desc, _ = cpu.run(per_step)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    total = sweep_bytes(shapes, batches)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / (value * 1e9) * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (f64 accumulate)", "data": "synthetic",
        "config": sweep_config(args.gpus), "path": "reference CPU path (oracle port of ops::gemv)",
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc, "single_thread": serial_baseline(shapes, batches)},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU

GEMM_SHAPES = [(4096, 12288), (12288, 4096)]   # (K, N)
GEMM_MS = [64, 512, 2048]


def bench_gemm(ctx, torch, stream, l2: int, world: int, rank: int, dist) -> dict:
    """The prefill GEMM configuration: per case TFLOP/s = 2MNK / launch time.
    Weights rotate over copies (>= 4x L2 per case) so the M=64 (HBM-bound)
    cases stream from HBM; at N > 1 the rows are sharded and gathered by the
    library (strata_cuda_gemm_sharded_dev)."""
    peak, peak_kind = tensor_peak()
    hbm, _ = peaks()
    cases = []
    xbits = {k: torch.from_numpy(bf16_bits(activations(77 + k, max(GEMM_MS), k)).view(np.int16)).cuda()
             for k, _ in GEMM_SHAPES}
    for q, qn, bb in ((Q5_K, "Q5_K", 176), (Q6_K, "Q6_K", 210)):
        for k, n in GEMM_SHAPES:
            full = quant_matrix(500 + k + q, q, n, k)
            part = sharding.row_shard(full, q, n, k, world, rank) if world > 1 else full
            copies = max(1, -(-4 * l2 // part.nbytes))
            ws = [ctx.upload(part, q, n // world, k) for _ in range(copies)]
            for m in GEMM_MS:
                y = torch.empty((m, n), dtype=torch.float32, device="cuda")
                it = [0]

                def fn():
                    w = ws[it[0] % len(ws)]
                    it[0] += 1
                    if world > 1:
                        ctx.gemm_sharded_dev(w, xbits[k].data_ptr(), y.data_ptr(), m, stream.cuda_stream)
                    else:
                        ctx.gemm_bf16_dev(w, xbits[k].data_ptr(), y.data_ptr(), m, stream.cuda_stream)
                reps = max(len(ws), {64: 60, 512: 30, 2048: 10}[m])
                ms = timed(torch, stream, fn, reps)
                if dist:
                    t = torch.tensor([ms], device="cuda")
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    ms = float(t.item())
                tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
                wbytes = n * (k // 256) * bb
                gbs = (wbytes + m * k * 2 + m * n * 4) / (ms * 1e-3) / 1e9
                cases.append({"quant": qn, "k": k, "n": n, "m": m, "us": round(ms * 1e3, 1),
                              "tflops": round(tf, 1), "frac_bf16_peak": round(tf / peak, 3),
                              "tensor_tflops_issued": round(2 * tf, 1),
                              "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3)})
            for w in ws:
                w.free()
    big = [c for c in cases if c["m"] >= 512]
    return {"cases": cases, "peak_tflops": peak, "peak_kind": peak_kind,
            "tflops_m512_2048_mean": round(statistics.mean(c["tflops"] for c in big), 1),
            "note": "2MNK per launch over the launch time (CUDA events, 10-60 launches on rotated weight copies); "
                    "the weights are staged as two bf16 terms (hi + residual), so the tensor cores issue "
                    "2x these FLOPs (tensor_tflops_issued); M = 64 is HBM-bound and reported as GB/s too"}


MOE_DIMS = dict(n_embd=2048, E=256, k=8, n_ff=512, n_ff_s=512)


def bench_moe(ctx, torch, stream, world: int, rank: int, dist, with_e2e: bool) -> dict:
    """The MoE FFN configuration at 1 and 64 tokens (strata_cuda_moe_ffn_dev;
    expert-parallel over the ranks with strata_cuda_moe_ffn_ep_dev). Each
    layer call reads its weights from HBM: the layer is replicated over
    enough copies to exceed 4x L2 and rotated."""
    d = MOE_DIMS
    e0, e1 = sharding.expert_range(d["E"], world, rank)
    ge = quant_matrix(1200 + 1, Q4_K, d["n_embd"], d["n_ff"], d["E"])
    ue = quant_matrix(1200 + 2, Q4_K, d["n_embd"], d["n_ff"], d["E"])
    de = quant_matrix(1200 + 3, Q4_K, d["n_ff"], d["n_embd"], d["E"])
    shared = {"gate_shexp": quant_matrix(1200 + 4, Q4_K, d["n_ff_s"], d["n_embd"]),
              "up_shexp": quant_matrix(1200 + 5, Q4_K, d["n_ff_s"], d["n_embd"]),
              "down_shexp": quant_matrix(1200 + 6, Q4_K, d["n_embd"], d["n_ff_s"]),
              "gate_inp_shexp": quant_matrix(1200 + 7, Q4_K, 1, d["n_embd"])}
    held = e1 - e0
    layer_bytes = 3 * held * d["n_embd"] * d["n_ff"] // 256 * 144 + sum(v.nbytes for v in shared.values())
    copies = max(1, -(-4 * 126 * 2**20 // layer_bytes))
    layers, handles = [], []
    for _ in range(copies):
        ws = {"gate_exps": ctx.upload(sharding.expert_shard(ge, d["E"], world, rank), Q4_K, d["n_embd"], d["n_ff"],
                                      n_expert=held),
              "up_exps": ctx.upload(sharding.expert_shard(ue, d["E"], world, rank), Q4_K, d["n_embd"], d["n_ff"],
                                    n_expert=held),
              "down_exps": ctx.upload(sharding.expert_shard(de, d["E"], world, rank), Q4_K, d["n_ff"], d["n_embd"],
                                      n_expert=held)}
        for nm, arr in shared.items():
            r, c = {"gate_shexp": (d["n_ff_s"], d["n_embd"]), "up_shexp": (d["n_ff_s"], d["n_embd"]),
                    "down_shexp": (d["n_embd"], d["n_ff_s"]), "gate_inp_shexp": (1, d["n_embd"])}[nm]
            ws[nm] = ctx.upload(arr, Q4_K, r, c)
        handles.append(ws)
        layers.append(ctx.moe_create(ws, d["n_embd"], d["E"], d["k"], d["n_ff"], d["n_ff_s"], expert_begin=e0,
                                     expert_end=e1, with_shared=(rank == 0)))
    out = {}
    R = 16  # routings rotated with the layer copies, so one token's experts are not L2-resident
    for T in (1, 64):
        x = torch.from_numpy(activations(1201 + T, T, d["n_embd"])).cuda()
        lg_np = [rng(1202 + 100 * T + r).standard_normal((T, d["E"])).astype(np.float32) for r in range(R)]
        lgs = [torch.from_numpy(a).cuda() for a in lg_np]
        y = torch.empty((T, d["n_embd"]), dtype=torch.float32, device="cuda")
        it = [0]

        def call(i):
            L, lg = layers[i % len(layers)], lgs[i % R]
            if world > 1:
                ctx.moe_ffn_ep_dev(L, x.data_ptr(), lg.data_ptr(), T, y.data_ptr(), stream.cuda_stream)
            else:
                ctx.moe_ffn_dev(L, x.data_ptr(), lg.data_ptr(), T, y.data_ptr(), stream=stream.cuda_stream)

        def fn():
            call(it[0])
            it[0] += 1
        graph_us = None
        # launch-bound at one token: also the layer replayed from a CUDA graph
        # (N > 1: every rank captures, and replays only if every rank could)
        with torch.cuda.stream(stream):
            call(0)
        stream.synchronize()
        n_cap = R * len(layers)
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g, stream=stream):
                for i in range(n_cap):
                    call(i)
            captured = 1
        except Exception as exc:  # noqa: BLE001 - stream timing only
            print(f"moe graph capture unavailable ({exc})", file=sys.stderr)
            captured = 0
        if dist:
            ok = torch.tensor([captured], device="cuda")
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            captured = int(ok.item())
        if captured:
            gms = timed(torch, stream, g.replay, 5) / n_cap
            if dist:
                t = torch.tensor([gms], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                gms = float(t.item())
            graph_us = round(gms * 1e3, 2)
        del g
        torch.cuda.synchronize()
        ms = timed(torch, stream, fn, max(R * len(layers), 48))
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        best_ms = min(ms, graph_us / 1e3) if graph_us else ms
        # bytes: the distinct experts each routing touches (x3 tensors) + the shared expert
        distinct = statistics.mean(len(np.unique(np.argsort(-a, axis=1)[:, :d["k"]])) for a in lg_np)
        wbytes = int(distinct * 3 * d["n_embd"] * d["n_ff"] // 256 * 144 + sum(v.nbytes for v in shared.values()))
        rec = {"tokens": T, "us_per_layer": round(best_ms * 1e3, 2), "us_per_layer_stream": round(ms * 1e3, 2),
               "us_per_layer_graph": graph_us, "tokens_per_s": round(T / (best_ms * 1e-3), 1),
               "distinct_experts": distinct, "weight_bytes": wbytes,
               "gbs": round(wbytes / (best_ms * 1e-3) / 1e9, 1)}
        if with_e2e and world == 1:
            import ctypes as C
            import strata_cuda as sc
            lib = sc.lib()
            hx = activations(1201 + T, T, d["n_embd"])
            lgc = [np.ascontiguousarray(v, dtype=np.float32) for v in lg_np]
            ho = np.empty((T, d["n_embd"]), np.float32)
            hids = np.empty((T, d["k"]), np.int32)
            hw = np.empty((T, d["k"]), np.float32)
            # the caller's buffers are fixed: their addresses are marshalled once (as
            # a compiled caller passes raw pointers); every call stages them through
            # the library inside the timed region
            fp = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
            px, po, pw = fp(hx), fp(ho), fp(hw)
            pids = hids.ctypes.data_as(C.POINTER(C.c_int32))
            plg = [fp(v) for v in lgc]

            def host_call(i):
                rc = lib.strata_cuda_moe_ffn(ctx.h, layers[i % len(layers)].handle, px, plg[i % R], T, po, pids, pw)
                if rc:
                    ctx.check(rc)
            for i in range(3):
                host_call(i)
            n_e = 64
            t0 = time.perf_counter()
            for i in range(n_e):
                host_call(i)
            dt = (time.perf_counter() - t0) / n_e
            rec["e2e"] = {"tokens_per_s": round(T / dt, 1), "us_per_layer": round(dt * 1e6, 1),
                          "h2d_bytes_per_step": hx.nbytes + lg_np[0].nbytes,
                          "d2h_bytes_per_step": T * d["n_embd"] * 4 + 2 * T * d["k"] * 4,
                          "timer": "host perf_counter around strata_cuda_moe_ffn (ctypes; the caller's buffer "
                                   "addresses marshalled once)"}
        out[f"T{T}"] = rec
    for L in layers:
        L.free()
    for ws in handles:
        for w in ws.values():
            w.free()
    return out


SHARDED_SHAPES = [(8192, 28672), (28672, 8192)]  # (K, N), Q4_K


def bench_q8_0(ctx, torch, stream, with_cpu: bool) -> dict:
    """The Q8_0 configuration: one 4096x4096 Q8_0 matrix (fp16 d ~ U(0.002, 0.02),
    int8 quants in [-127, 127]), f32 activation, batch 1, on rotated copies so
    every launch reads HBM; the CPU port of ops::gemv on the same matrix beside it."""
    k = n = 4096
    data = quant_matrix(8080, Q8_0, n, k)
    ws = [ctx.upload(data, Q8_0, n, k) for _ in range(max(1, -(-4 * 126 * 2**20 // data.nbytes)))]
    x = torch.from_numpy(activations(8081, 1, k)).cuda()
    y = torch.empty((1, n), dtype=torch.float32, device="cuda")
    it = [0]

    def fn():
        w = ws[it[0] % len(ws)]
        it[0] += 1
        ctx.gemv_dev(w, x.data_ptr(), y.data_ptr(), 1, stream.cuda_stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(len(ws)):
            fn()
    ms = timed(torch, stream, g.replay, 20) / len(ws)
    nbytes = data.nbytes + k * 4 + n * 4
    hbm, peak_kind = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    out = {"k": k, "n": n, "batch": 1, "us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
           "algorithmic_bytes": nbytes, "kernel": "q8::gemv_q8_0_bulk_kernel (CUDA cores, rows staged by bulk copies into a 4-stage shared-memory ring)"}
    if with_cpu:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle
        xv = activations(8081, 1, k)[0]
        for threads in (1, os.cpu_count() or 1):
            oracle.gemv_rows(Q8_0, data, n, k, xv, 0, 64, threads)
            reps, t = 0, time.perf_counter()
            while time.perf_counter() - t < 2.0:
                oracle.gemv_rows(Q8_0, data, n, k, xv, 0, n, threads)
                reps += 1
            dt = (time.perf_counter() - t) / reps
            out["cpu_threads_%d" % threads] = {"gbs": round(nbytes / dt / 1e9, 3), "cores": threads,
                                               "sample": "the whole matrix, ops::gemv port (oracle)"}
    for w in ws:
        w.free()
    return out


def bench_sharded(ctx, torch, stream, world: int, rank: int, dist) -> dict:
    """The large row-sharded projections: Q4_K batch-1 GEMV (GB/s of the whole
    weight) and M=1024 GEMM (TFLOP/s), rows split over the ranks and gathered
    by the library (one GPU: the unsharded call)."""
    out = []
    for k, n in SHARDED_SHAPES:
        full = quant_matrix(700 + k, Q4_K, n, k)
        part = sharding.row_shard(full, Q4_K, n, k, world, rank)
        ws = [ctx.upload(part, Q4_K, n // world, k) for _ in range(max(1, -(-4 * 126 * 2**20 // part.nbytes)))]
        x = torch.from_numpy(activations(701, 1, k)).cuda()
        y = torch.empty((1, n), dtype=torch.float32, device="cuda")
        xb = torch.from_numpy(bf16_bits(activations(702, 1024, k)).view(np.int16)).cuda()
        yb = torch.empty((1024, n), dtype=torch.float32, device="cuda")
        it = [0]

        def gemv():
            w = ws[it[0] % len(ws)]
            it[0] += 1
            if world > 1:
                ctx.gemv_sharded_dev(w, x.data_ptr(), y.data_ptr(), 1, stream.cuda_stream)
            else:
                ctx.gemv_dev(w, x.data_ptr(), y.data_ptr(), 1, stream.cuda_stream)

        def gemm():
            w = ws[it[0] % len(ws)]
            it[0] += 1
            if world > 1:
                ctx.gemm_sharded_dev(w, xb.data_ptr(), yb.data_ptr(), 1024, stream.cuda_stream)
            else:
                ctx.gemm_bf16_dev(w, xb.data_ptr(), yb.data_ptr(), 1024, stream.cuda_stream)
        res = {}
        for nm, fn, reps in (("gemv_b1", gemv, 100), ("gemm_m1024", gemm, 10)):
            ms = timed(torch, stream, fn, max(reps, len(ws)))
            if dist:
                t = torch.tensor([ms], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            res[nm] = ms
        wbytes = n * (k // 256) * 144
        out.append({"k": k, "n": n, "gemv_b1_us": round(res["gemv_b1"] * 1e3, 2),
                    "gemv_b1_gbs": round((wbytes + k * 4 + n * 4) / (res["gemv_b1"] * 1e-3) / 1e9, 1),
                    "gemm_m1024_us": round(res["gemm_m1024"] * 1e3, 1),
                    "gemm_m1024_tflops": round(2.0 * 1024 * n * k / (res["gemm_m1024"] * 1e-3) / 1e12, 1)})
        for w in ws:
            w.free()
    return {"cases": out, "parallelism": f"rows x{world}, library all-gather" if world > 1 else "single GPU"}


def run_gpu(args):
    import torch
    import strata_cuda as sc

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    shapes, batches = Q4K_SWEEP, SWEEP_BATCHES
    ctx = sc.Context(local)
    if world > 1:
        # the library's own communicator: rank 0's NCCL id reaches the others over torch.distributed
        uid = [sc.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.comm_init(rank, world, uid[0])
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    stream = torch.cuda.Stream()

    # this rank's row shard of every matrix, uploaded `copies` times
    weights, shard = {}, {}
    for (k, n) in shapes:
        r0, r1 = sharding.row_range(n, world, rank)
        full = quant_matrix(k + n, Q4_K, n, k)
        part = sharding.row_shard(full, Q4_K, n, k, world, rank)
        copies = max(1, -(-4 * l2 // max(part.nbytes, 1)))
        weights[(k, n)] = [ctx.upload(part, Q4_K, r1 - r0, k) for _ in range(copies)]
        shard[(k, n)] = (r0, r1)
    rot = max(len(v) for v in weights.values())
    xs = {b: torch.from_numpy(activations(900 + b, b, max(k for k, _ in shapes))).cuda() for b in batches}
    xk = {(b, k): xs[b][:, :k].contiguous() for b in batches for (k, _) in shapes}
    # single GPU: each GEMV writes its whole output; N GPUs: the library gathers every rank's rows
    ys = {(k, n, b): torch.empty(b, n, device="cuda") for (k, n) in shapes for b in batches}

    def enqueue(step_idx: int, s: int):
        if world > 1:  # the step's 16 gathers go out as one NCCL group
            ctx.comm_group_start()
        for b in batches:
            for (k, n) in shapes:
                w = weights[(k, n)][step_idx % len(weights[(k, n)])]
                if world > 1:
                    ctx.gemv_sharded_dev(w, xk[(b, k)].data_ptr(), ys[(k, n, b)].data_ptr(), b, s)
                else:
                    ctx.gemv_dev(w, xk[(b, k)].data_ptr(), ys[(k, n, b)].data_ptr(), b, s)
        if world > 1:
            ctx.comm_group_end()

    def capture():
        graphs = []
        with torch.cuda.stream(stream):
            enqueue(0, stream.cuda_stream)  # warm the kernels before capture
        stream.synchronize()
        try:  # N > 1: the library's gathers (peer kernels or NCCL group) are captured with the GEMVs
            for i in range(rot):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    enqueue(i, stream.cuda_stream)
                graphs.append(g)
            g = None  # the list holds the graphs (released before the communicator)
            captured = 1
        except Exception as exc:  # noqa: BLE001 - fall back to direct launches on every rank
            print(f"graph capture unavailable ({exc}); launching directly", file=sys.stderr)
            graphs = []
            captured = 0
        if dist:
            ok = torch.tensor([captured], device="cuda")
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if int(ok.item()) == 0:
                graphs = []
        torch.cuda.synchronize()
        return graphs

    peer = False
    if world > 1:
        peer = ctx.comm_peer_info()[0]
        ctx.comm_set_gather(ctx.GATHER_AUTO)  # peer gather fused into the GEMV where available
    graphs = capture()
    # every GEMV is two launches: the activation-limb prologue and the GEMV kernel;
    # with the peer gather one all-gather kernel per step (the step is one
    # collective group; the NCCL group's kernel of the NCCL gather is not counted)
    launches_per_step = 2 * len(batches) * len(shapes) + (1 if peer else 0)

    def step(i):
        if graphs:
            graphs[i % rot].replay()
        else:
            enqueue(i, stream.cuda_stream)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    t_clock0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    # keep the same load on for >= 1.5 s so the clock record covers it
    with torch.cuda.stream(stream):
        i = 0
        while time.perf_counter() - t_clock0 < 1.5:
            for _ in range(50):
                step(i)
                i += 1
            stream.synchronize()
    clk = clocks.stop()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    torch.cuda.synchronize()

    total = sweep_bytes(shapes, batches)
    value = total * args.steps / (ms / 1e3) / 1e9
    hbm, peak_kind = peaks()

    # N > 1: the same step with the NCCL all-gathers instead of the fused peer gather
    alt = None
    if world > 1 and peer:
        ctx.comm_set_gather(ctx.GATHER_NCCL)
        ngraphs = capture()

        def nstep(i):
            if ngraphs:
                ngraphs[i % rot].replay()
            else:
                enqueue(i, stream.cuda_stream)
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                nstep(i)
        stream.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for i in range(args.steps):
                nstep(i)
            a1.record(stream)
        a1.synchronize()
        t = torch.tensor([a0.elapsed_time(a1)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nms = float(t.item())
        alt = {"gather": "NCCL in-place all-gathers, the step's 16 in one NCCL group",
               "ms_per_step": round(nms / args.steps, 4), "value": round(total * args.steps / (nms / 1e3) / 1e9, 1),
               "unit": UNIT}
        del ngraphs
        torch.cuda.synchronize()
        ctx.comm_set_gather(ctx.GATHER_AUTO)

    # per-case device time: each case as its own graph over its rotated copies
    cases = []
    if not args.quick and world == 1:
        for b in batches:
            for (k, n) in shapes:
                ws = weights[(k, n)]
                reps = max(1, 64 // len(ws))
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for _ in range(reps):
                        for w in ws:
                            ctx.gemv_dev(w, xk[(b, k)].data_ptr(), ys[(k, n, b)].data_ptr(), b, stream.cuda_stream)
                with torch.cuda.stream(stream):
                    g.replay()
                    a0 = torch.cuda.Event(enable_timing=True)
                    a1 = torch.cuda.Event(enable_timing=True)
                    a0.record(stream)
                    for _ in range(5):
                        g.replay()
                    a1.record(stream)
                a1.synchronize()
                us = a0.elapsed_time(a1) * 1e3 / (5 * reps * len(ws))
                r0, r1 = shard[(k, n)]
                gb = gemv_bytes(k, r1 - r0, b) / (us * 1e-6) / 1e9
                cases.append({"k": k, "n": n, "batch": b, "us": round(us, 2), "gbs": round(gb, 1),
                              "frac_hbm": round(gb / hbm, 3)})
                del g

    # end to end through the host-buffer C ABI (pinned host input, result read back)
    e2e = None
    if not args.no_e2e and world == 1:
        # the caller's own (pageable) buffers, as a real caller's would be
        hx = {b: activations(900 + b, b, max(k for k, _ in shapes)) for b in batches}
        hxk = {(b, k): np.ascontiguousarray(hx[b][:, :k]) for b in batches for (k, _) in shapes}
        hy = {(k, n, b): np.empty((b, n), np.float32) for (k, n) in shapes for b in batches}
        lib = sc.lib()
        import ctypes as C
        # the caller's buffers are fixed, so their addresses are marshalled once (as
        # a compiled caller passes raw pointers); every call still stages x in and
        # y out through the library inside the timed region
        xp = {key: v.ctypes.data_as(C.POINTER(C.c_float)) for key, v in hxk.items()}
        yp = {key: v.ctypes.data_as(C.POINTER(C.c_float)) for key, v in hy.items()}
        calls = [(b, (k, n), xp[(b, k)], yp[(k, n, b)]) for b in batches for (k, n) in shapes]

        def host_step(i):
            for b, kn, x, y in calls:
                w = weights[kn][i % len(weights[kn])]
                rc = lib.strata_cuda_gemv(ctx.h, w.handle, x, y, b)
                if rc:
                    ctx.check(rc)
        for i in range(3):
            host_step(i)
        n_e2e = max(10, min(args.steps, 200))
        t = time.perf_counter()
        for i in range(n_e2e):
            host_step(i)
        dt = time.perf_counter() - t
        h2d = sum(b * k * 4 for b in batches for (k, _) in shapes)
        d2h = sum(b * n * 4 for b in batches for (_, n) in shapes)
        e2e = {"value": round(total * n_e2e / dt / 1e9, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n_e2e,
               "timer": "host perf_counter around strata_cuda_gemv (ctypes; the caller's buffer addresses marshalled once)"}

    if not args.no_e2e and world > 1:
        # N GPUs: the sharded C ABI call with the step's inputs copied in from pinned
        # host memory and every output copied back, all inside the timed region
        hx = {key: v.cpu().pin_memory() for key, v in xk.items()}
        hy = {key: torch.empty(v.shape, dtype=v.dtype).pin_memory() for key, v in ys.items()}

        def e2e_step(i):
            for b in batches:
                for (k, n) in shapes:
                    xk[(b, k)].copy_(hx[(b, k)], non_blocking=True)
                    w = weights[(k, n)][i % len(weights[(k, n)])]
                    ctx.gemv_sharded_dev(w, xk[(b, k)].data_ptr(), ys[(k, n, b)].data_ptr(), b, stream.cuda_stream)
                    hy[(k, n, b)].copy_(ys[(k, n, b)], non_blocking=True)
        n_e2e = max(10, min(args.steps, 200))
        ms_e = timed(torch, stream, lambda: e2e_step(0), 3, warm=2)  # warm
        with torch.cuda.stream(stream):
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for i in range(n_e2e):
                e2e_step(i)
            a1.record(stream)
        a1.synchronize()
        ms_e = a0.elapsed_time(a1)
        t = torch.tensor([ms_e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e = float(t.item())
        h2d = sum(b * k * 4 for b in batches for (k, _) in shapes)
        d2h = sum(b * n * 4 for b in batches for (_, n) in shapes)
        e2e = {"value": round(total * n_e2e / (ms_e / 1e3) / 1e9, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n_e2e,
               "timer": "CUDA events around pinned H2D + strata_cuda_gemv_sharded_dev + D2H, max over ranks"}

    # the other rows of the path (every rank takes part: their collectives run in the same order)
    gemm = moe = sharded_proj = q8 = None
    if not args.skip_sections and world == 1:
        q8 = bench_q8_0(ctx, torch, stream, with_cpu=not args.no_cpu)
    if not args.skip_sections:
        gemm = bench_gemm(ctx, torch, stream, l2, world, rank, dist)
        moe = bench_moe(ctx, torch, stream, world, rank, dist, with_e2e=not args.no_e2e)
        sharded_proj = bench_sharded(ctx, torch, stream, world, rank, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        v, desc, dt = CpuSweep(shapes, batches, threads).run(10.0)
        cpu = {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": desc,
               "single_thread": serial_baseline(shapes, batches)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded PCG64: fp16 d, dmin ~ U(0.001, 0.01), uniform random scale and quant "
                    "bits, N(0,1) activations)",
            "config": sweep_config(world),
            "collective": ((f"each GEMV writes its columns into this rank's exchange buffer; one peer all-gather "
                            f"kernel per step (16-byte pushes over NVLink, one signal per rank) inside the "
                            f"library's collective group" if peer else
                            f"local GEMV into its columns of y + in-place NCCL all-gathers inside "
                            f"strata_cuda_gemv_sharded_dev, the step's 16 in one NCCL group") if world > 1 else None),
            "launch": "CUDA graph per step" if graphs else "direct launches",
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(value / hbm, 3), "traffic": profiled_traffic(),
                         "algorithmic_bytes_per_launch": total // (len(batches) * len(shapes)),
                         "note": f"Q4_K GEMV over the timed sweep (16 GEMVs per step, each a prologue + "
                                 f"GEMV launch); peak = {peak_kind} copy bandwidth; traffic = DRAM bytes per "
                                 f"GEMV launch from profiles/gemv_q4k_sweep_dram.md"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "cases": cases,
            "nccl_gather": alt,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gemm": gemm,
            "moe": moe,
            "sharded_projection": sharded_proj,
            "q8_0": q8,
        }
        print(json.dumps(line), flush=True)

    del graphs
    for ws in weights.values():
        for w in ws:
            w.free()
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def parse_profile_case(spec: str):
    """K,N,B[,TYPE] -> (k, n, b, quant id); TYPE is a ggml type name (default Q4_K)."""
    import strata_cuda as sc
    parts = spec.split(",")
    if len(parts) not in (3, 4):
        raise SystemExit(f"--profile-case wants K,N,B[,TYPE], got {spec!r}")
    k, n, b = (int(v) for v in parts[:3])
    by_name = {name: q for q, name in sc.NAMES.items()}
    name = parts[3].strip().upper() if len(parts) == 4 else "Q4_K"
    if name not in by_name:
        raise SystemExit(f"--profile-case: unknown type {name!r} (one of {', '.join(sorted(by_name))})")
    return k, n, b, by_name[name]


def run_profile_case(args):
    """One GEMV case (K,N,B[,TYPE]) launched warmup + steps times on one weight
    copy: the small, single-kernel workload the ncu captures under profiles/
    use, and a quick look at the other block formats' GEMV."""
    import torch
    import strata_cuda as sc
    k, n, b, quant = parse_profile_case(args.profile_case)
    ctx = sc.Context(0)
    w = ctx.upload(quant_matrix(k + n, quant, n, k), quant, n, k)
    x = torch.from_numpy(activations(900 + b, b, k)).cuda()
    y = torch.empty(b, n, device="cuda")
    s = torch.cuda.current_stream()
    for _ in range(args.warmup):
        ctx.gemv_dev(w, x.data_ptr(), y.data_ptr(), b, s.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        ctx.gemv_dev(w, x.data_ptr(), y.data_ptr(), b, s.cuda_stream)
    e1.record(s)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / max(1, args.steps)
    nbytes = sc.byte_size(quant, k) * n + b * k * 4 + b * n * 4
    print(json.dumps({"profile_case": [k, n, b, sc.NAMES[quant]], "us_per_gemv": round(us, 2),
                      "gb_per_s": round(nbytes / (us * 1e-6) / 1e9, 1),
                      "note": "same weights every launch (L2-resident below ~126 MB): a profiling workload, "
                              "not a bench value"}))
    w.free()
    ctx.close()


def run_profile_gemm(args):
    """One prefill GEMM case (QUANT,K,N,M, e.g. Q5_K,4096,12288,2048) launched
    warmup + steps times: the workload of the GEMM ncu capture under profiles/."""
    import torch
    import strata_cuda as sc
    qn, k, n, m = args.profile_gemm.split(",")
    q = {"Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}[qn]
    k, n, m = int(k), int(n), int(m)
    ctx = sc.Context(0)
    w = ctx.upload(quant_matrix(500 + k + q, q, n, k), q, n, k)
    x = torch.from_numpy(bf16_bits(activations(77 + k, m, k)).view(np.int16)).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    ms = timed(torch, st, lambda: ctx.gemm_bf16_dev(w, x.data_ptr(), y.data_ptr(), m, st.cuda_stream),
               max(1, args.steps), warm=args.warmup)
    print(json.dumps({"profile_gemm": [qn, k, n, m], "us": round(ms * 1e3, 1),
                      "tflops": round(2.0 * m * n * k / (ms * 1e-3) / 1e12, 1),
                      "note": "same weights every launch: a profiling workload, not a bench value"}))
    w.free()
    ctx.close()


def run_profile_moe(args):
    """One MoE FFN configuration layer call at T tokens, warmup + steps times:
    the workload of the MoE ncu captures under profiles/."""
    import torch
    import strata_cuda as sc
    T = int(args.profile_moe)
    d = MOE_DIMS
    ctx = sc.Context(0)
    ws = {"gate_exps": ctx.upload(quant_matrix(1201, Q4_K, d["n_embd"], d["n_ff"], d["E"]), Q4_K, d["n_embd"],
                                  d["n_ff"], n_expert=d["E"]),
          "up_exps": ctx.upload(quant_matrix(1202, Q4_K, d["n_embd"], d["n_ff"], d["E"]), Q4_K, d["n_embd"],
                                d["n_ff"], n_expert=d["E"]),
          "down_exps": ctx.upload(quant_matrix(1203, Q4_K, d["n_ff"], d["n_embd"], d["E"]), Q4_K, d["n_ff"],
                                  d["n_embd"], n_expert=d["E"]),
          "gate_shexp": ctx.upload(quant_matrix(1204, Q4_K, d["n_ff_s"], d["n_embd"]), Q4_K, d["n_ff_s"], d["n_embd"]),
          "up_shexp": ctx.upload(quant_matrix(1205, Q4_K, d["n_ff_s"], d["n_embd"]), Q4_K, d["n_ff_s"], d["n_embd"]),
          "down_shexp": ctx.upload(quant_matrix(1206, Q4_K, d["n_embd"], d["n_ff_s"]), Q4_K, d["n_embd"], d["n_ff_s"]),
          "gate_inp_shexp": ctx.upload(quant_matrix(1207, Q4_K, 1, d["n_embd"]), Q4_K, 1, d["n_embd"])}
    L = ctx.moe_create(ws, d["n_embd"], d["E"], d["k"], d["n_ff"], d["n_ff_s"])
    x = torch.from_numpy(activations(1201 + T, T, d["n_embd"])).cuda()
    lg = torch.from_numpy(rng(1202 + T).standard_normal((T, d["E"])).astype(np.float32)).cuda()
    y = torch.empty((T, d["n_embd"]), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    ms = timed(torch, st, lambda: ctx.moe_ffn_dev(L, x.data_ptr(), lg.data_ptr(), T, y.data_ptr(),
                                                  stream=st.cuda_stream), max(1, args.steps), warm=args.warmup)
    print(json.dumps({"profile_moe": T, "us_per_layer": round(ms * 1e3, 2),
                      "note": "same weights and routing every call: a profiling workload, not a bench value"}))
    L.free()
    for w in ws.values():
        w.free()
    ctx.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="strata", choices=["strata", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--quick", action="store_true", help="skip the per-case table")
    ap.add_argument("--skip-sections", action="store_true", help="only the GEMV sweep (no gemm / moe / sharded lines)")
    ap.add_argument("--profile-case", default=None, metavar="K,N,B[,TYPE]",
                    help="launch one GEMV case (Q4_K unless TYPE names another ggml type) repeatedly "
                         "(for ncu captures) instead of the bench")
    ap.add_argument("--profile-gemm", default=None, metavar="QUANT,K,N,M",
                    help="launch one prefill GEMM case repeatedly (for ncu captures) instead of the bench")
    ap.add_argument("--profile-moe", default=None, metavar="T",
                    help="run the MoE configuration layer at T tokens repeatedly (for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        run_profile_case(args)
    elif args.profile_gemm:
        run_profile_gemm(args)
    elif args.profile_moe:
        run_profile_moe(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
