#!/usr/bin/env python3
"""Benchmark of the GLM-5.2 DSA indexer + top-k + absorbed-MLA attention substep.

Contract: ``python bench.py --gpus N --steps K --warmup W`` (N > 1 under
torchrun, one rank per GPU) prints ONE JSON line on rank 0.

Workload (``config.workload``): benchmark config 4 — one decode token for each
of 8 independent sequences, each with a 131072-key bf16 latent cache
[T, 576] and fp8-e4m3 index keys [T, 128] + per-key scale, top-2048, as an
indexer-owning layer. At N GPUs every cache is split into N contiguous key
shards (strong scaling: the same total work). A step = one layer-step of the
substep over all 8 sequences; the metric is microseconds per layer-step.
The caches (1.35 GB) exceed L2 (126 MB) at every N <= 8, so every step reads
HBM. Inputs are synthetic (seeded, the benchmark's distributions), generated on the
device. ``--impl reference`` times the reference's algorithm on the host cores
(the numpy port in oracle/, since the reference's own path is numpy).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG4 = dict(batch=8, T=131072, k=2048)
METRIC = "MLA+DSA attention substep latency, decode, 8 seq x 128K ctx, top-2048 (us/layer)"


# ---------------------------------------------------------------------------------------------
def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1/2/3 side measurements")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---- clocks sampler ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None

    def _read(self):
        for line in self.p.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        try:
            self.p.wait(timeout=2)
        except Exception:
            self.p.kill()
        self.t.join(timeout=1)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- device inputs ------------------------------------------------------------------------------
def make_device_inputs(torch, batch, T_local, t0, seed_base, device, n_q=1):
    """Seeded synthetic inputs on the device: c_kv ~ N(0,1) RMS-normalised rows,
    k_rot ~ N(0,1) roped at absolute positions (theta 1e6), bf16; index keys
    ~ N(0,1) quantised to e4m3 with per-key scale = amax/448; q ~ N(0,1) bf16,
    w ~ U(0,1). Sequence s uses seed seed_base + 1000*s (its shard: + t0)."""
    from windlass_b200 import attn as A
    kv = torch.empty(batch, T_local, 576, dtype=torch.bfloat16, device=device)
    keys = torch.empty(batch, T_local, 128, dtype=torch.uint8, device=device)
    scale = torch.empty(batch, T_local, dtype=torch.float32, device=device)
    qshape = (batch,) if n_q == 1 else (n_q,)
    g = torch.Generator(device=device)
    inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float64, device=device) / 64))
    for s in range(batch):
        g.manual_seed(seed_base + 1000 * s + 7919 * t0)
        x = torch.randn(T_local, 512, generator=g, device=device)
        kv[s, :, :512] = (x * torch.rsqrt((x * x).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
        r = torch.randn(T_local, 64, generator=g, device=device)
        ang = (torch.arange(t0, t0 + T_local, device=device, dtype=torch.float64)[:, None] * inv[None]).float()
        a, b = r[:, 0::2], r[:, 1::2]
        kv[s, :, 512:] = torch.cat([a * ang.cos() - b * ang.sin(), b * ang.cos() + a * ang.sin()], -1).to(torch.bfloat16)
        k = torch.randn(T_local, 128, generator=g, device=device)
        sc = (k.abs().amax(-1) / 448.0).clamp_min(1e-30)
        keys[s] = (k / sc[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
        scale[s] = sc
    g.manual_seed(seed_base + 17)
    q_abs = torch.randn(*qshape, 64, 576, generator=g, device=device).to(torch.bfloat16)
    q_idx = torch.randn(*qshape, 32, 128, generator=g, device=device).to(torch.bfloat16)
    w_idx = torch.rand(*qshape, 32, generator=g, device=device)
    return dict(kv=A.LatentKV.packed(kv), kv_raw=kv, keys=A.IndexKeys(keys, scale), q_abs=q_abs, q_idx=q_idx,
                w_idx=w_idx)


def elapsed_ms(torch, fn, steps, stream):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(steps):
        fn(i)
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e)


# ---- the reference arm (host cores) --------------------------------------------------------------
def host_threads() -> int:
    """Host cores this process may use (the same at every N: torch.distributed.run
    sets OMP_NUM_THREADS=1 for its ranks, which is not the reference's setting)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample_inputs(T, batch, pool=None):
    from oracle import attn_ref as o
    gen = lambda s: o.make_inputs(T, 4, seq=s)  # noqa: E731
    return list(pool.map(gen, range(batch))) if pool is not None else [gen(s) for s in range(batch)]


def cpu_step(inps, k, pool):
    """One layer-step of the workload through the reference's algorithm (numpy,
    fp32 like tools/ref_glm_chain.py): every sequence of the batch, the
    sequences spread over a thread pool (numpy releases the GIL in its
    kernels; each worker's BLAS gets an equal share of the cores)."""
    from oracle import attn_ref as o
    return list(pool.map(lambda inp: o.decode_step(inp, k, dtype=np.float32), inps))


class CpuArm:
    """The reference's CPU path for config 4 with every host core in use."""

    def __init__(self, batch):
        from concurrent.futures import ThreadPoolExecutor

        from threadpoolctl import threadpool_limits
        self.cores = host_threads()
        self.workers = max(1, min(batch, self.cores))
        self.limits = threadpool_limits(max(1, self.cores // self.workers))
        self.pool = ThreadPoolExecutor(self.workers)
        self.inps = cpu_sample_inputs(CFG4["T"], batch, self.pool)

    def step(self):
        cpu_step(self.inps, CFG4["k"], self.pool)

    def close(self):
        self.pool.shutdown()
        self.limits.restore_original_limits()

    def describe(self, steps):
        return (f"{steps} steps x all {len(self.inps)} sequences (T=131072, top-2048) through oracle/attn_ref.py "
                f"(numpy fp32), {self.workers} sequences in parallel x {max(1, self.cores // self.workers)} "
                f"BLAS threads on {self.cores} host cores")


def time_cpu(budget_s: float):
    """Whole layer-steps (all 8 sequences) of the workload on the host until the budget is spent."""
    arm = CpuArm(CFG4["batch"])
    arm.step()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        arm.step()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    arm.close()
    return el / n * 1e6, n, arm


def run_reference(args, rank):
    if rank != 0:
        return
    arm = CpuArm(CFG4["batch"])
    for _ in range(max(args.warmup, 1)):
        arm.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        arm.step()
        times.append(time.perf_counter() - t0)
    arm.close()
    us = statistics.mean(times) * 1e6
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/layer",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded, benchmark distributions)",
        "config": {"workload": "cfg4: decode, 8 seq x T=131072, top-2048, owner layer",
                   "batch": 8, "T": 131072, "index_topk": 2048},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": arm.cores, "kind": "port",
                         "sample": arm.describe(args.steps)},
        "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)



# ---- diagnostics run beside the timed region --------------------------------------------------
PHASES_P2P = ["indexer", "local_topk", "cand_exchange", "global_topk", "attention", "reduce_scatter",
              "all_gather"]
PHASES_NCCL = ["indexer", "local_topk", "cand_exchange", "global_topk", "attention", "local_merge",
               "all_gather", "merge"]
PHASES_1GPU = ["indexer", "topk", "attention", "merge"]


def phase_breakdown(torch, L, step, device, names, reps=20):
    """Per-phase device time of one layer-step (median over graph replays), from
    the library's global-timer stamps at its phase boundaries. The stamp
    launches break the overlap between phases, so the phases sum to a little
    more than the unstamped step."""
    buf = torch.zeros(64, dtype=torch.int64, device=device)
    L.wl_diag_phase_stamps(buf.data_ptr(), 64)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        n = L.wl_diag_phase_count()
    finally:
        L.wl_diag_phase_stamps(None, 0)
    rows = []
    for _ in range(reps + 2):
        g.replay()
        torch.cuda.synchronize()
        t = buf[:n].cpu().numpy().astype(np.float64)
        rows.append(np.diff(t) * 1e-3)
    d = np.median(np.array(rows[2:]), axis=0)
    if len(names) != len(d):  # e.g. an owner layer with index_topk >= T: no indexer or top-k phases
        names = names[-len(d):] if len(d) <= len(names) else [f"phase{i}" for i in range(len(d))]
    return {k: round(float(v), 2) for k, v in zip(names, d)}


def single_layer_us(torch, step, reps=20):
    """One eager call of the entry point, alone (synchronised on both sides):
    launch latency included, no graph."""
    ts = []
    for _ in range(reps):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    return round(float(np.median(ts)), 2)


def check_parity(torch, dist, A, _lib, cfg, data, sel, sel_n, ctx, lse, rank, world, seqs=(0, 1)):
    """The step's own outputs against the oracle on the same inputs: every rank's
    shard of sequences `seqs` is gathered to rank 0, which recomputes them on
    the host (oracle/attn_ref.py) and, at N > 1, on one GPU through
    wl_attn_decode. Returns (ok, summary) on rank 0, (True, None) elsewhere."""
    from oracle import attn_ref as o
    K = CFG4["k"]
    tol_rel = 1e-5  # the indexer's score tolerance (the reference's fp32 gate)
    res = {"checked": True, "seqs": list(seqs), "max_ulp": 0.0, "max_ulp_oracle_sel": 0.0, "max_lse_err": 0.0,
           "sel_mismatch": 0, "sel_in_gap": 0}
    if world > 1:
        res.update(single_gpu_sel_equal=True, max_ulp_vs_single_gpu=0.0)
    sel_c, n_c, ctx_c, lse_c = (t.cpu().numpy() for t in (sel, sel_n, ctx, lse))
    for s in seqs:
        parts = [data["kv_raw"][s].contiguous(), data["keys"].keys[s].contiguous(), data["keys"].scale[s].contiguous()]
        if world > 1:
            full = []
            for t in parts:
                lst = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(lst, t)
                full.append(torch.cat(lst, 0))
            parts = full
        if rank != 0:
            continue
        kv, bits, scale = parts
        inp = dict(c_kv=kv[:, :512].float().cpu().numpy(), k_rot=kv[:, 512:].float().cpu().numpy(),
                   q_abs=data["q_abs"][s].float().cpu().numpy(), q_idx=data["q_idx"][s].float().cpu().numpy(),
                   w_idx=data["w_idx"][s].cpu().numpy(), idx_bits=bits.cpu().numpy(),
                   idx_scale=scale.cpu().numpy(), scale=1.0 / 16.0)
        g_sel = sel_c[s, :int(n_c[s])]
        ref_index = o.indexer_scores(inp["q_idx"], o.dequant_e4m3(inp["idx_bits"], inp["idx_scale"]), inp["w_idx"])
        ref_sel = o.indexer_topk(ref_index, K)
        thr = np.sort(ref_index)[::-1][K - 1]
        tol = tol_rel * np.abs(ref_index).max()
        diff = set(ref_sel.tolist()) ^ set(g_sel.tolist())
        far = [t for t in diff if abs(ref_index[t] - thr) > tol]
        canonical = len(g_sel) == K and bool(np.all(np.diff(g_sel) > 0))
        res["sel_mismatch"] += len(far) + (0 if canonical else 1)
        res["sel_in_gap"] += len(diff) - len(far)
        rc, rl = o.mla_sparse(inp["q_abs"], inp["c_kv"], inp["k_rot"], g_sel, 1 / 16)
        res["max_ulp"] = max(res["max_ulp"], o.bf16_ulp_error(rc, ctx_c[s]))
        res["max_lse_err"] = max(res["max_lse_err"], float(np.abs(lse_c[s] - rl).max()))
        fc, _ = o.mla_sparse(inp["q_abs"], inp["c_kv"], inp["k_rot"], np.sort(ref_sel), 1 / 16)
        res["max_ulp_oracle_sel"] = max(res["max_ulp_oracle_sel"], o.bf16_ulp_error(fc, ctx_c[s]))
        if world > 1:
            one = A.attn_decode(A.glm52_cfg(kv.shape[0]), A.LatentKV.packed(kv[None]), data["q_abs"][s:s + 1],
                                keys=A.IndexKeys(bits[None], scale[None]), q_idx=data["q_idx"][s:s + 1],
                                w_idx=data["w_idx"][s:s + 1])
            torch.cuda.synchronize()
            s1 = one["sel"].cpu().numpy()[0]
            res["single_gpu_sel_equal"] &= bool(np.array_equal(s1, g_sel))
            res["max_ulp_vs_single_gpu"] = max(res["max_ulp_vs_single_gpu"],
                                               o.bf16_ulp_error(one["ctx"].cpu().numpy()[0], ctx_c[s]))
    if rank != 0:
        return True, None
    for k in ("max_ulp", "max_ulp_oracle_sel", "max_lse_err", "max_ulp_vs_single_gpu"):
        if k in res:
            res[k] = round(float(res[k]), 4)
    ok = (res["sel_mismatch"] == 0 and res["max_ulp"] <= 2.0 and res["max_lse_err"] < 1e-3
          and res["max_ulp_oracle_sel"] <= 2.0 and res.get("single_gpu_sel_equal", True)
          and res.get("max_ulp_vs_single_gpu", 0.0) <= 2.0)
    res["ok"] = bool(ok)
    return ok, res


# ---- our arm ------------------------------------------------------------------------------------
def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch
    import torch.distributed as dist

    from windlass_b200 import _lib
    from windlass_b200 import attn as A

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    B, T, K = CFG4["batch"], CFG4["T"], CFG4["k"]
    T_local = T // world
    t0 = rank * T_local
    cfg = A.glm52_cfg(T)
    data = make_device_inputs(torch, B, T_local, t0, 20260805, device)
    stream = torch.cuda.current_stream()
    L = _lib.lib()

    # ---- the step: one owner layer-step over 8 sequences ----
    ctx = torch.empty(B, 64, 512, dtype=torch.float32, device=device)
    lse = torch.empty(B, 64, dtype=torch.float32, device=device)
    sel = torch.empty(B, K, dtype=torch.int32, device=device)
    sel_n = torch.empty(B, dtype=torch.int32, device=device)
    io, keep = A.decode_io(cfg, data["kv"], data["q_abs"], keys=data["keys"], q_idx=data["q_idx"],
                           w_idx=data["w_idx"], sel_out=sel, sel_n_out=sel_n, ctx=ctx, lse=lse)
    comm = None
    if world > 1:
        comm = A.Comm(rank, world)
        shard = _lib.Shard(t0, T)
        nbytes = L.wl_attn_sharded_workspace_bytes(C.byref(cfg), T_local, B, world)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)

        def call(io_):
            _lib.check(L.wl_attn_decode_sharded(C.byref(cfg), C.byref(io_), C.byref(shard), comm.h, ws.data_ptr(),
                                                nbytes, torch.cuda.current_stream().cuda_stream))

        def step(i=0):
            call(io)
        # peer exchange: histogram zeroing, indexer, local top-k, candidate put,
        # global top-k, attention, reduce-scatter, all-gather; NCCL: histogram
        # zeroing, indexer, local top-k, global top-k, attention, local merge,
        # final merge (+ NCCL's own kernels)
        launches_per_step = 8 if comm.p2p else 7
    else:
        nbytes = L.wl_attn_workspace_bytes(C.byref(cfg), T, B)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)

        def call(io_):
            _lib.check(L.wl_attn_decode(C.byref(cfg), C.byref(io_), ws.data_ptr(), nbytes,
                                        torch.cuda.current_stream().cuda_stream))

        def step(i=0):
            call(io)
        launches_per_step = 5  # histogram zeroing, indexer, top-k, attention, merge

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # Capture one step in a CUDA graph (the launch chain of a layer-step).
    graph = None
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        torch.cuda.synchronize()
        graph = g
    except Exception as ex:  # pragma: no cover - reported, not hidden
        print(f"# graph capture failed ({ex}); timing eager launches", file=sys.stderr)
    run = (lambda i: graph.replay()) if graph is not None else step
    for _ in range(3):
        run(0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = elapsed_ms(torch, run, args.steps, stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    t_step = torch.tensor([ms / args.steps], device=device)
    if world > 1:
        dist.all_reduce(t_step, op=dist.ReduceOp.MAX)
    us = t_step.item() * 1e3
    _lib.check(A.device_error(clear=True)[0], "device error word after the timed region")

    # ---- e2e: public API with host buffers (queries in, ctx and selection out, every step) ----
    # A serving loop's pipeline: two sets of device buffers; step i computes on
    # one stream while the next step's queries go up and the previous step's
    # results come down on copy streams. Every step still carries its own H2D
    # and D2H copies; the time is from the first upload to the last download.
    qn = ("q_abs", "q_idx", "w_idx")
    h_q = [torch.empty_like(data[n], device="cpu").pin_memory() for n in qn]
    for h, n in zip(h_q, qn):
        h.copy_(data[n].cpu())
    h_ctx = torch.empty(B, 64, 512, dtype=torch.float32).pin_memory()
    h_sel = torch.empty(B, K, dtype=torch.int32).pin_memory()
    bufs = []
    for b in range(2):
        qb = {n: torch.empty_like(data[n]) for n in qn}
        ob = dict(ctx=torch.empty_like(ctx), lse=torch.empty_like(lse), sel=torch.empty_like(sel),
                  sel_n=torch.empty_like(sel_n))
        io_b, keep_b = A.decode_io(cfg, data["kv"], qb["q_abs"], keys=data["keys"], q_idx=qb["q_idx"],
                                   w_idx=qb["w_idx"], sel_out=ob["sel"], sel_n_out=ob["sel_n"], ctx=ob["ctx"],
                                   lse=ob["lse"])
        bufs.append((qb, ob, io_b, keep_b))
    s_comp, s_in, s_out = stream, torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in", "comp", "out")}

    def e2e_pipelined(n, s_comp=s_comp):
        def upload(j):
            qb = bufs[j % 2][0]
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev["comp"][j % 2])  # step j - 2 has read these buffers
                for h, nme in zip(h_q, qn):
                    qb[nme].copy_(h, non_blocking=True)
                ev["in"][j % 2].record(s_in)
        for e in ev["comp"] + ev["out"]:
            e.record(s_comp)
        upload(0)
        for i in range(n):
            b = i % 2
            s_comp.wait_event(ev["in"][b])
            s_comp.wait_event(ev["out"][b])  # step i - 2's results have been read out
            with torch.cuda.stream(s_comp):
                call(bufs[b][2])
            ev["comp"][b].record(s_comp)
            if i + 1 < n:
                upload(i + 1)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev["comp"][b])
                h_ctx.copy_(bufs[b][1]["ctx"], non_blocking=True)
                h_sel.copy_(bufs[b][1]["sel"], non_blocking=True)
                ev["out"][b].record(s_out)

    e2e_pipelined(4)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_a, t_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_a.record(s_comp)
    s_in.wait_event(t_a)
    e2e_pipelined(args.steps)
    s_comp.wait_stream(s_out)
    t_b.record(s_comp)
    t_b.synchronize()
    ms_e2e = t_a.elapsed_time(t_b)
    e2e_mode = ("pipelined: two buffer sets, each step's H2D and D2H on copy streams overlapping the "
                "neighbouring steps' compute; eager calls through the C ABI (no graph)")
    e2e_eager_us = ms_e2e / args.steps * 1e3
    # The same K pipelined steps — every step's uploads, call and downloads —
    # captured once as one CUDA graph and replayed once: the host's per-call
    # launch cost leaves the timed region, the copies and kernels do not.
    try:
        s_g = torch.cuda.Stream(device)
        g_e2e = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g_e2e, stream=s_g):
            e2e_pipelined(args.steps, s_g)
            s_g.wait_stream(s_out)
        torch.cuda.synchronize()
        with torch.cuda.stream(s_g):
            for _ in range(2):
                g_e2e.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t_a.record(s_g)
        with torch.cuda.stream(s_g):
            g_e2e.replay()
        t_b.record(s_g)
        t_b.synchronize()
        ms_e2e = t_a.elapsed_time(t_b)
        e2e_mode = ("pipelined: two buffer sets, each step's H2D and D2H on copy streams overlapping the "
                    "neighbouring steps' compute; the K steps' calls through the C ABI and their copies "
                    "captured as one CUDA graph, replayed once")
    except Exception as ex:  # pragma: no cover - reported, not hidden
        print(f"# e2e graph capture failed ({ex}); e2e is the eager loop's", file=sys.stderr)
        torch.cuda.synchronize()
    t_e2e = torch.tensor([ms_e2e / args.steps], device=device)
    if world > 1:
        dist.all_reduce(t_e2e, op=dist.ReduceOp.MAX)
    assert torch.equal(h_sel, sel.cpu()), "e2e selection differs from the timed step's"
    h2d = sum(h.numel() * h.element_size() for h in h_q)
    d2h = h_ctx.numel() * 4 + h_sel.numel() * 4

    # ---- outside the timed regions: phase breakdown, un-graphed latency, self-check ----
    names = (PHASES_P2P if comm.p2p else PHASES_NCCL) if comm is not None else PHASES_1GPU
    phases = phase_breakdown(torch, L, step, device, names)
    phases_min = None
    if world > 1:
        pv = torch.tensor(list(phases.values()), device=device)
        pm = pv.clone()
        dist.all_reduce(pv, op=dist.ReduceOp.MAX)
        dist.all_reduce(pm, op=dist.ReduceOp.MIN)
        phases_min = {k: round(float(v), 2) for k, v in zip(phases, pm.tolist())}
        phases = {k: round(float(v), 2) for k, v in zip(phases, pv.tolist())}
    single_us = single_layer_us(torch, step)
    if world > 1:
        su = torch.tensor([single_us], device=device)
        dist.all_reduce(su, op=dist.ReduceOp.MAX)
        single_us = round(su.item(), 2)
    step()
    torch.cuda.synchronize()
    par_ok, parity = check_parity(torch, dist, A, _lib, cfg, data, sel, sel_n, ctx, lse, rank, world)
    if world > 1:
        okt = torch.tensor([1 if par_ok else 0], device=device)
        dist.broadcast(okt, 0)
        par_ok = bool(okt.item())

    # ---- per-kernel breakdown through the individual entry points (roofline) ----
    roof = None
    breakdown = None
    if world == 1:
        breakdown, roof = kernel_breakdown(torch, A, _lib, cfg, data, args.steps, stream)

    extras = {}
    if world == 1 and not args.no_extras:
        extras = side_configs(torch, A, _lib, device, stream)

    if world > 1 and comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        cpu = None
        if world == 1:
            cpu_us, n, arm = time_cpu(args.cpu_seconds)
            cpu = {"value": round(cpu_us, 1), "unit": "us/layer", "cores": arm.cores, "kind": "port",
                   "sample": arm.describe(n)}
        line = {
            "metric": METRIC, "value": round(us, 2), "unit": "us/layer", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(us / 1e3, 5), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded on device, benchmark distributions)",
            "config": {"workload": "cfg4: decode, 8 seq x T=131072, top-2048, owner layer",
                       "batch": B, "T": T, "index_topk": K, "parallelism": f"kv-seq shard x{world}" + ("" if comm is None else
                                                                  (" (NVLink peer exchange)" if comm.p2p else " (NCCL)")),
                       "l2": "inputs (1.35 GB of caches) larger than L2", "graph": graph is not None},
            "tokens_per_s": round(B / (us * 1e-6), 1),
            "e2e": {"value": round(t_e2e.item() * 1e3, 2), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "mode": e2e_mode,
                    "eager_loop_value": round(e2e_eager_us, 2)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "roofline": roof,
            "kernels_us": breakdown,
            "phases_us": phases,
            "phases_us_min_over_ranks": phases_min,
            "single_layer_us": single_us,
            "parity": parity,
            "cpu_baseline": cpu,
            "extras": extras,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        # Multi-rank teardown: graphs that captured NCCL work keep the
        # communicator referenced, and destroying it (or the process group)
        # under them can block. Everything is printed and synchronised, so the
        # ranks leave directly after a final barrier.
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0 if par_ok else 1)
    if not par_ok:
        sys.exit(1)


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def traffic_per_key(kernel: str):
    """DRAM bytes per unit measured by ncu, from the committed summary
    profiles/<kernel>.txt (line 'dram_bytes_per_unit: X'), else None."""
    p = os.path.join(ROOT, "profiles", f"{kernel}.txt")
    try:
        for line in open(p):
            if line.startswith("dram_bytes_per_unit:"):
                return float(line.split(":")[1])
    except Exception:
        pass
    return None


def kernel_breakdown(torch, A, _lib, cfg, data, steps, stream):
    """Each kernel of the layer-step timed with CUDA events on the launching stream."""
    L = _lib.lib()
    B, T, K = CFG4["batch"], CFG4["T"], CFG4["k"]
    dev = data["q_abs"].device
    index = torch.empty(B, T, dtype=torch.float32, device=dev)
    sel = torch.empty(B, K, dtype=torch.int32, device=dev)
    cnt = torch.empty(B, dtype=torch.int32, device=dev)
    S = 16
    o_part = torch.empty(B, S, 64, 512, dtype=torch.float32, device=dev)
    l_part = torch.empty(B, S, 64, dtype=torch.float32, device=dev)
    ctx = torch.empty(B, 64, 512, dtype=torch.float32, device=dev)
    lse = torch.empty(B, 64, dtype=torch.float32, device=dev)
    rows = _lib.Rows(B, 1, T, 0)
    kc, lc = data["keys"].c(), data["kv"].c()
    # a second copy of the index keys: the indexer's timed launches alternate
    # between the two (2 x 138 MB, twice the L2), so no launch finds its keys
    # left in L2 by the one before
    keys2 = type(data["keys"])(data["keys"].keys.clone(), data["keys"].scale.clone())
    kcs = [kc, keys2.c()]
    tws = torch.empty(L.wl_indexer_topk_workspace_bytes(B, T), dtype=torch.uint8, device=dev)
    calls = {
        "indexer_scores": lambda st, i: L.wl_indexer_scores(C.byref(cfg), C.byref(kcs[i % 2]), T, C.byref(rows),
                                                      data["q_idx"].data_ptr(), data["w_idx"].data_ptr(),
                                                      index.data_ptr(), T, st),
        "topk": lambda st, i: L.wl_indexer_topk(index.data_ptr(), T, C.byref(rows), T, K, None, sel.data_ptr(), K,
                                             cnt.data_ptr(), tws.data_ptr(), tws.numel(), st),
        "mla_sparse_attn": lambda st, i: L.wl_mla_sparse_attn(C.byref(cfg), C.byref(lc), T, C.byref(rows),
                                                        data["q_abs"].data_ptr(), sel.data_ptr(), K,
                                                        cnt.data_ptr(), 0, 0, T, 128, o_part.data_ptr(),
                                                        l_part.data_ptr(), S, st),
        "lse_merge": lambda st, i: L.wl_lse_merge(o_part.data_ptr(), l_part.data_ptr(), B, S, S * 64 * 512, 64 * 512,
                                            S * 64, 64, 64, 512, ctx.data_ptr(), lse.data_ptr(), st),
    }
    st_now = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    reps = 20
    us = {}
    for name, fn in calls.items():
        _lib.check(fn(st_now(), 0), name)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                _lib.check(fn(st_now(), i), name)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        n = 5
        ms = elapsed_ms(torch, lambda i: g.replay(), n, stream)
        us[name] = ms / (n * reps) * 1e3
    # algorithmic bytes per launch
    algo = {
        "indexer_scores": B * T * (128 + 4 + 4) + B * (32 * 128 * 2 + 32 * 4),
        "topk": B * T * 4 + B * K * 4,
        "mla_sparse_attn": B * K * 1152 + B * S * (64 * 576 * 2) + B * S * 64 * 512 * 4,
        "lse_merge": B * S * 64 * 512 * 4 + B * 64 * 512 * 4,
    }
    dom = max(us, key=us.get)
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    achieved = algo[dom] / (us[dom] * 1e-6) / 1e9
    per_key = traffic_per_key(dom)
    units = B * T if dom in ("indexer_scores", "topk") else B * K
    roof = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": "fallback" if peaks.get("fallback") else "measured",
            "traffic": round(per_key * units) if per_key else None, "algo_bytes": algo[dom]}
    return {k: round(v, 2) for k, v in us.items()}, roof


def side_configs(torch, A, _lib, device, stream):
    """Short measurements of benchmark configs 0, 1, 2 (decode, batch 1) and 3 (prefill) on this GPU."""
    out = {}
    L = _lib.lib()
    # decode, batch 1: config 2 (T=32768) and config 1 (T=4096), owner + consumer;
    # enough cache instances that each step reads HBM (> 2x L2 in total).
    peaks = load_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    src = "fallback" if peaks.get("fallback") else "measured"
    qbytes = 64 * 576 * 2 + 32 * 128 * 2 + 32 * 4 + 64 * 512 * 4 + 64 * 4  # queries in, ctx + lse out
    for name, T in (("cfg2_decode_32k", 32768), ("cfg1_decode_4k", 4096), ("cfg0_decode_1k", 1024)):
        per = T * (1152 + 132)
        n_inst = max(2, int(np.ceil(300e6 / per)))
        cfg = A.glm52_cfg(T)
        insts = [make_device_inputs(torch, 1, T, 0, 20260802 + i, device) for i in range(n_inst)]
        nbytes = L.wl_attn_workspace_bytes(C.byref(cfg), T, 1)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        ios = []
        for d in insts:
            io, keep = A.decode_io(cfg, d["kv"], d["q_abs"], keys=d["keys"], q_idx=d["q_idx"], w_idx=d["w_idx"])
            io2, keep2 = A.decode_io(cfg, d["kv"], d["q_abs"], mode=_lib.WL_MODE_CONSUMER,
                                     sel_in=keep["sel_out"], sel_n_in=keep["sel_n_out"], canonical=True)
            ios.append((io, keep, io2, keep2))
        res = {}
        for mode in (0, 1):
            fns = []
            for i in range(n_inst):
                io = ios[i][0] if mode == 0 else ios[i][2]
                fns.append(lambda io=io: _lib.check(L.wl_attn_decode(C.byref(cfg), C.byref(io), ws.data_ptr(),
                                                                     nbytes, torch.cuda.current_stream().cuda_stream)))
            for f in fns:
                f()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()  # one graph = one step on each instance, round robin
            with torch.cuda.graph(g):
                for f in fns:
                    f()
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            reps = 20
            ms = elapsed_ms(torch, lambda i: g.replay(), reps, stream)
            us = ms / (reps * n_inst) * 1e3
            algo = (T * 132 if mode == 0 else 0) + min(2048, T) * 1152 + qbytes
            gbs = algo / (us * 1e-6) / 1e9
            ent = {"us_per_layer": round(us, 2), "algo_bytes": algo, "tokens_per_s": round(1e6 / us, 1),
                   "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                "frac": round(gbs / hbm, 4), "peak_source": src}}
            f0 = fns[0]
            ent["single_layer_us"] = single_layer_us(torch, f0)
            ent["phases_us"] = phase_breakdown(torch, L, f0, device,
                                               PHASES_1GPU if mode == 0 else PHASES_1GPU[2:])
            res["owner" if mode == 0 else "consumer"] = ent
        out[name] = res
        del insts, ios
        torch.cuda.empty_cache()
    # chunked prefill: config 3 (4096 rows on a 4096 prefix, top-2048)
    pos0, n_q = 4096, 4096
    T = pos0 + n_q
    cfg = A.glm52_cfg(T)
    d = make_device_inputs(torch, 1, T, 0, 20260803, device, n_q=n_q)
    fn = lambda i=0: A.attn_prefill(cfg, d["kv"], d["q_abs"], pos0, keys=d["keys"], q_idx=d["q_idx"],
                                    w_idx=d["w_idx"])
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    ms = elapsed_ms(torch, fn, 5, stream) / 5
    idx_flops = 2 * 32 * 128 * sum(pos0 + 1 + i for i in range(n_q))
    att_flops = n_q * 2048 * 64 * (2 * 576 + 2 * 512)
    tf = (idx_flops + att_flops) / (ms * 1e-3) / 1e12
    pk = peaks.get("bf16_tflops", 1590.0)
    gather = n_q * 2048 * 1152  # bytes of latent rows the attention gathers (mostly L2 hits)
    out["cfg3_prefill"] = {"ms": round(ms, 3), "tflops": round(tf, 1),
                           "attn_gather_bytes": gather,
                           "attn_gather_gbs": round(gather / (ms * 1e-3) / 1e9, 1),
                           "idx_gflop": round(idx_flops / 1e9, 1), "attn_gflop": round(att_flops / 1e9, 1),
                           "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk, "unit": "TFLOP/s",
                                        "frac": round(tf / pk, 4), "peak_source": src + " bf16 burst"}}
    del d
    torch.cuda.empty_cache()
    out["around"] = around_kernels(torch, A, device, stream)
    out["reference_gpu_kernels"] = reference_gpu_kernels()
    return out


def reference_gpu_kernels():
    """The reference's own CUDA kernels for the same block (indexer scores,
    combine, one-CTA top-k, index mask, mla_decode_absorbed; bf16 keys, fp32
    latent cache), compiled unmodified for sm_100a into oracle/_ref by
    oracle/build_ref.sh and timed there with CUDA events, batch 1. The GPU row
    to compare configs 0-2 with; absent when the binary was not built."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_kernels_bench")
    if not os.path.exists(exe):
        return {"unavailable": "oracle/_ref/ref_kernels_bench not built (needs the reference sources)"}
    try:
        r = subprocess.run([exe, "10"], capture_output=True, text=True, timeout=300)
        rows = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
        return {"source": "reference src/glm_kernels.cuh + src/glm_layer_runner.cuh, unmodified, sm_100a",
                "rows": rows, "rc": r.returncode}
    except Exception as ex:  # reported, not hidden
        return {"unavailable": f"{type(ex).__name__}: {ex}"}


def around_kernels(torch, A, device, stream):
    """The kernels either side of the substep at config 4's decode batch (8
    rows) and config 3's prefill chunk (4096 tokens): the absorption GEMVs and
    the indexer's query projection (weights rotated over 8 instances, larger
    than L2 in total, so they stream from HBM) and the cache write. Each timed as a CUDA graph of back-to-back calls."""
    res = {}
    cfg = A.glm52_cfg(8192)
    g = torch.Generator(device=device)
    g.manual_seed(7)
    n_w = 8
    kvbs = [(torch.randn(64 * 448, 512, device=device, generator=g) * 0.05).to(torch.bfloat16) for _ in range(n_w)]
    B = 8
    q = torch.randn(B, 64, 256, device=device, generator=g)
    ctx = torch.randn(B, 64, 512, device=device, generator=g)

    def graph_us(fns, reps=20):
        for f in fns:
            f()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for f in fns:
                f()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        return elapsed_ms(torch, lambda i: gr.replay(), reps, stream) / (reps * len(fns)) * 1e3

    us = graph_us([lambda w=w: A.mla_absorb_q(cfg, q, w) for w in kvbs])
    wb = 64 * 192 * 512 * 2
    res["absorb_q_b8"] = {"us": round(us, 2), "weight_bytes": wb, "achieved_gbs": round(wb / (us * 1e-6) / 1e9, 1)}
    us = graph_us([lambda w=w: A.mla_project_v(cfg, ctx, w) for w in kvbs])
    wb = 64 * 256 * 512 * 2
    res["project_v_b8"] = {"us": round(us, 2), "weight_bytes": wb, "achieved_gbs": round(wb / (us * 1e-6) / 1e9, 1)}
    del kvbs
    # the indexer's query side at B = 8 (wq_b 16.8 MB bf16 + weights_proj 0.8 MB fp32, rotated over 8)
    wqs = [(torch.randn(4096, 2048, device=device, generator=g) * 0.02).to(torch.bfloat16) for _ in range(n_w)]
    wp = torch.randn(32, 6144, device=device, generator=g) * 0.02
    qr, xh = torch.randn(B, 2048, device=device, generator=g), torch.randn(B, 6144, device=device, generator=g)
    cq, sq = torch.rand(B, 32, device=device, generator=g), torch.rand(B, 32, device=device, generator=g)
    us = graph_us([lambda w=w: A.indexer_query(cfg, qr, w, xh, wp, cq, sq) for w in wqs])
    wb = 4096 * 2048 * 2 + 32 * 6144 * 4
    res["indexer_query_b8"] = {"us": round(us, 2), "weight_bytes": wb, "achieved_gbs": round(wb / (us * 1e-6) / 1e9, 1)}
    del wqs
    for name, n, T_max in (("cache_append_decode_b8", 8, 8192), ("cache_append_prefill_4096", 4096, 8192)):
        n_seq = 8 if n == 8 else 1
        keys = A.IndexKeys(torch.empty(n_seq, T_max, 128, dtype=torch.uint8, device=device),
                           torch.empty(n_seq, T_max, dtype=torch.float32, device=device))
        kv = A.LatentKV.packed(torch.empty(n_seq, T_max, 576, dtype=torch.bfloat16, device=device))
        pos = (torch.arange(n, device=device, dtype=torch.int32) % T_max) if n_seq == 1 else \
            torch.full((n,), T_max - 1, dtype=torch.int32, device=device)
        seq = torch.arange(n, device=device, dtype=torch.int32) if n_seq > 1 else None
        cs, sn = torch.rand(n, 32, device=device, generator=g), torch.rand(n, 32, device=device, generator=g)
        k_raw, kv_raw = torch.randn(n, 128, device=device, generator=g), torch.randn(n, 576, device=device, generator=g)
        kw = torch.ones(128, dtype=torch.bfloat16, device=device)
        kb = torch.zeros(128, dtype=torch.bfloat16, device=device)
        kvw = torch.ones(512, dtype=torch.bfloat16, device=device)
        fn = lambda: A.cache_append(cfg, pos, cs, sn, keys=keys, k_raw=k_raw, k_norm_w=kw, k_norm_b=kb, kv=kv,  # noqa: E731
                                    kv_raw=kv_raw, kv_norm_w=kvw, seq=seq)
        us = graph_us([fn] * 8)
        nb = n * (128 * 4 + 576 * 4 + 2 * 32 * 4 + 4 + 128 + 4 + 576 * 2)
        res[name] = {"us": round(us, 2), "bytes": nb, "achieved_gbs": round(nb / (us * 1e-6) / 1e9, 1)}
    return res


if __name__ == "__main__":
    main()
