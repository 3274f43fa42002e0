"""Benchmark of the B200 linear-layer path (mruntime's Backend::gemm).

Workload (default): the Qwen2.5-7B projection sweep -- one decoder layer's
four projections, qkv 3584->4608, o 3584->3584, gate+up 3584->37888 and
down 18944->3584, BF16 weights uploaded once as FP16, FP16 activations
x[M,3584] and x_down[M,18944] ~ N(0,1), seed 4 (mruntime_b200/workloads.py).
A step is one pass of the four GEMMs over one batch of M = 2048 tokens; the
headline metric is matmul TFLOP/s.  The same run also times every M of the
sweep (1 .. 2048; M <= 16 is the HBM-bound decode regime, reported in GB/s).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With N > 1 (launched by torchrun, one rank per GPU) the weights are sharded
tensor-parallel: qkv and gate/up by rows (column-parallel, no exchange), o and
down by K (row-parallel, FP32 partials all-reduced over NVLink by NCCL, then
rounded once to FP16).  Total work is fixed, so scaling is strong.

``--impl reference`` times the reference's own CPU gemm (built from its
sources into oracle/_ref) on a bounded sample of the same workload on the
host cores; under torchrun only rank 0 runs it.

Weights total 466 MB per step (larger than the 126 MB L2), so every timed
step streams them from HBM; no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import hashlib
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

from mruntime_b200 import workloads as WL  # noqa: E402

METRIC = "matmul TFLOP/s (Qwen2.5-7B projection sweep, M=2048 prefill step)"
UNIT = "TFLOP/s"
HEADLINE_M = 2048
# Per-launch DRAM traffic of the dominant kernel (the gate+up GEMM at
# M=2048, 2048x37888x3584): dram__bytes_read.sum + dram__bytes_write.sum of
# one launch in an ncu capture of this kernel build (the capture's command
# and date are kept with the kernel's profile summary).
GATEUP_TRAFFIC_BYTES = 427336448


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="mruntime_b200", choices=["mruntime_b200", "reference"])
    ap.add_argument("--m", type=int, default=HEADLINE_M, help="tokens per step (headline 2048)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-M sweep extras")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every step eagerly instead of replaying one captured CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-decode", action="store_true", help="skip the 7B greedy-decode measurement")
    ap.add_argument("--decode-tokens", type=int, default=64, help="tokens generated in the decode measurement")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed loop runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "power_w_max": max(power) if power else None, "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

class Proj:
    """One projection of the sweep as held by this rank."""

    def __init__(self, name, kind, weight, x, y, partial, n_full, k_full):
        self.name, self.kind, self.w, self.x, self.y, self.partial = name, kind, weight, x, y, partial
        self.n_full, self.k_full = n_full, k_full


def setup_gpu(rank: int, world: int, local: int, max_m: int):
    import torch

    from mruntime_b200 import capi

    torch.cuda.set_device(local)
    capi.init(local)
    stream = torch.cuda.current_stream().cuda_stream
    tp = None
    if world > 1:
        import torch.distributed as dist

        uid = [capi.TensorParallel.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        tp = capi.TensorParallel(rank, world, uid[0])
    d = WL.sweep_7b(max_m=max_m)
    projs = []
    for name, parts, k in WL.SWEEP_7B:
        w = np.ascontiguousarray(d[name])
        n = sum(parts)
        kind = WL.SWEEP_7B_PARALLEL[name]
        xfull = d["x_down"] if name == "down" else d["x"]
        if world > 1 and kind == "row":
            k0, k1 = capi.shard_cols(k, world, rank)
            wt = capi.Weight(w.ctypes.data, capi.BF16, False, n, k, None, (k0, k1), stream)
            xin = np.ascontiguousarray(xfull[:, k0:k1])
        else:
            ranges = capi.shard_rows(list(parts), world, rank) if world > 1 else None
            wt = capi.Weight(w.ctypes.data, capi.BF16, False, n, k, ranges, None, stream)
            xin = xfull
        x = torch.from_numpy(np.ascontiguousarray(xin).view(np.int16)).cuda()
        y = torch.empty((max_m, wt.n), dtype=torch.int16, device="cuda")
        partial = torch.empty((max_m, wt.n), dtype=torch.float32, device="cuda") if (world > 1 and kind == "row") else None
        projs.append(Proj(name, kind, wt, x, y, partial, n, k))
    del d
    if tp is not None:
        # Row-parallel outputs through the library's NVLink peer exchange when
        # every rank can map its peers' memory; NCCL otherwise.
        tp.p2p = False
        try:
            tp.p2p_init(max_m * max(p.w.n for p in projs if p.partial is not None))
            tp.p2p = True
        except capi.MrtError:
            pass
    torch.cuda.synchronize()
    return projs, tp, stream


def run_step(projs, tp, stream, M, ev=None):
    """One pass of the four projections over M tokens.  ev = (start, end)
    events recorded around the gate+up GEMM (the dominant kernel)."""
    from mruntime_b200 import capi

    for p in projs:
        if p.name == "gateup" and ev is not None:
            ev[0].record()
        if p.partial is None:
            capi.gemm(p.w, p.x.data_ptr(), p.x.shape[1], p.y.data_ptr(), p.w.n, M, False, stream)
        elif tp.p2p:
            # FP32 partial into the exchange region, summed across ranks over
            # NVLink and rounded once; the FP16 rows land in p.y on every rank
            tp.gemm_rowpar(p.w, p.x.data_ptr(), p.x.shape[1], M, p.y.data_ptr(), p.w.n, stream)
        else:
            capi.gemm_f32(p.w, p.x.data_ptr(), p.x.shape[1], p.partial.data_ptr(), p.w.n, M, stream)
            tp.allreduce_f32_to_f16(p.partial.data_ptr(), p.y.data_ptr(), M * p.w.n, stream)
        if p.name == "gateup" and ev is not None:
            ev[1].record()


def barrier_sync(world):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def capture(fn):
    """Record fn(stream) into a CUDA graph (scratch buffers were sized by the
    warm-up calls, so nothing allocates during capture)."""
    import torch

    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(s.cuda_stream)  # one eager pass on the capture stream
        torch.cuda.synchronize()
        g.capture_begin()
        fn(s.cuda_stream)
        g.capture_end()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return g


def time_steps(projs, tp, stream, M, steps, world, dominant=False, graph=None):
    """Device time of `steps` steps (max over ranks), replaying `graph` when
    given; with dominant=True also the mean time of the gate+up GEMM alone
    (eager launches, CUDA events around each call)."""
    import torch

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier_sync(world)
    start.record()
    for _ in range(steps):
        if graph is not None:
            graph.replay()
        else:
            run_step(projs, tp, stream, M)
    end.record()
    torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    dom_ms = None
    if dominant:
        gate = [p for p in projs if p.name == "gateup"]
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in evs:
            a.record()
            run_step(gate, tp, stream, M)
            b.record()
        torch.cuda.synchronize()
        dom_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    return max_over_ranks(total_ms, world), dom_ms


def time_projections(projs, tp, stream, M, iters):
    """Mean device time of each projection alone (ms): a CUDA graph of the
    one projection replayed `iters` times between two events."""
    import torch

    out = {}
    world = tp.world if tp is not None else 1
    for p in projs:
        g = capture(lambda s, p=p: run_step([p], tp, s, M))
        barrier_sync(world)  # ranks start together (a row-parallel call waits for its peers)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        out[p.name] = a.elapsed_time(b) / iters
        del g
    return out


def e2e_host_buffers(projs, tp, stream, M, steps, world):
    """Same step through the host-buffer entry point (N=1: mrt_gemm_host, the
    reference's calling convention) or, under TP, pinned-host copies around the
    device calls.  Returns (ms per step, h2d bytes, d2h bytes)."""
    import torch

    from mruntime_b200 import capi

    hx = [torch.empty((M, p.x.shape[1]), dtype=torch.int16, pin_memory=True) for p in projs]
    for h, p in zip(hx, projs):
        h.copy_(p.x[:M].cpu())
    hy = [torch.empty((M, p.w.n), dtype=torch.int16, pin_memory=True) for p in projs]
    h2d = sum(h.numel() * 2 for h in hx)
    d2h = sum(h.numel() * 2 for h in hy)

    # Queue order: PCIe carries both directions at once (~84 GB/s together on
    # B200 hosts, ~55 one way), so the call with the largest output goes
    # first (its copies to the host start early and run longest), the
    # input-heavy down projection next to it so its copies to the device
    # overlap them, and a small call last (measured 4.16 ms per step against
    # 4.36 in projection order).
    rank_of = {"gateup": 0, "qkv": 1, "down": 2, "o": 3}
    order = sorted(range(len(projs)), key=lambda i: rank_of.get(projs[i].name, 9))

    def one():
        if world == 1:
            # the four products queued on pinned host buffers, one wait per step
            for i in order:
                capi.gemm_host_async(projs[i].w, hx[i].data_ptr(), hy[i].data_ptr(), M, False, stream)
            capi.sync(stream)
        else:
            for h, p in zip(hx, projs):
                p.x[:M].copy_(h, non_blocking=True)
            run_step(projs, tp, stream, M)
            for g, p in zip(hy, projs):
                g.copy_(p.y[:M], non_blocking=True)
            torch.cuda.current_stream().synchronize()

    for _ in range(2):
        one()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier_sync(world)
    start.record()
    for _ in range(steps):
        one()
    end.record()
    torch.cuda.synchronize()
    return max_over_ranks(start.elapsed_time(end), world) / steps, h2d, d2h


def WL_plan_pair(M: int, N: int, K: int) -> bool:
    from mruntime_b200 import capi

    return bool(capi.gemm_plan(M, N, K).get("pair"))


def step_flops(M: int) -> float:
    return WL.sweep_flops(M)


def gpu_arm(args, rank, world, local):
    import torch

    from mruntime_b200 import capi

    peaks = load_peaks()
    M = args.m
    projs, tp, stream = setup_gpu(rank, world, local, max(M, max(WL.SWEEP_M) if not args.no_sweep else M))
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler attach; it runs through warm-up and the timed region
    for _ in range(args.warmup):
        run_step(projs, tp, stream, M)
    capi.sync(stream)
    launches0 = capi.launch_count()
    run_step(projs, tp, stream, M)
    per_step_launches = capi.launch_count() - launches0
    graph = None if args.no_graph else capture(lambda s: run_step(projs, tp, s, M))
    total_ms, dom_ms = time_steps(projs, tp, stream, M, args.steps, world, dominant=True, graph=graph)
    launches = per_step_launches * args.steps
    clk = clocks.stop()
    del graph
    capi.sync(stream)  # raises if any bounded wait inside a kernel gave up
    ms = total_ms / args.steps
    value = step_flops(M) / (ms * 1e-3) / 1e12

    gate = next(p for p in projs if p.name == "gateup")
    dom_flops = 2.0 * M * gate.w.n * gate.w.k
    dom_tflops = dom_flops / (dom_ms * 1e-3) / 1e12
    # The dominant kernel is timed alone in a short loop (steps launches of
    # ~0.4 ms), at the clocks of a burst, so the denominator is the burst
    # cuBLAS figure; the sustained figure (a seconds-long loop under the
    # power cap) is reported beside it.
    peak = peaks["bf16_tflops"]
    roofline = {"bound": "tensor", "achieved": round(dom_tflops, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(dom_tflops / peak, 4), "traffic": GATEUP_TRAFFIC_BYTES,
                "kernel": f"{'tc_pair_kernel' if WL_plan_pair(M, gate.w.n, gate.w.k) else 'tc_gemm_kernel'} gate+up "
                          f"{M}x{gate.w.n}x{gate.w.k} (rank-local shard)",
                "peak_source": f"{peaks['source']} bf16 cuBLAS 8192^3, burst (timed alone like this kernel)",
                "frac_of_sustained": round(dom_tflops / peaks["bf16_tflops_sustained"], 4),
                "sustained_peak": peaks["bf16_tflops_sustained"],
                "algorithmic_flops_per_launch": dom_flops, "ms_per_launch": round(dom_ms, 5),
                "launches_timed": args.steps,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch, same kernel build"}

    e2e_ms, h2d, d2h = e2e_host_buffers(projs, tp, stream, M, max(3, min(args.steps, 10)), world)
    e2e = {"value": round(step_flops(M) / (e2e_ms * 1e-3) / 1e12, 2), "unit": UNIT, "ms_per_step": round(e2e_ms, 3),
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "path": "mrt_gemm_host_async x 4 (gate+up, q|k|v, down, o) + mrt_sync per step (pinned host buffers; "
                   "row chunks pipelined over copy-in, compute and copy-out streams, consecutive calls overlapping "
                   "through four staging sets; copies inside the timed region)" if world == 1 else
           "pinned-host copies + mrt_gemm / " + ("mrt_tp_gemm_rowpar (NVLink peer exchange)" if tp.p2p else
                                                  "mrt_gemm_f32 + mrt_tp_allreduce_f32_to_f16 (NCCL)")}

    sweep = []
    if not args.no_sweep:
        for m in WL.SWEEP_M:
            for _ in range(3):
                run_step(projs, tp, stream, m)
            n_it = 50 if m <= 128 else 20
            g = None if args.no_graph else capture(lambda s, m=m: run_step(projs, tp, s, m))
            t_ms, _ = time_steps(projs, tp, stream, m, n_it, world, graph=g)
            del g
            t = t_ms / n_it
            # Decode shapes also back to back: one graph of 8 consecutive
            # steps (as the layers of a decoder follow each other), so each
            # step's first GEMM overlaps the previous step's last one.
            chained = None
            if m <= 128 and not args.no_graph:
                gc = capture(lambda s, m=m: [run_step(projs, tp, s, m) for _ in range(8)])
                c_ms, _ = time_steps(projs, tp, stream, m, 7, world, graph=gc)
                del gc
                chained = c_ms / 56
            tf = step_flops(m) / (t * 1e-3) / 1e12
            gbs = WL.sweep_bytes(m) / (t * 1e-3) / 1e9
            bound = "hbm" if m <= 128 else "tensor"
            frac = gbs / peaks["hbm_gbs"] if bound == "hbm" else tf / peaks["bf16_tflops"]
            per = time_projections(projs, tp, stream, m, 10)
            plans = {p.name: capi.gemm_plan(m, p.w.n, p.w.k) for p in projs}
            row = {"M": m, "ms": round(t, 4), "TFLOP/s": round(tf, 1), "GB/s": round(gbs, 1), "bound": bound,
                   "frac": round(frac, 4)}
            if chained is not None:
                c_gbs = WL.sweep_bytes(m) / (chained * 1e-3) / 1e9
                row.update({"ms_back_to_back": round(chained, 4), "GB/s_back_to_back": round(c_gbs, 1),
                            "frac_back_to_back": round(c_gbs / peaks["hbm_gbs"], 4)})
            sweep.append({**row, "per_projection_ms": {k: round(v, 4) for k, v in per.items()},
                          "plans": {k: "{kernel} bn={bn} full={full_tiles} splits={tail_splits} kb={kb_per} "
                                       "grid={grid}{c}".format(c=" cluster" if v["cluster"] else "", **v)
                                    for k, v in plans.items()}})
        capi.sync(stream)
    return {"ms": ms, "value": value, "roofline": roofline, "e2e": e2e, "clocks": clk, "launches": launches,
            "sweep": sweep, "peaks": peaks, "projs": projs, "tp": tp}


# ---------------------------------------------------------------------------
# The smaller reference configurations, timed on one GPU (extras)
# ---------------------------------------------------------------------------

def configs_arm(peaks) -> dict:
    """Device time of the reference's smaller configurations through the C ABI
    (each a graph of repeated calls, CUDA events around the replays; random
    device-made operands, the values do not change the work):

    * decode GEMV, M=1, W 4864x896 FP16 (8.7 MB): cold = 30 weight copies
      called in turn (262 MB, more than the 126 MB L2), hot = one copy 30 times;
    * Qwen2.5-0.5B layer at M=512: the seven projections as the reference
      calls them (q/k/v with their biases, o, gate, up, down), BF16 weights;
    * 0.5B lm_head (151936x896 FP16, 272 MB) with the greedy argmax at M=1 and
      M=128 (mrt_lm_head_argmax).

    GB/s counts 2NK + 2MK + 2MN bytes per call, TFLOP/s 2MNK; HBM fractions
    against the measured copy bandwidth, tensor fractions against the measured
    burst bf16 peak (each call runs alone for microseconds)."""
    import torch

    from mruntime_b200 import capi

    s0 = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)

    def weight(n, k, dt=torch.float16):
        t = (torch.randn(n, k, generator=gen, device="cuda") * 0.02).to(dt)
        w = capi.Weight(t.data_ptr(), capi.FP16 if dt == torch.float16 else capi.BF16, True, n, k, None, None, s0)
        torch.cuda.synchronize()
        return w

    def act(m, k):
        return torch.randn(m, k, generator=gen, device="cuda").half()

    def per_call_ms(fn, calls, reps=20):
        g = capture(fn)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(3):
            g.replay()
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) / reps / calls

    out = {}
    # decode GEMV
    N, K = 4864, 896
    ws = [weight(N, K) for _ in range(30)]
    x, y = act(1, K), torch.empty(1, N, dtype=torch.float16, device="cuda")
    nbytes = 2 * N * K + 2 * K + 2 * N
    cold = per_call_ms(lambda s: [capi.gemm(w, x.data_ptr(), K, y.data_ptr(), N, 1, False, s) for w in ws], 30)
    hot = per_call_ms(lambda s: [capi.gemm(ws[0], x.data_ptr(), K, y.data_ptr(), N, 1, False, s) for _ in ws], 30)
    for w in ws:
        w.free()
    out["decode_gemv_4864x896_m1"] = {
        "cold_us": round(cold * 1e3, 2), "cold_GB/s": round(nbytes / (cold * 1e-3) / 1e9, 1),
        "cold_frac_hbm": round(nbytes / (cold * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
        "hot_us": round(hot * 1e3, 2), "hot_GB/s": round(nbytes / (hot * 1e-3) / 1e9, 1),
        "note": "hot: the weight stays in L2, so the HBM fraction does not apply"}
    # 0.5B layer at M = 512
    M = 512
    shapes = WL.LAYER_05B
    lw = {nm: weight(n, k, torch.bfloat16) for nm, n, k in shapes}
    keep = []
    for nm, n in (("q", 896), ("k", 128), ("v", 128)):
        b = (torch.randn(n, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
        keep.append(b)
        lw[nm].attach_bias(b.data_ptr(), capi.BF16, True, s0)
    torch.cuda.synchronize()
    xl, xd = act(M, 896), act(M, 4864)
    ys = {nm: torch.empty(M, n, dtype=torch.float16, device="cuda") for nm, n, _ in shapes}

    def layer(s):
        for nm, n, k in shapes:
            src = xd if nm == "down" else xl
            capi.gemm(lw[nm], src.data_ptr(), k, ys[nm].data_ptr(), n, M, nm in ("q", "k", "v"), s)

    t = per_call_ms(layer, 1)
    flops = sum(2.0 * M * n * k for _, n, k in shapes)
    # The same outputs from four calls: q|k|v stacked into one 1152-row weight
    # (with the three biases) and gate|up into one 9728-row weight, as a
    # decoder holds them; rows are independent, so every output is the same.
    src = {nm: (torch.randn(n, k, generator=gen, device="cuda") * 0.02).to(torch.bfloat16) for nm, n, k in shapes}
    fw = {"qkv": capi.Weight(torch.cat([src["q"], src["k"], src["v"]]).data_ptr(), capi.BF16, True, 1152, 896,
                             None, None, s0),
          "o": capi.Weight(src["o"].data_ptr(), capi.BF16, True, 896, 896, None, None, s0),
          "gateup": capi.Weight(torch.cat([src["gate"], src["up"]]).data_ptr(), capi.BF16, True, 9728, 896,
                                None, None, s0),
          "down": capi.Weight(src["down"].data_ptr(), capi.BF16, True, 896, 4864, None, None, s0)}
    qkv_bias = torch.cat(keep)
    fw["qkv"].attach_bias(qkv_bias.data_ptr(), capi.BF16, True, s0)
    torch.cuda.synchronize()
    fy = {nm: torch.empty(M, w.n, dtype=torch.float16, device="cuda") for nm, w in fw.items()}

    def layer_fused(s):
        for nm, w in fw.items():
            src_x = xd if nm == "down" else xl
            capi.gemm(w, src_x.data_ptr(), w.k, fy[nm].data_ptr(), w.n, M, nm == "qkv", s)

    tf = per_call_ms(layer_fused, 1)
    for w in list(lw.values()) + list(fw.values()):
        w.free()
    out["layer_05b_m512"] = {"us": round(tf * 1e3, 2), "TFLOP/s": round(flops / (tf * 1e-3) / 1e12, 1),
                             "frac_tensor_burst": round(flops / (tf * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
                             "calls": 4, "note": "q|k|v and gate|up stacked into one weight each",
                             "seven_calls_us": round(t * 1e3, 2),
                             "seven_calls_frac_tensor_burst": round(flops / (t * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)}
    # lm_head + argmax
    V, H = 151936, 896
    wl = weight(V, H)
    for m in (1, 128):
        xm = act(m, H)
        logits = torch.empty(m, V, dtype=torch.float16, device="cuda")
        idx = torch.empty(m, dtype=torch.int64, device="cuda")
        t = per_call_ms(lambda s, m=m, xm=xm, logits=logits, idx=idx: capi.lm_head_argmax(
            wl, xm.data_ptr(), H, m, logits.data_ptr(), 0, idx.data_ptr(), None, s), 1)
        nbytes = 2 * V * H + 2 * m * H + 2 * m * V
        out[f"lm_head_05b_argmax_m{m}"] = {
            "us": round(t * 1e3, 2), "GB/s": round(nbytes / (t * 1e-3) / 1e9, 1),
            "frac_hbm": round(nbytes / (t * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
            "TFLOP/s": round(2.0 * m * V * H / (t * 1e-3) / 1e12, 1)}
    wl.free()
    return out


# ---------------------------------------------------------------------------
# Greedy decode of the 7B-shaped decoder (mrt_decoder_*), one GPU
# ---------------------------------------------------------------------------

DECODE_PROMPT = 512


def decode_arm(peaks: dict, max_new: int, tp=None, world: int = 1) -> dict:
    """tok/s of batch-1 greedy decoding on the Qwen2.5-7B-shaped decoder
    (random N(0, 0.02) FP16 weights made on the GPU, RMSNorm gains 1, seeded
    512-token prompt): prefill once, then `max_new` tokens; the decode rate
    counts the graph-replayed steps (every step after the first).  With a
    tensor-parallel handle every rank runs its shard; times are the max over
    ranks."""
    import torch

    from mruntime_b200 import capi

    cfg = WL.DECODER_7B
    dec = capi.Decoder(cfg, DECODE_PROMPT + max_new, tp)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    wbytes = 0
    for name, shape, kind in WL.decoder_tensor_specs(cfg):
        if kind == "ones":
            t = torch.ones(shape, dtype=torch.float16, device="cuda")
        else:
            t = (torch.randn(shape, generator=g, device="cuda", dtype=torch.float32) * 0.02).half()
            if name != "model.embed_tokens.weight":
                wbytes += t.numel() * 2
        dec.load(name, t.data_ptr(), capi.FP16, True, shape)
        del t
    prompt = WL.decoder_prompt(3, DECODE_PROMPT, cfg["vocab_size"])
    launches0 = capi.launch_count()
    dec.generate(prompt, max_new)  # warm: builds tables, sizes scratch
    per_run = capi.launch_count() - launches0
    toks, st = dec.generate(prompt, max_new)
    dec.free()
    ms = max_over_ranks(st.decode_ms, world) / max(1, st.decode_steps)
    prefill_ms = max_over_ranks(st.prefill_ms, world)
    first_ms = max_over_ranks(st.first_step_ms, world)
    st.prefill_ms, st.first_step_ms = prefill_ms, first_ms
    wbytes //= world  # each GPU streams its shard (replicated heads at 8 ranks add a little)
    gbs = wbytes / (ms * 1e-3) / 1e9
    return {"metric": f"Qwen2.5-7B-shaped greedy decode tokens/s (batch 1, 512-token prompt, {world} GPU"
                      f"{'s, tensor parallel' if world > 1 else ''})",
            "value": round(1000.0 / ms, 1), "unit": "tokens/s", "ms_per_token": round(ms, 4),
            "decode_steps_timed": st.decode_steps, "first_step_ms": round(st.first_step_ms, 3),
            "prefill_ms": round(st.prefill_ms, 2), "prefill_tokens_per_s": round(DECODE_PROMPT / (st.prefill_ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "algorithmic_bytes_per_token": wbytes,
                         "note": "per GPU: its weight shard streamed once per token (all projections + lm_head); "
                                 "KV cache, activations and all-reduces excluded"},
            "gpu_launches_per_generate": per_run, "tokens_head": toks[:8],
            "tokens_sha256_16": hashlib.sha256(np.asarray(toks, dtype=np.int64).tobytes()).hexdigest()[:16],
            "tokens_generated": len(toks),
            "data": "synthetic (torch-seeded N(0,0.02) FP16 weights on the GPU, seeded prompt)"}


# ---------------------------------------------------------------------------
# CPU: the reference's own gemm (oracle/_ref, built from the reference sources)
# ---------------------------------------------------------------------------

class RefSample:
    """A bounded sample of the sweep step for the reference's CPU gemm:
    `rows` rows of x through every projection, restricted to the first
    `n_frac` of each weight's output rows when even one row is too slow.
    Rows are independent in the reference (cpu_backend.cpp:143-166), so the
    sample's throughput is the full step's."""

    def __init__(self, M: int, threads: int = 0):
        from oracle import oracle as O

        self.O = O
        self.rb = O.RefBackend(threads)
        d = WL.sweep_7b(max_m=M)
        self.items = []
        for name, parts, k in WL.SWEEP_7B:
            x = d["x_down"] if name == "down" else d["x"]
            self.items.append((name, x, d[name]))
        self.rows, self.n_frac = 1, 1.0

    def flops(self) -> float:
        return sum(2.0 * self.rows * int(w.shape[0] * self.n_frac) * w.shape[1] for _, _, w in self.items)

    def run(self):
        for _, x, w in self.items:
            n = max(1, int(w.shape[0] * self.n_frac))
            self.rb.gemm(x[: self.rows], self.O.FP16, w[:n], self.O.BF16, trans_b=True)

    def calibrate(self, seconds: float):
        """Choose rows / n_frac so that one run() takes about `seconds`."""
        self.rows, self.n_frac = 1, 0.05
        self.run()  # first call pays for thread start-up and page faults
        t0 = time.perf_counter()
        self.run()
        t = max(time.perf_counter() - t0, 1e-4)
        per_full_row = t / 0.05
        if per_full_row <= seconds:
            self.n_frac = 1.0
            self.rows = max(1, min(64, int(seconds / per_full_row)))
        else:
            self.n_frac = max(0.002, seconds / per_full_row)

    def describe(self, M: int) -> str:
        return (f"{self.rows} of {M} rows x {self.n_frac:.3f} of each weight's output rows, all four projections "
                f"(qkv, o, gate+up, down), {self.flops() / 1e9:.2f} GFLOP per sample")


def cpu_baseline(M: int, seconds: float) -> dict:
    s = RefSample(M)
    s.calibrate(seconds / 3)
    s.run()  # warm
    reps, t_total = 0, 0.0
    while t_total < seconds * 0.66 or reps < 2:
        t0 = time.perf_counter()
        s.run()
        t_total += time.perf_counter() - t0
        reps += 1
    value = s.flops() * reps / t_total / 1e12
    return {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
            "sample": s.describe(M) + f"; {reps} samples in {t_total:.1f} s"}


def reference_arm(args, rank, world):
    if rank != 0:
        return None
    M = args.m
    budget = 150.0  # seconds for the whole --warmup + --steps run
    per_step = min(20.0, max(0.05, budget / max(1, args.steps + args.warmup)))
    s = RefSample(M)
    s.calibrate(per_step)
    for _ in range(args.warmup):
        s.run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s.run()
    dt = time.perf_counter() - t0
    value = s.flops() * args.steps / dt / 1e12
    cpu = {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
           "sample": s.describe(M)}
    return {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 accumulate (fp16 x, bf16 w)",
            "data": "synthetic (seeded N(0,1) FP16 activations, N(0,0.02) BF16 weights)",
            "config": workload_config(M, world), "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def workload_config(M: int, world: int, graph: bool = True) -> dict:
    return {"workload": "qwen2.5-7b projection sweep (qkv 3584->4608, o 3584->3584, gate+up 3584->37888, "
                        "down 18944->3584), one step = the four GEMMs at M tokens",
            "M": M, "seed": 4, "weights": "bf16 source, uploaded once as fp16",
            "parallelism": f"tp{world}" if world > 1 else "single gpu",
            "launch": "each timed step replays one CUDA graph of the step" if graph else "eager launches",
            "l2": "inputs larger than L2 (466 MB of fp16 weights streamed per step)"}


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    if args.impl == "reference":
        line = reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line))
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    r = gpu_arm(args, rank, world, local)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(args.m, args.cpu_seconds)
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {e}"}
    configs = None
    if world == 1 and not args.no_sweep:
        configs = configs_arm(r["peaks"])
    decode = None
    if not args.no_decode:
        r["projs"] = None  # release the sweep's weights first
        decode = decode_arm(r["peaks"], args.decode_tokens, r["tp"], world)
    if rank == 0:
        line = {"metric": METRIC, "value": round(r["value"], 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(r["ms"], 5), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
                "data": "synthetic (seeded N(0,1) FP16 activations, N(0,0.02) BF16 weights)",
                "config": workload_config(args.m, world, not args.no_graph), "e2e": r["e2e"], "roofline": r["roofline"],
                "cpu_baseline": cpu, "clocks": r["clocks"], "gpu_launches": r["launches"], "sweep": r["sweep"],
                "configs": configs, "decode": decode}
        if r["tp"] is not None:
            line["config"]["row_parallel_exchange"] = (
                "NVLink peer exchange in the library's kernels (mrt_tp_gemm_rowpar)" if r["tp"].p2p else
                "NCCL all-reduce of FP32 partials + one FP16 rounding")
        print(json.dumps(line))
    if r["tp"] is not None:
        import gc

        gc.collect()  # graphs holding NCCL calls are gone before the communicator
        r["tp"].destroy()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
