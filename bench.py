#!/usr/bin/env python
"""MoE-layer throughput of the B200 implementation (and, with --impl reference, of the reference's CPU path).

Workload: one MoE layer (hidden 2048, 512 experts of intermediate 512, top-10,
Q2_0 experts, sigmoid-gated shared expert), 64 decode tokens per step, Zipf(1.1) expert popularity.
A step is one smoe_moe_forward over one batch: router, dispatch, expert products, combine.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]

Timing: W untimed steps, then exactly K steps between CUDA events on the launching stream, bracketed by a
barrier and a synchronize, max over ranks.  Each step's expert bytes (~200 MB) exceed the 126 MB L2 and the
steps rotate over --layers distinct seeded layers, so weights stream from HBM.  Rank 0 prints one JSON line.
N > 1 runs independent replicas (decode does not shard: "replicas only"), value = all ranks' tokens / time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s (decode b1/b64, prefill 4k); expert-weight HBM GB/s vs peak"
UNIT = "tokens/s"
STAGES = ["router_gemv", "router_topk_q8", "dispatch", "expert_gate_up", "expert_down", "combine"]
KERNEL_OF_STAGE = {"router_gemv": "bf16_gemv_kernel", "router_topk_q8": "router_topk_kernel",
                   "dispatch": "group_kernel", "expert_gate_up": "layer_gate_up_kernel",
                   "expert_down": "layer_down_kernel", "combine": "combine_kernel"}
KERNEL_OF_STAGE_TC = dict(KERNEL_OF_STAGE, expert_gate_up="tc_expert_kernel<0>", expert_down="tc_expert_kernel<1>")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4])
    ap.add_argument("--expert-path", type=int, default=0, choices=[0, 1, 2],
                    help="0 automatic, 1 SIMT expert kernels, 2 tensor-core expert kernels")
    ap.add_argument("--layers", type=int, default=4, help="distinct layers rotated through the steps")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------------
# clocks during the timed region (read-only NVML queries)
# ---------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
               "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int, period: float = 0.01):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period, self.stop_flag = period, threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self.stop_flag.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.stop_flag.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "err", "no samples")}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_unit():
    """DRAM bytes per expert tile from the committed ncu summary (profiles/traffic_per_unit.txt), if any."""
    p = ROOT / "profiles" / "traffic_per_unit.txt"
    out = {}
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and not line.startswith("#"):
                out[parts[0]] = float(parts[1])
    return out


# ---------------------------------------------------------------------------------------------------
# the reference's CPU path (oracle/_ref: StrataMetal's own host references, else the oracle port)
# ---------------------------------------------------------------------------------------------------
def cpu_layer_runner(lay):
    import ctypes as C

    import numpy as np

    from oracle import oracle as O
    t = {k: np.ascontiguousarray(v.cpu().numpy()) for k, v in lay.tensors.items()}
    sp = lay.spec
    R = O.ref()
    threads = os.cpu_count() or 1
    vp = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    if R is not None:
        R.ref_moe_layer.restype = C.c_int

        def run(x):
            out = np.empty_like(x)
            rc = R.ref_moe_layer(sp.n_embd, sp.n_ff, sp.n_expert, sp.k, sp.gu_type, sp.d_type,
                                 vp(t["ffn_gate_inp.weight"]), vp(t["ffn_gate_exps.weight"]),
                                 vp(t["ffn_up_exps.weight"]), vp(t["ffn_down_exps.weight"]), 1, sp.sg_type,
                                 sp.sd_type, vp(t["ffn_gate_shexp.weight"]), vp(t["ffn_up_shexp.weight"]),
                                 vp(t["ffn_down_shexp.weight"]), vp(t["ffn_gate_inp_shexp.weight"]), vp(x),
                                 x.shape[0], vp(out), threads)
            assert rc == 0
            return out
        return run, "reference", threads
    sh = dict(sg_type=sp.sg_type, su_type=sp.su_type, sd_type=sp.sd_type, sgate=t["ffn_gate_shexp.weight"],
              sup=t["ffn_up_shexp.weight"], sdown=t["ffn_down_shexp.weight"],
              ginp=t["ffn_gate_inp_shexp.weight"].view(np.uint16))
    hl = O.HostLayer(sp.n_embd, sp.n_ff, sp.n_expert, sp.k, sp.gu_type, sp.d_type,
                     t["ffn_gate_inp.weight"].view(np.uint16), t["ffn_gate_exps.weight"], t["ffn_up_exps.weight"],
                     t["ffn_down_exps.weight"], sh)
    return (lambda x: O.moe_layer(hl, x, n_threads=threads)), "port", threads


def cpu_baseline(lay, x_host, seconds: float):
    run, kind, threads = cpu_layer_runner(lay)
    T = x_host.shape[0]
    run(x_host[:1])
    n, t0 = 0, time.perf_counter()
    while True:
        run(x_host)
        n += 1
        el = time.perf_counter() - t0
        if el > seconds or n >= 50:
            break
    return {"value": n * T / el, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n} full steps of the bench workload ({T} tokens each, layer 0), {el:.1f} s"}


# ---------------------------------------------------------------------------------------------------
def setup_dist(args):
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def config_dict(args, spec, T, D_mean):
    return {"workload": f"configs[{args.config}]: one MoE layer, {T} {'decode' if T <= 64 else 'prefill'} tokens/step"
                        + (", Zipf(1.1) expert popularity" if spec.zipf else "")
                        + (", IQ2_S gate/up" if spec.gu_type == 22 else ""),
            "tokens_per_step": T, "n_embd": spec.n_embd, "n_ff": spec.n_ff, "n_expert": spec.n_expert,
            "top_k": spec.k, "expert_format": "IQ2_S gate/up + Q2_0 down" if spec.gu_type == 22 else "Q2_0",
            "shared_expert": True, "distinct_experts_per_step": D_mean, "layers_rotated": args.layers,
            "l2": "inputs larger than L2: each step streams its experts' weights (> 126 MB), layers rotate",
            "parallelism": f"replicas x{args.gpus}", "seed": spec.seed}


def run_reference(args, ws, rank):
    """--impl reference: the reference's CPU implementation on this host's cores (rank 0 only)."""
    import numpy as np

    from stratametal_b200 import synth
    if rank != 0:
        return
    spec, T = synth.config_spec(args.config)
    lay = synth.make_layer(spec, 0, "cpu")
    x = synth.make_x(spec.seed, T, spec.n_embd).numpy()
    run, kind, threads = cpu_layer_runner(lay)
    t0 = time.perf_counter()
    run(x[:1])
    t_tok = time.perf_counter() - t0
    budget = 150.0 / max(1, args.steps + args.warmup)      # whole run within a few minutes
    s = int(max(1, min(T, budget / max(t_tok, 1e-6))))
    xs = np.ascontiguousarray(x[:s])
    for _ in range(args.warmup):
        run(xs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run(xs)
    el = time.perf_counter() - t0
    value = args.steps * s / el
    sample = f"{s} of the {T} tokens per step (layer 0 of configs[{args.config}]), {args.steps} steps, {el:.1f} s"
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int2 dot, f32/f64 sums", "data": "synthetic",
            "config": config_dict(args, spec, T, None), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, ws, rank, local):
    import ctypes as C

    import numpy as np
    import torch

    from stratametal_b200 import api, build, synth
    from stratametal_b200._lib import lib
    build.build()
    dev = torch.device("cuda", local)
    torch.cuda.set_stream(torch.cuda.Stream(dev))  # the C ABI wants an explicit non-null stream
    spec, T = synth.config_spec(args.config)
    api.set_expert_path(args.expert_path)
    layers = [api.MoeLayer(synth.make_layer(spec, li, dev), T, dev) for li in range(args.layers)]
    tc = lib().smoe_expert_path_for(C.byref(layers[0].c), T) == 2
    n_batches = 4
    xs = [synth.make_x(spec.seed + 1000 * local, T, spec.n_embd, dev, stream=b) for b in range(n_batches)]
    out = torch.empty(T, spec.n_embd, device=dev)
    stream = torch.cuda.current_stream()

    # distinct experts per (layer, batch), for the algorithmic bytes
    D = {}
    for li, m in enumerate(layers):
        for b, x in enumerate(xs):
            tr = m.make_trace(T)
            m.forward(x, out, tr)
            D[(li, b)] = int(torch.unique(tr.ids).numel())
    torch.cuda.synchronize()
    assert api.device_status() == 0

    def step(i):
        layers[i % args.layers].forward(xs[(i // args.layers) % n_batches], out)

    K, W = args.steps, args.warmup
    for i in range(W):
        step(i)
    # stage events for every timed step
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(STAGES) + 1)] for _ in range(K)]
    for row in ev:  # torch creates the CUDA event on its first record
        for e in row:
            e.record(stream)
    handles = [(C.c_void_p * len(STAGES))(*[e.cuda_event for e in row[1:]]) for row in ev]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(K):
            ev[i][0].record(stream)
            lib().smoe_set_stage_events(handles[i], len(STAGES))
            step(i)
        end.record(stream)
        lib().smoe_set_stage_events(None, 0)
        torch.cuda.synchronize()
    barrier(ws)
    el_ms = start.elapsed_time(end)
    el_ms = max_over_ranks(el_ms, ws)
    ms_step = el_ms / K
    value = ws * T / (ms_step * 1e-3)
    # per-stage device time
    stage_ms = {s: 0.0 for s in STAGES}
    for i in range(K):
        for j, s in enumerate(STAGES):
            stage_ms[s] += ev[i][j].elapsed_time(ev[i][j + 1])
    dominant = max(stage_ms, key=stage_ms.get)
    hbm_peak, peak_kind = peaks()
    E_BYTES = spec.expert_bytes()
    rbg = synth.row_bytes(spec.gu_type, spec.n_embd) * spec.n_ff
    rbd = synth.row_bytes(spec.d_type, spec.n_ff) * spec.n_embd
    Ds = [D[(i % args.layers, (i // args.layers) % n_batches)] for i in range(K)]
    D_mean = float(np.mean(Ds))
    q8x, q8h = (spec.n_embd // 32) * 36, (spec.n_ff // 32) * 36
    rows = T * spec.k + T
    alg = {"expert_gate_up": lambda d: (d + 1) * 2 * rbg + T * q8x + rows * q8h,
           "expert_down": lambda d: (d + 1) * rbd + rows * q8h + rows * spec.n_embd * 4,
           "router_gemv": lambda d: spec.n_expert * spec.n_embd * 2 + T * spec.n_embd * 4 + T * spec.n_expert * 4,
           "combine": lambda d: rows * spec.n_embd * 4 + T * spec.n_embd * 4}
    dom_bytes = float(np.mean([alg[dominant](d) for d in Ds])) if dominant in alg else None
    dom_ms = stage_ms[dominant] / K
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9 if dom_bytes else None
    tpu = traffic_per_unit()
    traffic = None
    if dominant == "expert_gate_up" and "expert_gate_up_per_expert" in tpu:
        traffic = tpu["expert_gate_up_per_expert"] * (D_mean + 1)
    expert_gbs = (D_mean + 1) * E_BYTES / (ms_step * 1e-3) / 1e9

    # end to end through the public API with host buffers
    x_host = [x.cpu().pin_memory() for x in xs]
    out_host = torch.empty(T, spec.n_embd).pin_memory()
    x_dev = torch.empty(T, spec.n_embd, device=dev)
    Ke = min(K, 1000)
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(Ke):
        x_dev.copy_(x_host[(i // args.layers) % n_batches], non_blocking=True)
        layers[i % args.layers].forward(x_dev, out)
        out_host.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws) / Ke
    e2e = {"value": ws * T / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": T * spec.n_embd * 4,
           "d2h_bytes_per_step": T * spec.n_embd * 4, "ms_per_step": e2e_ms}
    assert api.device_status() == 0

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(synth.make_layer(spec, 0, "cpu"), xs[0].cpu().numpy(), args.cpu_seconds)

    if rank == 0:
        # router GEMV, top-k (+ q8_1), dispatch, gate/up, [SwiGLU], down, combine; the tensor-core path adds the
        # hi/lo activation image and fuses SwiGLU into gate/up
        if tc:
            launches_per_step = 7
        else:
            launches_per_step = 7 + (0 if spec.sg_type == spec.gu_type else 2) + \
                (0 if spec.sd_type == spec.d_type else 2)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
                "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": ("fp16 x fp16 tcgen05 (exact hi/lo q8_1 image), f32 accumulate" if tc
                          else "int8 x int2 dot (q8_1 contract), f32/f64 sums"), "data": "synthetic",
                "expert_path": "tensor cores (tcgen05)" if tc else "SIMT",
                "config": config_dict(args, spec, T, D_mean),
                "expert_weight_gbs": expert_gbs, "expert_weight_frac_of_peak": expert_gbs / hbm_peak,
                "roofline": {"bound": "hbm", "kernel": (KERNEL_OF_STAGE_TC if tc else KERNEL_OF_STAGE)[dominant],
                             "achieved": achieved,
                             "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
                             "frac": achieved / hbm_peak if achieved else None, "traffic": traffic,
                             "algorithmic_bytes_per_launch": dom_bytes, "ms_per_launch": dom_ms},
                "stage_ms_per_step": {s: v / K for s, v in stage_ms.items()},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": K * launches_per_step,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, ws, rank)
        return
    ws, rank, local = setup_dist(args)
    try:
        run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
