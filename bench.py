#!/usr/bin/env python
"""MoE-layer throughput of the B200 implementation (and, with --impl reference, of the reference's CPU path).

Headline workload: one MoE layer (hidden 2048, 512 experts of intermediate 512, top-10,
Q2_0 experts, sigmoid-gated shared expert), 64 decode tokens per step, Zipf(1.1) expert popularity.  A step is
one smoe_moe_forward over one batch: router, dispatch, expert products, combine.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C] [--subs LIST]

The same JSON line carries a sub-record per other BASELINE configuration ("configs"): configs[0] (one decode
token), configs[2] (4096-token prefill), configs[3] (the 48-layer stack at batch 1 and at batch 16) and configs[4]
(IQ2_S gate/up, batch 8), each timed the same way with the same K and W.

Timing: each step's smoe_moe_forward calls are captured once as a CUDA graph (one graph per (layer, batch)
forward; for configs[3] one graph for the whole 48-layer stack with its residual add + RMSNorm); W untimed
replays, then exactly K replays between CUDA events on the replay stream, bracketed by a barrier and a
synchronize, max over ranks.  Per-stage times come from a separate eager pass with stage events.  Each step's
expert bytes exceed the 126 MB L2 or the steps rotate over enough distinct seeded layers that they do, so
weights stream from HBM.  Rank 0 prints one JSON line.  N > 1 runs independent replicas for the decode configs
(decode does not shard: "replicas only"), value = all ranks' tokens / time; configs[2] and configs[3] at batch 16
run expert-parallel instead: the step's tokens split over the N ranks, E / N experts per rank, token rows and down
rows exchanged over peer memory inside smoe_ep_forward (strong scaling).

  python bench.py --config 3 [--tokens 16] --subs none   # the 48-layer stack at batch 1 (or 16) alone
  python bench.py --config 2 --subs none                 # 4096-token prefill alone
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

STACK_LAYERS = 48
RMS_EPS = 1e-6
METRIC = "MoE-layer tokens/s (decode b1/b64, prefill 4k); expert-weight HBM GB/s vs peak"
UNIT = "tokens/s"
STAGES = ["router_gemv", "router_topk_q8", "dispatch", "expert_gate_up", "expert_down", "combine"]
KERNEL_OF_STAGE = {"router_gemv": "bf16_gemv_kernel", "router_topk_q8": "router_topk_kernel",
                   "dispatch": "group_kernel", "expert_gate_up": "layer_gate_up_kernel",
                   "expert_down": "layer_down_kernel", "combine": "combine_kernel"}
KERNEL_OF_STAGE_TC = dict(KERNEL_OF_STAGE, expert_gate_up="tc_expert_kernel<0>", expert_down="tc_expert_kernel<1>")
KERNEL_OF_STAGE_TQ = dict(KERNEL_OF_STAGE, expert_gate_up="tq_expert_kernel<0>", expert_down="tq_expert_kernel<1>")
FUSED_KERNEL = "decode_stack_kernel"
# sub-records: name -> (config, tokens per step, single-layer configs: distinct layers x batches rotated)
SUBS = {"cfg0_b1": (0, 1, (16, 1)), "cfg2_prefill4096": (2, 4096, (2, 1)), "cfg3_stack48_b1": (3, 1, None),
        "cfg3_stack48_b16": (3, 16, None), "cfg4_iq2s_b8": (4, 8, (4, 4))}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4])
    ap.add_argument("--expert-path", type=int, default=0, choices=[0, 1, 2, 4],
                    help="0 automatic, 1 SIMT expert kernels, 2 fp16 tensor-core kernels, 4 int8 tensor-core kernels")
    ap.add_argument("--layers", type=int, default=4, help="distinct layers rotated through the headline's steps")
    ap.add_argument("--tokens", type=int, default=0, help="override the config's tokens per step (configs[3]: 1 or 16)")
    ap.add_argument("--subs", default="auto",
                    help="sub-records to add: 'auto' (every other config when the headline is configs[1]), 'none', "
                         "or a comma list of " + ",".join(SUBS))
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    if a.subs == "auto":
        a.sub_list = list(SUBS) if (a.config == 1 and not a.tokens and a.expert_path == 0) else []
    elif a.subs == "none":
        a.sub_list = []
    else:
        a.sub_list = [s for s in a.subs.split(",") if s]
        for s in a.sub_list:
            if s not in SUBS:
                raise SystemExit(f"unknown sub-record {s}")
    return a


# ---------------------------------------------------------------------------------------------------
# clocks during the timed regions (read-only NVML queries)
# ---------------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples the SM clock and the throttle reasons every few milliseconds while a timed region is open
    (`with sampler.timed(): ...`), over every timed region of the run."""
    REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
               "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int, period: float = 0.004):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period, self.stop_flag, self.active = period, threading.Event(), threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = str(e)
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def _sample(self):
        nv = self.nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            for name, bit in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    self.reasons.add(name)
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self.stop_flag.is_set():
            if self.active.is_set():
                self._sample()
            time.sleep(self.period)

    @contextlib.contextmanager
    def timed(self):
        self.active.set()
        try:
            yield
        finally:
            self.active.clear()
            if self.ok:
                self._sample()  # at least one sample per timed region, however short

    def stop(self):
        if self.ok:
            self.stop_flag.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "err", "no samples")}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples),
                "window": "every timed region of this run (headline and sub-records)"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


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


def cpu_baseline(lay, x_host, seconds: float, n_layers: int = 1):
    """The reference's CPU path on this host: layer 0 on the step's tokens, repeated within the time budget.  For
    the stack the per-layer time is multiplied by the layer count (every layer has the same shape)."""
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
    per_step = el / n * n_layers
    sample = f"{n} layer calls of the bench workload ({T} tokens each, layer 0), {el:.1f} s"
    if n_layers > 1:
        sample += f"; tokens/s for the stack = T / ({n_layers} x the per-layer time)"
    return {"value": T / per_step, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample}


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


def schedule(K: int, n_layers: int, n_batches: int) -> list[tuple[int, int]]:
    """The (layer, batch) forward that timed step i replays, for the first K steps."""
    return [(i % n_layers, (i // n_layers) % n_batches) for i in range(K)]


def config_dict(gpus, cfg, spec, T, D_mean, n_layers, n_batches, stack=False):
    if stack:
        return {"workload": f"configs[3]: stack of {n_layers} MoE layers (residual add + RMSNorm between them), "
                            f"{T} decode tokens/step",
                "tokens_per_step": T, "layers": n_layers, "n_embd": spec.n_embd, "n_ff": spec.n_ff,
                "n_expert": spec.n_expert, "top_k": spec.k, "expert_format": "Q2_0", "shared_expert": True,
                "distinct_experts_per_layer": D_mean, "rms_eps": RMS_EPS,
                "l2": "inputs larger than L2: one step streams every layer's routed experts (> 400 MB)",
                "parallelism": f"replicas x{gpus}", "seed": spec.seed}
    return {"workload": f"configs[{cfg}]: one MoE layer, {T} {'decode' if T <= 64 else 'prefill'} tokens/step"
                        + (", Zipf(1.1) expert popularity" if spec.zipf else "")
                        + (", IQ2_S gate/up" if spec.gu_type == 22 else ""),
            "tokens_per_step": T, "n_embd": spec.n_embd, "n_ff": spec.n_ff, "n_expert": spec.n_expert,
            "top_k": spec.k, "expert_format": "IQ2_S gate/up + Q2_0 down" if spec.gu_type == 22 else "Q2_0",
            "shared_expert": True, "distinct_experts_per_step": D_mean, "layers_rotated": n_layers,
            "batches_rotated": n_batches,
            "l2": "inputs larger than L2: the (layer, batch) forwards a step cycles through stream > 126 MB of "
                  "expert weights",
            "parallelism": f"replicas x{gpus}", "seed": spec.seed}


def reference_distinct_experts(spec, T, n_layers, n_batches, K):
    """The mean number of distinct routed experts per step of the headline schedule, from the oracle's router
    stage on the same seeded routers and tokens (the GPU arm reads the same figure from its own traces)."""
    import numpy as np

    from oracle import oracle as O
    from stratametal_b200 import synth
    D = {}
    for li in range(n_layers):
        r = synth.router_weights(spec, li, "cpu").numpy().view(np.uint16)
        for b in range(n_batches):
            x = synth.make_x(spec.seed, T, spec.n_embd, "cpu", stream=b).numpy()
            D[(li, b)] = int(np.unique(O.router(r, x, spec.k)[1]).size)
    return float(np.mean([D[s] for s in schedule(K, n_layers, n_batches)]))


def run_reference(args, ws, rank):
    """--impl reference: the reference's CPU implementation on this host's cores (rank 0 only)."""
    import numpy as np

    from stratametal_b200 import synth
    if rank != 0:
        return
    spec, T = synth.config_spec(args.config)
    if args.tokens:
        T = args.tokens
    stack = args.config == 3
    n_layers, n_batches = (STACK_LAYERS, 1) if stack else (args.layers, 4)
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
    if stack:  # the stack's layers share one shape: tokens/s through all of them
        value /= STACK_LAYERS
        sample += f"; stack tokens/s = layer tokens/s / {STACK_LAYERS}"
    D_mean = None if stack else reference_distinct_experts(spec, T, n_layers, n_batches, args.steps)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int2 dot, f32/f64 sums", "data": "synthetic",
            "config": config_dict(args.gpus, args.config, spec, T, D_mean, n_layers, n_batches, stack),
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------------
def measure(args, ws, rank, local, clk, cfg, T_req, rot):
    """Times one configuration; returns its record (rank 0) after releasing its device memory.  rot = (distinct
    layers, batches) rotated through the steps of a single-layer config; None for the stack."""
    import ctypes as C

    import numpy as np
    import torch

    from stratametal_b200 import api, synth
    from stratametal_b200._lib import lib
    dev = torch.device("cuda", local)
    spec, T = synth.config_spec(cfg)
    if T_req:
        T = T_req
    H = spec.n_embd
    stack = cfg == 3
    n_layers, n_batches = (STACK_LAYERS, 1) if stack else rot
    # expert parallelism for the batched and prefill workloads on N > 1 GPUs: the step's tokens split evenly over
    # the ranks (strong scaling), E / N routed experts per rank, the exchange inside smoe_ep_forward
    ep_mode = ws > 1 and (cfg == 2 or (stack and T > 1))
    T_all = T
    areas = None
    if ep_mode:
        from stratametal_b200 import ep
        if T % ws:
            raise SystemExit(f"{T} tokens do not split over {ws} ranks")
        T = T // ws
        areas = ep.EpAreas.distributed(spec, T)
        layers = [ep.EpLayer(ep.shard_layer(spec, li, rank, ws, dev), areas, dev) for li in range(n_layers)]
        path = lib().smoe_expert_path_for(C.byref(layers[0].c), T_all)
        xs = [synth.make_x(spec.seed, T_all, H, dev, stream=b)[rank * T:(rank + 1) * T].contiguous()
              for b in range(n_batches)]
    else:
        layers = [api.MoeLayer(synth.make_layer(spec, li, dev), T, dev) for li in range(n_layers)]
        path = lib().smoe_expert_path_for(C.byref(layers[0].c), T)
        xs = [synth.make_x(spec.seed + 1000 * local, T, H, dev, stream=b) for b in range(n_batches)]
    tc, fused, tq = path == 2, path == 3, path == 4
    out = torch.empty(T, H, device=dev)
    stream = torch.cuda.current_stream()
    # the stack ping-pongs between two buffers: layer l reads cur, writes MoE(cur) to nxt, then
    # nxt = rms_norm(nxt + cur)
    sbuf = [torch.empty(T, H, device=dev) for _ in range(2)]

    def forward_once(li, b, dst):
        layers[li].forward(xs[b], dst)

    # the batch-1 stack runs as one persistent launch per 48 layers (smoe_stack_decode) when its layers qualify
    stack_kernel = stack and fused and not ep_mode
    stack_scratch = torch.empty(1 << 20, dtype=torch.uint8, device=dev) if stack_kernel else None

    def stack_once():
        if stack_kernel:
            return api.stack_decode(layers, xs[0], sbuf[(n_layers - 1) & 1], RMS_EPS, scratch=stack_scratch)
        cur = xs[0]
        for li in range(n_layers):
            nxt = sbuf[li & 1]
            layers[li].forward(cur, nxt)
            api.add_rms_norm(nxt, cur, None, T, H, RMS_EPS)
            cur = nxt
        return cur

    # distinct experts per (layer, batch), for the algorithmic bytes (eager, with a trace)
    D = {}
    cur = xs[0]
    for li, m in enumerate(layers):
        for b in range(n_batches):
            tr = m.make_trace(T)
            xin = cur if stack else xs[b]
            m.forward(xin, out, tr)
            if ep_mode:  # the experts of this rank that any rank's tokens reach
                import torch.distributed as dist
                allids = [torch.empty_like(tr.ids) for _ in range(ws)]
                dist.all_gather(allids, tr.ids)
                u = torch.unique(torch.cat(allids))
                lo_e = rank * (spec.n_expert // ws)
                D[(li, b)] = int(((u >= lo_e) & (u < lo_e + spec.n_expert // ws)).sum())
            else:
                D[(li, b)] = int(torch.unique(tr.ids).numel())
            if stack:  # follow the stack's own activations
                api.add_rms_norm(out, xin, None, T, H, RMS_EPS)
                cur = out.clone()
    torch.cuda.synchronize()
    assert api.device_status() == 0

    # one CUDA graph per step kind: every (layer, batch) forward, or the whole stack
    G = 1 if stack else n_layers * n_batches
    # each single-layer graph reads and writes buffers of its own (its batch's tokens), so consecutive steps never
    # share one and the end-to-end loop below can upload the next step's input while this one computes
    g_in = [xs[0]] if stack else [xs[(gi // n_layers) % n_batches].clone() for gi in range(G)]
    g_out = [sbuf[(n_layers - 1) & 1]] if stack else [torch.empty(T, H, device=dev) for _ in range(G)]
    graphs = []
    for gi in range(G):
        g = torch.cuda.CUDAGraph()
        for _ in range(2):  # warm the allocator and any first-call set-up outside the capture
            stack_once() if stack else layers[gi % n_layers].forward(g_in[gi], g_out[gi])
        torch.cuda.synchronize()
        with torch.cuda.graph(g, capture_error_mode="relaxed"):
            stack_once() if stack else layers[gi % n_layers].forward(g_in[gi], g_out[gi])
        g.replay()  # set-up, not a step: a graph's first launch uploads it to the device
        graphs.append(g)
    torch.cuda.synchronize()
    gstream = torch.cuda.current_stream()

    K, W = args.steps, args.warmup
    for i in range(W):
        graphs[i % G].replay()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    with clk.timed():
        start.record(gstream)
        for i in range(K):
            graphs[i % G].replay()
        end.record(gstream)
        torch.cuda.synchronize()
    barrier(ws)
    el_ms = max_over_ranks(start.elapsed_time(end), ws)
    ms_step = el_ms / K
    value = ws * T / (ms_step * 1e-3)
    assert api.device_status() == 0

    # per-stage device time: an eager pass with stage events (single layers, one rank per layer)
    stage_ms = None
    if not stack and not ep_mode:
        Ks = min(K, 500)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(STAGES) + 1)] for _ in range(Ks)]
        for row in ev:  # torch creates the CUDA event on its first record
            for e in row:
                e.record(stream)
        handles = [(C.c_void_p * len(STAGES))(*[e.cuda_event for e in row[1:]]) for row in ev]
        torch.cuda.synchronize()
        for i in range(Ks):
            ev[i][0].record(stream)
            lib().smoe_set_stage_events(handles[i], len(STAGES))
            forward_once(i % n_layers, (i // n_layers) % n_batches, out)
        lib().smoe_set_stage_events(None, 0)
        torch.cuda.synchronize()
        stage_ms = {s: 0.0 for s in STAGES}
        for i in range(Ks):
            for j, s in enumerate(STAGES):
                stage_ms[s] += ev[i][j].elapsed_time(ev[i][j + 1]) / Ks

    hbm_peak, tensor_peak, peak_kind = peaks()
    E_BYTES = spec.expert_bytes()
    rbg = synth.row_bytes(spec.gu_type, spec.n_embd) * spec.n_ff
    rbd = synth.row_bytes(spec.d_type, spec.n_ff) * spec.n_embd
    q8x, q8h = (spec.n_embd // 32) * 36, (spec.n_ff // 32) * 36
    rows = T * spec.k + T  # slots per rank (in expectation the same with expert parallelism)
    flop_gu = 2.0 * rows * 2 * spec.n_embd * spec.n_ff   # useful FLOPs of the gate/up products
    flop_dn = 2.0 * rows * spec.n_embd * spec.n_ff
    if stack:
        Ds = [D[(li, 0)] for li in range(n_layers)]
        step_bytes = float(sum((d + 1) * E_BYTES for d in Ds))
        D_mean = float(np.mean(Ds))
        expert_gbs = step_bytes / (ms_step * 1e-3) / 1e9 * (ws if ep_mode else 1)
        roof = {"bound": "hbm", "kernel": ("decode_stack_kernel (the whole stack, one launch)" if stack_kernel else
                                           f"whole {n_layers}-layer stack (CUDA graph"
                                           + (f", {ws} ranks" if ep_mode else "") + ")"),
                "achieved": expert_gbs, "peak": hbm_peak * (ws if ep_mode else 1), "peak_kind": peak_kind,
                "unit": "GB/s", "frac": expert_gbs / (hbm_peak * (ws if ep_mode else 1)), "traffic": None,
                "algorithmic_bytes_per_launch": step_bytes, "ms_per_launch": ms_step,
                "per_layer_us": 1e3 * ms_step / n_layers}
    elif ep_mode:
        Ds = [D[s] for s in schedule(K, n_layers, n_batches)]
        D_mean = float(np.mean(Ds))
        flops = ws * (flop_gu + flop_dn)
        achieved = flops / (ms_step * 1e-3) / 1e12
        expert_gbs = ws * (D_mean + 1) * E_BYTES / (ms_step * 1e-3) / 1e9
        roof = {"bound": "tensor", "kernel": f"whole expert-parallel step over {ws} ranks",
                "achieved": achieved, "peak": tensor_peak * ws, "peak_kind": peak_kind + " (bf16 dense, burst)",
                "unit": "TFLOP/s", "frac": achieved / (tensor_peak * ws), "traffic": None,
                "algorithmic_flops_per_launch": flops, "ms_per_launch": ms_step}
    else:
        Ds = [D[s] for s in schedule(K, n_layers, n_batches)]
        D_mean = float(np.mean(Ds))
        alg = {"expert_gate_up": lambda d: (d + 1) * 2 * rbg + T * q8x + rows * q8h,
               "expert_down": lambda d: (d + 1) * rbd + rows * q8h + rows * spec.n_embd * 4,
               "router_gemv": lambda d: spec.n_expert * spec.n_embd * 2 + T * spec.n_embd * 4 + T * spec.n_expert * 4,
               "combine": lambda d: rows * spec.n_embd * 4 + T * spec.n_embd * 4}
        if fused:  # one kernel for the whole block: its bytes are the router's and the experts'
            dominant = "fused"
            alg["fused"] = lambda d: (d + 1) * E_BYTES + spec.n_expert * spec.n_embd * 2
            stage_ms = {"fused_block": sum(stage_ms.values())}
            dom_ms = ms_step  # the step is this one kernel: its duration is the timed replays' (the eager stage
            # events around a lone launch add the launch latency)
        else:
            dominant = max(stage_ms, key=stage_ms.get)
            dom_ms = stage_ms[dominant]
        expert_gbs = (D_mean + 1) * E_BYTES / (ms_step * 1e-3) / 1e9
        kos = KERNEL_OF_STAGE_TC if tc else KERNEL_OF_STAGE_TQ if tq else KERNEL_OF_STAGE
        if 2 <= T <= 64:
            kos = dict(kos, router_gemv="router_gemm_kernel (split K; the top-k launch adds the partials)")
        kname = FUSED_KERNEL if fused else kos[dominant]
        if tc and dominant in ("expert_gate_up", "expert_down"):
            flops = flop_gu if dominant == "expert_gate_up" else flop_dn
            achieved = flops / (dom_ms * 1e-3) / 1e12
            roof = {"bound": "tensor", "kernel": kname, "achieved": achieved, "peak": tensor_peak,
                    "peak_kind": peak_kind + " (bf16 dense, burst)", "unit": "TFLOP/s",
                    "frac": achieved / tensor_peak, "traffic": None, "algorithmic_flops_per_launch": flops,
                    "ms_per_launch": dom_ms,
                    "hbm_gbs_of_weights": float(np.mean([alg[dominant](d) for d in Ds])) / (dom_ms * 1e-3) / 1e9}
        else:
            dom_bytes = float(np.mean([alg[dominant](d) for d in Ds])) if dominant in alg else None
            achieved = dom_bytes / (dom_ms * 1e-3) / 1e9 if dom_bytes else None
            tpu = traffic_per_unit()
            traffic = None
            if dominant == "expert_gate_up" and not tc and not tq and "expert_gate_up_per_expert" in tpu:
                traffic = tpu["expert_gate_up_per_expert"] * (D_mean + 1)
            elif dominant == "expert_gate_up" and tq and "tq_gate_up_per_expert" in tpu:
                traffic = tpu["tq_gate_up_per_expert"] * (D_mean + 1)
            roof = {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm_peak, "peak_kind": peak_kind,
                    "unit": "GB/s", "frac": achieved / hbm_peak if achieved else None, "traffic": traffic,
                    "algorithmic_bytes_per_launch": dom_bytes, "ms_per_launch": dom_ms}

    # end to end: every step uploads its input from pinned host memory into the buffer its captured forward reads,
    # replays the captured API calls and reads its result back into pinned host memory, all inside the timed
    # region.  The copies run on two copy streams, pipelined with the replays as a serving loop runs them: step
    # i + 1's upload and step i - 1's read-back overlap step i's compute.  A step's upload waits until the previous
    # step that used the same buffers has been read back (events), and each replay waits for its own upload.
    x_host = [t.cpu().pin_memory() for t in g_in]
    out_host = [torch.empty(T, H).pin_memory() for _ in range(2)]
    hs, ds = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    Ke = min(K, 1000)
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    go = torch.cuda.Event()
    # one event of each kind per buffer set, created and first recorded here, outside the timed loop (a stream wait
    # takes an event's latest record, so each is recorded again for every step that uses its buffers)
    up_ev, done_ev, rb_ev = ([torch.cuda.Event() for _ in range(G)] for _ in range(3))
    for evs in (up_ev, done_ev, rb_ev, [go]):
        for ev in evs:
            ev.record(gstream)
    torch.cuda.synchronize()
    e0.record(gstream)
    go.record(gstream)
    hs.wait_event(go)
    ds.wait_event(go)
    drv = _driver_calls(graphs)
    if drv is not None:  # the same operations through the driver API, so the Python loop stays off the critical path
        d, execs = drv
        gs_h, hs_h, ds_h = gstream.cuda_stream, hs.cuda_stream, ds.cuda_stream
        up_h, done_h, rb_h = ([e.cuda_event for e in evs] for evs in (up_ev, done_ev, rb_ev))
        nbytes = T * H * 4
        in_p, out_p = [t.data_ptr() for t in g_in], [t.data_ptr() for t in g_out]
        xh_p, oh_p = [t.data_ptr() for t in x_host], [t.data_ptr() for t in out_host]
        bad = 0
        for i in range(Ke):
            gi = i % G
            bad |= d.cuStreamWaitEvent(hs_h, rb_h[gi], 0)
            bad |= d.cuMemcpyHtoDAsync_v2(in_p[gi], xh_p[gi], nbytes, hs_h)
            bad |= d.cuEventRecord(up_h[gi], hs_h)
            bad |= d.cuStreamWaitEvent(gs_h, up_h[gi], 0)
            bad |= d.cuGraphLaunch(execs[gi], gs_h)
            bad |= d.cuEventRecord(done_h[gi], gs_h)
            bad |= d.cuStreamWaitEvent(ds_h, done_h[gi], 0)
            bad |= d.cuMemcpyDtoHAsync_v2(oh_p[i % 2], out_p[gi], nbytes, ds_h)
            bad |= d.cuEventRecord(rb_h[gi], ds_h)
        if bad:
            raise RuntimeError("end-to-end loop: a CUDA driver call failed")
    for i in range(Ke if drv is None else 0):
        gi = i % G
        with torch.cuda.stream(hs):
            hs.wait_event(rb_ev[gi])  # the previous step on these buffers has been read back
            g_in[gi].copy_(x_host[gi], non_blocking=True)
            up_ev[gi].record(hs)
        gstream.wait_event(up_ev[gi])
        graphs[gi].replay()
        done_ev[gi].record(gstream)
        with torch.cuda.stream(ds):
            ds.wait_event(done_ev[gi])
            out_host[i % 2].copy_(g_out[gi], non_blocking=True)
            rb_ev[gi].record(ds)
    gstream.wait_stream(hs)
    gstream.wait_stream(ds)
    e1.record(gstream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws) / Ke
    e2e = {"value": ws * T / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
           "d2h_bytes_per_step": T * H * 4, "ms_per_step": e2e_ms,
           "how": "per step: H2D of the input from pinned memory, replay of the captured smoe_moe_forward calls, "
                  "D2H of the output; the copies on two copy streams, overlapping the neighbouring steps' compute"}
    assert api.device_status() == 0

    # router (GEMV, or split-K GEMM from 2 to 64 tokens, whose partials the top-k launch adds), top-k, grouping
    # (3 launches above 256 tokens), gate/up, SwiGLU (SIMT only), down, combine; the fp16 tensor-core path adds the
    # hi/lo image
    router_l = 1
    group_l = 3 if T > 256 else 1
    if tc:
        per_fwd = router_l + 1 + 1 + group_l + 3
    elif tq:
        per_fwd = router_l + 1 + group_l + 3
    else:
        per_fwd = router_l + 1 + group_l + 4 + (0 if spec.sg_type == spec.gu_type else 2) + \
            (0 if spec.sd_type == spec.d_type else 2)
    if fused:
        per_fwd = 1
    if ep_mode:  # router, top-k, dispatch, receive, grouping over the ws * T received rows, experts, wait, combine
        per_fwd = router_l + 1 + 1 + 1 + (3 if ws * T > 256 else 1) + (2 if tc or tq else 3) + 1 + 1
    launches_per_step = n_layers * (per_fwd + 1) if stack else per_fwd
    if stack_kernel:
        launches_per_step = (n_layers + 47) // 48

    cfgd = config_dict(args.gpus, cfg, spec, T_all, D_mean, n_layers, n_batches, stack)
    if ep_mode:
        cfgd["parallelism"] = (f"expert parallel x{ws}: {spec.n_expert // ws} routed experts and {T} of the "
                               f"{T_all} tokens per GPU; dispatch and return over peer memory (CUDA IPC, "
                               f"NVLink), no collective on the data path")
        cfgd["distinct_experts_per_step"] = f"{D_mean} on rank 0 (of its {spec.n_expert // ws})"
    rec = {"value": value, "unit": UNIT, "ms_per_step": ms_step, "n_gpus": ws,
           "scaling": "strong" if ep_mode else "weak",
           "dtype": ("fp16 x fp16 tcgen05 (exact hi/lo q8_1 image), f32 accumulate" if tc
                     else "int8 x int8 tcgen05 (q8_1 contract, s32 per 32-value partial), f32 epilogue in the "
                          "reference's order" if tq
                     else "int8 x int2 dot (q8_1 contract), f32/f64 sums"),
           "expert_path": ("fp16 tensor cores (tcgen05)" if tc else "int8 tensor cores (tcgen05 kind::i8)" if tq
                           else "fused single-token stack kernel (one cooperative launch for the 48 layers)"
                           if stack_kernel else "fused single-token kernel (one cooperative launch)" if fused
                           else "SIMT"),
           "config": cfgd,
           "timing": "CUDA events around CUDA-graph replays (one captured forward per step"
                     + (", the whole 48-layer stack" if stack else "") + ")",
           "expert_weight_gbs": expert_gbs, "expert_weight_frac_of_peak": expert_gbs / (hbm_peak * (ws if ep_mode else 1)),
           "roofline": roof, "stage_ms_per_step": stage_ms, "e2e": e2e, "gpu_launches_per_step": launches_per_step,
           "gpu_launches": K * launches_per_step, "_T": T, "_spec": spec, "_x0": xs[0].cpu().numpy(),
           "_n_layers": n_layers}

    # release this configuration's graphs and buffers before the next one
    del graphs
    torch.cuda.synchronize()
    barrier(ws)
    if areas is not None:  # every rank's kernels are done before any rank unmaps or frees an exchange area
        areas.close()
    del layers, xs, out, sbuf
    torch.cuda.empty_cache()
    barrier(ws)
    return rec


def public(rec: dict) -> dict:
    return {k: v for k, v in rec.items() if not k.startswith("_")}


def run_ours(args, ws, rank, local):
    import torch

    from stratametal_b200 import api, build, synth
    build.build()
    dev = torch.device("cuda", local)
    torch.cuda.set_stream(torch.cuda.Stream(dev))  # the C ABI wants an explicit non-null stream
    api.set_expert_path(args.expert_path)
    clk = ClockSampler(local)
    try:
        rot = (STACK_LAYERS, 1) if args.config == 3 else (args.layers, 4)
        head = measure(args, ws, rank, local, clk, args.config, args.tokens, rot)
        subs = {}
        for name in args.sub_list:
            cfg, T, srot = SUBS[name]
            subs[name] = measure(args, ws, rank, local, clk, cfg, T, srot)
    finally:
        clk.stop()

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        spec = head["_spec"]
        cpu = cpu_baseline(synth.make_layer(spec, 0, "cpu"), head["_x0"], args.cpu_seconds,
                           head["_n_layers"] if args.config == 3 else 1)

    if rank == 0:
        K, W = args.steps, args.warmup
        line = {"metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
                "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": head["scaling"],
                "vs_baseline": None, "dtype": head["dtype"], "data": "synthetic", "expert_path": head["expert_path"],
                "config": head["config"], "timing": head["timing"], "expert_weight_gbs": head["expert_weight_gbs"],
                "expert_weight_frac_of_peak": head["expert_weight_frac_of_peak"], "roofline": head["roofline"],
                "stage_ms_per_step": head["stage_ms_per_step"], "cpu_baseline": cpu, "e2e": head["e2e"],
                "gpu_launches": head["gpu_launches"], "clocks": clk.summary()}
        if subs:
            line["configs"] = {name: public(r) for name, r in subs.items()}
        print(json.dumps(line), flush=True)


def _driver_calls(graphs):
    """The CUDA driver entry points the end-to-end loop issues (through ctypes) and the graphs' executable handles,
    or None when either is unavailable (the loop then goes through torch)."""
    import ctypes as C
    try:
        d = C.CDLL("libcuda.so.1")
        execs = [g.raw_cuda_graph_exec() for g in graphs]
    except (OSError, AttributeError, RuntimeError):
        return None
    if any(not isinstance(e, int) or not e for e in execs):
        return None
    sig = {"cuStreamWaitEvent": [C.c_void_p, C.c_void_p, C.c_uint],
           "cuMemcpyHtoDAsync_v2": [C.c_uint64, C.c_void_p, C.c_size_t, C.c_void_p],
           "cuMemcpyDtoHAsync_v2": [C.c_void_p, C.c_uint64, C.c_size_t, C.c_void_p],
           "cuEventRecord": [C.c_void_p, C.c_void_p],
           "cuGraphLaunch": [C.c_void_p, C.c_void_p]}
    for name, args in sig.items():
        f = getattr(d, name)
        f.argtypes = args
        f.restype = C.c_int
    return d, execs


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
