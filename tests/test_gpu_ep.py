"""Expert parallelism (smoe_ep_forward) against the single-GPU block on the same tokens.

Every rank's output, ids, weights and per-slot down rows must equal smoe_moe_forward's on the concatenated
tokens bit for bit: the exchange only moves rows, the owners run the same kernels over the same slots, and the
token's rank combines in router order.  On one GPU the ranks share the device and run phase by phase
(run_local_step); with two or more GPUs a second test runs one process per GPU over CUDA IPC."""
import os

import numpy as np
import pytest
import torch

from stratametal_b200 import api, ep, synth

pytestmark = pytest.mark.gpu


def single_reference(cuda, spec, xs, path):
    """smoe_moe_forward over all ranks' tokens at once (the whole expert pool on one device)."""
    api.set_expert_path(path)
    try:
        full = api.MoeLayer(synth.make_layer(spec, 0, cuda), sum(x.shape[0] for x in xs), cuda)
        x = torch.cat(xs)
        tr = full.make_trace(x.shape[0])
        out = full.forward(x, trace=tr)
        torch.cuda.synchronize()
    finally:
        api.set_expert_path(0)
    return out, tr


def run_group(cuda, spec, xs, max_tokens, path, steps=1):
    world = len(xs)
    views = ep.EpAreas.local(spec, world, max_tokens)
    api.set_expert_path(path)
    try:
        layers = [ep.EpLayer(ep.shard_layer(spec, 0, r, world, cuda), views[r], cuda) for r in range(world)]
        outs = [torch.full((max(x.shape[0], 1), spec.n_embd), 7.0, device=cuda) for x in xs]
        trs = [L.make_trace(max(x.shape[0], 1)) for L, x in zip(layers, xs)]
        api.device_status(clear=True)
        for _ in range(steps):
            ep.run_local_step(layers, xs, outs, trs)
        torch.cuda.synchronize()
        assert api.device_status() == 0
    finally:
        api.set_expert_path(0)
    return layers, views, outs, trs


def check_equal(xs, outs, trs, want, wtr):
    t0 = 0
    for x, o, tr in zip(xs, outs, trs):
        T = x.shape[0]
        if T == 0:
            assert torch.all(o == 7.0), "a rank without tokens wrote an output"
            continue
        sl = slice(t0, t0 + T)
        assert torch.equal(tr.ids[:T], wtr.ids[sl])
        assert torch.equal(tr.weights[:T], wtr.weights[sl])
        assert torch.equal(tr.parts[:T], wtr.parts[sl]), "routed down rows differ"
        assert torch.equal(o[:T], want[sl]), "block output differs"
        t0 += T


@pytest.mark.parametrize("world", [2, 4])
def test_ep_int8_tensor_cores_match_single(cuda, world):
    # the int8 tensor-core kernels (path 4) store the down rows to the token ranks and signal from their epilogue
    spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=10, seed=55)
    sizes = [16, 5, 0, 11][:world]
    xs = [synth.make_x(65 + r, n, spec.n_embd, cuda) for r, n in enumerate(sizes)]
    want, wtr = single_reference(cuda, spec, xs, 4)
    layers, views, outs, trs = run_group(cuda, spec, xs, 16, 4)
    check_equal(xs, outs, trs, want, wtr)
    views[0].close()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_simt_matches_single(cuda, world):
    spec = synth.LayerSpec(n_embd=1024, n_ff=256, n_expert=64, k=8, seed=51)
    sizes = [13, 0, 7, 16][:world]  # ragged, one rank without tokens
    xs = [synth.make_x(60 + r, n, spec.n_embd, cuda) for r, n in enumerate(sizes)]
    want, wtr = single_reference(cuda, spec, xs, 1)
    layers, views, outs, trs = run_group(cuda, spec, xs, 16, 1)
    check_equal(xs, outs, trs, want, wtr)
    views[0].close()


def test_ep_tensor_cores_match_single(cuda):
    spec, _ = synth.config_spec(2)
    sizes = [300, 212]
    xs = [synth.make_x(70 + r, n, spec.n_embd, cuda) for r, n in enumerate(sizes)]
    want, wtr = single_reference(cuda, spec, xs, 2)
    layers, views, outs, trs = run_group(cuda, spec, xs, 320, 2)
    check_equal(xs, outs, trs, want, wtr)
    views[0].close()


def test_ep_steps_and_graph_replay(cuda):
    """Several steps in a row (the flags count steps), then the whole local step captured once and replayed."""
    spec = synth.LayerSpec(n_embd=512, n_ff=128, n_expert=32, k=4, seed=53)
    world, Tm = 2, 8
    xa = [synth.make_x(80 + r, Tm, spec.n_embd, cuda) for r in range(world)]
    xb = [synth.make_x(90 + r, Tm, spec.n_embd, cuda) for r in range(world)]
    want_a, _ = single_reference(cuda, spec, xa, 1)
    want_b, _ = single_reference(cuda, spec, xb, 1)
    api.set_expert_path(1)
    views = ep.EpAreas.local(spec, world, Tm)
    try:
        layers = [ep.EpLayer(ep.shard_layer(spec, 0, r, world, cuda), views[r], cuda) for r in range(world)]
        xs = [torch.empty_like(x) for x in xa]
        outs = [torch.empty(Tm, spec.n_embd, device=cuda) for _ in range(world)]
        for x, src in zip(xs, xa):
            x.copy_(src)
        for _ in range(3):
            ep.run_local_step(layers, xs, outs)
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(outs), want_a)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="relaxed"):
            ep.run_local_step(layers, xs, outs)
        for src, want in ((xb, want_b), (xa, want_a), (xb, want_b)):
            for x, s in zip(xs, src):
                x.copy_(s)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(torch.cat(outs), want)
        del g
        assert api.device_status() == 0
    finally:
        api.set_expert_path(0)
        views[0].close()


def test_ep_absent_rank_times_out(cuda):
    """Rank 1 never takes part: rank 0's waits give up after their bound, record DEVICE_TIMEOUT and return; the
    device stays usable."""
    spec = synth.LayerSpec(n_embd=512, n_ff=128, n_expert=32, k=4, seed=57)
    views = ep.EpAreas.local(spec, 2, 4)
    L0 = ep.EpLayer(ep.shard_layer(spec, 0, 0, 2, cuda), views[0], cuda)
    x = synth.make_x(5, 4, spec.n_embd, cuda)
    api.device_status(clear=True)
    L0.forward(x)
    torch.cuda.synchronize()
    st = api.device_status(clear=True)
    assert st & 1, f"status {st:#x}: the wait for the absent rank must give up"
    # the device still works
    m = api.MoeLayer(synth.make_layer(spec, 0, cuda), 4, cuda)
    y = m.forward(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all() and api.device_status() == 0
    views[0].close()


def _two_gpu_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.cuda.set_stream(torch.cuda.Stream(dev))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=10, seed=61)
        Tm = 24
        sizes = [24, 17, 9, 24][:world]
        xs = [synth.make_x(100 + r, n, spec.n_embd, dev) for r, n in enumerate(sizes)]
        api.set_expert_path(4)  # the int8 tensor-core kernels, whose down epilogue stores to the other GPU
        full = api.MoeLayer(synth.make_layer(spec, 0, dev), sum(sizes), dev)
        want = full.forward(torch.cat(xs))
        areas = ep.EpAreas.distributed(spec, Tm)
        L = ep.EpLayer(ep.shard_layer(spec, 0, rank, world, dev), areas, dev)
        x = xs[rank]
        out = torch.empty(Tm, spec.n_embd, device=dev)
        dist.barrier()
        api.device_status(clear=True)
        for _ in range(4):
            L.forward(x, out)
        torch.cuda.synchronize()
        t0 = sum(sizes[:rank])
        ok = torch.equal(out[:sizes[rank]], want[t0:t0 + sizes[rank]]) and api.device_status() == 0
        dist.barrier()
        areas.close()
        q.put((rank, bool(ok), ""))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_over_ipc(cuda):
    import socket

    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
