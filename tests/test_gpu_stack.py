"""The layer stack of configs[3] (x = rms_norm(x + MoE_l(x)) per layer) against the oracle, and CUDA-graph
capture of smoe_moe_forward: replays of a captured forward must reproduce eager calls bit for bit."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import api, synth

from test_gpu_layer import host_layer

pytestmark = pytest.mark.gpu

EPS = 1e-6


def gpu_stack(layers, x, T, H):
    bufs = [torch.empty(T, H, device=x.device) for _ in range(2)]
    cur = x
    for li, m in enumerate(layers):
        nxt = bufs[li & 1]
        m.forward(cur, nxt)
        api.add_rms_norm(nxt, cur, None, T, H, EPS)
        cur = nxt
    return cur


def test_stack_vs_oracle(cuda):
    spec = synth.LayerSpec(n_embd=512, n_ff=128, n_expert=32, k=4, seed=31)
    T, H = 4, spec.n_embd
    lays = [synth.make_layer(spec, li, cuda) for li in range(3)]
    mods = [api.MoeLayer(lay, T, cuda) for lay in lays]
    x = synth.make_x(9, T, H, cuda)
    got = gpu_stack(mods, x, T, H).cpu().numpy()
    torch.cuda.synchronize()
    assert api.device_status() == 0
    want = O.moe_stack([host_layer(lay) for lay in lays], x.cpu().numpy(), EPS)
    assert O.rel_l1(want, got) <= 1e-5
    # every row leaves the norm with mean square 1
    assert np.allclose((got.astype(np.float64) ** 2).mean(axis=1), 1.0, atol=1e-4)


@pytest.mark.parametrize("path,T", [(1, 8), (2, 64), (0, 1)])  # SIMT, tensor cores, fused single token
def test_graph_replay_matches_eager(cuda, path, T):
    spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=10, seed=41)
    api.set_expert_path(path)
    try:
        m = api.MoeLayer(synth.make_layer(spec, 0, cuda), T, cuda)
        xa, xb = synth.make_x(1, T, 2048, cuda), synth.make_x(2, T, 2048, cuda)
        x = torch.empty_like(xa)
        out = torch.empty(T, 2048, device=cuda)
        eager = []
        for xi in (xa, xb):
            eager.append(m.forward(xi).clone())
        x.copy_(xa)
        m.forward(x, out)  # first call outside the capture (one-time set-up)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="relaxed"):
            m.forward(x, out)
        for xi, want in zip((xa, xb, xa), (eager[0], eager[1], eager[0])):
            x.copy_(xi)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        del g
        assert api.device_status() == 0
    finally:
        api.set_expert_path(0)
