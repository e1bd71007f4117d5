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


@pytest.mark.parametrize("H,F,E,k,L,weighted", [(2048, 512, 64, 10, 6, False), (2560, 640, 32, 10, 3, True),
                                                (512, 128, 16, 4, 50, False)])
def test_stack_decode_equals_layer_by_layer(cuda, H, F, E, k, L, weighted):
    # one launch per 48 layers (smoe_stack_decode) == L x (smoe_moe_forward + smoe_add_rms_norm), bit for bit
    spec = synth.LayerSpec(n_embd=H, n_ff=F, n_expert=E, k=k, seed=H + L)
    mods = [api.MoeLayer(synth.make_layer(spec, li, cuda), 1, cuda) for li in range(L)]
    assert api.expert_path_for(mods[0], 1) == 3
    x = synth.make_x(5, 1, H, cuda)
    norm_w = [1.0 + 0.1 * torch.randn(H, device=cuda) for _ in range(L)] if weighted else None
    bufs = [torch.empty(1, H, device=cuda) for _ in range(2)]
    cur = x
    for li, m in enumerate(mods):
        nxt = bufs[li & 1]
        m.forward(cur, nxt)
        api.add_rms_norm(nxt, cur, None if norm_w is None else norm_w[li], 1, H, EPS)
        cur = nxt
    out = torch.full((1, H + 8), 7.0, device=cuda)
    api.device_status(clear=True)
    api.stack_decode(mods, x, out[:, :H], EPS, norm_w)
    torch.cuda.synchronize()
    assert api.device_status() == 0
    assert torch.equal(out[:, :H], cur)
    assert torch.all(out[:, H:] == 7.0)
    # twice in a row (the barrier words are zeroed before every launch)
    out2 = torch.empty(1, H, device=cuda)
    api.stack_decode(mods, x, out2, EPS, norm_w)
    torch.cuda.synchronize()
    assert torch.equal(out2, cur)


def test_stack_decode_graph_replay(cuda):
    spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=10, seed=77)
    mods = [api.MoeLayer(synth.make_layer(spec, li, cuda), 1, cuda) for li in range(4)]
    xa, xb = synth.make_x(1, 1, 2048, cuda), synth.make_x(2, 1, 2048, cuda)
    want = [api.stack_decode(mods, xi, torch.empty(1, 2048, device=cuda)).clone() for xi in (xa, xb)]
    x, out = xa.clone(), torch.empty(1, 2048, device=cuda)
    scratch = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    api.stack_decode(mods, x, out, scratch=scratch)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="relaxed"):
        api.stack_decode(mods, x, out, scratch=scratch)
    for xi, w in ((xa, want[0]), (xb, want[1]), (xa, want[0])):
        x.copy_(xi)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, w)
    del g
