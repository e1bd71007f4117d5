"""The tensor-core expert path (tcgen05 grouped GEMMs, smoe_set_expert_path(2)) against the oracle and against
the SIMT path on the same seeded inputs.

The tensor-core kernels multiply fp16 weights ((code - 1) * d, exact) by an exact hi/lo fp16 split of the q8_1
activation, accumulating in f32: each expert dot product equals the reference's integer contract up to the
order of the f32 additions.  That order still matters downstream: h is re-quantized to q8_1 before the down
product, and an h within a few f32 ulps of a rounding boundary lands on the other code (about 4e-5 of the h
values at these shapes), moving that slot's down output by one quantum.  So the checks are: ids, logits and the
q8_1 of x exact; at least half of the routed slots within the reference walk's stage bar (pack_parity.cpp:
8764-8768, 1e-5 rel_l1); the whole parts, shared and block outputs within 2e-4 rel_l1; and the block within
2e-3 of the host result normwise, the tolerance the MoE block is specified to."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import _lib, api, synth

from test_gpu_layer import bits, host_layer

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc_path():
    api.set_expert_path(2)
    yield
    api.set_expert_path(0)


def forward(cuda, lay, T, x, path):
    api.set_expert_path(path)
    m = api.MoeLayer(lay, T, cuda)
    assert _lib.lib().smoe_expert_path_for(C.byref(m.c), T) == (2 if path == 2 else 1)
    H = lay.spec.n_embd
    out = torch.full((T * H + 16,), 7.0, device=cuda)
    tr = m.make_trace(T)
    api.device_status(clear=True)
    m.forward(x, out[:T * H].view(T, H), tr)
    torch.cuda.synchronize()
    assert api.device_status() == 0
    got = out.cpu().numpy()
    assert np.all(got[T * H:] == 7.0), "wrote past the output"
    return got[:T * H].reshape(T, H), tr


def check_vs_oracle(cuda, spec, T, x_seed=1):
    lay = synth.make_layer(spec, 0, cuda)
    x = synth.make_x(x_seed, T, spec.n_embd, cuda)
    got, tr = forward(cuda, lay, T, x, 2)
    want, otr = O.moe_layer(host_layer(lay), x.cpu().numpy(), mode=0, trace=True)
    assert np.array_equal(bits(tr.logits.cpu().numpy()), bits(otr["logits"]))
    assert np.array_equal(tr.ids.cpu().numpy(), otr["ids"]), "expert ids must be exact"
    assert np.array_equal(tr.xq.cpu().numpy(), otr["xq"])
    gp, wp = tr.parts.cpu().numpy(), otr["parts"]
    per_slot = np.abs(gp - wp).sum(-1) / np.maximum(np.abs(wp).sum(-1), 1e-30)
    assert np.median(per_slot) <= 1e-5, "most slots must match to f32 summation order"
    assert O.rel_l1(wp, gp) <= 2e-4
    if spec.has_shared:
        assert O.rel_l1(otr["shared"], tr.shared.cpu().numpy()) <= 2e-4
    assert O.rel_l1(want, got) <= 2e-4
    assert np.abs(got - want).max() / np.abs(want).max() <= 2e-3
    return got, want


def test_tc_cfg1_zipf_b64(cuda, tc_path):
    spec, T = synth.config_spec(1)
    check_vs_oracle(cuda, spec, T)


def test_tc_single_token(cuda, tc_path):
    spec, _ = synth.config_spec(0)
    check_vs_oracle(cuda, spec, 1)


def test_tc_many_tokens_per_expert(cuda, tc_path):
    # 64 experts, 192 tokens, k 10: ~30 slots per expert, several experts above one 64-slot chunk, and the
    # shared expert in three chunks
    spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=10, seed=7)
    check_vs_oracle(cuda, spec, 192)


def test_tc_no_shared_wide_ff(cuda, tc_path):
    spec = synth.LayerSpec(n_embd=1024, n_ff=1024, n_expert=32, k=4, has_shared=False, seed=11)
    check_vs_oracle(cuda, spec, 40)


def test_tc_matches_simt_at_prefill_scale(cuda):
    # BASELINE shapes at 1024 tokens: the two GPU paths agree to f32 summation order
    spec, _ = synth.config_spec(2)
    T = 1024
    lay = synth.make_layer(spec, 0, cuda)
    x = synth.make_x(3, T, spec.n_embd, cuda)
    try:
        a, tra = forward(cuda, lay, T, x, 1)
        b, trb = forward(cuda, lay, T, x, 2)
    finally:
        api.set_expert_path(0)
    assert np.array_equal(tra.ids.cpu().numpy(), trb.ids.cpu().numpy())
    pa, pb = tra.parts.cpu().numpy(), trb.parts.cpu().numpy()
    per_slot = np.abs(pa - pb).sum(-1) / np.maximum(np.abs(pa).sum(-1), 1e-30)
    assert np.median(per_slot) <= 1e-5
    assert O.rel_l1(pa, pb) <= 2e-4
    assert O.rel_l1(a, b) <= 2e-4


def test_path_selection(cuda):
    spec, _ = synth.config_spec(1)
    m = api.MoeLayer(synth.make_layer(spec, 0, cuda), 8, cuda)
    f = _lib.lib().smoe_expert_path_for
    assert f(C.byref(m.c), 8) == 4 and f(C.byref(m.c), 4096) == 2 and f(C.byref(m.c), 1) == 3
    iq = synth.LayerSpec(n_embd=512, n_ff=512, n_expert=16, k=4, gu_type=synth.IQ2_S, seed=3)
    mi = api.MoeLayer(synth.make_layer(iq, 0, cuda), 8, cuda)
    assert f(C.byref(mi.c), 4096) == 1 and f(C.byref(mi.c), 8) == 1  # IQ2_S stays on the SIMT kernels
    with pytest.raises(api.SmoeError):
        api.set_expert_path(5)
