"""The int8 tensor-core expert path (tcgen05 kind::i8, smoe_set_expert_path(4)) against the SIMT kernels and the
oracle: both evaluate the reference's q8_1 integer contract in its summation order, so every per-slot down row,
the shared expert's output and the block output must agree bit for bit."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import _lib, api, synth

from test_gpu_layer import bits, host_layer

pytestmark = pytest.mark.gpu


def run(cuda, lay, x, path):
    T = x.shape[0]
    api.set_expert_path(path)
    try:
        m = api.MoeLayer(lay, T, cuda)
        assert _lib.lib().smoe_expert_path_for(C.byref(m.c), T) == path
        H = lay.spec.n_embd
        out = torch.full((T * H + 16,), 7.0, device=cuda)
        tr = m.make_trace(T)
        api.device_status(clear=True)
        m.forward(x, out[:T * H].view(T, H), tr)
        torch.cuda.synchronize()
        assert api.device_status() == 0
    finally:
        api.set_expert_path(0)
    got = out.cpu()
    assert torch.all(got[T * H:] == 7.0), "wrote past the output"
    return got[:T * H].view(T, H), tr


@pytest.mark.parametrize("H,F,E,k,T,shared", [
    (2048, 512, 512, 10, 64, True),     # configs[1] shapes
    (2048, 512, 64, 10, 200, True),     # experts with many 8-slot chunks
    (1024, 1024, 32, 4, 37, False),
    (512, 2048, 16, 4, 9, True),
    (512, 512, 8, 2, 2, True),
    (2048, 2048, 128, 8, 511, True),
])
def test_tq_equals_simt(cuda, H, F, E, k, T, shared):
    spec = synth.LayerSpec(n_embd=H, n_ff=F, n_expert=E, k=k, has_shared=shared, seed=H + F + E + T)
    lay = synth.make_layer(spec, 0, cuda)
    x = synth.make_x(11, T, H, cuda)
    a, tra = run(cuda, lay, x, 1)
    b, trb = run(cuda, lay, x, 4)
    assert torch.equal(tra.ids, trb.ids)
    assert torch.equal(tra.parts, trb.parts), "routed down rows differ"
    if shared:
        assert torch.equal(tra.shared, trb.shared), "shared expert differs"
    assert torch.equal(a, b), "block output differs"


def test_tq_cfg1_vs_oracle(cuda):
    spec, T = synth.config_spec(1)
    lay = synth.make_layer(spec, 0, cuda)
    x = synth.make_x(3, T, spec.n_embd, cuda)
    got, tr = run(cuda, lay, x, 4)
    want, otr = O.moe_layer(host_layer(lay), x.cpu().numpy(), mode=0, trace=True)
    assert np.array_equal(tr.ids.cpu().numpy(), otr["ids"])
    assert np.array_equal(bits(tr.parts.cpu().numpy()), bits(otr["parts"]))
    assert np.array_equal(bits(got.numpy()), bits(want))
