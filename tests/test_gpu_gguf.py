"""The model boundary on the B200: MoE layers read from a GGUF file by tensor name (smoe_gguf_load_layer, the
reference's FfnExec::load over blk.<L>.* names, layer_exec.cpp:369-452) run the same block as the same planes given
directly, bit for bit, at the reference model's own geometry (n_embd 2560, n_ff 640, layout.hpp:43-53)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import api, synth

from test_gpu_layer import bits, host_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gu,d,T", [(O.Q2_0, O.Q2_0, 1), (O.Q2_0, O.Q2_0, 6), (O.IQ3_S, O.IQ4_NL, 3)])
def test_gguf_layers_at_model_geometry(cuda, tmp_path, gu, d, T):
    spec = synth.LayerSpec(n_embd=2560, n_ff=640, n_expert=32, k=10, gu_type=gu, d_type=d, sg_type=gu, su_type=gu,
                           sd_type=d, seed=640 + gu)
    lays = [synth.make_layer(spec, li) for li in range(2)]
    path = tmp_path / "model.gguf"
    synth.write_gguf(path, synth.layer_gguf_tensors(lays[0], 0) + synth.layer_gguf_tensors(lays[1], 1, router_f32=True),
                     {"general.architecture": "qwen4exp", "qwen4exp.expert_used_count": 10})
    model = api.GgufModel(path)
    x = synth.make_x(11, T, 2560, cuda)
    try:
        for li in range(2):
            g = model.load_layer(li, with_shared=True)
            assert (g.c.n_embd, g.c.n_ff, g.c.n_expert, g.c.k) == (2560, 640, 32, 10)
            api.device_status(clear=True)
            got = g.forward(x)
            direct = api.MoeLayer(synth.Layer(spec, li, lays[li].tensors), T, cuda).forward(x)
            torch.cuda.synchronize()
            assert api.device_status() == 0
            assert torch.equal(got, direct), f"layer {li}"
            want = O.moe_layer(host_layer(lays[li]), x.cpu().numpy())
            assert np.array_equal(bits(got.cpu().numpy()), bits(want)), f"layer {li} vs the oracle"
            g.close()
    finally:
        model.close()
