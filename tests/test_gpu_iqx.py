"""The other expert formats of the reference's MMVQ family (IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S) on the B200: the
stage entry point smoe_iq_mmvq and the any-format layer path of smoe_moe_forward (iqx.cu), bitwise against the
reference's own results (golden rows and expert pairs, iq_parity.cpp:153-222, 504-539) and the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import api, synth

from test_gpu_layer import bits, check_block, run_case
from test_oracle import PAIRS

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("name,t,n_in", [("iq3xxs_2048", O.IQ3_XXS, 2048), ("iq3s_2048", O.IQ3_S, 2048)])
def test_mmvq_iq3_golden_bitwise(golden, cuda, name, t, n_in):
    w, xq, want = golden[f"dot_{name}_w"], golden[f"dot_{name}_x"], golden[f"dot_{name}_y"]
    y = torch.full((want.size + 16,), 7.0, device=cuda)
    api.iq_mmvq(t, dev(w, cuda), dev(xq, cuda), n_in, want.size, 1, y)
    got = y.cpu().numpy()
    assert np.array_equal(bits(got[:want.size]), bits(want))
    assert np.all(got[want.size:] == 7.0), "wrote past the output"


@pytest.mark.parametrize("t,n_in,n_out,n_col", [(O.IQ3_XXS, 2048, 70, 3), (O.IQ3_XXS, 256, 9, 2),
                                                (O.IQ3_S, 4096, 33, 2), (O.IQ3_S, 512, 40, 3)])
def test_mmvq_iq3_random_bitwise(cuda, t, n_in, n_out, n_col):
    w = synth.quant_matrix(t, 1000 + n_in + n_out, n_out, n_in, "cpu").numpy()
    xq = O.quant_q8_1(np.random.default_rng(n_in).standard_normal(n_col * n_in).astype(np.float32))
    y = torch.empty(n_col * n_out, device=cuda)
    api.iq_mmvq(t, dev(w, cuda), dev(xq, cuda), n_in, n_out, n_col, y)
    assert np.array_equal(bits(y.cpu().numpy()), bits(O.mmvq(t, w, xq, n_in, n_out, n_col).ravel()))


@pytest.mark.parametrize("name", PAIRS)
def test_expert_pairs_golden(golden, cuda, name):
    # one expert, top-1, no shared expert: the block's output is the expert's (the reference's ref_expert bits)
    gt, dt, H, F = (int(v) for v in golden[f"pair_{name}_geom"])
    blob = golden[f"pair_{name}_blob"]
    ngu = F * O.row_bytes(gt, H)
    spec = synth.LayerSpec(n_embd=H, n_ff=F, n_expert=1, k=1, gu_type=gt, d_type=dt, has_shared=False)
    t = {"ffn_gate_inp.weight": torch.full((1, H), 0x3C00, dtype=torch.int16),
         "ffn_gate_exps.weight": torch.from_numpy(blob[:ngu].copy()),
         "ffn_up_exps.weight": torch.from_numpy(blob[ngu:2 * ngu].copy()),
         "ffn_down_exps.weight": torch.from_numpy(blob[2 * ngu:].copy())}
    m = api.MoeLayer(synth.Layer(spec, 0, t), 2, cuda)
    assert api.expert_path_for(m, 2) == (1 if (gt, dt) in ((O.IQ2_S, O.Q2_0), (O.Q2_0, O.Q2_0)) else 5)
    api.device_status(clear=True)
    got = m.forward(dev(golden[f"pair_{name}_x"], cuda))
    torch.cuda.synchronize()
    assert api.device_status() == 0
    assert np.array_equal(bits(got.cpu().numpy().ravel()), bits(golden[f"pair_{name}_y"]))


@pytest.mark.parametrize("gu,d,sg,sd,T", [(O.IQ3_S, O.IQ4_NL, O.Q2_0, O.Q2_0, 5),
                                          (O.IQ4_XS, O.Q2_0, O.IQ4_XS, O.Q2_0, 1),
                                          (O.IQ3_XXS, O.Q2_0, O.IQ3_XXS, O.IQ4_NL, 40),
                                          (O.IQ2_S, O.IQ4_NL, O.IQ2_S, O.IQ4_NL, 12)])
def test_any_format_layer_vs_oracle(cuda, gu, d, sg, sd, T):
    spec = synth.LayerSpec(n_embd=2048, n_ff=512, n_expert=64, k=8, gu_type=gu, d_type=d, sg_type=sg, su_type=sg,
                           sd_type=sd, seed=gu * 100 + d)
    got, want, tr, otr, hl, x = run_case(cuda, spec, T)
    check_block(got, want, tr, otr, T, spec.k)
    # every stage follows the reference's operation order: bitwise
    assert np.array_equal(bits(got), bits(want))
    assert np.array_equal(bits(tr.parts.cpu().numpy()), bits(otr["parts"]))


def test_any_format_model_geometry(cuda):
    # the reference model's own widths (n_embd 2560, n_ff 640) in an IQ3_S / IQ4_NL pack
    spec = synth.LayerSpec(n_embd=2560, n_ff=640, n_expert=32, k=8, gu_type=O.IQ3_S, d_type=O.IQ4_NL,
                           sg_type=O.IQ3_S, su_type=O.IQ3_S, sd_type=O.IQ4_NL, seed=2560)
    got, want, tr, otr, hl, x = run_case(cuda, spec, 3)
    check_block(got, want, tr, otr, 3, spec.k)
    assert np.array_equal(bits(got), bits(want))
