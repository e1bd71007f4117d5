"""The seeded generator: deterministic, in the reference's block formats, with the configured distributions."""
import numpy as np
import torch

from stratametal_b200 import synth


def test_deterministic_and_shardable():
    sp = synth.LayerSpec(n_embd=256, n_ff=64, n_expert=8, k=2, seed=3)
    a = synth.make_layer(sp, 1)
    b = synth.make_layer(sp, 1)
    for k in a.tensors:
        assert torch.equal(a[k], b[k]), k
    shard = synth.make_layer(sp, 1, experts=range(4, 8))
    n = a["ffn_gate_exps.weight"].numel() // 8
    assert torch.equal(shard["ffn_gate_exps.weight"], a["ffn_gate_exps.weight"][4 * n:])
    c = synth.make_layer(sp, 2)
    assert not torch.equal(a["ffn_gate_exps.weight"], c["ffn_gate_exps.weight"])


def test_q2_0_format_and_distributions():
    sp = synth.LayerSpec(n_embd=2048, n_ff=64, n_expert=4, k=2, seed=9)
    L = synth.make_layer(sp, 0)
    w = L["ffn_gate_exps.weight"].numpy().reshape(-1, 18)
    d = w[:, :2].copy().view(np.float16).astype(np.float64).ravel()
    assert np.all(d >= 0)
    assert abs(d.mean() - 0.05 * np.sqrt(2 / np.pi)) < 0.003      # |N(0, 0.05)|
    codes = np.stack([(w[:, 2:] >> s) & 3 for s in (0, 2, 4, 6)]).ravel()
    hist = np.bincount(codes, minlength=4) / codes.size
    assert np.all(np.abs(hist - 0.25) < 0.01)
    r = L["ffn_gate_inp.weight"].view(torch.bfloat16).float().numpy()
    assert abs(r.std() - 0.02) < 0.002
    x = synth.make_x(1, 64, 2048).numpy()
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1) < 0.02


def test_iq2_s_blocks():
    sp = synth.LayerSpec(n_embd=256, n_ff=32, n_expert=2, k=1, gu_type=synth.IQ2_S, seed=4)
    L = synth.make_layer(sp, 0)
    w = L["ffn_gate_exps.weight"].numpy().reshape(-1, 82)
    assert w.shape[0] == 2 * 32
    sc = w[:, 74:82]
    assert set(np.unique(sc & 15)) <= set(range(16))


def test_zipf_calibration_is_heavy_tailed():
    f = synth.zipf_row_scales(512, 10)
    assert f[0] > 3 * np.median(f)
    g = np.random.default_rng(1).standard_normal((2000, 512)) * f
    top = np.argpartition(-g, 9, axis=1)[:, :10]
    freq = np.bincount(top.ravel(), minlength=512) / 2000
    assert freq[0] > 0.3 and freq[400:].mean() < 0.01
