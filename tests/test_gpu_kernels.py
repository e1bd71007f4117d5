"""Stage parity on the B200: every C-ABI stage entry point against the oracle and the golden vectors the
reference's own host code produced.  Integer and byte results are compared bitwise; the float stages too,
because the kernels reproduce the reference's operation order (iq.metal:459-514, iq_parity.cpp:275-292)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from stratametal_b200 import api

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_q8_1_bitwise(golden, cuda):
    x = dev(golden["q8_x"], cuda)
    y = torch.empty(golden["q8_y"].size, dtype=torch.uint8, device=cuda)
    api.iq_quantize_q8_1(x, x.numel(), y)
    assert np.array_equal(y.cpu().numpy(), golden["q8_y"])
    rng = np.random.default_rng(3)
    xs = (rng.standard_normal(64 * 2048) * np.repeat(10.0 ** rng.integers(-6, 7, 2048), 64)).astype(np.float32)
    y2 = torch.empty(xs.size // 32 * 36, dtype=torch.uint8, device=cuda)
    api.iq_quantize_q8_1(dev(xs, cuda), xs.size, y2)
    assert np.array_equal(y2.cpu().numpy(), O.quant_q8_1(xs))


def test_bf16_bulk_bitwise(golden, cuda):
    v = dev(golden["bits_v"], cuda)
    y = torch.empty(v.numel(), dtype=torch.int16, device=cuda)
    api.f32_to_bf16_bulk(v, y)
    assert np.array_equal(y.cpu().numpy().view(np.uint16), golden["bits_bf16"])


@pytest.mark.parametrize("name,t,n_in", [("q2_2048", O.Q2_0, 2048), ("q2_512", O.Q2_0, 512),
                                         ("iq2s_2048", O.IQ2_S, 2048), ("q2_64", O.Q2_0, 64),
                                         ("iq4nl_512", O.IQ4_NL, 512), ("iq4xs_2048", O.IQ4_XS, 2048)])
def test_mmvq_golden_bitwise(golden, cuda, name, t, n_in):
    w, xq, want = golden[f"dot_{name}_w"], golden[f"dot_{name}_x"], golden[f"dot_{name}_y"]
    y = torch.full((want.size + 16,), 7.0, device=cuda)
    api.iq_mmvq(t, dev(w, cuda), dev(xq, cuda), n_in, want.size, 1, y)
    got = y.cpu().numpy()
    assert np.array_equal(bits(got[:want.size]), bits(want))
    assert np.all(got[want.size:] == 7.0), "wrote past the output"


@pytest.mark.parametrize("t,n_in,n_out,n_col", [(O.Q2_0, 2048, 512, 5), (O.Q2_0, 512, 2048, 3),
                                                (O.IQ2_S, 2048, 96, 4), (O.Q2_0, 256, 40, 3), (O.IQ2_S, 512, 40, 3),
                                                (O.Q2_0, 2560, 100, 2), (O.Q2_0, 640, 70, 2),
                                                (O.IQ4_NL, 2048, 70, 3), (O.IQ4_NL, 32, 9, 2), (O.IQ4_XS, 4096, 33, 2),
                                                (O.IQ4_XS, 256, 8, 3)])
def test_mmvq_random_bitwise(cuda, t, n_in, n_out, n_col):
    rng = np.random.default_rng(n_in * 7 + n_out)
    rb = O.row_bytes(t, n_in)
    w = rng.integers(0, 256, n_out * rb, dtype=np.uint8)
    bs = {O.Q2_0: 18, O.IQ2_S: 82, O.IQ4_NL: 18, O.IQ4_XS: 136}[t]
    for o in range(0, w.size, bs):
        h = int(np.float16(abs(rng.standard_normal()) * 0.05).view(np.uint16))
        w[o], w[o + 1] = h & 255, h >> 8
    xq = O.quant_q8_1(rng.standard_normal(n_col * n_in).astype(np.float32))
    y = torch.empty(n_col * n_out, device=cuda)
    api.iq_mmvq(t, dev(w, cuda), dev(xq, cuda), n_in, n_out, n_col, y)
    assert np.array_equal(bits(y.cpu().numpy()), bits(O.mmvq(t, w, xq, n_in, n_out, n_col).ravel()))


def test_swiglu_q8(cuda):
    rng = np.random.default_rng(11)
    g = (rng.standard_normal(512 * 64) * 3).astype(np.float32)
    u = rng.standard_normal(512 * 64).astype(np.float32)
    y = torch.empty(g.size // 32 * 36, dtype=torch.uint8, device=cuda)
    api.iq_swiglu_q8(dev(g, cuda), dev(u, cuda), g.size, y)
    got, want = y.cpu().numpy().reshape(-1, 36), O.swiglu_q8(g, u).reshape(-1, 36)
    # SwiGLU's exp is the correctly rounded one; the host libm expf may differ in its last bit on rare inputs
    assert (got != want).any(axis=1).mean() < 1e-3


@pytest.mark.parametrize("name", ["random", "equal", "tie12", "dominant", "e7k3", "e1024", "k64"])
def test_router_top10_golden(golden, cuda, name):
    lg, ids_w, w_w = golden[f"route_{name}_logits"], golden[f"route_{name}_ids"], golden[f"route_{name}_w"]
    T, E = lg.shape
    k = ids_w.shape[1]
    ids = torch.full((T * k + 1,), 7, dtype=torch.int32, device=cuda)
    w = torch.full((T * k + 1,), 7.0, device=cuda)
    api.router_top10(dev(lg, cuda), T, E, k, ids, w)
    ids_h, w_h = ids.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(ids_h[:-1].reshape(T, k), ids_w)
    rel = np.abs(w_h[:-1].reshape(T, k).astype(np.float64) - w_w) / np.abs(w_w)
    assert rel.max() <= 1e-6
    assert ids_h[-1] == 7 and w_h[-1] == 7.0


def test_router_zero_tokens_leaves_outputs(cuda):
    ids = torch.full((4,), 7, dtype=torch.int32, device=cuda)
    api.router_top10(torch.zeros(4, device=cuda), 0, 512, 10, ids, ids)
    torch.cuda.synchronize()
    assert ids.cpu().tolist() == [7, 7, 7, 7]


@pytest.mark.parametrize("T", [33, 200])  # 200 tokens take the tiled fp64 GEMM (partial tiles included)
def test_router_fused_logits_bitwise(cuda, T):
    from stratametal_b200 import synth
    sp = synth.LayerSpec(n_embd=2048, n_ff=64, n_expert=512, k=10, seed=8)
    lay = synth.make_layer(sp, 0, cuda)
    x = synth.make_x(5, T, 2048, cuda)
    wr = lay["ffn_gate_inp.weight"]
    logits = torch.empty(T, 512, device=cuda)
    ids = torch.empty(T, 10, dtype=torch.int32, device=cuda)
    w = torch.empty(T, 10, device=cuda)
    api.router(x, wr, T, 2048, 512, 10, logits, ids, w)
    xh = x.cpu().numpy()
    wh = wr.cpu().numpy().view(np.uint16)
    L = O.lib()
    lg_ref = np.empty((T, 512), np.float32)
    for t in range(T):
        xr = np.array([L.orc_bf16_from_f32(float(v)) for v in xh[t]], np.uint16)
        xr = (xr.astype(np.uint32) << 16).view(np.float32)
        for e in range(512):
            lg_ref[t, e] = L.orc_bf16_dot(O._ptr(xr, O._f32p), O._ptr(wh[e], O._u16p), 2048)
    assert np.array_equal(bits(logits.cpu().numpy()), bits(lg_ref))
    ids_ref, w_ref = O.route(lg_ref, 10)
    assert np.array_equal(ids.cpu().numpy(), ids_ref)
    assert np.abs(w.cpu().numpy() / w_ref - 1).max() <= 1e-6


def test_combine_golden(golden, cuda):
    parts, w, sh = golden["combine_parts"], golden["combine_w"], golden["combine_shared"]
    y = torch.full((256 + 16,), 7.0, device=cuda)
    api.moe_combine(dev(parts, cuda), dev(w, cuda), dev(sh, cuda), y, 256, 10)
    got = y.cpu().numpy()
    assert np.array_equal(bits(got[:256]), bits(golden["combine_right"]))
    assert np.all(got[256:] == 7.0)
    api.moe_combine(dev(parts, cuda), dev(w, cuda), None, y, 256, 10)
    assert np.array_equal(bits(y.cpu().numpy()[:256]), bits(golden["combine_noshared"]))


@pytest.mark.parametrize("T,E,k", [(1, 512, 10), (64, 512, 10), (300, 512, 10), (5, 7, 3), (2, 1024, 64)])
def test_group_stable(cuda, T, E, k):
    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    scratch = torch.empty(api.moe_group_scratch_bytes(T, k, E), dtype=torch.uint8, device=cuda)
    slot = torch.empty(T * k, dtype=torch.int32, device=cuda)
    src = torch.empty(T * k, dtype=torch.int32, device=cuda)
    api.moe_group(dev(ids, cuda), T, k, E, scratch, slot, src)
    tab = scratch.cpu().numpy().view(np.int32)
    counts, offsets = tab[:E], tab[E:2 * E + 1]
    n_active = tab[3 * E + 1]
    active = tab[2 * E + 1:2 * E + 1 + n_active]
    flat = ids.ravel()
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(counts)]))
    assert np.array_equal(active, np.nonzero(counts)[0])
    order = np.argsort(flat, kind="stable")          # stable by expert, then by pair index = token order
    want_slot = np.empty_like(order)
    want_slot[order] = np.arange(order.size)
    assert np.array_equal(slot.cpu().numpy(), want_slot)
    assert np.array_equal(src.cpu().numpy(), order // k)


@pytest.mark.parametrize("T", [5, 300])  # one CTA; the any-size two-pass CTA
def test_group_refuses_a_repeated_expert(cuda, T):
    # a token whose ids name one expert twice: the second pair gets no row (slot -1) and BAD_ID is recorded;
    # every other pair is grouped as if the repeat were absent
    E, k = 64, 6
    rng = np.random.default_rng(T)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[3, 4] = ids[3, 1]
    scratch = torch.empty(api.moe_group_scratch_bytes(T, k, E), dtype=torch.uint8, device=cuda)
    slot = torch.empty(T * k, dtype=torch.int32, device=cuda)
    src = torch.empty(T * k, dtype=torch.int32, device=cuda)
    api.device_status(clear=True)
    api.moe_group(dev(ids, cuda), T, k, E, scratch, slot, src)
    torch.cuda.synchronize()
    assert api.device_status() == 2
    got = slot.cpu().numpy()
    bad = 3 * k + 4
    assert got[bad] == -1
    keep = np.ones(T * k, bool)
    keep[bad] = False
    flat = ids.ravel()
    counts = scratch.cpu().numpy().view(np.int32)[:E]
    assert np.array_equal(counts, np.bincount(flat[keep], minlength=E))
    order = np.nonzero(keep)[0][np.argsort(flat[keep], kind="stable")]
    want = np.full(T * k, -1)
    want[order] = np.arange(order.size)
    assert np.array_equal(got, want)
    assert np.array_equal(src.cpu().numpy()[:order.size], order // k)


@pytest.mark.parametrize("rows,cols,resid,weighted", [(1, 2048, True, False), (16, 2048, True, True),
                                                      (5, 1000, False, True)])
def test_add_rms_norm(cuda, rows, cols, resid, weighted):
    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    r = rng.standard_normal((rows, cols)).astype(np.float32) if resid else None
    w = (0.5 + rng.random(cols)).astype(np.float32) if weighted else None
    xd = torch.tensor(np.concatenate([x.ravel(), np.full(8, 7.0, np.float32)]), device=cuda)
    api.add_rms_norm(xd, None if r is None else dev(r, cuda), None if w is None else dev(w, cuda), rows, cols, 1e-6)
    got = xd.cpu().numpy()
    assert np.all(got[rows * cols:] == 7.0)
    want = O.add_rms_norm(x, r, w, 1e-6)
    ulp = np.abs(bits(got[:rows * cols]).astype(np.int64) - bits(want.ravel()).astype(np.int64))
    assert ulp.max() <= 1 and (ulp == 0).mean() >= 0.999   # only the fp64 order of the sum of squares differs
