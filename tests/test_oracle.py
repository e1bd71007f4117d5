"""The CPU oracle (oracle/oracle.c) pinned against the reference's own host code.

golden.npz was produced by the reference's parity-test references compiled from its sources
(tests/golden/make_golden.py); when oracle/_ref was built here the same functions are also called live on
fresh random inputs.  The trap cases are the reference's own (iq_parity.cpp:490-538,
moe_combine_parity.cpp:126-134, router_parity.cpp:160-180): each plausible misreading must land far away.
"""
import numpy as np
import pytest

from oracle import oracle as O
from stratametal_b200 import synth


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_bit_conversions(golden):
    L = O.lib()
    v = golden["bits_v"]
    assert [L.orc_bf16_from_f32(float(a)) for a in v] == golden["bits_bf16"].tolist()
    assert [L.orc_f16_from_f32(float(a)) for a in v] == golden["bits_f16"].tolist()


def test_q8_1_bitwise_including_clamped_scale(golden):
    y = O.quant_q8_1(golden["q8_x"])
    assert np.array_equal(y, golden["q8_y"])
    # the 1e10 block stores the clamped scale 65504 (0x7BFF)
    assert int(y[0]) | (int(y[1]) << 8) == 0x7BFF


@pytest.mark.parametrize("name,t,n_in", [("q2_2048", O.Q2_0, 2048), ("q2_512", O.Q2_0, 512),
                                         ("iq2s_2048", O.IQ2_S, 2048), ("q2_64", O.Q2_0, 64),
                                         ("iq4nl_512", O.IQ4_NL, 512), ("iq4xs_2048", O.IQ4_XS, 2048),
                                         ("iq3xxs_2048", O.IQ3_XXS, 2048), ("iq3s_2048", O.IQ3_S, 2048)])
def test_row_dot_bitwise(golden, name, t, n_in):
    w, xq, want = golden[f"dot_{name}_w"], golden[f"dot_{name}_x"], golden[f"dot_{name}_y"]
    got = O.mmvq(t, w, xq, n_in, want.size, 1)[0]
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("name", ["q2", "iq2s", "q2_wide"])
def test_expert_chain_bitwise(golden, name):
    gt, H, F = golden[f"exp_{name}_geom"].tolist()
    blob, xq, want = golden[f"exp_{name}_blob"], golden[f"exp_{name}_xq"], golden[f"exp_{name}_y"]
    rb = O.row_bytes(gt, H)
    g = O.mmvq(gt, blob[:F * rb], xq, H, F, 2)
    u = O.mmvq(gt, blob[F * rb:2 * F * rb], xq, H, F, 2)
    hq = O.swiglu_q8(g.ravel(), u.ravel())
    y = O.mmvq(O.Q2_0, blob[2 * F * rb:], hq, F, H, 2).ravel()
    assert np.array_equal(bits(y), bits(want))
    # the two tokens do not share an output (iq_parity.cpp:527-528)
    assert O.rel_l1(y[:H], y[H:]) > 0.05


@pytest.mark.parametrize("name", ["random", "equal", "tie12", "dominant", "e7k3", "e1024", "k64"])
def test_route_matches_reference(golden, name):
    lg, ids_w, w_w = golden[f"route_{name}_logits"], golden[f"route_{name}_ids"], golden[f"route_{name}_w"]
    ids, w = O.route(lg, ids_w.shape[1])
    assert np.array_equal(ids, ids_w)
    assert np.array_equal(bits(w), bits(w_w))


def test_route_known_answers(golden):
    ids, w = O.route(golden["route_equal_logits"], 10)
    assert ids[0].tolist() == list(range(10))          # ties keep the lower index
    assert np.all(w == np.float32(0.1))
    # renormalisation left out would be 98% away (router_parity.cpp:174-180)
    raw = np.float32(1.0 / 512)
    assert abs(raw - w[0, 0]) / w[0, 0] > 0.5
    ids, w = O.route(golden["route_dominant_logits"], 10)
    assert ids[:, 0].tolist() == [0, 1, 2, 3]
    assert (10 / 512) / 6.103515625e-05 == 320        # the clamp is 320x below the smallest top-10 sum


def test_combine_and_traps(golden):
    parts, w, sh = golden["combine_parts"], golden["combine_w"], golden["combine_shared"]
    y = O.combine(parts[None], w[None], sh[None])[0]
    assert np.array_equal(bits(y), bits(golden["combine_right"]))
    y0 = O.combine(parts[None], w[None], None)[0]
    assert np.array_equal(bits(y0), bits(golden["combine_noshared"]))
    assert O.rel_l1(golden["combine_right"], golden["combine_unweighted"]) > 0.05
    assert O.rel_l1(golden["combine_right"], golden["combine_shared_weighted"]) > 0.05
    assert O.rel_l1(golden["combine_right"], y0) > 0.05


def test_q2_minus_one_trap(golden):
    w, xq, want = golden["dot_q2_2048_w"], golden["dot_q2_2048_x"], golden["dot_q2_2048_y"]
    rb = O.row_bytes(O.Q2_0, 2048)
    bare = np.array([O.lib().orc_row_dot_variant(O.Q2_0, O._ptr(w[r * rb:], O._u8p), O._ptr(xq, O._u8p), 2048, 1)
                     for r in range(want.size)], np.float32)
    assert O.rel_l1(want, bare) > 0.05


def test_swapped_gate_up_trap(golden):
    gt, H, F = golden["exp_q2_geom"].tolist()
    blob, xq, want = golden["exp_q2_blob"], golden["exp_q2_xq"], golden["exp_q2_y"]
    rb = O.row_bytes(gt, H)
    g = O.mmvq(gt, blob[F * rb:2 * F * rb], xq, H, F, 2)   # up read as gate
    u = O.mmvq(gt, blob[:F * rb], xq, H, F, 2)
    y = O.mmvq(O.Q2_0, blob[2 * F * rb:], O.swiglu_q8(g.ravel(), u.ravel()), F, H, 2).ravel()
    assert O.rel_l1(want, y) > 0.05


def test_live_reference_cross_check():
    R = O.ref()
    if R is None:
        pytest.skip("oracle/_ref not built here (the reference tree is absent)")
    rng = np.random.default_rng(7)
    for t, n_in in ((O.Q2_0, 2048), (O.IQ2_S, 2048), (O.Q2_0, 512), (O.IQ4_NL, 512), (O.IQ4_XS, 2048),
                    (O.IQ3_XXS, 512), (O.IQ3_S, 512)):
        rb = O.row_bytes(t, n_in)
        w = rng.integers(0, 256, 8 * rb, dtype=np.uint8)
        bs = {O.Q2_0: 18, O.IQ2_S: 82, O.IQ4_NL: 18, O.IQ4_XS: 136, O.IQ3_XXS: 98, O.IQ3_S: 110}[t]
        for o in range(0, w.size, bs):
            h = int(np.float16(abs(rng.standard_normal()) * 0.05).view(np.uint16))
            w[o], w[o + 1] = h & 255, h >> 8
        xq = O.quant_q8_1(rng.standard_normal(n_in).astype(np.float32))
        got = O.mmvq(t, w, xq, n_in, 8, 1)[0]
        for r in range(8):
            wr = np.ascontiguousarray(w[r * rb:(r + 1) * rb])
            ref = R.ref_row_dot(t, O._ptr(wr, O._u8p), O._ptr(xq, O._u8p), n_in, 0)
            assert bits(got[r]) == bits(ref)
    for _ in range(50):
        lg = rng.standard_normal((1, 512)).astype(np.float32) * rng.uniform(0.1, 5)
        ids, w = O.route(lg, 10)
        ri, rw = np.empty(10, np.int32), np.empty(10, np.float32)
        R.ref_route(O._ptr(lg[0], O._f32p), 512, 10, O._ptr(ri, O._i32p), O._ptr(rw, O._f32p))
        assert np.array_equal(ids[0], ri) and np.array_equal(bits(w[0]), bits(rw))


def _small_layer(rng, gu_type=O.Q2_0, H=256, F=64, E=16, k=4, shared=True):
    def rows(t, n, n_in):
        rb = O.row_bytes(t, n_in)
        w = rng.integers(0, 256, n * rb, dtype=np.uint8)
        bs = 18 if t == O.Q2_0 else 82
        for o in range(0, w.size, bs):
            h = int(np.float16(abs(rng.standard_normal()) * 0.05).view(np.uint16))
            w[o], w[o + 1] = h & 255, h >> 8
        return w
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    rb16 = np.array([O.lib().orc_bf16_from_f32(float(v)) for v in router.ravel()], np.uint16).reshape(E, H)
    sh = None
    if shared:
        ginp = np.array([O.lib().orc_bf16_from_f32(float(v)) for v in rng.standard_normal(H) * 0.02], np.uint16)
        sh = dict(sg_type=O.Q2_0, su_type=O.Q2_0, sd_type=O.Q2_0, sgate=rows(O.Q2_0, F, H), sup=rows(O.Q2_0, F, H),
                  sdown=rows(O.Q2_0, H, F), ginp=ginp)
    return O.HostLayer(H, F, E, k, gu_type, O.Q2_0, rb16, rows(gu_type, E * F, H), rows(gu_type, E * F, H),
                       rows(O.Q2_0, E * H, F), sh)


@pytest.mark.parametrize("gu_type", [O.Q2_0, O.IQ2_S])
def test_layer_composition(gu_type):
    """orc_moe_layer equals the stage functions chained by hand, serial and threaded alike."""
    rng = np.random.default_rng(77)
    L = _small_layer(rng, gu_type)
    x = rng.standard_normal((3, L.n_embd)).astype(np.float32)
    out, tr = O.moe_layer(L, x, trace=True, n_threads=1)
    out4 = O.moe_layer(L, x, n_threads=4)
    assert np.array_equal(bits(out), bits(out4))
    H, F, K = L.n_embd, L.n_ff, L.k
    rbg, rbd = O.row_bytes(gu_type, H), O.row_bytes(O.Q2_0, F)
    for t in range(3):
        xr = np.array([O.lib().orc_bf16_from_f32(float(v)) for v in x[t]], np.uint16)
        xr = (xr.astype(np.uint32) << 16).view(np.float32)
        lg = np.array([O.lib().orc_bf16_dot(O._ptr(xr, O._f32p), O._ptr(L.router[e], O._u16p), H)
                       for e in range(L.n_expert)], np.float32)
        assert np.array_equal(bits(lg), bits(tr["logits"][t]))
        ids, w = O.route(lg[None], K)
        assert np.array_equal(ids[0], tr["ids"][t])
        xq = O.quant_q8_1(x[t])
        parts = []
        for e in ids[0]:
            g = O.mmvq(gu_type, L.gate[e * F * rbg:(e + 1) * F * rbg], xq, H, F, 1)
            u = O.mmvq(gu_type, L.up[e * F * rbg:(e + 1) * F * rbg], xq, H, F, 1)
            parts.append(O.mmvq(O.Q2_0, L.down[e * H * rbd:(e + 1) * H * rbd], O.swiglu_q8(g, u), F, H, 1)[0])
        parts = np.array(parts, np.float32)
        assert np.array_equal(bits(parts), bits(tr["parts"][t]))
        s = L.shared
        g = O.mmvq(O.Q2_0, s["sgate"], xq, H, F, 1)
        u = O.mmvq(O.Q2_0, s["sup"], xq, H, F, 1)
        sd = O.mmvq(O.Q2_0, s["sdown"], O.swiglu_q8(g, u), F, H, 1)[0]
        gl = O.lib().orc_bf16_dot(O._ptr(xr, O._f32p), O._ptr(s["ginp"], O._u16p), H)
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(np.float32(-gl)))
        shared = (sd * sig).astype(np.float32)
        assert np.allclose(shared, tr["shared"][t], rtol=1e-6, atol=0)
        y = O.combine(parts[None], w, tr["shared"][t][None])[0]
        assert np.array_equal(bits(y), bits(out[t]))


def test_fp32_mode_is_close_to_contract_mode():
    rng = np.random.default_rng(5)
    L = _small_layer(rng, O.Q2_0, H=512, F=128)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    c = O.moe_layer(L, x, mode=0, n_threads=2)
    f = O.moe_layer(L, x, mode=1, n_threads=2)
    # the q8_1 activation contract moves the block by about a percent, not more
    assert 1e-4 < O.rel_l1(f, c) < 0.05


def test_rms_norm_rule():
    # the reference's own test inputs (elementwise_parity.cpp:102-112): x = sin(0.017 i) * 1.7 + 0.4,
    # w = 0.5 + 0.002 (c % 97); checked against an independent fp64 evaluation of the same formula
    rows, cols = 3, 2048
    i = np.arange(rows * cols, dtype=np.float64)
    x = (np.sin(i * 0.017).astype(np.float32) * np.float32(1.7) + np.float32(0.4)).reshape(rows, cols)
    w = (np.float32(0.5) + np.float32(0.002) * (np.arange(cols) % 97).astype(np.float32)).astype(np.float32)
    got = O.add_rms_norm(x, None, w, 1e-6)
    xd = x.astype(np.float64)
    den = np.sqrt((xd * xd).sum(axis=1, keepdims=True) / cols + np.float64(np.float32(1e-6)))
    want = ((xd / den) * w.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, want)
    # unit weight: mean of squares 1; the residual is added in f32 first
    r = np.ones_like(x)
    g2 = O.add_rms_norm(x, r, None, 1e-6)
    assert np.allclose((g2.astype(np.float64) ** 2).mean(axis=1), 1.0, atol=1e-5)
    assert np.array_equal(g2, O.add_rms_norm((x + r).astype(np.float32), None, None, 1e-6))


def test_iq4_fields_are_observable(golden):
    """The IQ4 partials read each code byte's two nibbles as values i and i + 16, and IQ4_XS's 6-bit scales take
    two high bits from the scales_h word: swapping the nibbles, or clearing scales_h, must move the rows far."""
    for name, t, n_in, bs in (("iq4nl_512", O.IQ4_NL, 512, 18), ("iq4xs_2048", O.IQ4_XS, 2048, 136)):
        w, xq, want = golden[f"dot_{name}_w"], golden[f"dot_{name}_x"], golden[f"dot_{name}_y"]
        qs0 = 2 if t == O.IQ4_NL else 8
        sw = w.copy()
        for o in range(0, sw.size, bs):
            b = sw[o + qs0:o + bs]
            sw[o + qs0:o + bs] = (b >> 4) | ((b & 15) << 4)
        assert O.rel_l1(want, O.mmvq(t, sw, xq, n_in, want.size, 1)[0]) > 0.05
        if t == O.IQ4_XS:
            hz = w.copy()
            for o in range(0, hz.size, bs):
                hz[o + 2] = hz[o + 3] = 0
            assert O.rel_l1(want, O.mmvq(t, hz, xq, n_in, want.size, 1)[0]) > 0.05


PAIRS = ["iq2s_iq4nl", "iq3xxs_q2", "iq3s_iq4nl", "iq4xs_q2", "iq3s_iq4nl_wide"]


def pair_layer(golden, name):
    """The reference's expert pair as a one-expert, top-1 layer without a shared expert: the router must pick
    expert 0 with weight 1, so the block's output is the expert's output (golden pair_*, iq_parity.cpp:504-539)."""
    gt, dt, H, F = (int(v) for v in golden[f"pair_{name}_geom"])
    blob = golden[f"pair_{name}_blob"]
    ngu = F * O.row_bytes(gt, H)
    router = np.full(H, 0x3C00, np.uint16)  # any bf16 row
    return O.HostLayer(H, F, 1, 1, gt, dt, router, blob[:ngu], blob[ngu:2 * ngu], blob[2 * ngu:], None)


@pytest.mark.parametrize("name", PAIRS)
def test_expert_pairs_through_the_layer(golden, name):
    # the oracle's block over the other formats reproduces the reference's ref_expert bit for bit
    got = O.moe_layer(pair_layer(golden, name), golden[f"pair_{name}_x"])
    assert np.array_equal(got.ravel().view(np.uint32), golden[f"pair_{name}_y"].view(np.uint32))


def test_s2_expert_is_the_gguf_expert():
    # An S2 blob is a re-layout of GGUF Q2_0 rows, and its rows are evaluated in the reference's row_dot order: on
    # the same int8 activations and scales it gives the reference's own GGUF expert chain (the one-expert block
    # below, pinned bitwise to ref_expert by test_expert_pairs_through_the_layer) bit for bit.  The Q8_0 and q8_1
    # rules round the same values the same way except at exact half-way ties, which these inputs do not hit.
    H, F = 512, 128
    rows = [synth.quant_matrix(42, k, n_out, n_in, "cpu").numpy() for k, n_out, n_in in ((1, F, H), (2, F, H), (3, H, F))]
    x = np.random.default_rng(77).standard_normal((1, H)).astype(np.float32)
    q80, q81 = O.quant_q8_0(x), O.quant_q8_1(x.ravel())
    for b in range(H // 32):
        assert np.array_equal(q80[b * 34:b * 34 + 2], q81[b * 36:b * 36 + 2])
        assert np.array_equal(q80[b * 34 + 2:b * 34 + 34], q81[b * 36 + 4:b * 36 + 36])
    s2 = O.s2_expert(O.s2_pack(*rows, H, F), H, F, q80)
    layer = O.HostLayer(H, F, 1, 1, O.Q2_0, O.Q2_0, np.full(H, 0x3C00, np.uint16), rows[0], rows[1], rows[2], None)
    gguf = O.moe_layer(layer, x).ravel()
    assert np.array_equal(s2.view(np.uint32), gguf.view(np.uint32))
