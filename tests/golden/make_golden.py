"""Generate tests/golden/golden.npz from the reference's OWN host references (oracle/_ref/libstrata_ref.so,
compiled from StrataMetal's metal/src/{iq,router,moe_combine}_parity.cpp and its bf16/f16 headers).

Run in a checkout that has the reference tree (make -C oracle builds _ref/ from it):
    python tests/golden/make_golden.py
The fixture holds every input and the reference's output, so the tests need neither the reference tree
nor this script.  Seeds are the ones the reference's parity tests use (iq_parity.cpp:454, router_parity.cpp:130,
moe_combine_parity.cpp:121).
"""
import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

R = O.ref()
if R is None:
    raise SystemExit("oracle/_ref/libstrata_ref.so is missing: build it with `make -C oracle` next to the reference")
f32p, u8p, i32p = O._f32p, O._u8p, O._i32p
P = O._ptr


def rand_rows(rng, t, rows, n_in):
    """Random weight rows with fp16 scales of exponent 7..11, a quarter negative (iq_parity.cpp:316-332)."""
    rb = O.row_bytes(t, n_in)
    bs = {O.Q2_0: 18, O.IQ2_S: 82, O.IQ4_NL: 18, O.IQ4_XS: 136, O.IQ3_XXS: 98, O.IQ3_S: 110}[t]
    w = rng.integers(0, 256, rows * rb, dtype=np.uint8)
    for o in range(0, w.size, bs):
        h = (0x8000 if rng.integers(0, 4) == 0 else 0) | (int(rng.integers(7, 12)) << 10) | int(rng.integers(0, 1024))
        w[o] = h & 255
        w[o + 1] = h >> 8
    return w


def ref_q8(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.size // 32 * 36, np.uint8)
    for b in range(x.size // 32):
        xb = np.ascontiguousarray(x[b * 32:(b + 1) * 32])
        yb = np.empty(36, np.uint8)
        R.ref_quant_q8_1_block(P(xb, f32p), P(yb, u8p))
        y[b * 36:(b + 1) * 36] = yb
    return y


def ref_rows(t, w, xq, n_in, n_out):
    rb = O.row_bytes(t, n_in)
    out = np.empty(n_out, np.float32)
    for r in range(n_out):
        wr = np.ascontiguousarray(w[r * rb:(r + 1) * rb])
        out[r] = R.ref_row_dot(t, P(wr, u8p), P(xq, u8p), n_in, 0)
    return out


def main():
    g = {}
    rng = np.random.default_rng(20261014)
    # q8_1, including the reference's clamped-scale case (iq_parity.cpp:456-464)
    x = rng.standard_normal(256).astype(np.float32)
    x[3] = 1e10
    x[40] = -8e6
    x[64:96] = 0.0
    x[96:128] *= 1e-6
    g["q8_x"] = x
    g["q8_y"] = ref_q8(x)
    # row dots: Q2_0 gate geometry, Q2_0 down geometry, IQ2_S gate geometry
    for name, t, n_in, n_out in (("q2_2048", O.Q2_0, 2048, 24), ("q2_512", O.Q2_0, 512, 24),
                                 ("iq2s_2048", O.IQ2_S, 2048, 24), ("q2_64", O.Q2_0, 64, 8)):
        w = rand_rows(rng, t, n_out, n_in)
        xq = ref_q8(rng.standard_normal(n_in).astype(np.float32))
        g[f"dot_{name}_w"] = w
        g[f"dot_{name}_x"] = xq
        g[f"dot_{name}_y"] = ref_rows(t, w, xq, n_in, n_out)
    # expert chains (ref_expert, iq_parity.cpp:386-411): 2 tokens, the second -0.5 x + 0.25 (:513)
    for name, gt, H, F in (("q2", O.Q2_0, 256, 64), ("iq2s", O.IQ2_S, 256, 64), ("q2_wide", O.Q2_0, 2048, 64)):
        blob = np.concatenate([rand_rows(rng, gt, 2 * F, H), rand_rows(rng, O.Q2_0, H, F)])
        xx = rng.standard_normal((2, H)).astype(np.float32)
        xx[1] = -0.5 * xx[0] + 0.25
        xq = ref_q8(xx.ravel())
        y = np.empty(2 * H, np.float32)
        R.ref_expert_q8(gt, O.Q2_0, H, F, P(blob, u8p), blob.size, P(xq, u8p), 2, P(y, f32p))
        g[f"exp_{name}_blob"] = blob
        g[f"exp_{name}_xq"] = xq
        g[f"exp_{name}_y"] = y
        g[f"exp_{name}_geom"] = np.array([gt, H, F], np.int32)
    # router cases (router_parity.cpp:130-193)
    rr = np.random.default_rng(2024)
    cases = {
        "random": rr.standard_normal((8, 512)).astype(np.float32),
        "equal": np.full((2, 512), 0.5, np.float32),
        "tie12": np.where(np.arange(512) < 12, 2.0, rr.standard_normal((4, 512))).astype(np.float32),
        "dominant": np.zeros((4, 512), np.float32),
        "e7k3": rr.standard_normal((4, 7)).astype(np.float32),
        "e1024": rr.standard_normal((4, 1024)).astype(np.float32),
        "k64": rr.standard_normal((2, 64)).astype(np.float32),
    }
    for t in range(4):
        cases["dominant"][t, t] = 20.0
    ks = {"e7k3": 3, "k64": 64}
    for name, lg in cases.items():
        k = ks.get(name, 10)
        T, E = lg.shape
        ids = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        for t in range(T):
            row = np.ascontiguousarray(lg[t])
            R.ref_route(P(row, f32p), E, k, P(ids[t], i32p), P(w[t], f32p))
        g[f"route_{name}_logits"] = lg
        g[f"route_{name}_ids"] = ids
        g[f"route_{name}_w"] = w
    # combine (moe_combine_parity.cpp:121-134) with its two traps
    rc = np.random.default_rng(31337)
    parts = rc.standard_normal((10, 256)).astype(np.float32)
    wv = (np.abs(rc.standard_normal(10)) + 0.05).astype(np.float32)
    wv = (wv / wv.astype(np.float64).sum()).astype(np.float32)
    sh = (rc.standard_normal(256) * 3.0).astype(np.float32)
    for name, wr, ws in (("right", 1, 0), ("unweighted", 0, 0), ("shared_weighted", 1, 1)):
        y = np.empty(256, np.float32)
        R.ref_combine(P(parts, f32p), P(wv, f32p), P(sh, f32p), P(y, f32p), 256, 10, wr, ws)
        g[f"combine_{name}"] = y
    y = np.empty(256, np.float32)
    R.ref_combine(P(parts, f32p), P(wv, f32p), None, P(y, f32p), 256, 10, 1, 0)
    g["combine_noshared"] = y
    g["combine_parts"], g["combine_w"], g["combine_shared"] = parts, wv, sh
    # bit conversions of awkward values (bf16 ties, fp16 subnormals and overflow)
    v = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 65504.0, 65520.0, 1e30, 6e-8, 3e-8, 5.96e-8, 1e-5,
                  -2.5e-6, np.inf, -np.inf, 3.14159265, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9] +
                 list(rng.standard_normal(64) * 10.0 ** rng.integers(-8, 6, 64)), np.float32)
    g["bits_v"] = v
    g["bits_bf16"] = np.array([R.ref_bf16_from_f32(float(a)) for a in v], np.uint16)
    g["bits_f16"] = np.array([R.ref_f16_from_f32(float(a)) for a in v], np.uint16)
    # the IQ4 formats (the reference's next gate/up and down formats; oracle only): their own generator, so the
    # arrays above do not change
    r4 = np.random.default_rng(4420)
    for name, t, n_in, n_out in (("iq4nl_512", O.IQ4_NL, 512, 48), ("iq4xs_2048", O.IQ4_XS, 2048, 48)):
        w = rand_rows(r4, t, n_out, n_in)
        xq = ref_q8(r4.standard_normal(n_in).astype(np.float32))
        g[f"dot_{name}_w"] = w
        g[f"dot_{name}_x"] = xq
        g[f"dot_{name}_y"] = ref_rows(t, w, xq, n_in, n_out)
    r3 = np.random.default_rng(4421)
    for name, t, n_in, n_out in (("iq3xxs_2048", O.IQ3_XXS, 2048, 48), ("iq3s_2048", O.IQ3_S, 2048, 48)):
        w = rand_rows(r3, t, n_out, n_in)
        xq = ref_q8(r3.standard_normal(n_in).astype(np.float32))
        g[f"dot_{name}_w"] = w
        g[f"dot_{name}_x"] = xq
        g[f"dot_{name}_y"] = ref_rows(t, w, xq, n_in, n_out)
    # the reference's expert pairs of other formats (iq_parity.cpp:504-539), with the f32 tokens kept so the whole
    # block can be driven through them: 2 tokens, the second -0.5 x + 0.25; their own generator as above
    rp = np.random.default_rng(504)
    for name, gt, dt, H, F in (("iq2s_iq4nl", O.IQ2_S, O.IQ4_NL, 256, 64), ("iq3xxs_q2", O.IQ3_XXS, O.Q2_0, 256, 64),
                               ("iq3s_iq4nl", O.IQ3_S, O.IQ4_NL, 256, 64), ("iq4xs_q2", O.IQ4_XS, O.Q2_0, 256, 64),
                               ("iq3s_iq4nl_wide", O.IQ3_S, O.IQ4_NL, 1280, 128)):
        blob = np.concatenate([rand_rows(rp, gt, 2 * F, H), rand_rows(rp, dt, H, F)])
        xx = rp.standard_normal((2, H)).astype(np.float32)
        xx[1] = -0.5 * xx[0] + 0.25
        xq = ref_q8(xx.ravel())
        y = np.empty(2 * H, np.float32)
        R.ref_expert_q8(gt, dt, H, F, P(blob, u8p), blob.size, P(xq, u8p), 2, P(y, f32p))
        g[f"pair_{name}_blob"] = blob
        g[f"pair_{name}_x"] = xx
        g[f"pair_{name}_y"] = y
        g[f"pair_{name}_geom"] = np.array([gt, dt, H, F], np.int32)
    out = Path(__file__).with_name("golden.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
