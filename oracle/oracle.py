"""ctypes front end of the CPU checker (TEST INFRASTRUCTURE ONLY).

``liboracle.so`` is the plain-C restatement of StrataMetal's host MoE reference (oracle.c cites the
reference file:line of every function).  ``_ref/libstrata_ref.so``, when it was built, holds the
reference's OWN host references compiled from its parity sources; tests use it to pin the restatement.
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline / reference arm use this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
Q2_0 = 42
IQ2_S = 22
IQ4_NL = 20
IQ4_XS = 23
IQ3_XXS = 18
IQ3_S = 21

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_i32p = C.POINTER(C.c_int32)


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and _ref/ when the reference tree is present)."""
    out = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class OrcLayer(C.Structure):
    _fields_ = [
        ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_expert", C.c_int), ("k", C.c_int),
        ("gu_type", C.c_int), ("d_type", C.c_int),
        ("router", _u16p), ("gate", _u8p), ("up", _u8p), ("down", _u8p),
        ("has_shared", C.c_int), ("sg_type", C.c_int), ("su_type", C.c_int), ("sd_type", C.c_int),
        ("sgate", _u8p), ("sup", _u8p), ("sdown", _u8p), ("ginp", _u16p),
    ]


class OrcTrace(C.Structure):
    _fields_ = [("logits", _f32p), ("ids", _i32p), ("weights", _f32p), ("parts", _f32p),
                ("shared", _f32p), ("xq", _u8p)]


_lib = None
_ref = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            build()
        L = C.CDLL(str(so))
        L.orc_bf16_from_f32.restype = C.c_uint16
        L.orc_bf16_from_f32.argtypes = [C.c_float]
        L.orc_f16_from_f32.restype = C.c_uint16
        L.orc_f16_from_f32.argtypes = [C.c_float]
        L.orc_f32_from_f16.restype = C.c_float
        L.orc_f32_from_f16.argtypes = [C.c_uint16]
        L.orc_row_bytes.restype = C.c_size_t
        L.orc_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.orc_q8_1_bytes.restype = C.c_size_t
        L.orc_q8_1_bytes.argtypes = [C.c_int64]
        L.orc_quant_q8_1.argtypes = [_f32p, C.c_int64, _u8p]
        L.orc_row_dot.restype = C.c_float
        L.orc_row_dot.argtypes = [C.c_int, _u8p, _u8p, C.c_int]
        L.orc_row_dot_variant.restype = C.c_float
        L.orc_row_dot_variant.argtypes = [C.c_int, _u8p, _u8p, C.c_int, C.c_int]
        L.orc_mmvq.argtypes = [C.c_int, _u8p, _u8p, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_swiglu_q8.argtypes = [_f32p, _f32p, C.c_int64, _u8p]
        L.orc_bf16_dot.restype = C.c_float
        L.orc_bf16_dot.argtypes = [_f32p, _u16p, C.c_int]
        L.orc_route.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        L.orc_router.argtypes = [_f32p, C.c_int, _u16p, C.c_int, C.c_int, C.c_int, _f32p, _i32p, _f32p]
        L.orc_router.restype = None
        L.orc_s2_blob_bytes.restype = C.c_size_t
        L.orc_s2_blob_bytes.argtypes = [C.c_int, C.c_int]
        L.orc_s2_pack.argtypes = [_u8p, _u8p, _u8p, C.c_int, C.c_int, _u8p]
        L.orc_quant_q8_0.argtypes = [_f32p, C.c_int64, _u8p, _f32p]
        L.orc_s2_expert.argtypes = [_u8p, C.c_int, C.c_int, _u8p, _f32p, _f32p]
        L.orc_combine.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int]
        L.orc_dequant_row.argtypes = [C.c_int, _u8p, C.c_int, _f32p]
        L.orc_add_rms_norm.argtypes = [_f32p, _f32p, _f32p, C.c_int64, C.c_int64, C.c_float, _f32p]
        L.orc_add_rms_norm.restype = None
        L.orc_moe_layer.restype = C.c_int
        L.orc_moe_layer.argtypes = [C.POINTER(OrcLayer), _f32p, C.c_int, _f32p, C.POINTER(OrcTrace), C.c_int,
                                    C.c_int]
        _lib = L
    return _lib


def ref() -> C.CDLL | None:
    """The reference's own host references, or None when oracle/_ref was not built."""
    global _ref
    if _ref is None:
        so = HERE / "_ref" / "libstrata_ref.so"
        if not so.exists():
            return None
        R = C.CDLL(str(so))
        R.ref_quant_q8_1_block.argtypes = [_f32p, _u8p]
        R.ref_row_dot.restype = C.c_float
        R.ref_row_dot.argtypes = [C.c_int, _u8p, _u8p, C.c_int, C.c_int]
        R.ref_expert_q8.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _u8p, C.c_size_t, _u8p, C.c_int, _f32p]
        R.ref_route.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        R.ref_combine.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        R.ref_bf16_from_f32.restype = C.c_uint16
        R.ref_bf16_from_f32.argtypes = [C.c_float]
        R.ref_f16_from_f32.restype = C.c_uint16
        R.ref_f16_from_f32.argtypes = [C.c_float]
        R.ref_f32_from_f16.restype = C.c_float
        R.ref_f32_from_f16.argtypes = [C.c_uint16]
        _ref = R
    return _ref


# ---------------------------------------------------------------------------------------------------
# numpy conveniences
# ---------------------------------------------------------------------------------------------------

def row_bytes(t: int, n: int) -> int:
    return int(lib().orc_row_bytes(t, n))


def q8_1_bytes(n: int) -> int:
    return int(lib().orc_q8_1_bytes(n))


def quant_q8_1(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(q8_1_bytes(x.size), np.uint8)
    lib().orc_quant_q8_1(_ptr(x, _f32p), x.size, _ptr(y, _u8p))
    return y


def mmvq(t: int, w: np.ndarray, xq: np.ndarray, n_in: int, n_out: int, n_col: int) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint8)
    xq = np.ascontiguousarray(xq, np.uint8)
    y = np.empty(n_col * n_out, np.float32)
    lib().orc_mmvq(t, _ptr(w, _u8p), _ptr(xq, _u8p), n_in, n_out, n_col, _ptr(y, _f32p))
    return y.reshape(n_col, n_out)


def swiglu_q8(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    y = np.empty(q8_1_bytes(g.size), np.uint8)
    lib().orc_swiglu_q8(_ptr(g, _f32p), _ptr(u, _f32p), g.size, _ptr(y, _u8p))
    return y


def route(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    for t in range(T):
        lib().orc_route(_ptr(logits[t], _f32p), E, k, _ptr(ids[t], _i32p), _ptr(w[t], _f32p))
    return ids, w


def router(router_bf16: np.ndarray, x: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The block's router stage for x [T, n_embd]: (logits [T, E], ids [T, k], weights [T, k])."""
    x = np.ascontiguousarray(x, np.float32)
    r = np.ascontiguousarray(router_bf16, np.uint16)
    T, H = x.shape
    E = r.size // H
    logits = np.empty((T, E), np.float32)
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().orc_router(_ptr(x, _f32p), T, _ptr(r, _u16p), E, H, k, _ptr(logits, _f32p), _ptr(ids, _i32p),
                     _ptr(w, _f32p))
    return logits, ids, w


def s2_blob_bytes(H: int, F: int) -> int:
    return int(lib().orc_s2_blob_bytes(H, F))


def s2_pack(gate: np.ndarray, up: np.ndarray, down: np.ndarray, H: int, F: int) -> np.ndarray:
    """One expert's GGUF Q2_0 gate / up / down rows -> the pack's planar S2 blob."""
    g, u, d = (np.ascontiguousarray(a, np.uint8) for a in (gate, up, down))
    blob = np.empty(s2_blob_bytes(H, F), np.uint8)
    lib().orc_s2_pack(_ptr(g, _u8p), _ptr(u, _u8p), _ptr(d, _u8p), H, F, _ptr(blob, _u8p))
    return blob


def quant_q8_0(x: np.ndarray, scaled: bool = False):
    """Q8_0 blocks of x (34 B per 32 values); with scaled=True also the fp32 scales (the CPU contract)."""
    x = np.ascontiguousarray(x, np.float32).ravel()
    y = np.empty(x.size // 32 * 34, np.uint8)
    sc = np.empty(x.size // 32, np.float32) if scaled else None
    lib().orc_quant_q8_0(_ptr(x, _f32p), x.size, _ptr(y, _u8p), None if sc is None else _ptr(sc, _f32p))
    return (y, sc) if scaled else y


def s2_expert(blob: np.ndarray, H: int, F: int, xq: np.ndarray, xs: np.ndarray | None = None) -> np.ndarray:
    """One S2 expert on one token's Q8_0 activation row (and fp32 scales)."""
    b = np.ascontiguousarray(blob, np.uint8)
    q = np.ascontiguousarray(xq, np.uint8)
    s = None if xs is None else np.ascontiguousarray(xs, np.float32)
    out = np.empty(H, np.float32)
    lib().orc_s2_expert(_ptr(b, _u8p), H, F, _ptr(q, _u8p), None if s is None else _ptr(s, _f32p), _ptr(out, _f32p))
    return out


def combine(parts: np.ndarray, w: np.ndarray, shared: np.ndarray | None) -> np.ndarray:
    parts = np.ascontiguousarray(parts, np.float32)
    T, K, N = parts.shape
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty((T, N), np.float32)
    for t in range(T):
        sp = None
        if shared is not None:
            s = np.ascontiguousarray(shared[t], np.float32)
            sp = _ptr(s, _f32p)
        lib().orc_combine(_ptr(parts[t], _f32p), _ptr(w[t], _f32p), sp, _ptr(y[t], _f32p), N, K)
    return y


def dequant_rows(t: int, w: np.ndarray, n_rows: int, n_in: int) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint8)
    rb = row_bytes(t, n_in)
    out = np.empty((n_rows, n_in), np.float32)
    for r in range(n_rows):
        lib().orc_dequant_row(t, _ptr(w[r * rb:], _u8p), n_in, _ptr(out[r], _f32p))
    return out


class HostLayer:
    """Host copies of one MoE layer's tensors, named as the GGUF names them."""

    def __init__(self, n_embd, n_ff, n_expert, k, gu_type, d_type, router, gate, up, down,
                 shared=None):
        self.n_embd, self.n_ff, self.n_expert, self.k = n_embd, n_ff, n_expert, k
        self.gu_type, self.d_type = gu_type, d_type
        self.router = np.ascontiguousarray(router, np.uint16)
        self.gate = np.ascontiguousarray(gate, np.uint8)
        self.up = np.ascontiguousarray(up, np.uint8)
        self.down = np.ascontiguousarray(down, np.uint8)
        self.shared = shared  # dict(sg_type, su_type, sd_type, sgate, sup, sdown, ginp) or None
        if shared is not None:
            for key in ("sgate", "sup", "sdown"):
                shared[key] = np.ascontiguousarray(shared[key], np.uint8)
            shared["ginp"] = np.ascontiguousarray(shared["ginp"], np.uint16)

    def c_struct(self) -> OrcLayer:
        L = OrcLayer()
        L.n_embd, L.n_ff, L.n_expert, L.k = self.n_embd, self.n_ff, self.n_expert, self.k
        L.gu_type, L.d_type = self.gu_type, self.d_type
        L.router = _ptr(self.router, _u16p)
        L.gate, L.up, L.down = _ptr(self.gate, _u8p), _ptr(self.up, _u8p), _ptr(self.down, _u8p)
        if self.shared is not None:
            s = self.shared
            L.has_shared = 1
            L.sg_type, L.su_type, L.sd_type = s["sg_type"], s["su_type"], s["sd_type"]
            L.sgate, L.sup, L.sdown = _ptr(s["sgate"], _u8p), _ptr(s["sup"], _u8p), _ptr(s["sdown"], _u8p)
            L.ginp = _ptr(s["ginp"], _u16p)
        return L


def moe_layer(layer: HostLayer, x: np.ndarray, mode: int = 0, n_threads: int | None = None,
              trace: bool = False):
    """The whole block for T tokens: out [T, n_embd]; with trace, also the stage outputs."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    H, E, K = layer.n_embd, layer.n_expert, layer.k
    out = np.empty((T, H), np.float32)
    tr = None
    bufs = {}
    if trace:
        bufs = dict(logits=np.empty((T, E), np.float32), ids=np.empty((T, K), np.int32),
                    weights=np.empty((T, K), np.float32), parts=np.empty((T, K, H), np.float32),
                    shared=np.zeros((T, H), np.float32), xq=np.empty((T, q8_1_bytes(H)), np.uint8))
        tr = OrcTrace(_ptr(bufs["logits"], _f32p), _ptr(bufs["ids"], _i32p), _ptr(bufs["weights"], _f32p),
                      _ptr(bufs["parts"], _f32p), _ptr(bufs["shared"], _f32p), _ptr(bufs["xq"], _u8p))
    if n_threads is None:
        n_threads = os.cpu_count() or 1
    L = layer.c_struct()
    rc = lib().orc_moe_layer(C.byref(L), _ptr(x, _f32p), T, _ptr(out, _f32p), C.byref(tr) if tr else None,
                             mode, n_threads)
    if rc != 0:
        raise ValueError("oracle: bad layer geometry or routed id")
    return (out, bufs) if trace else out


def add_rms_norm(x: np.ndarray, residual: np.ndarray | None = None, w: np.ndarray | None = None,
                 eps: float = 1e-6) -> np.ndarray:
    """rms_norm_weighted's host rule (elementwise_parity.cpp:84-100) after an optional residual add."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    out = np.empty_like(x)
    r = None if residual is None else np.ascontiguousarray(residual, np.float32)
    ww = None if w is None else np.ascontiguousarray(w, np.float32)
    lib().orc_add_rms_norm(_ptr(x, _f32p), None if r is None else _ptr(r, _f32p),
                           None if ww is None else _ptr(ww, _f32p), rows, cols, eps, _ptr(out, _f32p))
    return out


def moe_stack(layers: list, x: np.ndarray, eps: float = 1e-6, mode: int = 0) -> np.ndarray:
    """The configs[3] stack: per layer x = rms_norm(x + moe_layer(x)) with unit weight."""
    for hl in layers:
        x = add_rms_norm(moe_layer(hl, x, mode=mode), x, None, eps)
    return x


def rel_l1(a: np.ndarray, b: np.ndarray) -> float:
    """sum |a - b| / sum |a| over all elements (the reference's rel_l1, pack_parity.cpp:2425-2433)."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.abs(a).sum()
    num = np.abs(a - b).sum()
    if den == 0:
        return 0.0 if num == 0 else 1.0
    return float(num / den)
