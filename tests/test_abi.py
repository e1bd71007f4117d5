"""The C ABI library without a GPU: it loads, exports every symbol include/smoe.h declares, and refuses or
no-ops the argument cases the reference refuses or no-ops (router.mm:32-37, iq.mm:150-158,
moe_combine.mm:31-38) before any CUDA call."""
import ctypes as C
import re
from pathlib import Path

import pytest

from stratametal_b200 import _lib, build

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def L():
    build.build()
    return _lib.lib()


def declared_symbols():
    text = (ROOT / "include" / "smoe.h").read_text()
    return sorted(set(re.findall(r"\b(smoe_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(L):
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "the ctypes table and the header disagree"


def test_geometry(L):
    assert L.smoe_row_bytes(42, 2048) == 576
    assert L.smoe_row_bytes(42, 512) == 144
    assert L.smoe_row_bytes(22, 2048) == 656
    assert L.smoe_row_bytes(22, 2000) == 0
    assert L.smoe_row_bytes(29, 256) == 0          # IQ1_M blocks are not this product (iq_parity.cpp:570-575)
    assert L.smoe_q8_1_bytes(2048) == 2304
    assert L.smoe_q8_1_bytes(33) == 0


def test_router_refusals(L):
    bad = 1
    assert L.smoe_router_top10(None, 1, 128, 65, None, None, None) == bad      # k = 65
    assert L.smoe_router_top10(None, 1, 1025, 1, None, None, None) == bad     # 1025 experts
    assert L.smoe_router_top10(None, -1, 32, 4, None, None, None) == bad      # negative count
    assert L.smoe_router_top10(None, 1, 4, 8, None, None, None) == bad        # k above n_expert
    assert b"k exceeds n_expert" in L.smoe_last_error()
    assert L.smoe_router_top10(None, 0, 512, 10, None, None, None) == 0      # zero tokens: no launch
    assert L.smoe_last_error() == b""


def test_mmvq_and_combine_refusals(L):
    assert L.smoe_iq_mmvq(29, None, None, 256, 4, 1, None, None) == 2         # unsupported type
    assert L.smoe_iq_mmvq(42, None, None, 100, 4, 1, None, None) == 1         # not whole blocks
    assert L.smoe_iq_mmvq(42, None, None, -64, 4, 1, None, None) == 1         # negative
    assert L.smoe_iq_mmvq(42, None, None, 0, 4, 1, None, None) == 0           # zero: no launch
    assert L.smoe_iq_mmvq(20, None, None, 48, 4, 1, None, None) == 1         # IQ4_NL: not whole blocks
    assert L.smoe_iq_mmvq(23, None, None, 256, 4, 1, None, None) == 1        # IQ4_XS: no stream
    assert L.smoe_moe_combine(None, None, None, None, 16, 65, 1, None) == 1   # k = 65
    assert L.smoe_moe_combine(None, None, None, None, -1, 4, 1, None) == 1    # negative
    assert L.smoe_moe_combine(None, None, None, None, 0, 10, 1, None) == 0    # zero length
    assert L.smoe_moe_combine(None, None, None, None, 256, 0, 1, None) == 0
    assert L.smoe_iq_swiglu_q8(None, None, 48, None, None) == 1               # partial block
    assert L.smoe_iq_quantize_q8_1(None, 40, None, None) == 1
    assert L.smoe_iq_quantize_q8_1(None, 0, None, None) == 0


def test_null_stream_is_refused(L):
    # every call enqueues on an explicit stream; null is refused before anything runs
    assert L.smoe_router_top10(C.c_void_p(16), 1, 512, 10, C.c_void_p(16), C.c_void_p(16), None) == 1
    assert b"stream" in L.smoe_last_error()


def layer_struct(**kw):
    c = _lib.SmoeLayer()
    c.n_embd, c.n_ff, c.n_expert, c.k = 2048, 512, 512, 10
    c.gu_type = c.d_type = 42
    c.router = c.gate = c.up = c.down = 256
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_layer_check(L):
    assert L.smoe_layer_check(C.byref(layer_struct())) == 0
    assert L.smoe_layer_check(C.byref(layer_struct(k=65))) == 1
    assert L.smoe_layer_check(C.byref(layer_struct(n_expert=1025))) == 1
    assert L.smoe_layer_check(C.byref(layer_struct(gu_type=14))) == 2
    assert L.smoe_layer_check(C.byref(layer_struct(gate=258))) == 1            # misaligned plane
    assert L.smoe_layer_check(C.byref(layer_struct(gu_type=22))) == 0
    # the other formats of the reference's expert packs take the any-format path (5)
    for gu, d in ((21, 20), (18, 42), (23, 42), (22, 20)):
        assert L.smoe_layer_check(C.byref(layer_struct(gu_type=gu, d_type=d))) == 0
        assert L.smoe_expert_path_for(C.byref(layer_struct(gu_type=gu, d_type=d)), 8) == 5
    assert L.smoe_expert_path_for(C.byref(layer_struct()), 64) in (1, 4)
    assert L.smoe_row_bytes(18, 512) == 196 and L.smoe_row_bytes(21, 256) == 110 and L.smoe_row_bytes(20, 64) == 36
    assert L.smoe_layer_check(C.byref(layer_struct(gu_type=20, n_embd=2112))) == 0   # IQ4_NL: 32-value blocks
    assert L.smoe_layer_check(C.byref(layer_struct(gu_type=21, n_embd=2112))) == 2   # IQ3_S: not whole blocks
    assert L.smoe_moe_scratch_bytes(C.byref(layer_struct()), 64) > 64 * 11 * 2048 * 4
    # zero tokens: OK before any launch
    assert L.smoe_moe_forward(C.byref(layer_struct()), None, 0, None, None, 0, None, None) == 0
