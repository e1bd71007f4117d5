"""The GGUF reader of the model boundary (smoe_gguf_*, include/smoe_gguf.hpp) on the host: the tensor directory,
shapes, types and data of a synthetic model written in the GGUF v3 format, metadata of every value type, and the
files it refuses (bad magic or version, a tensor listed twice, data past the end, a misaligned offset)."""
import ctypes as C
import struct

import numpy as np
import pytest

from stratametal_b200 import api, synth
from stratametal_b200._lib import SmoeError


def small_model(path, alignment=32):
    spec = synth.LayerSpec(n_embd=256, n_ff=64, n_expert=8, k=2, seed=3)
    lays = [synth.make_layer(spec, li) for li in range(2)]
    tensors = synth.layer_gguf_tensors(lays[0], 0) + synth.layer_gguf_tensors(lays[1], 1, router_f32=True)
    meta = {"general.architecture": "qwen4exp", "qwen4exp.expert_used_count": 2, "qwen4exp.block_count": 2,
            "general.name": "synthetic", "qwen4exp.rope.freq_base": 1.0e6, "tokenizer.ggml.tokens": ["a", "bb", "ccc"],
            "qwen4exp.layer_types": [0, 1], "general.big": 2 ** 40, "general.flag": True}
    synth.write_gguf(path, tensors, meta, alignment=alignment)
    return tensors, lays


@pytest.mark.parametrize("alignment", [32, 64])
def test_tensor_directory(tmp_path, alignment):
    p = tmp_path / "m.gguf"
    tensors, _ = small_model(p, alignment)
    m = api.GgufModel(p)
    try:
        for name, ttype, ne, data in tensors:
            t = m.tensor(name)
            assert t["type"] == ttype and t["ne"][:len(ne)] == tuple(ne) and t["bytes"] == len(data), name
            assert C.string_at(t["data"], len(data)) == bytes(data), name
        with pytest.raises(SmoeError):
            m.tensor("blk.2.ffn_gate_exps.weight")
    finally:
        m.close()


def corrupt(tmp_path, fn):
    p = tmp_path / "m.gguf"
    small_model(p)
    b = bytearray(p.read_bytes())
    b = fn(b)
    p.write_bytes(bytes(b))
    return p


@pytest.mark.parametrize("fn,why", [
    (lambda b: b"XXXX" + b[4:], "magic"),
    (lambda b: b[:4] + struct.pack("<I", 1) + b[8:], "version"),
    (lambda b: b[:2000], "truncated"),
])
def test_refusals(tmp_path, fn, why):
    with pytest.raises(SmoeError) as e:
        api.GgufModel(corrupt(tmp_path, fn))
    assert why in str(e.value) or why == "truncated"


def test_duplicate_and_past_the_end(tmp_path):
    t = [("a", 0, (8,), bytes(32)), ("a", 0, (8,), bytes(32))]
    synth.write_gguf(tmp_path / "d.gguf", t, {})
    with pytest.raises(SmoeError) as e:
        api.GgufModel(tmp_path / "d.gguf")
    assert "twice" in str(e.value)
    synth.write_gguf(tmp_path / "e.gguf", [("a", 0, (64,), bytes(256))], {})
    p = tmp_path / "e.gguf"
    p.write_bytes(p.read_bytes()[:-100])
    with pytest.raises(SmoeError) as e:
        api.GgufModel(p)
    assert "past the end" in str(e.value)
