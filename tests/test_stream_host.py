"""The pack's expert file reader (smoe_native_experts_*: native_experts.txt over a mapped experts.bin) on the host:
the offsets and bytes it picks, and the index errors the reference's reader refuses (metal/src/pack.cpp:367-416).
The admission rules of the VRAM tier (Residency, include/smoe_stream.hpp) are checked by tests/cpp/stream_test.cpp."""
import ctypes as C

import numpy as np
import pytest

from stratametal_b200 import api, synth
from stratametal_b200._lib import SmoeError


def blobs(n_layers, n_expert, nbytes, seed=1):
    rng = np.random.default_rng(seed)
    return [[rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(n_expert)] for _ in range(n_layers)]


def test_pick_offsets_and_bytes(tmp_path):
    L = blobs(3, 5, 96)
    synth.write_native_pack(tmp_path, L, 21, 20)
    nx = api.NativeExperts(tmp_path)
    try:
        for li in range(3):
            for e in range(5):
                p = nx.pick(li, e)
                assert (p["gu_type"], p["d_type"], p["blob_bytes"]) == (21, 20, 96)
                assert p["file_off"] == (li * 5 + e) * 96
                got = np.frombuffer(C.string_at(p["host_blob"], 96), np.uint8)
                assert np.array_equal(got, L[li][e])
        with pytest.raises(SmoeError):
            nx.pick(0, 5)          # expert outside 0..n_expert-1
        with pytest.raises(SmoeError):
            nx.pick(3, 0)          # layer not in the index
    finally:
        nx.close()


@pytest.mark.parametrize("text,why", [
    ("# strata native experts v4 (n_expert 2)\n0 42 42 0 16\n0 42 42 32 16\n", "repeated"),
    ("# strata native experts v4 (n_expert 2)\n0 42 42 zero 16\n", "malformed"),
    ("# strata native experts v5 (n_expert 2)\n0 42 42 0 16\n", "v5"),
    ("# strata native experts v4\n0 42 42 0 16\n", "n_expert"),
])
def test_index_refusals(tmp_path, text, why):
    (tmp_path / "native_experts.txt").write_text(text)
    (tmp_path / "experts.bin").write_bytes(bytes(64))
    with pytest.raises(SmoeError) as e:
        api.NativeExperts(tmp_path)
    assert why in str(e.value)


def test_non_contiguous_layers_are_refused(tmp_path):
    (tmp_path / "native_experts.txt").write_text("# strata native experts v4 (n_expert 2)\n0 42 42 0 16\n1 42 42 48 16\n")
    (tmp_path / "experts.bin").write_bytes(bytes(96))
    nx = api.NativeExperts(tmp_path)
    try:
        assert nx.pick(0, 1)["file_off"] == 16
        with pytest.raises(SmoeError) as e:
            nx.pick(1, 0)          # layer 1 must start at 2 x 16
        assert "contiguous" in str(e.value)
    finally:
        nx.close()


def test_short_experts_bin_is_refused(tmp_path):
    synth.write_native_pack(tmp_path, blobs(1, 2, 32), 42, 42)
    (tmp_path / "experts.bin").write_bytes(bytes(40))
    nx = api.NativeExperts(tmp_path)
    try:
        with pytest.raises(SmoeError):
            nx.pick(0, 1)
    finally:
        nx.close()
