"""ctypes binding of libsmoe.so, the C ABI declared in include/smoe.h.

The library is the product: there is no fallback.  Loading fails loudly when libsmoe.so is missing.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_SO = Path(__file__).resolve().parent / "libsmoe.so"

SMOE_OK, SMOE_INVALID_ARG, SMOE_UNSUPPORTED, SMOE_CUDA_ERROR, SMOE_DEVICE_TIMEOUT = range(5)
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "CUDA_ERROR", 4: "DEVICE_TIMEOUT"}

_vp = C.c_void_p


class SmoeLayer(C.Structure):
    _fields_ = [
        ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_expert", C.c_int), ("k", C.c_int),
        ("gu_type", C.c_int), ("d_type", C.c_int),
        ("router", _vp), ("gate", _vp), ("up", _vp), ("down", _vp),
        ("has_shared", C.c_int), ("sg_type", C.c_int), ("su_type", C.c_int), ("sd_type", C.c_int),
        ("sgate", _vp), ("sup", _vp), ("sdown", _vp), ("gate_inp_shexp", _vp),
    ]


class SmoeTrace(C.Structure):
    _fields_ = [("logits", _vp), ("ids", _vp), ("weights", _vp), ("xq", _vp), ("parts", _vp), ("shared", _vp)]


EP_MAX_WORLD = 8
EP_HANDLE_BYTES = 64


class SmoeEp(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("max_tokens", C.c_int), ("areas", _vp * EP_MAX_WORLD)]


# name -> (restype, argtypes); every symbol include/smoe.h declares
SIGNATURES = {
    "smoe_last_error": (C.c_char_p, []),
    "smoe_device_status": (C.c_uint, [C.c_int]),
    "smoe_row_bytes": (C.c_size_t, [C.c_int, C.c_int64]),
    "smoe_q8_1_bytes": (C.c_size_t, [C.c_int64]),
    "smoe_f32_to_bf16_bulk": (C.c_int, [_vp, _vp, C.c_int64, _vp]),
    "smoe_bf16_gemv": (C.c_int, [_vp, _vp, _vp, C.c_int64, C.c_int64, C.c_int64, _vp]),
    "smoe_router_top10": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp]),
    "smoe_router": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp]),
    "smoe_iq_quantize_q8_1": (C.c_int, [_vp, C.c_int64, _vp, _vp]),
    "smoe_iq_mmvq": (C.c_int, [C.c_int, _vp, _vp, C.c_int64, C.c_int64, C.c_int64, _vp, _vp]),
    "smoe_iq_swiglu_q8": (C.c_int, [_vp, _vp, C.c_int64, _vp, _vp]),
    "smoe_moe_combine": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int64, C.c_int, C.c_int, _vp]),
    "smoe_moe_group_scratch_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "smoe_moe_group": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp]),
    "smoe_set_stage_events": (None, [C.POINTER(_vp), C.c_int]),
    "smoe_moe_group_noalloc": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp]),
    "smoe_rms_norm_weighted": (C.c_int, [_vp, _vp, C.c_int64, C.c_int64, C.c_float, _vp]),
    "smoe_add_rms_norm": (C.c_int, [_vp, _vp, _vp, C.c_int64, C.c_int64, C.c_float, _vp]),
    "smoe_set_expert_path": (C.c_int, [C.c_int]),
    "smoe_s2_blob_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "smoe_s2_pack_expert": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, _vp, _vp]),
    "smoe_quantize_q8_0": (C.c_int, [_vp, _vp, _vp, C.c_int64, _vp]),
    "smoe_moe_grouped_scratch_bytes": (C.c_size_t, [C.c_int64, C.c_int64, C.c_int64]),
    "smoe_moe_grouped_s2": (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_int64, C.c_int64, C.c_int, C.c_int, _vp, _vp,
                                      _vp, _vp, _vp]),
    "smoe_moe_group_resident": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "smoe_moe_hit_select": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp]),
    "smoe_moe_hit_grouped_s2": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int64, C.c_int64, C.c_int, C.c_int, _vp, _vp,
                                          C.c_int, _vp, _vp, _vp]),
    "smoe_moe_hit_add": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int64, C.c_int64, _vp]),
    "smoe_native_experts_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "smoe_native_experts_close": (None, [_vp]),
    "smoe_native_experts_pick": (C.c_int, [_vp, C.c_int64, C.c_int64, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                           C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(_vp)]),
    "smoe_expert_cache_open": (C.c_int, [C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.POINTER(_vp)]),
    "smoe_expert_cache_close": (None, [_vp]),
    "smoe_expert_cache_ensure": (C.c_int, [_vp, C.c_int64, C.c_int64, _vp, C.c_int64, _vp, C.POINTER(C.c_int32)]),
    "smoe_expert_cache_slot_of": (C.c_int32, [_vp, C.c_int64, C.c_int64]),
    "smoe_expert_cache_arena": (_vp, [_vp]),
    "smoe_expert_cache_row": (_vp, [_vp, C.c_int64]),
    "smoe_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "smoe_gguf_close": (None, [_vp]),
    "smoe_gguf_tensor": (C.c_int, [_vp, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_uint64),
                                   C.POINTER(_vp)]),
    "smoe_gguf_load_layer": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(SmoeLayer), C.POINTER(_vp)]),
    "smoe_gguf_free_layer": (None, [_vp]),
    "smoe_stack_decode_scratch_bytes": (C.c_size_t, [C.POINTER(SmoeLayer)]),
    "smoe_stack_decode": (C.c_int, [C.POINTER(SmoeLayer), C.c_int, C.POINTER(_vp), C.c_float, _vp, _vp, _vp,
                                    C.c_size_t, _vp]),
    "smoe_expert_path_for": (C.c_int, [C.POINTER(SmoeLayer), C.c_int]),
    "smoe_layer_check": (C.c_int, [C.POINTER(SmoeLayer)]),
    "smoe_moe_scratch_bytes": (C.c_size_t, [C.POINTER(SmoeLayer), C.c_int]),
    "smoe_moe_forward": (C.c_int, [C.POINTER(SmoeLayer), _vp, C.c_int, _vp, _vp, C.c_size_t,
                                   C.POINTER(SmoeTrace), _vp]),
    "smoe_ep_area_bytes": (C.c_size_t, [C.POINTER(SmoeLayer), C.c_int, C.c_int]),
    "smoe_ep_area_alloc": (C.c_int, [C.c_size_t, C.POINTER(_vp), _vp]),
    "smoe_ep_area_open": (C.c_int, [_vp, C.POINTER(_vp)]),
    "smoe_ep_area_close": (C.c_int, [_vp]),
    "smoe_ep_area_free": (C.c_int, [_vp]),
    "smoe_ep_init": (C.c_int, [C.POINTER(SmoeEp), C.POINTER(SmoeLayer)]),
    "smoe_ep_scratch_bytes": (C.c_size_t, [C.POINTER(SmoeLayer), C.POINTER(SmoeEp)]),
    "smoe_ep_forward": (C.c_int, [C.POINTER(SmoeLayer), C.POINTER(SmoeEp), _vp, C.c_int, _vp, _vp, C.c_size_t,
                                  C.POINTER(SmoeTrace), C.c_int, _vp]),
}

_lib: C.CDLL | None = None


def lib_path() -> Path:
    return _SO


def lib() -> C.CDLL:
    """The loaded library (RTLD_GLOBAL so one copy serves every caller)."""
    global _lib
    if _lib is None:
        if not _SO.exists():
            raise RuntimeError(f"{_SO} is missing: run `python -m stratametal_b200.build` (no fallback exists)")
        L = C.CDLL(str(_SO), mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class SmoeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def check(status: int) -> None:
    if status != SMOE_OK:
        raise SmoeError(status, lib().smoe_last_error().decode())
