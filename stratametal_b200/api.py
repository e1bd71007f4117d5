"""Python front end of the C ABI, for tests, benches and Python callers (torch tensors in, device pointers out).

Function names and argument meaning follow the reference's per-kernel host API
(metal/include/strata/metal/{router,moe_combine,iq,bf16_gemv}.hpp); errors raise SmoeError where the
reference throws MetalError.  Every call enqueues on torch's current CUDA stream.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import synth
from ._lib import SmoeError, SmoeLayer, SmoeTrace, check, lib

__all__ = ["SmoeError", "f32_to_bf16_bulk", "bf16_gemv", "router_top10", "router", "iq_quantize_q8_1", "iq_mmvq",
           "iq_swiglu_q8", "moe_combine", "moe_group", "row_bytes", "q8_1_bytes", "MoeLayer", "device_status",
           "set_expert_path", "rms_norm_weighted", "add_rms_norm"]


def _s() -> int:
    """torch's current stream.  The C ABI refuses the null (legacy default) stream, as the reference's
    contract does (native_router.hpp:15): run under `torch.cuda.stream(...)` / `torch.cuda.set_stream`."""
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def row_bytes(t: int, n: int) -> int:
    return int(lib().smoe_row_bytes(t, n))


def q8_1_bytes(n: int) -> int:
    return int(lib().smoe_q8_1_bytes(n))


def device_status(clear: bool = True) -> int:
    return int(lib().smoe_device_status(1 if clear else 0))


def rms_norm_weighted(x: torch.Tensor, w: torch.Tensor | None, rows: int, cols: int, eps: float) -> None:
    check(lib().smoe_rms_norm_weighted(_p(x), _p(w), rows, cols, eps, _s()))


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor | None, w: torch.Tensor | None, rows: int, cols: int,
                 eps: float) -> None:
    """x = rms_norm(x + residual) * w in place: the step between two MoE blocks of a layer stack."""
    check(lib().smoe_add_rms_norm(_p(x), _p(residual), _p(w), rows, cols, eps, _s()))


def set_expert_path(path: int) -> None:
    """0 automatic, 1 the SIMT expert kernels, 2 the fp16 tensor-core expert kernels where the layer qualifies,
    3 the fused single-token kernel where the batch is one token and the layer qualifies, 4 the int8 tensor-core
    kernels of the integer contract where the layer qualifies."""
    check(lib().smoe_set_expert_path(path))


def f32_to_bf16_bulk(x: torch.Tensor, y: torch.Tensor, n: int | None = None) -> None:
    check(lib().smoe_f32_to_bf16_bulk(_p(x), _p(y), x.numel() if n is None else n, _s()))


def bf16_gemv(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, n_in: int, n_out: int, n_col: int = 1) -> None:
    check(lib().smoe_bf16_gemv(_p(x), _p(w), _p(y), n_in, n_out, n_col, _s()))


def router_top10(logits: torch.Tensor, n_tokens: int, n_expert: int, k: int, ids: torch.Tensor,
                 weights: torch.Tensor) -> None:
    check(lib().smoe_router_top10(_p(logits), n_tokens, n_expert, k, _p(ids), _p(weights), _s()))


def router(x: torch.Tensor, w: torch.Tensor, n_tokens: int, n_embd: int, n_expert: int, k: int,
           logits: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> None:
    check(lib().smoe_router(_p(x), _p(w), n_tokens, n_embd, n_expert, k, _p(logits), _p(ids), _p(weights), _s()))


def iq_quantize_q8_1(x: torch.Tensor, n: int, y: torch.Tensor) -> None:
    check(lib().smoe_iq_quantize_q8_1(_p(x), n, _p(y), _s()))


def iq_mmvq(t: int, w: torch.Tensor, x_q8: torch.Tensor, n_in: int, n_out: int, n_col: int, y: torch.Tensor) -> None:
    check(lib().smoe_iq_mmvq(t, _p(w), _p(x_q8), n_in, n_out, n_col, _p(y), _s()))


def iq_swiglu_q8(gate: torch.Tensor, up: torch.Tensor, n: int, y: torch.Tensor) -> None:
    check(lib().smoe_iq_swiglu_q8(_p(gate), _p(up), n, _p(y), _s()))


def moe_combine(parts: torch.Tensor, weights: torch.Tensor, shared: torch.Tensor | None, y: torch.Tensor,
                n_embd: int, k: int, n_tok: int = 1) -> None:
    check(lib().smoe_moe_combine(_p(parts), _p(weights), _p(shared), _p(y), n_embd, k, n_tok, _s()))


def moe_group(ids: torch.Tensor, n_tok: int, k: int, n_expert: int, scratch: torch.Tensor, slot: torch.Tensor,
              src: torch.Tensor | None) -> None:
    check(lib().smoe_moe_group(_p(ids), n_tok, k, n_expert, _p(scratch), _p(slot), _p(src), _s()))


def moe_group_scratch_bytes(n_tok: int, k: int, n_expert: int) -> int:
    return int(lib().smoe_moe_group_scratch_bytes(n_tok, k, n_expert))


@dataclass
class Trace:
    logits: torch.Tensor
    ids: torch.Tensor
    weights: torch.Tensor
    xq: torch.Tensor
    parts: torch.Tensor
    shared: torch.Tensor


def layer_struct(t: dict, sp: synth.LayerSpec) -> SmoeLayer:
    """The C ABI's layer descriptor over device tensors keyed by their GGUF names."""
    c = SmoeLayer()
    c.n_embd, c.n_ff, c.n_expert, c.k = sp.n_embd, sp.n_ff, sp.n_expert, sp.k
    c.gu_type, c.d_type = sp.gu_type, sp.d_type
    c.router = _p(t["ffn_gate_inp.weight"])
    c.gate = _p(t["ffn_gate_exps.weight"])
    c.up = _p(t["ffn_up_exps.weight"])
    c.down = _p(t["ffn_down_exps.weight"])
    if sp.has_shared:
        c.has_shared = 1
        c.sg_type, c.su_type, c.sd_type = sp.sg_type, sp.su_type, sp.sd_type
        c.sgate = _p(t["ffn_gate_shexp.weight"])
        c.sup = _p(t["ffn_up_shexp.weight"])
        c.sdown = _p(t["ffn_down_shexp.weight"])
        c.gate_inp_shexp = _p(t["ffn_gate_inp_shexp.weight"])
    return c


def trace_struct(trace: "Trace | None") -> SmoeTrace | None:
    if trace is None:
        return None
    return SmoeTrace(_p(trace.logits), _p(trace.ids), _p(trace.weights), _p(trace.xq), _p(trace.parts),
                     _p(trace.shared))


def make_trace(sp: synth.LayerSpec, T: int, device) -> "Trace":
    return Trace(logits=torch.empty(T, sp.n_expert, dtype=torch.float32, device=device),
                 ids=torch.empty(T, sp.k, dtype=torch.int32, device=device),
                 weights=torch.empty(T, sp.k, dtype=torch.float32, device=device),
                 xq=torch.empty(T, q8_1_bytes(sp.n_embd), dtype=torch.uint8, device=device),
                 parts=torch.empty(T, sp.k, sp.n_embd, dtype=torch.float32, device=device),
                 shared=torch.zeros(T, sp.n_embd, dtype=torch.float32, device=device))


class MoeLayer:
    """One MoE layer resident on the device plus its scratch arena; `forward` is smoe_moe_forward."""

    def __init__(self, layer: synth.Layer, max_tokens: int, device: torch.device | str = "cuda"):
        sp = layer.spec
        self.spec = sp
        self.device = torch.device(device)
        self.t = {k: v.to(self.device).contiguous() for k, v in layer.tensors.items()}
        c = layer_struct(self.t, sp)
        self.c = c
        check(lib().smoe_layer_check(c))
        self.max_tokens = max_tokens
        nbytes = int(lib().smoe_moe_scratch_bytes(c, max_tokens))
        self.scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        off = (-self.scratch.data_ptr()) % 256
        self.scratch_ptr = self.scratch.data_ptr() + off
        self.scratch_bytes = nbytes

    def make_trace(self, T: int) -> Trace:
        return make_trace(self.spec, T, self.device)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, trace: Trace | None = None) -> torch.Tensor:
        T = x.shape[0]
        if T > self.max_tokens:
            raise SmoeError(1, f"{T} tokens exceed the arena's {self.max_tokens}")
        if out is None:
            out = torch.empty(T, self.spec.n_embd, dtype=torch.float32, device=self.device)
        tr = trace_struct(trace)
        import ctypes as C
        check(lib().smoe_moe_forward(C.byref(self.c), _p(x), T, _p(out), self.scratch_ptr, self.scratch_bytes,
                                     C.byref(tr) if tr is not None else None, _s()))
        return out


def expert_path_for(m: "MoeLayer", n_tokens: int) -> int:
    """The expert path smoe_moe_forward takes for this layer and batch (smoe_expert_path_for): 1 SIMT, 2 fp16 tensor
    cores, 3 fused single-token kernel, 4 int8 tensor cores."""
    import ctypes as C
    return int(lib().smoe_expert_path_for(C.byref(m.c), n_tokens))


# ---- the pack's planar S2 experts, the grouped / hit decode API, and expert streaming -------------------------------
def s2_blob_bytes(n_embd: int, n_ff: int) -> int:
    return int(lib().smoe_s2_blob_bytes(n_embd, n_ff))


def s2_pack_expert(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, n_embd: int, n_ff: int,
                   blob: torch.Tensor) -> None:
    """One expert's GGUF Q2_0 rows (device) -> its planar S2 blob (device)."""
    check(lib().smoe_s2_pack_expert(_p(gate), _p(up), _p(down), n_embd, n_ff, _p(blob), _s()))


def quantize_q8_0(x: torch.Tensor, n: int, blocks: torch.Tensor, scales: torch.Tensor | None = None) -> None:
    check(lib().smoe_quantize_q8_0(_p(x), _p(blocks), _p(scales), n, _s()))


def moe_grouped_scratch_bytes(cap_entries: int, n_embd: int, n_ff: int) -> int:
    return int(lib().smoe_moe_grouped_scratch_bytes(cap_entries, n_embd, n_ff))


def moe_grouped_s2(grp_ptr, grp_start, n_groups, ent_dst, ent_tok, cap_groups: int, cap_entries: int, n_embd: int,
                   n_ff: int, x_q8_0, x_scales, scratch, out) -> None:
    check(lib().smoe_moe_grouped_s2(_p(grp_ptr), _p(grp_start), _p(n_groups), _p(ent_dst), _p(ent_tok), cap_groups,
                                    cap_entries, n_embd, n_ff, _p(x_q8_0), _p(x_scales), _p(scratch), _p(out), _s()))


def moe_group_resident(ids, n: int, k_per_tok: int, base: int, blob_bytes: int, grp_ptr, grp_start, counts, ent_dst,
                       ent_tok) -> None:
    check(lib().smoe_moe_group_resident(_p(ids), n, k_per_tok, base, blob_bytes, _p(grp_ptr), _p(grp_start),
                                        _p(counts), _p(ent_dst), _p(ent_tok), _s()))


def moe_hit_select(ids, res_row: int, n: int, n_expert: int, slot, dst, count) -> None:
    """res_row: a device address (an ExpertCache row, or a tensor's data_ptr())."""
    check(lib().smoe_moe_hit_select(_p(ids), res_row, n, n_expert, _p(slot), _p(dst), _p(count), _s()))


def moe_hit_grouped_s2(blob_base: int, slot_index, dst_index, d_count, cap: int, blob_bytes: int, n_embd: int, n_ff: int,
                       x_q8_0, x_scales, k_per_token: int, scratch, out) -> None:
    check(lib().smoe_moe_hit_grouped_s2(blob_base, _p(slot_index), _p(dst_index), _p(d_count), cap, blob_bytes, n_embd,
                                        n_ff, _p(x_q8_0), _p(x_scales), k_per_token, _p(scratch), _p(out), _s()))


def moe_hit_add(parts, hit_out, dst, count, cap: int, n_embd: int) -> None:
    check(lib().smoe_moe_hit_add(_p(parts), _p(hit_out), _p(dst), _p(count), cap, n_embd, _s()))


class NativeExperts:
    """The pack's expert file (native_experts.txt over a mapped experts.bin): pick(layer, expert)."""

    def __init__(self, pack_dir: str):
        import ctypes as C
        h = C.c_void_p()
        check(lib().smoe_native_experts_open(str(pack_dir).encode(), C.byref(h)))
        self.h = h

    def pick(self, layer: int, expert: int) -> dict:
        import ctypes as C
        gu, d = C.c_int(), C.c_int()
        off, nb = C.c_uint64(), C.c_uint64()
        ptr = C.c_void_p()
        check(lib().smoe_native_experts_pick(self.h, layer, expert, C.byref(gu), C.byref(d), C.byref(off),
                                             C.byref(nb), C.byref(ptr)))
        return {"gu_type": gu.value, "d_type": d.value, "file_off": off.value, "blob_bytes": nb.value,
                "host_blob": ptr.value}

    def close(self) -> None:
        if self.h:
            lib().smoe_native_experts_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


class ExpertCache:
    """The VRAM expert tier: ensure(layer, expert, host_ptr, nbytes) -> slot (or -1 when full)."""

    def __init__(self, n_slots: int, n_layers: int, n_expert: int, blob_bytes: int, per_layer: bool = False):
        import ctypes as C
        h = C.c_void_p()
        check(lib().smoe_expert_cache_open(n_slots, n_layers, n_expert, blob_bytes, 1 if per_layer else 0, C.byref(h)))
        self.h, self.blob_bytes = h, blob_bytes

    def ensure(self, layer: int, expert: int, host_ptr: int, nbytes: int) -> int:
        import ctypes as C
        slot = C.c_int32()
        check(lib().smoe_expert_cache_ensure(self.h, layer, expert, host_ptr, nbytes, _s(), C.byref(slot)))
        return slot.value

    def slot_of(self, layer: int, expert: int) -> int:
        return int(lib().smoe_expert_cache_slot_of(self.h, layer, expert))

    def arena(self) -> int:
        return int(lib().smoe_expert_cache_arena(self.h))

    def row(self, layer: int) -> int:
        return int(lib().smoe_expert_cache_row(self.h, layer) or 0)

    def close(self) -> None:
        if self.h:
            torch.cuda.synchronize()
            lib().smoe_expert_cache_close(self.h)
            self.h = None


class GgufModel:
    """A GGUF file mapped read-only (smoe_gguf_*): tensors by name, and MoE layers uploaded to the device."""

    def __init__(self, path):
        import ctypes as C
        h = C.c_void_p()
        check(lib().smoe_gguf_open(str(path).encode(), C.byref(h)))
        self.h = h

    def tensor(self, name: str) -> dict:
        import ctypes as C
        t, nb, ptr = C.c_int(), C.c_uint64(), C.c_void_p()
        ne = (C.c_int64 * 4)()
        check(lib().smoe_gguf_tensor(self.h, name.encode(), C.byref(t), ne, C.byref(nb), C.byref(ptr)))
        return {"type": t.value, "ne": tuple(ne), "bytes": nb.value, "data": ptr.value}

    def load_layer(self, layer: int, with_shared: bool = True, k: int = 0) -> "GgufMoeLayer":
        return GgufMoeLayer(self, layer, with_shared, k)

    def close(self) -> None:
        if self.h:
            lib().smoe_gguf_close(self.h)
            self.h = None


class GgufMoeLayer:
    """One MoE layer uploaded from a GGUF model (the device planes are owned here); forward as MoeLayer."""

    def __init__(self, model: GgufModel, layer: int, with_shared: bool, k: int, max_tokens: int = 64,
                 device: torch.device | str = "cuda"):
        import ctypes as C
        self.c = SmoeLayer()
        owner = C.c_void_p()
        check(lib().smoe_gguf_load_layer(model.h, layer, 1 if with_shared else 0, k, C.byref(self.c), C.byref(owner)))
        self.owner = owner
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        nbytes = int(lib().smoe_moe_scratch_bytes(C.byref(self.c), max_tokens))
        self.scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        self.scratch_ptr = self.scratch.data_ptr() + (-self.scratch.data_ptr()) % 256
        self.scratch_bytes = nbytes

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        import ctypes as C
        T = x.shape[0]
        if out is None:
            out = torch.empty(T, self.c.n_embd, dtype=torch.float32, device=self.device)
        check(lib().smoe_moe_forward(C.byref(self.c), _p(x), T, _p(out), self.scratch_ptr, self.scratch_bytes, None,
                                     _s()))
        return out

    def close(self) -> None:
        if self.owner:
            torch.cuda.synchronize()
            lib().smoe_gguf_free_layer(self.owner)
            self.owner = None


def stack_decode(layers: list, x: torch.Tensor, out: torch.Tensor, eps: float = 1e-6,
                 norm_w: list | None = None, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """smoe_stack_decode: one token through every layer (x = rms_norm(MoE_l(x) + x)) in one launch per 48 layers.
    layers: MoeLayer objects of one geometry."""
    import ctypes as C
    n = len(layers)
    arr = (SmoeLayer * n)(*[m.c for m in layers])
    nbytes = int(lib().smoe_stack_decode_scratch_bytes(C.byref(layers[0].c)))
    if scratch is None:
        scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=x.device)
    ptr = scratch.data_ptr() + (-scratch.data_ptr()) % 256
    nw = None if norm_w is None else (C.c_void_p * n)(*[None if w is None else w.data_ptr() for w in norm_w])
    check(lib().smoe_stack_decode(arr, n, nw, eps, _p(x), _p(out), ptr, nbytes, _s()))
    return out
