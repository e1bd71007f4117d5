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
