"""Expert parallelism for the MoE block (smoe_ep_* in include/smoe.h).

Rank r of `world` keeps the router and the shared expert whole and routed experts
[r * E / world, (r + 1) * E / world).  The exchange itself (token rows to the owners of their experts, down rows
back to the token's rank) runs inside the library over peer memory; this module sets it up: it allocates each
rank's exchange area, swaps the areas' IPC handles through torch.distributed (any backend: NCCL on the GPU box,
gloo in the CPU tests) and refuses, on every rank, a group whose ranks disagree on the geometry.

Two ways to hold a group:
  * `EpAreas.distributed(...)`: one process per GPU, the normal deployment;
  * `EpAreas.local(...)`: every rank in this process on one device (tests): run phase 1 of every rank, then
    phase 2 of every rank, then phase 4 (`run_local_step`), so that no kernel waits for one launched after it.

Reference counterpart: none for the data path (the reference has no collective layer; its second GPU is an
expert tier reached through peer reads or mapped host memory, include/strata/core/peer_experts.hpp:35-104).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import synth
from ._lib import EP_HANDLE_BYTES, EP_MAX_WORLD, SmoeEp, SmoeError, SmoeLayer, check, lib
from .api import Trace, _p, _s, layer_struct, make_trace, trace_struct

__all__ = ["expert_range", "geometry_key", "agree", "EpAreas", "EpLayer", "run_local_step", "shard_layer"]


def expert_range(n_expert: int, rank: int, world: int) -> range:
    """The routed experts rank `rank` owns."""
    if not 1 <= world <= EP_MAX_WORLD or not 0 <= rank < world:
        raise SmoeError(1, f"ep: need 1 <= world <= {EP_MAX_WORLD} and 0 <= rank < world")
    if n_expert % world:
        raise SmoeError(1, f"ep: {n_expert} experts do not split over {world} ranks")
    n = n_expert // world
    return range(rank * n, (rank + 1) * n)


def shard_layer(spec: synth.LayerSpec, index: int, rank: int, world: int, device) -> synth.Layer:
    """Layer `index` as rank `rank` holds it: router and shared expert whole, its own routed experts."""
    return synth.make_layer(spec, index, device, experts=expert_range(spec.n_expert, rank, world))


def geometry_key(spec: synth.LayerSpec, world: int, max_tokens: int) -> tuple:
    """What every rank of a group must agree on."""
    return (world, max_tokens, spec.n_embd, spec.n_ff, spec.n_expert, spec.k, spec.gu_type, spec.d_type,
            bool(spec.has_shared))


def agree(payload, key: tuple, group=None) -> list:
    """All-gather (payload, key) over the process group; every rank raises when the keys differ, so no rank
    goes on to a step that the others will not take."""
    import torch.distributed as dist
    ws = dist.get_world_size(group)
    objs = [None] * ws
    dist.all_gather_object(objs, (payload, key), group=group)
    keys = [o[1] for o in objs]
    if any(k != keys[0] for k in keys):
        raise SmoeError(1, f"ep: ranks disagree on the group geometry: {keys}")
    return [o[0] for o in objs]


def _area_bytes(spec: synth.LayerSpec, max_tokens: int, world: int) -> int:
    c = SmoeLayer()
    c.n_embd, c.n_ff, c.n_expert, c.k = spec.n_embd, spec.n_ff, spec.n_expert, spec.k
    n = int(lib().smoe_ep_area_bytes(C.byref(c), max_tokens, world))
    if n == 0:
        raise SmoeError(1, "ep: no exchange area for this geometry (n_embd % 128, k, max_tokens, world)")
    return n


class EpAreas:
    """The exchange areas of one group as this process addresses them (one rank's view)."""

    def __init__(self, rank: int, world: int, max_tokens: int, areas: list[int], owned: list[int],
                 opened: list[int]):
        self.rank, self.world, self.max_tokens = rank, world, max_tokens
        self.areas = areas
        self._owned, self._opened = owned, opened
        self._inited = False

    def desc(self) -> SmoeEp:
        d = SmoeEp()
        d.rank, d.world, d.max_tokens = self.rank, self.world, self.max_tokens
        for i, a in enumerate(self.areas):
            d.areas[i] = a
        return d

    @staticmethod
    def _alloc(nbytes: int, want_handle: bool) -> tuple[int, bytes | None]:
        p = C.c_void_p()
        h = (C.c_ubyte * EP_HANDLE_BYTES)() if want_handle else None
        check(lib().smoe_ep_area_alloc(nbytes, C.byref(p), h))
        return p.value, (bytes(h) if want_handle else None)

    @classmethod
    def local(cls, spec: synth.LayerSpec, world: int, max_tokens: int) -> list["EpAreas"]:
        """`world` ranks inside this process on the current device: one view per rank."""
        nbytes = _area_bytes(spec, max_tokens, world)
        areas = [cls._alloc(nbytes, False)[0] for _ in range(world)]
        views = [cls(r, world, max_tokens, list(areas), [], []) for r in range(world)]
        views[0]._owned = list(areas)  # freed once, through rank 0's view
        return views

    @classmethod
    def distributed(cls, spec: synth.LayerSpec, max_tokens: int, group=None) -> "EpAreas":
        """This process's rank of a group spanning torch.distributed's process group (one GPU per rank)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        expert_range(spec.n_expert, rank, world)
        nbytes = _area_bytes(spec, max_tokens, world)
        own, handle = cls._alloc(nbytes, True)
        try:
            handles = agree(handle, geometry_key(spec, world, max_tokens) + (nbytes,), group)
        except Exception:
            lib().smoe_ep_area_free(C.c_void_p(own))
            raise
        areas, opened = [], []
        for p, h in enumerate(handles):
            if p == rank:
                areas.append(own)
                continue
            ptr = C.c_void_p()
            buf = (C.c_ubyte * EP_HANDLE_BYTES).from_buffer_copy(h)
            check(lib().smoe_ep_area_open(buf, C.byref(ptr)))
            areas.append(ptr.value)
            opened.append(ptr.value)
        return cls(rank, world, max_tokens, areas, [own], opened)

    def init(self, c: SmoeLayer) -> None:
        if not self._inited:
            check(lib().smoe_ep_init(C.byref(self.desc()), C.byref(c)))
            self._inited = True

    def close(self) -> None:
        """Unmap the other ranks' areas and free this rank's (after every rank finished its last step)."""
        for a in self._opened:
            lib().smoe_ep_area_close(C.c_void_p(a))
        for a in self._owned:
            lib().smoe_ep_area_free(C.c_void_p(a))
        self._opened, self._owned = [], []


class EpLayer:
    """One rank's part of an expert-parallel MoE layer; `forward` is smoe_ep_forward."""

    def __init__(self, layer: synth.Layer, areas: EpAreas, device: torch.device | str = "cuda"):
        sp = layer.spec
        self.spec, self.areas = sp, areas
        self.device = torch.device(device)
        self.t = {k: v.to(self.device).contiguous() for k, v in layer.tensors.items()}
        n_local = sp.n_expert // areas.world
        if self.t["ffn_gate_exps.weight"].numel() != n_local * sp.n_ff * synth.row_bytes(sp.gu_type, sp.n_embd):
            raise SmoeError(1, "ep: the routed planes must hold exactly this rank's experts")
        self.c = layer_struct(self.t, sp)
        self.ep = areas.desc()
        areas.init(self.c)
        nbytes = int(lib().smoe_ep_scratch_bytes(C.byref(self.c), C.byref(self.ep)))
        if nbytes == 0:
            check(lib().smoe_ep_init(C.byref(self.ep), C.byref(self.c)))  # raises with the reason
        self.scratch = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        self.scratch_ptr = self.scratch.data_ptr() + (-self.scratch.data_ptr()) % 256
        self.scratch_bytes = nbytes

    def make_trace(self, T: int) -> Trace:
        return make_trace(self.spec, T, self.device)

    def forward(self, x: torch.Tensor | None, out: torch.Tensor | None = None, trace: Trace | None = None,
                phases: int = 7, n_tokens: int | None = None) -> torch.Tensor | None:
        T = (x.shape[0] if x is not None else 0) if n_tokens is None else n_tokens
        if out is None and (phases & 4):
            out = torch.empty(max(T, 1), self.spec.n_embd, dtype=torch.float32, device=self.device)
        tr = trace_struct(trace)
        check(lib().smoe_ep_forward(C.byref(self.c), C.byref(self.ep), _p(x), T, _p(out), self.scratch_ptr,
                                    self.scratch_bytes, C.byref(tr) if tr is not None else None, phases, _s()))
        return out


def run_local_step(layers: list[EpLayer], xs: list[torch.Tensor], outs: list[torch.Tensor],
                   traces: list[Trace | None] | None = None) -> None:
    """One step of a group whose ranks all live in this process (EpAreas.local), phase by phase over the ranks:
    every wait a kernel makes is already satisfied when it starts."""
    traces = traces or [None] * len(layers)
    for ph in (1, 2, 4):
        for L, x, o, tr in zip(layers, xs, outs, traces):
            L.forward(x, o, tr, phases=ph, n_tokens=x.shape[0])
