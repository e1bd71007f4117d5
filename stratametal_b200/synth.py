"""Seeded synthetic MoE layers in the reference's GGUF block formats.

Every value is a pure function of (seed, layer, tensor, expert, index): a 32-bit counter hash, evaluated
with torch integer ops, so a layer is generated identically on any device and any expert-parallel shard
can generate just its own experts.  Normal variates use Box-Muller in float64.

Distributions (the choices the configs leave open are marked *):
  x                     fp32 ~ N(0, 1)                                   [T, n_embd]
  ffn_gate_inp          fp32 ~ N(0, 0.02), stored bf16 (RNE)             [n_expert, n_embd]
                        cfg1: row e scaled by a calibrated factor so expert popularity follows Zipf(1.1)
  ffn_{gate,up,down}_exps, *_shexp   Q2_0: codes uniform in {0..3}, fp16 d = |N(0, 0.05)| per 64-block
  IQ2_S gate/up (cfg4)  qs / qh bytes uniform (10-bit grid index uniform over 1024), sign bytes uniform,
                        4-bit sub-scales uniform in [0, 15]*, fp16 d = |N(0, 0.05)| per 256-block
  ffn_gate_inp_shexp*   fp32 ~ N(0, 0.02), stored bf16
"""
from __future__ import annotations

import functools
import struct
import math
from dataclasses import dataclass, field

import numpy as np
import torch

Q2_0 = 42
IQ2_S = 22
IQ4_NL = 20
IQ4_XS = 23
IQ3_XXS = 18
IQ3_S = 21
M32 = 0xFFFFFFFF
# (values, bytes) per block of each format
BLOCKS = {Q2_0: (64, 18), IQ2_S: (256, 82), IQ4_NL: (32, 18), IQ4_XS: (256, 136), IQ3_XXS: (256, 98), IQ3_S: (256, 110)}

# tensor ids inside a layer's key
T_ROUTER, T_GINP, T_GATE, T_UP, T_DOWN, T_SGATE, T_SUP, T_SDOWN, T_X = range(1, 10)


def _mix_py(*vals: int) -> int:
    """Host-side key derivation (Python ints, splitmix64 finalizer)."""
    h = 0x9E3779B97F4A7C15
    for v in vals:
        h = (h ^ (v & 0xFFFFFFFFFFFFFFFF)) * 0xBF58476D1CE4E5B9 & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
        h = h * 0x94D049BB133111EB & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 29
    return h


def _mul32(x: torch.Tensor, c: int) -> torch.Tensor:
    # x * c mod 2^32 without any int64 overflow: split x into 16-bit halves
    hi = ((x >> 16) * c) & 0xFFFF
    return ((hi << 16) + (x & 0xFFFF) * c) & M32


def _hash32(x: torch.Tensor) -> torch.Tensor:
    x = x & M32
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    x = x ^ (x >> 16)
    return x


def hash_u32(key: int, idx: torch.Tensor) -> torch.Tensor:
    """Uniform 32-bit values (as int64) for counter `idx` under `key`."""
    ka, kb = key & M32, (key >> 32) & M32
    return _hash32(_hash32(idx ^ ka) ^ kb)


def uniform01(key: int, idx: torch.Tensor) -> torch.Tensor:
    return (hash_u32(key, idx).to(torch.float64) + 0.5) * (1.0 / 4294967296.0)


def normal(key: int, n: int, device) -> torch.Tensor:
    """n standard normals (float64) by Box-Muller over counters 2i, 2i + 1."""
    i = torch.arange(n, dtype=torch.int64, device=device)
    u1 = uniform01(key, 2 * i)
    u2 = uniform01(key, 2 * i + 1)
    return torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * math.pi * u2)


def random_bytes(key: int, n: int, device) -> torch.Tensor:
    """n uniform bytes (uint8), n a multiple of 4."""
    assert n % 4 == 0
    h = hash_u32(key, torch.arange(n // 4, dtype=torch.int64, device=device))
    b = torch.stack([(h >> (8 * j)) & 0xFF for j in range(4)], dim=1)
    return b.reshape(-1).to(torch.uint8)


def fp16_bytes(v: torch.Tensor) -> torch.Tensor:
    """float64 -> fp16 (round to nearest even) -> 2 little-endian bytes per value."""
    h = v.to(torch.float32).to(torch.float16).view(torch.int16).to(torch.int64) & 0xFFFF
    return torch.stack([h & 0xFF, h >> 8], dim=1).to(torch.uint8)


def row_bytes(t: int, n: int) -> int:
    if t not in BLOCKS:
        raise ValueError(f"type {t}")
    v, b = BLOCKS[t]
    assert n % v == 0
    return n // v * b


def quant_matrix(t: int, key: int, rows: int, n_in: int, device, d_sigma: float = 0.05) -> torch.Tensor:
    """rows x n_in weights of type t as raw blocks (uint8 [rows * row_bytes])."""
    if t == Q2_0:
        nb = rows * (n_in // 64)
        d = fp16_bytes(normal(_mix_py(key, 1), nb, device).abs() * d_sigma)
        qs = random_bytes(_mix_py(key, 2), nb * 16, device).view(nb, 16)
        return torch.cat([d, qs], dim=1).reshape(-1)
    if t in BLOCKS:
        # every other format: fp16 d then uniform bytes (every byte pattern is a valid block: grid indices, signs
        # and sub-scales span their whole fields).  IQ2_S: qs[32] signs[32] qh[8] scales[8]; IQ4_NL: qs[16];
        # IQ4_XS: scales_h, scales_l[4], qs[128]; IQ3_XXS: qs[64], sign/scale words[8]; IQ3_S: qs[64] qh[8]
        # signs[32] scales[4]
        v, b = BLOCKS[t]
        nb = rows * (n_in // v)
        d = fp16_bytes(normal(_mix_py(key, 1), nb, device).abs() * d_sigma)
        nr = (b - 2 + 3) // 4 * 4
        rest = random_bytes(_mix_py(key, 2), nb * nr, device).view(nb, nr)[:, :b - 2]
        return torch.cat([d, rest], dim=1).reshape(-1)
    raise ValueError(f"type {t}")


def bf16_bits(v: torch.Tensor) -> torch.Tensor:
    """float -> bf16 (round to nearest even) bits as uint16-valued int16 storage."""
    return v.to(torch.float32).to(torch.bfloat16).view(torch.int16)


# ---------------------------------------------------------------------------------------------------
# Zipf routing calibration (cfg1)
# ---------------------------------------------------------------------------------------------------

@functools.lru_cache(maxsize=8)
def zipf_row_scales(n_expert: int, k: int, s: float = 1.1, seed: int = 110, cap: float = 0.45,
                    iters: int = 40, n_sim: int = 4096) -> np.ndarray:
    """Factors f[rank] for router rows so that the chance a token selects the rank-r expert follows
    Zipf(s) (capped at `cap`; scaling a row cannot push it past 1/2 for a symmetric activation).

    The logit of expert e is ~ f_e * g_e with g_e iid normal, so the calibration simulates that directly
    and moves each f multiplicatively toward its target inclusion rate.  Deterministic (seeded)."""
    rng = np.random.default_rng(seed)
    r = np.arange(1, n_expert + 1, dtype=np.float64)
    p = r ** -s
    q = k * p / p.sum()
    for _ in range(50):  # cap and hand the excess to the uncapped ranks
        over = q > cap
        if not over.any():
            break
        excess = (q[over] - cap).sum()
        q[over] = cap
        free = ~over
        q[free] += excess * q[free] / q[free].sum()
    f = np.ones(n_expert)
    g = rng.standard_normal((n_sim, n_expert))
    for _ in range(iters):
        logits = g * f
        top = np.argpartition(-logits, k - 1, axis=1)[:, :k]
        freq = np.bincount(top.ravel(), minlength=n_expert) / n_sim
        f *= np.clip((q / np.maximum(freq, 0.5 / n_sim)) ** 0.5, 0.5, 2.0)
        f /= np.exp(np.log(f).mean())
    f.flags.writeable = False  # cached: shared by every caller
    return f


# ---------------------------------------------------------------------------------------------------
# layers
# ---------------------------------------------------------------------------------------------------

@dataclass
class LayerSpec:
    n_embd: int = 2048
    n_ff: int = 512
    n_expert: int = 512
    k: int = 10
    gu_type: int = Q2_0
    d_type: int = Q2_0
    has_shared: bool = True
    sg_type: int = Q2_0
    su_type: int = Q2_0
    sd_type: int = Q2_0
    zipf: float | None = None     # cfg1: Zipf exponent of expert popularity
    seed: int = 2024

    def expert_bytes(self) -> int:
        return 2 * self.n_ff * row_bytes(self.gu_type, self.n_embd) + self.n_embd * row_bytes(self.d_type, self.n_ff)


@dataclass
class Layer:
    """One layer's tensors (torch, on `device`), keyed by their GGUF names."""
    spec: LayerSpec
    index: int
    tensors: dict = field(default_factory=dict)

    def __getitem__(self, name):
        return self.tensors[name]


def router_weights(spec: LayerSpec, index: int, device="cpu") -> torch.Tensor:
    """Layer `index`'s ffn_gate_inp (bf16 bits [n_expert, n_embd]) alone, as make_layer generates it."""
    H, E = spec.n_embd, spec.n_expert
    base = _mix_py(spec.seed, index)
    w = normal(_mix_py(base, T_ROUTER), E * H, device).view(E, H) * 0.02
    if spec.zipf is not None:
        f = zipf_row_scales(E, spec.k, spec.zipf)
        perm = np.random.default_rng(_mix_py(base, 77) & M32).permutation(E)
        scale = np.empty(E)
        scale[perm] = f  # expert perm[r] gets the rank-r factor
        w = w * torch.from_numpy(scale).to(device=device, dtype=torch.float64).view(E, 1)
    return bf16_bits(w).contiguous()


def make_layer(spec: LayerSpec, index: int, device="cpu", experts: range | None = None) -> Layer:
    """Generate layer `index` of `spec` on `device`.  `experts` limits the routed planes to a subset
    (an expert-parallel shard); the default generates all n_expert."""
    H, F, E = spec.n_embd, spec.n_ff, spec.n_expert
    base = _mix_py(spec.seed, index)
    L = Layer(spec, index)
    L.tensors["ffn_gate_inp.weight"] = router_weights(spec, index, device)
    ex = experts if experts is not None else range(E)
    for name, tid, t, rows, n_in in (("ffn_gate_exps.weight", T_GATE, spec.gu_type, F, H),
                                     ("ffn_up_exps.weight", T_UP, spec.gu_type, F, H),
                                     ("ffn_down_exps.weight", T_DOWN, spec.d_type, H, F)):
        parts = [quant_matrix(t, _mix_py(base, tid, e), rows, n_in, device) for e in ex]
        L.tensors[name] = torch.cat(parts).contiguous()
    if spec.has_shared:
        L.tensors["ffn_gate_inp_shexp.weight"] = bf16_bits(normal(_mix_py(base, T_GINP), H, device) * 0.02)
        L.tensors["ffn_gate_shexp.weight"] = quant_matrix(spec.sg_type, _mix_py(base, T_SGATE), F, H, device)
        L.tensors["ffn_up_shexp.weight"] = quant_matrix(spec.su_type, _mix_py(base, T_SUP), F, H, device)
        L.tensors["ffn_down_shexp.weight"] = quant_matrix(spec.sd_type, _mix_py(base, T_SDOWN), H, F, device)
    return L


def make_x(seed: int, T: int, n_embd: int, device="cpu", stream: int = 0) -> torch.Tensor:
    """T tokens of N(0, 1) activations (float32)."""
    return normal(_mix_py(seed, T_X, stream), T * n_embd, device).view(T, n_embd).to(torch.float32)


# The five BASELINE configurations.
def config_spec(cfg: int, seed: int | None = None) -> tuple[LayerSpec, int]:
    """(layer spec, tokens per call) of BASELINE configs[cfg]."""
    if cfg == 0:
        return LayerSpec(seed=seed or 20240), 1
    if cfg == 1:
        return LayerSpec(zipf=1.1, seed=seed or 20241), 64
    if cfg == 2:
        return LayerSpec(seed=seed or 20242), 4096
    if cfg == 3:
        return LayerSpec(seed=seed or 20243), 1
    if cfg == 4:
        return LayerSpec(gu_type=IQ2_S, seed=seed or 20244), 8
    raise ValueError(cfg)


def write_native_pack(pack_dir, layers: list[list[np.ndarray]], gu_type: int, d_type: int, version: int = 4) -> None:
    """A pack's expert file: experts.bin = every layer's expert blobs back to back (layers in order), and
    native_experts.txt with the header and one "layer gu_type d_type offset blob_bytes" line per layer (the format
    metal/src/pack.cpp:367-416 reads).  layers[l][e] is expert e's blob (uint8) of layer l."""
    from pathlib import Path
    d = Path(pack_dir)
    d.mkdir(parents=True, exist_ok=True)
    n_expert = len(layers[0])
    lines = [f"# strata native experts v{version} (n_expert {n_expert})"]
    off = 0
    with open(d / "experts.bin", "wb") as f:
        for li, blobs in enumerate(layers):
            assert len(blobs) == n_expert and len({b.size for b in blobs}) == 1
            lines.append(f"{li} {gu_type} {d_type} {off} {blobs[0].size}")
            for b in blobs:
                f.write(np.ascontiguousarray(b, np.uint8).tobytes())
            off += blobs[0].size * n_expert
    (d / "native_experts.txt").write_text("\n".join(lines) + "\n")


GGUF_BF16, GGUF_F32 = 30, 0


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _gguf_value(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<IB", 7, int(v))
    if isinstance(v, int):
        return struct.pack("<IQ", 10, v) if v >= 2 ** 32 else struct.pack("<II", 4, v)
    if isinstance(v, float):
        return struct.pack("<If", 6, v)
    if isinstance(v, str):
        return struct.pack("<I", 8) + _gguf_str(v)
    if isinstance(v, list):  # arrays of strings or of int32
        if all(isinstance(x, str) for x in v):
            return struct.pack("<IIQ", 9, 8, len(v)) + b"".join(_gguf_str(x) for x in v)
        return struct.pack("<IIQ", 9, 5, len(v)) + b"".join(struct.pack("<i", x) for x in v)
    raise TypeError(type(v))


def write_gguf(path, tensors: list, meta: dict, alignment: int = 32, version: int = 3) -> None:
    """A GGUF file: the header, the metadata `meta` (int, float, bool, str, list of str or int), then each tensor
    (name, ggml type, ne tuple with ne[0] fastest, raw bytes) at an aligned offset of the data section."""
    kv = dict(meta)
    if alignment != 32:
        kv["general.alignment"] = alignment
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kv))
    head += b"".join(_gguf_str(k) + _gguf_value(v) for k, v in kv.items())
    off, infos, datas = 0, [], []
    for name, ttype, ne, data in tensors:
        infos.append(_gguf_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne) +
                     struct.pack("<IQ", ttype, off))
        data = bytes(data)
        pad = (-len(data)) % alignment
        datas.append(data + bytes(pad))
        off += len(data) + pad
    head += b"".join(infos)
    head += bytes((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for d in datas:
            f.write(d)


def layer_gguf_tensors(lay: Layer, index: int, router_f32: bool = False) -> list:
    """The MoE tensors of a synthetic layer under the names of layer `index` of a GGUF model (blk.<L>.<name>)."""
    sp = lay.spec
    H, F, E = sp.n_embd, sp.n_ff, sp.n_expert
    t = {k: v.cpu().numpy() for k, v in lay.tensors.items()}
    pre = f"blk.{index}."
    r = t["ffn_gate_inp.weight"].view(np.uint16)
    if router_f32:  # stored as f32 (its bf16 values exactly)
        rt, rb = GGUF_F32, (r.astype(np.uint32) << 16).view(np.float32).tobytes()
    else:
        rt, rb = GGUF_BF16, r.tobytes()
    out = [(pre + "ffn_gate_inp.weight", rt, (H, E), rb),
           (pre + "ffn_gate_exps.weight", sp.gu_type, (H, F, E), t["ffn_gate_exps.weight"].tobytes()),
           (pre + "ffn_up_exps.weight", sp.gu_type, (H, F, E), t["ffn_up_exps.weight"].tobytes()),
           (pre + "ffn_down_exps.weight", sp.d_type, (F, H, E), t["ffn_down_exps.weight"].tobytes())]
    if sp.has_shared:
        out += [(pre + "ffn_gate_shexp.weight", sp.sg_type, (H, F), t["ffn_gate_shexp.weight"].tobytes()),
                (pre + "ffn_up_shexp.weight", sp.su_type, (H, F), t["ffn_up_shexp.weight"].tobytes()),
                (pre + "ffn_down_shexp.weight", sp.sd_type, (F, H), t["ffn_down_shexp.weight"].tobytes()),
                (pre + "ffn_gate_inp_shexp.weight", GGUF_BF16, (H,), t["ffn_gate_inp_shexp.weight"].view(np.uint16).tobytes())]
    return out
