"""Seeded synthetic MoE layers in the MLX affine format.

Distribution (per workload): router weight N(0, gate_std) fp16 [E, H];
integer codes uniform over 0..2^bits-1 packed LSB-first into uint32 words;
per-64-group fp16 scale = |N(0, scale_std)| / ((2^bits - 1) / 2) and bias
= -2^(bits-1) * scale; optional per-expert fp32 correction bias N(0, e_bias_std);
activations N(0, 1) in the activation dtype.

Two generators: ``make_layer_np`` (numpy PCG64, CPU; small layers, golden
fixtures) and ``make_layer_torch`` (torch generator on the target device; large
layers).  Both are deterministic for a given seed; they do not produce the same
values as each other.
"""
from __future__ import annotations

import hashlib

import numpy as np

from .spec import MoESpec


def _f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def act_bits_np(x: np.ndarray, act_dtype: str) -> np.ndarray:
    """fp32 array -> uint16 bit patterns of the activation dtype."""
    if act_dtype == "float16":
        return _f16(x).view(np.uint16)
    return _bf16_bits(x)


def _qmat_np(rng: np.random.Generator, spec: MoESpec, n: int, out_dim: int, in_dim: int):
    words = in_dim * spec.bits // 32
    w = rng.integers(0, 1 << 32, size=(n, out_dim, words), dtype=np.uint64).astype(np.uint32)
    ng = in_dim // spec.group_size
    s = _f16(np.abs(rng.standard_normal((n, out_dim, ng), dtype=np.float32) * spec.scale_std) / spec.scale_den)
    b = _f16(-float(spec.code_mid) * s.astype(np.float32))
    return w, s, b


def make_layer_np(spec: MoESpec, seed: int = 0) -> dict:
    """Numpy layer: dict with gate_w (fp16 [E,H]), e_bias (fp32 [E] or None),
    gate/up/down (w, s, b) stacks and shared (three single-expert triples) or None."""
    spec.validate()
    rng = np.random.default_rng(seed)
    E, H, I = spec.n_experts, spec.hidden, spec.inter
    gate_w = _f16(rng.standard_normal((E, H), dtype=np.float32) * spec.gate_std)
    e_bias = None
    if spec.router == "sigmoid_group":
        e_bias = (rng.standard_normal(E, dtype=np.float32) * spec.e_bias_std).astype(np.float32)
    gate = _qmat_np(rng, spec, E, I, H)
    up = _qmat_np(rng, spec, E, I, H)
    down = _qmat_np(rng, spec, E, H, I)
    shared = None
    if spec.n_shared:
        Is = I * spec.n_shared
        sg = _qmat_np(rng, spec, 1, Is, H)
        su = _qmat_np(rng, spec, 1, Is, H)
        sd = _qmat_np(rng, spec, 1, H, Is)
        shared = tuple(tuple(a[0] for a in m) for m in (sg, su, sd))
    return {"gate_w": gate_w, "e_bias": e_bias, "gate": gate, "up": up, "down": down, "shared": shared}


def make_x_np(spec: MoESpec, T: int, seed: int = 1) -> np.ndarray:
    """Activation bit patterns [T, H] (uint16) of N(0,1) values."""
    rng = np.random.default_rng(seed)
    return act_bits_np(rng.standard_normal((T, spec.hidden), dtype=np.float32), spec.act_dtype)


def layer_digest(layer: dict) -> str:
    """sha256 over every array of a layer (detects generator drift)."""
    h = hashlib.sha256()

    def add(a):
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())

    add(layer["gate_w"])
    add(layer["e_bias"])
    for m in ("gate", "up", "down"):
        for a in layer[m]:
            add(a)
    if layer["shared"] is not None:
        for m in layer["shared"]:
            for a in m:
                add(a)
    return h.hexdigest()


# ---------------------------------------------------------------------------
# torch (device) generator for full-size workloads
# ---------------------------------------------------------------------------
def make_layer_torch(spec: MoESpec, seed: int = 0, device="cuda") -> dict:
    import torch

    spec.validate()
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E, H, I = spec.n_experts, spec.hidden, spec.inter

    def normal(shape, std):
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std

    def qmat(n, out_dim, in_dim):
        words = in_dim * spec.bits // 32
        w = torch.randint(-(1 << 31), 1 << 31, (n, out_dim, words), generator=g, device=device,
                          dtype=torch.int64).to(torch.int32)
        ng = in_dim // spec.group_size
        s = (normal((n, out_dim, ng), spec.scale_std).abs() / spec.scale_den).to(torch.float16)
        b = (-float(spec.code_mid) * s.float()).to(torch.float16)
        return w, s, b

    gate_w = normal((E, H), spec.gate_std).to(torch.float16)
    e_bias = normal((E,), spec.e_bias_std) if spec.router == "sigmoid_group" else None
    out = {"gate_w": gate_w, "e_bias": e_bias, "gate": qmat(E, I, H), "up": qmat(E, I, H),
           "down": qmat(E, H, I), "shared": None}
    if spec.n_shared:
        Is = I * spec.n_shared
        out["shared"] = tuple(tuple(a[0] for a in m) for m in (qmat(1, Is, H), qmat(1, Is, H), qmat(1, H, Is)))
    return out


def make_x_torch(spec: MoESpec, T: int, seed: int = 1, device="cuda"):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    dt = torch.float16 if spec.act_dtype == "float16" else torch.bfloat16
    return torch.randn((T, spec.hidden), generator=g, device=device, dtype=torch.float32).to(dt)
