"""MLX safetensors -> the library's expert layout (no repacking).

mlx_lm stores a quantised MoE layer's experts stacked per projection:
``model.layers.{i}.mlp.switch_mlp.{gate,up,down}_proj.{weight,scales,biases}``
(``weight`` uint32 codes ``[E, out, in*bits/32]``, ``scales``/``biases``
``[E, out, in/group]``), which is the layout the reference reads
(ef_engine_v2.py:88-91) and the one the kernels take.  This module reads a
model's safetensors files (one file, or a directory with
``model.safetensors.index.json``) with the header parsing the reference uses
for its prefetcher (8-byte little-endian header length, JSON header with
``data_offsets`` relative to the end of the header;
experiments/ef_v17_pinned.py:135-152, experiments/ef_v18_prefetch2.py:120-146),
memory-maps each tensor, and assembles one MoE layer: router weight (dequantised
when the checkpoint quantised it), DeepSeek-V3 ``e_score_correction_bias``,
the three stacked projections and ``shared_experts``.

Tensor-name prefixes tried per layer, as the reference's prefetchers do
(experiments/ef_v17_pinned.py:165-169): ``model.layers.{i}.mlp`` (Qwen-MoE,
DeepSeek) and ``model.layers.{i}.block_sparse_moe`` (Mixtral).

Scales and biases are fp16 on the device.  Checkpoints that store them as bf16
are converted; a bf16 value converts exactly whenever it lies in fp16's normal
range, and a layer with any value outside it is rejected rather than rounded.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np

from .spec import MoESpec

# safetensors dtype -> (numpy storage dtype, element bytes); BF16 is kept as its uint16 bits
_DTYPES = {"U32": (np.uint32, 4), "I32": (np.int32, 4), "F32": (np.float32, 4), "F16": (np.float16, 2),
           "BF16": (np.uint16, 2), "U16": (np.uint16, 2), "U8": (np.uint8, 1), "I8": (np.int8, 1)}


@dataclass(frozen=True)
class TensorInfo:
    file: str
    offset: int          # absolute byte offset of the data in `file`
    nbytes: int
    dtype: str           # safetensors dtype string ("U32", "F16", "BF16", ...)
    shape: Tuple[int, ...]


def read_header(path: str) -> Tuple[dict, int]:
    """(header dict, absolute offset of the data section) of one safetensors file."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        n = struct.unpack("<Q", raw)[0]
        if n > 100 * 1024 * 1024:
            raise ValueError(f"{path}: header of {n} bytes")
        header = json.loads(f.read(n))
    return header, 8 + n


class SafetensorsIndex:
    """Tensor name -> location over one safetensors file or a model directory."""

    def __init__(self, path: str):
        self.path = path
        self.tensors: Dict[str, TensorInfo] = {}
        self.config: dict = {}
        if os.path.isdir(path):
            files = []
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    files = sorted(set(json.load(f).get("weight_map", {}).values()))
            else:
                files = sorted(n for n in os.listdir(path) if n.endswith(".safetensors"))
            files = [os.path.join(path, n) for n in files]
            cfg = os.path.join(path, "config.json")
            if os.path.exists(cfg):
                with open(cfg) as f:
                    self.config = json.load(f)
        else:
            files = [path]
        if not files:
            raise FileNotFoundError(f"no safetensors files under {path}")
        for fp in files:
            header, data_start = read_header(fp)
            size = os.path.getsize(fp)
            for name, info in header.items():
                if name == "__metadata__":
                    continue
                a, b = info["data_offsets"]
                if info["dtype"] not in _DTYPES:
                    raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
                ti = TensorInfo(fp, data_start + a, b - a, info["dtype"], tuple(info["shape"]))
                want = int(np.prod(ti.shape, dtype=np.int64)) * _DTYPES[ti.dtype][1]
                if ti.nbytes != want or data_start + b > size:
                    raise ValueError(f"{name}: byte range does not match its shape / the file")
                self.tensors[name] = ti

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def array(self, name: str) -> np.ndarray:
        """Read-only memory map of a tensor (BF16 as its uint16 bit patterns)."""
        ti = self.tensors[name]
        dt = _DTYPES[ti.dtype][0]
        return np.memmap(ti.file, dtype=dt, mode="r", offset=ti.offset, shape=ti.shape)


# ---------------------------------------------------------------------------
_PREFIXES = ("model.layers.{i}.mlp", "model.layers.{i}.block_sparse_moe")
_PROJ = ("gate_proj", "up_proj", "down_proj")


def layer_prefix(index: SafetensorsIndex, layer: int) -> str:
    for p in _PREFIXES:
        pre = p.format(i=layer)
        if f"{pre}.switch_mlp.gate_proj.weight" in index:
            return pre
    raise KeyError(f"layer {layer}: no switch_mlp experts under {[p.format(i=layer) for p in _PREFIXES]}")


def _bf16_to_f16(bits: np.ndarray, what: str) -> np.ndarray:
    f32 = (bits.astype(np.uint32) << 16).view(np.float32)
    f16 = f32.astype(np.float16)
    back = f16.astype(np.float32)
    bad = (back != f32) & np.isfinite(f32)
    if bad.any():
        raise ValueError(f"{what}: {int(bad.sum())} bf16 values are not exact in fp16 (outside its normal range)")
    return f16


def _half(index: SafetensorsIndex, name: str) -> np.ndarray:
    ti = index.tensors[name]
    a = index.array(name)
    if ti.dtype == "F16":
        return np.asarray(a)
    if ti.dtype == "BF16":
        return _bf16_to_f16(np.asarray(a), name)
    if ti.dtype == "F32":
        f16 = np.asarray(a).astype(np.float16)
        if (f16.astype(np.float32) != a).any():
            raise ValueError(f"{name}: fp32 values not exact in fp16")
        return f16
    raise ValueError(f"{name}: expected a float tensor, got {ti.dtype}")


def _qtriple(index: SafetensorsIndex, pre: str):
    w = index.array(f"{pre}.weight")
    if index.tensors[f"{pre}.weight"].dtype not in ("U32", "I32"):
        raise ValueError(f"{pre}.weight: expected packed uint32 codes")
    w = np.asarray(w).view(np.uint32)
    s = _half(index, f"{pre}.scales")
    if f"{pre}.biases" not in index:
        raise ValueError(f"{pre}: no biases (only the affine MLX format is supported)")
    b = _half(index, f"{pre}.biases")
    return w, s, b


def dequantize_np(w: np.ndarray, s: np.ndarray, b: np.ndarray, bits: int, group: int) -> np.ndarray:
    """fp32 s*q + b of MLX affine codes (LSB-first in uint32 words); [..., out, in]."""
    per = 32 // bits
    mask = (1 << bits) - 1
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = (w[..., None] >> shifts) & mask  # [..., out, words, per]
    q = q.reshape(*w.shape[:-1], w.shape[-1] * per).astype(np.float32)
    sf = np.repeat(s.astype(np.float32), group, axis=-1)
    bf = np.repeat(b.astype(np.float32), group, axis=-1)
    return sf * q + bf


def _cfg_get(cfg: dict, *names, default=None):
    for n in names:
        if n in cfg:
            return cfg[n]
    return default


def infer_spec(path_or_index, layer: int, group_size: Optional[int] = None, bits: Optional[int] = None) -> MoESpec:
    """The MoESpec of one MoE layer from its tensors' shapes and dtypes and
    config.json (when the index has one); reads no tensor data."""
    index = path_or_index if isinstance(path_or_index, SafetensorsIndex) else SafetensorsIndex(path_or_index)
    cfg = index.config
    qcfg = cfg.get("quantization", cfg.get("quantization_config", {})) or {}
    group = group_size or int(qcfg.get("group_size", 64))
    pre = layer_prefix(index, layer)
    shape = {p: index.tensors[f"{pre}.switch_mlp.{p}.weight"].shape for p in _PROJ}
    if any(len(v) != 3 for v in shape.values()):
        raise ValueError(f"{pre}.switch_mlp: stacked [E, out, words] codes expected")
    E, inter, words = shape["gate_proj"]
    sname = f"{pre}.switch_mlp.gate_proj.scales"
    if sname not in index:
        raise ValueError(f"{pre}.switch_mlp.gate_proj: no scales")
    hidden = index.tensors[sname].shape[-1] * group
    b = bits or (words * 32 // hidden)
    if words * 32 != hidden * b or b not in (4, 8):
        raise ValueError(f"{pre}: {words} words per row do not give a 4/8-bit code at hidden {hidden}")
    for name, shp in (("up_proj", (E, inter, words)), ("down_proj", (E, hidden, inter * b // 32))):
        if shape[name] != shp:
            raise ValueError(f"{pre}.switch_mlp.{name}: shape {shape[name]}, expected {shp}")
    gname = f"{pre}.gate.weight"
    if f"{pre}.gate.scales" in index:
        gate_dtype = "float16"  # a quantised router is dequantised to fp16
    else:
        gate_dtype = "bfloat16" if index.tensors[gname].dtype == "BF16" else "float16"
    has_bias = f"{pre}.gate.e_score_correction_bias" in index
    n_shared = 0
    sgn = f"{pre}.shared_experts.gate_proj.weight"
    if sgn in index:
        s_inter = index.tensors[sgn].shape[0]
        if s_inter % inter:
            raise ValueError(f"{pre}.shared_experts: inter {s_inter} is not a multiple of {inter}")
        n_shared = s_inter // inter
    sigmoid = has_bias or _cfg_get(cfg, "scoring_func") == "sigmoid"
    spec = MoESpec(
        hidden=hidden, n_experts=E, top_k=int(_cfg_get(cfg, "num_experts_per_tok", "num_experts_per_token",
                                                     default=8)),
        inter=inter, bits=b, group_size=group, router="sigmoid_group" if sigmoid else "softmax",
        norm_topk=bool(_cfg_get(cfg, "norm_topk_prob", default=True)),
        n_group=int(_cfg_get(cfg, "n_group", default=1)) if sigmoid else 1,
        topk_group=int(_cfg_get(cfg, "topk_group", default=1)) if sigmoid else 1,
        routed_scaling=float(_cfg_get(cfg, "routed_scaling_factor", default=1.0)) if sigmoid else 1.0,
        n_shared=n_shared, act_dtype="float16" if _cfg_get(cfg, "torch_dtype") == "float16" else "bfloat16",
        gate_dtype=gate_dtype)
    spec.validate()
    return spec


def load_layer_arrays(path_or_index, layer: int, group_size: Optional[int] = None,
                      bits: Optional[int] = None) -> Tuple[dict, MoESpec]:
    """One MoE layer as the library's layer dict (numpy, memory-mapped codes)
    and the MoESpec that describes it (shapes from the tensors, routing from
    config.json when the index has one)."""
    index = path_or_index if isinstance(path_or_index, SafetensorsIndex) else SafetensorsIndex(path_or_index)
    spec = infer_spec(index, layer, group_size, bits)
    qcfg = index.config.get("quantization", index.config.get("quantization_config", {})) or {}
    pre = layer_prefix(index, layer)
    gate = _qtriple(index, f"{pre}.switch_mlp.gate_proj")
    up = _qtriple(index, f"{pre}.switch_mlp.up_proj")
    down = _qtriple(index, f"{pre}.switch_mlp.down_proj")
    # router
    gname = f"{pre}.gate.weight"
    if f"{pre}.gate.scales" in index:  # quantised router: dequantise once (fp32 -> fp16)
        gw, gs, gb = _qtriple(index, f"{pre}.gate")
        gate_w = dequantize_np(gw, gs, gb, int(qcfg.get("bits", spec.bits)), spec.group_size).astype(np.float16)
    elif index.tensors[gname].dtype == "BF16":
        gate_w = np.asarray(index.array(gname))  # uint16 bit patterns
    else:
        gate_w = _half(index, gname)
    e_bias = None
    ebn = f"{pre}.gate.e_score_correction_bias"
    if ebn in index:
        raw = np.asarray(index.array(ebn))
        e_bias = ((raw.astype(np.uint32) << 16).view(np.float32) if index.tensors[ebn].dtype == "BF16"
                  else raw.astype(np.float32))
    shared = None
    if spec.n_shared:
        shared = tuple(_qtriple(index, f"{pre}.shared_experts.{p}") for p in _PROJ)
    layer_dict = {"gate_w": gate_w, "e_bias": e_bias, "gate": gate, "up": up, "down": down, "shared": shared}
    return layer_dict, spec


def moe_layers(index: SafetensorsIndex) -> list:
    """Layer indices (ascending) whose switch_mlp experts the index holds."""
    out = set()
    for name in index.tensors:
        if name.endswith(".switch_mlp.gate_proj.weight") and name.startswith("model.layers."):
            part = name.split(".")[2]
            if part.isdigit():
                out.add(int(part))
    return sorted(out)


def expert_ranges(index: SafetensorsIndex, layer: int, spec: MoESpec) -> list:
    """Where each expert's bytes lie in the files: 9 ``(file, bf16, offset,
    stride)`` in the order gate w, s, b, up w, s, b, down w, s, b.  A stacked
    tensor [E, ...] is contiguous, so expert e's slice starts at
    ``offset + e * stride`` with stride = tensor bytes / E -- the per-expert
    offsets of the reference's prefetcher (experiments/ef_v18_prefetch2.py:137-146).
    Scales / biases may be F16 or BF16 (bf16 = True: converted on read)."""
    pre = layer_prefix(index, layer)
    H, I, bits, E = spec.hidden, spec.inter, spec.bits, spec.n_experts
    dims = {"gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}
    out = []
    for p in _PROJ:
        rows, cols = dims[p]
        want = {"weight": (rows, cols * bits // 32), "scales": (rows, cols // spec.group_size),
                "biases": (rows, cols // spec.group_size)}
        for part in ("weight", "scales", "biases"):
            name = f"{pre}.switch_mlp.{p}.{part}"
            if name not in index:
                raise KeyError(f"{name}: missing")
            ti = index.tensors[name]
            if ti.shape != (E, *want[part]):
                raise ValueError(f"{name}: shape {ti.shape}, expected {(E, *want[part])}")
            if part == "weight" and ti.dtype not in ("U32", "I32"):
                raise ValueError(f"{name}: expected packed uint32 codes, got {ti.dtype}")
            if part != "weight" and ti.dtype not in ("F16", "BF16"):
                raise ValueError(f"{name}: scales / biases must be F16 or BF16 to stream, got {ti.dtype}")
            out.append((ti.file, ti.dtype == "BF16", ti.offset, ti.nbytes // E))
    return out


def load_moe_layer(path_or_index, layer: int, device="cuda", spec: Optional[MoESpec] = None, **kw):
    """An ``expertflow_b200.moe.MoELayer`` for layer `layer` of a safetensors
    checkpoint, its weights copied to `device` once."""
    import torch
    from .moe import MoELayer

    arrays, inferred = load_layer_arrays(path_or_index, layer, **kw)
    spec = spec or inferred
    if arrays["gate_w"].dtype == np.uint16:  # bf16 router bits
        arrays = dict(arrays, gate_w=torch.from_numpy(np.ascontiguousarray(arrays["gate_w"]).view(np.int16))
                      .view(torch.bfloat16))
    return MoELayer.from_arrays(spec, arrays, device=device)


# ---------------------------------------------------------------------------
def write_safetensors(path: str, tensors: Dict[str, Tuple[np.ndarray, str]], metadata: Optional[dict] = None):
    """Write {name: (array, safetensors dtype)} (arrays in name order, 8-byte
    aligned data); BF16 arrays are given as their uint16 bit patterns."""
    header, off = {}, 0
    names = sorted(tensors)
    for name in names:
        arr, dt = tensors[name]
        n = int(np.asarray(arr).nbytes)
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + n]}
        off += n
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:  # tensor by tensor: no copy of the whole model in memory
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for name in names:
            arr = np.ascontiguousarray(np.asarray(tensors[name][0]))
            f.write(memoryview(arr.reshape(-1).view(np.uint8)))


def layer_tensors(layer_dict: dict, layer: int, prefix: str = "model.layers.{i}.mlp",
                  gate_dtype: str = "F16") -> Dict[str, Tuple[np.ndarray, str]]:
    """A layer dict under mlx_lm tensor names (for tests and exports)."""
    pre = prefix.format(i=layer)
    out = {f"{pre}.gate.weight": (layer_dict["gate_w"], gate_dtype)}
    if layer_dict.get("e_bias") is not None:
        out[f"{pre}.gate.e_score_correction_bias"] = (np.asarray(layer_dict["e_bias"], np.float32), "F32")
    for m, p in zip(("gate", "up", "down"), _PROJ):
        w, s, b = layer_dict[m]
        out[f"{pre}.switch_mlp.{p}.weight"] = (np.asarray(w).view(np.uint32), "U32")
        out[f"{pre}.switch_mlp.{p}.scales"] = (np.asarray(s, np.float16), "F16")
        out[f"{pre}.switch_mlp.{p}.biases"] = (np.asarray(b, np.float16), "F16")
    if layer_dict.get("shared") is not None:
        for (w, s, b), p in zip(layer_dict["shared"], _PROJ):
            out[f"{pre}.shared_experts.{p}.weight"] = (np.asarray(w).view(np.uint32), "U32")
            out[f"{pre}.shared_experts.{p}.scales"] = (np.asarray(s, np.float16), "F16")
            out[f"{pre}.shared_experts.{p}.biases"] = (np.asarray(b, np.float16), "F16")
    return out
