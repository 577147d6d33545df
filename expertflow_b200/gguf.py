"""GGUF checkpoints: header parsing, expert byte ranges, a writer for tests.

The reference reads DeepSeek-style GGUF models by parsing each file's header
(magic, version, tensor and key/value counts, typed metadata values, tensor
infos, data section aligned to ``general.alignment``; ef_deepseek_mmap.py:148-270)
and slicing single experts out of the stacked ``blk.{i}.ffn_{gate,up,down}_exps``
tensors (``expert_bytes = tensor_bytes // n_experts``) or reading the per-expert
``blk.{i}.ffn_{gate,up,down}.{e}.weight`` tensors of Mixtral-style files
(ef_deepseek_mmap.py:431-568).  This module restates that reader (same
function names and error behaviour: ``ValueError("Not a GGUF file")`` for a bad
magic, ``struct.error`` for a truncated header, ``FileNotFoundError`` for a
directory without ``.gguf`` files) and adds ``write_gguf`` so tests and
benchmarks can build files.  K-quant blocks (Q2_K / Q3_K / Q4_K) are decoded on
the GPU by ``ef_kquant_*``.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
GGUF_VERSION = 3

# GGML tensor types
GGML_TYPE_F32, GGML_TYPE_F16 = 0, 1
GGML_TYPE_Q4_0, GGML_TYPE_Q4_1, GGML_TYPE_Q5_0, GGML_TYPE_Q5_1, GGML_TYPE_Q8_0, GGML_TYPE_Q8_1 = 2, 3, 6, 7, 8, 9
GGML_TYPE_Q2_K, GGML_TYPE_Q3_K, GGML_TYPE_Q4_K, GGML_TYPE_Q5_K, GGML_TYPE_Q6_K, GGML_TYPE_Q8_K = 10, 11, 12, 13, 14, 15
GGML_TYPE_IQ2_XXS, GGML_TYPE_IQ2_XS, GGML_TYPE_IQ3_XXS, GGML_TYPE_IQ1_S = 16, 17, 18, 19
GGML_TYPE_IQ4_NL, GGML_TYPE_IQ3_S, GGML_TYPE_IQ2_S, GGML_TYPE_IQ4_XS = 20, 21, 22, 23
GGML_TYPE_IQ1_M, GGML_TYPE_BF16 = 29, 30

QK_K = 256
# type -> (elements per block, bytes per block)
GGML_BLOCK_SIZES = {
    GGML_TYPE_F32: (1, 4), GGML_TYPE_F16: (1, 2), GGML_TYPE_BF16: (1, 2),
    GGML_TYPE_Q4_0: (32, 18), GGML_TYPE_Q4_1: (32, 20), GGML_TYPE_Q5_0: (32, 22), GGML_TYPE_Q5_1: (32, 24),
    GGML_TYPE_Q8_0: (32, 34), GGML_TYPE_Q8_1: (32, 36),
    GGML_TYPE_Q2_K: (QK_K, 84), GGML_TYPE_Q3_K: (QK_K, 110), GGML_TYPE_Q4_K: (QK_K, 144),
    GGML_TYPE_Q5_K: (QK_K, 176), GGML_TYPE_Q6_K: (QK_K, 210), GGML_TYPE_Q8_K: (QK_K, 292),
    GGML_TYPE_IQ1_S: (QK_K, 50), GGML_TYPE_IQ1_M: (QK_K, 56), GGML_TYPE_IQ2_XXS: (QK_K, 66),
    GGML_TYPE_IQ2_XS: (QK_K, 74), GGML_TYPE_IQ2_S: (QK_K, 84), GGML_TYPE_IQ3_XXS: (QK_K, 98),
    GGML_TYPE_IQ3_S: (QK_K, 110), GGML_TYPE_IQ4_NL: (32, 18), GGML_TYPE_IQ4_XS: (QK_K, 136),
}
KQUANT_TYPES = (GGML_TYPE_Q2_K, GGML_TYPE_Q3_K, GGML_TYPE_Q4_K)

# metadata value types
(GGUF_TYPE_UINT8, GGUF_TYPE_INT8, GGUF_TYPE_UINT16, GGUF_TYPE_INT16, GGUF_TYPE_UINT32, GGUF_TYPE_INT32,
 GGUF_TYPE_FLOAT32, GGUF_TYPE_BOOL, GGUF_TYPE_STRING, GGUF_TYPE_ARRAY, GGUF_TYPE_UINT64, GGUF_TYPE_INT64,
 GGUF_TYPE_FLOAT64) = range(13)
_SCALAR = {GGUF_TYPE_UINT8: "<B", GGUF_TYPE_INT8: "<b", GGUF_TYPE_UINT16: "<H", GGUF_TYPE_INT16: "<h",
           GGUF_TYPE_UINT32: "<I", GGUF_TYPE_INT32: "<i", GGUF_TYPE_FLOAT32: "<f", GGUF_TYPE_UINT64: "<Q",
           GGUF_TYPE_INT64: "<q", GGUF_TYPE_FLOAT64: "<d"}


@dataclass
class GGUFTensorInfo:
    name: str
    n_dims: int
    shape: tuple          # GGML order: shape[0] is the contiguous dimension
    dtype: int
    offset: int           # from the start of the file's data section
    file_idx: int = 0
    total_bytes: int = 0


@dataclass
class GGUFFileInfo:
    path: str
    version: int
    n_tensors: int
    metadata: dict
    tensors: dict
    data_offset: int
    alignment: int = 32


def tensor_byte_size(shape, dtype) -> int:
    """Bytes of a tensor: whole blocks of its type (a partial block rounds up)."""
    if dtype not in GGML_BLOCK_SIZES:
        raise ValueError(f"Unsupported GGML type: {dtype}")
    per, nbytes = GGML_BLOCK_SIZES[dtype]
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    return (n + per - 1) // per * nbytes


def _read_exact(f, n: int) -> bytes:
    b = f.read(n)
    if len(b) != n:
        raise struct.error(f"unpack requires a buffer of {n} bytes")
    return b


def _u32(f) -> int:
    return struct.unpack("<I", f.read(4))[0]


def _u64(f) -> int:
    return struct.unpack("<Q", f.read(8))[0]


def _read_string(f) -> str:
    return _read_exact(f, _u64(f)).decode("utf-8")


def _read_value(f, vtype: int):
    if vtype in _SCALAR:
        fmt = _SCALAR[vtype]
        return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
    if vtype == GGUF_TYPE_BOOL:
        return bool(struct.unpack("<B", f.read(1))[0])
    if vtype == GGUF_TYPE_STRING:
        return _read_string(f)
    if vtype == GGUF_TYPE_ARRAY:
        et, n = _u32(f), _u64(f)
        return [_read_value(f, et) for _ in range(n)]
    raise ValueError(f"Unknown GGUF value type: {vtype}")


def parse_gguf(path) -> GGUFFileInfo:
    """Header, metadata and tensor infos of one GGUF file."""
    with open(path, "rb") as f:
        magic = struct.unpack("<I", f.read(4))[0]
        if magic != GGUF_MAGIC:
            raise ValueError(f"Not a GGUF file: {path} (magic={hex(magic)})")
        version = _u32(f)
        n_tensors, n_kv = _u64(f), _u64(f)
        metadata = {}
        for _ in range(n_kv):
            key = _read_string(f)
            metadata[key] = _read_value(f, _u32(f))
        alignment = int(metadata.get("general.alignment", 32))
        tensors = {}
        for _ in range(n_tensors):
            name = _read_string(f)
            n_dims = _u32(f)
            shape = tuple(_u64(f) for _ in range(n_dims))
            dtype = _u32(f)
            offset = _u64(f)
            tensors[name] = GGUFTensorInfo(name, n_dims, shape, dtype, offset,
                                           total_bytes=tensor_byte_size(shape, dtype))
        data_offset = f.tell()
        data_offset += (-data_offset) % alignment
    return GGUFFileInfo(str(path), version, n_tensors, metadata, tensors, data_offset, alignment)


def parse_split_gguf(model_dir):
    """Every ``*.gguf`` file of a directory (sorted): (file infos, merged tensor
    infos with their file index, the first file's metadata)."""
    if not os.path.isdir(model_dir):
        raise FileNotFoundError(f"No such directory: {model_dir}")
    files = sorted(n for n in os.listdir(model_dir) if n.endswith(".gguf"))
    if not files:
        raise FileNotFoundError(f"No .gguf files in {model_dir}")
    infos, tensors, metadata = [], {}, {}
    for i, n in enumerate(files):
        info = parse_gguf(os.path.join(model_dir, n))
        infos.append(info)
        if i == 0:
            metadata = info.metadata
        for name, t in info.tensors.items():
            t.file_idx = i
            tensors[name] = t
    return infos, tensors, metadata


# ---------------------------------------------------------------------------
_PROJ = ("gate", "up", "down")


@dataclass
class ExpertSlice:
    file: str
    offset: int           # absolute byte offset of expert 0 (stacked) or of this expert
    expert_bytes: int
    dtype: int
    shape: tuple          # (cols, rows) of one expert, GGML order
    stacked: bool = True


class GGUFExperts:
    """Expert byte ranges of a GGUF model (one file or a directory of splits):
    ``slice(layer, proj)`` for stacked ``blk.{i}.ffn_{proj}_exps.weight``
    tensors (expert e at ``offset + e * expert_bytes``), and per-expert
    Mixtral-style tensors ``blk.{i}.ffn_{proj}.{e}.weight``."""

    def __init__(self, path):
        if os.path.isdir(path):
            self.file_infos, self.tensors, self.metadata = parse_split_gguf(path)
        else:
            info = parse_gguf(path)
            self.file_infos, self.tensors, self.metadata = [info], info.tensors, info.metadata
        self.n_experts = int(self.metadata.get("deepseek2.expert_count", self.metadata.get("llama.expert_count", 0)))
        self._stacked: Dict[Tuple[int, str], ExpertSlice] = {}
        self._single: Dict[Tuple[int, str, int], ExpertSlice] = {}
        for name, t in self.tensors.items():
            parts = name.split(".")
            if len(parts) < 4 or parts[0] != "blk" or not parts[1].isdigit() or not parts[2].startswith("ffn_"):
                continue
            layer, kind = int(parts[1]), parts[2][4:]
            fi = self.file_infos[t.file_idx]
            absoff = fi.data_offset + t.offset
            if kind.endswith("_exps") and kind[:-5] in _PROJ and parts[-1] == "weight":
                E = t.shape[-1] if len(t.shape) >= 3 else self.n_experts
                if self.n_experts and E != self.n_experts:
                    raise ValueError(f"{name}: {E} stacked experts, metadata says {self.n_experts}")
                if E <= 0 or t.total_bytes % E:
                    raise ValueError(f"{name}: {t.total_bytes} bytes do not split into {E} experts")
                self._stacked[(layer, kind[:-5])] = ExpertSlice(fi.path, absoff, t.total_bytes // E, t.dtype,
                                                                tuple(t.shape[:-1]))
                if not self.n_experts:
                    self.n_experts = E
            elif kind in _PROJ and len(parts) == 5 and parts[3].isdigit() and parts[4] == "weight":
                self._single[(layer, kind, int(parts[3]))] = ExpertSlice(fi.path, absoff, t.total_bytes, t.dtype,
                                                                          tuple(t.shape), stacked=False)

    def layers(self) -> List[int]:
        return sorted({k[0] for k in self._stacked} | {k[0] for k in self._single})

    def expert(self, layer: int, e: int, proj: str) -> ExpertSlice:
        """Where expert e's `proj` matrix lies (absolute offset of that expert)."""
        if (layer, proj, e) in self._single:
            return self._single[(layer, proj, e)]
        s = self._stacked.get((layer, proj))
        if s is None:
            raise KeyError(f"No expert layout for layer {layer}, proj {proj}")
        if not 0 <= e < self.n_experts:
            raise KeyError(f"Expert {e} not found in layer {layer}, proj {proj}")
        return ExpertSlice(s.file, s.offset + e * s.expert_bytes, s.expert_bytes, s.dtype, s.shape)

    def stacked(self, layer: int, proj: str) -> ExpertSlice:
        """The stacked ``blk.{layer}.ffn_{proj}_exps`` tensor (expert 0's slice;
        expert e at ``offset + e * expert_bytes``)."""
        s = self._stacked.get((layer, proj))
        if s is None:
            raise KeyError(f"No stacked experts for layer {layer}, proj {proj}")
        return s

    def shared_slice(self, layer: int, proj: str) -> Optional[ExpertSlice]:
        """The shared expert's matrix under the names GGUF conversions use
        (``ffn_{proj}_shexp``, ``ffn_{proj}_shared``, ``ffn_{proj}``), as the
        reference's ``load_shared_expert`` looks them up (ef_deepseek_mmap.py:611-639);
        None when the layer has none."""
        for name in (f"blk.{layer}.ffn_{proj}_shexp.weight", f"blk.{layer}.ffn_{proj}_shared.weight",
                     f"blk.{layer}.ffn_{proj}.weight"):
            t = self.tensors.get(name)
            if t is not None:
                fi = self.file_infos[t.file_idx]
                return ExpertSlice(fi.path, fi.data_offset + t.offset, t.total_bytes, t.dtype, tuple(t.shape),
                                   stacked=False)
        return None

    def load_expert_raw(self, layer: int, e: int, proj: str = "gate"):
        """(raw bytes, dtype, shape) of one expert's matrix."""
        s = self.expert(layer, e, proj)
        with open(s.file, "rb") as f:
            f.seek(s.offset)
            raw = f.read(s.expert_bytes)
        if len(raw) != s.expert_bytes:
            raise ValueError(f"{s.file}: expert range past the end of the file")
        return raw, s.dtype, s.shape


# ---------------------------------------------------------------------------
def _write_string(f, s: str) -> None:
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _value_type(v) -> int:
    if isinstance(v, bool):
        return GGUF_TYPE_BOOL
    if isinstance(v, int):
        return GGUF_TYPE_UINT32 if 0 <= v < 2 ** 32 else GGUF_TYPE_INT64
    if isinstance(v, float):
        return GGUF_TYPE_FLOAT32
    if isinstance(v, str):
        return GGUF_TYPE_STRING
    if isinstance(v, (list, tuple)):
        return GGUF_TYPE_ARRAY
    raise TypeError(f"no GGUF type for {type(v).__name__}")


def _write_value(f, v, vtype: int) -> None:
    if vtype in _SCALAR:
        f.write(struct.pack(_SCALAR[vtype], v))
    elif vtype == GGUF_TYPE_BOOL:
        f.write(struct.pack("<B", int(v)))
    elif vtype == GGUF_TYPE_STRING:
        _write_string(f, v)
    elif vtype == GGUF_TYPE_ARRAY:
        et = _value_type(v[0]) if len(v) else GGUF_TYPE_UINT32
        f.write(struct.pack("<IQ", et, len(v)))
        for x in v:
            _write_value(f, x, et)
    else:
        raise ValueError(f"Unknown GGUF value type: {vtype}")


def write_gguf(path: str, tensors: Dict[str, Tuple[Sequence[int], int, bytes]],
               metadata: Optional[dict] = None, alignment: int = 32) -> None:
    """Write a GGUF v3 file.  tensors: name -> (GGML shape, GGML type, raw
    bytes of exactly tensor_byte_size(shape, type)); tensor data in name order,
    each aligned to `alignment`."""
    md = dict(metadata or {})
    if alignment != 32:
        md["general.alignment"] = alignment
    names = sorted(tensors)
    offs, off = {}, 0
    for n in names:
        shape, dt, raw = tensors[n]
        if len(raw) != tensor_byte_size(shape, dt):
            raise ValueError(f"{n}: {len(raw)} bytes for a {tensor_byte_size(shape, dt)}-byte tensor")
        offs[n] = off
        off += len(raw)
        off += (-off) % alignment
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(names), len(md)))
        for k, v in md.items():
            _write_string(f, k)
            vt = _value_type(v)
            f.write(struct.pack("<I", vt))
            _write_value(f, v, vt)
        for n in names:
            shape, dt, _ = tensors[n]
            _write_string(f, n)
            f.write(struct.pack("<I", len(shape)))
            for d in shape:
                f.write(struct.pack("<Q", int(d)))
            f.write(struct.pack("<IQ", dt, offs[n]))
        pos = f.tell()
        f.write(b"\0" * ((-pos) % alignment))
        base = f.tell()
        for n in names:
            f.seek(base + offs[n])
            f.write(tensors[n][2])


def random_kquant_blocks(dtype: int, n_blocks: int, rng: np.random.Generator, d_scale: float = 0.01) -> bytes:
    """Seeded K-quant blocks: random code / scale bytes, fp16 super-block
    scales |N(0, d_scale)| (and mins |N(0, d_scale)|) at the format's offsets."""
    per, bb = GGML_BLOCK_SIZES[dtype]
    raw = rng.integers(0, 256, size=(n_blocks, bb), dtype=np.uint8)
    d = np.abs(rng.standard_normal(n_blocks) * d_scale).astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
    m = np.abs(rng.standard_normal(n_blocks) * d_scale).astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
    if dtype == GGML_TYPE_Q2_K:      # scales[16] qs[64] d dmin
        raw[:, 80:82], raw[:, 82:84] = d, m
    elif dtype == GGML_TYPE_Q3_K:    # hmask[32] qs[64] scales[12] d
        raw[:, 108:110] = d
    elif dtype == GGML_TYPE_Q4_K:    # d dmin scales[12] qs[128]
        raw[:, 0:2], raw[:, 2:4] = d, m
    else:
        raise ValueError(f"not a K-quant type: {dtype}")
    return raw.tobytes()
