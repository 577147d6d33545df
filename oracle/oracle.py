"""CPU oracle for the ExpertFlow MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only as the checker.  The product package never does.

Two restatements of the same algorithm live here:

* the C library ``_build/libeforacle.so`` built from ``ef_oracle.c``
  (fast, OpenMP; used at full configuration sizes and as the CPU baseline), and
* a numpy twin of every routing function (``np_*``), used to cross-check the C
  code bit-for-bit and against the golden fixtures in ``tests/golden``.

What they restate (reference file:line, relative to the reference root):

* ``ef_engine.py:609-619``   router: Mixtral-style top-k of logits + softmax
  over the selected k; ``(inds, scores)`` gate for DeepSeek/Qwen models.
* ``ef_engine.py:678-704``   per-(token, k) SwiGLU with three quantized
  matmuls, ``out * score`` summed over k in k order, ``+ shared``.
* ``ef_cpu_fast.py:70-125``  dequantise-then-matmul CPU path (mx.dequantize).
* ``ef_engine_v2.py:88-91``  stacked expert layout ``[E, out, in*bits/32]``
  uint32 codes, ``[E, out, in/group]`` fp16 scales and biases.
* ``ef_deepseek_mmap.py:330-378, 655-773``  the reference's GGUF K-quant
  decoders (Q2_K, Q3_K, Q4_K blocks of 256 -> fp16), as ``np_dequant_kquant``;
  pinned by ``tests/golden/kquant_gguf.npz`` (generator:
  ``tests/golden/make_gguf_golden.py``, which runs the reference's own
  decoders), and the GEMV over such rows as ``np_kquant_matmul``.

Parity pin: the reference's routing/combine code (``streaming_moe_forward``)
and its expert cache (``FrequencyWeightedCache``) are executed on this
machine through a numpy restatement of the few MLX ops they call; their
outputs are the golden fixtures in ``tests/golden`` (generator:
``tests/golden/make_golden.py``).  The MLX arithmetic itself (mlx is an
unvendored third-party dependency of the reference; version not pinned in the
reference, mlx-lm 0.31.2 per ``experiments/v25_research_findings.md:117``) is
restated from its published affine-quantisation definition.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libeforacle.so")
_lib = None


def build() -> str:
    """Compile the C restatement (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "ef_oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i = ctypes.c_int
        f = ctypes.c_float
        L.efo_expf.restype = f
        L.efo_expf.argtypes = [f]
        L.efo_router_logits.argtypes = [P, i, P, i, i, i, i, P]
        L.efo_route_softmax.argtypes = [P, i, i, i, i, P, P]
        L.efo_route_sigmoid_group.argtypes = [P, P, i, i, i, i, i, i, f, P, P]
        L.efo_dequantize.argtypes = [P, P, P, i, i, i, i, P]
        L.efo_moe_ffn.restype = i
        L.efo_moe_ffn.argtypes = [P, i, i, i, i, i, i, i, i, P, P] + [_QMat] * 3 + [P, P, P, P]
        L.efo_num_threads.restype = i
        L.efo_set_num_threads.argtypes = [i]
        _lib = L
    return _lib


class _QMat(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("s", ctypes.c_void_p), ("b", ctypes.c_void_p)]


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().efo_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().efo_num_threads())


# ---------------------------------------------------------------------------
# 16-bit helpers: arrays of uint16 bit patterns
# ---------------------------------------------------------------------------
def f16_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)


def bf16_bits_from_f32(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bits_to_f32(bits: np.ndarray, is_bf16: bool) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    if is_bf16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# numpy twin of the deterministic exp / sigmoid
# ---------------------------------------------------------------------------
_LOG2E = np.float32(1.44269502162933349609375)
_LN2_HI = np.float32(0.693145751953125)
_LN2_LO = np.float32(1.428606765330187045e-06)
_C = [np.float32(v) for v in (1.98412698412698412698e-04, 1.38888888888888888889e-03,
                               8.33333333333333333333e-03, 4.16666666666666666667e-02,
                               1.66666666666666666667e-01, 0.5, 1.0, 1.0)]


def np_expf(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        t = x * _LOG2E
        n = np.rint(t).astype(np.float32)
        r = (x - n * _LN2_HI).astype(np.float32)
        r = (r - n * _LN2_LO).astype(np.float32)
        p = _C[0]
        for c in _C[1:]:
            p = (p * r).astype(np.float32)
            p = (p + c).astype(np.float32)
        ni = np.clip(n, -200, 200).astype(np.int32)
        out = np.ldexp(p, ni).astype(np.float32)
    out = np.where(x > np.float32(88.7228393554688), np.float32(np.inf), out)
    out = np.where(x < np.float32(-103.972084045410), np.float32(0.0), out)
    out = np.where(np.isnan(x), x, out)
    return out.astype(np.float32)


def np_sigmoidf(x) -> np.ndarray:
    e = np_expf(-np.asarray(x, dtype=np.float32))
    return (np.float32(1.0) / (np.float32(1.0) + e)).astype(np.float32)


# ---------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------
def _butterfly(acc: np.ndarray) -> np.ndarray:
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        acc = (acc + acc[..., lanes ^ off]).astype(np.float32)
    return acc[..., 0]


def np_router_logits(x_bits: np.ndarray, x_bf16: bool, w_bits: np.ndarray, w_bf16: bool) -> np.ndarray:
    """Canonical-order fp32 logits [T, E] (slot-interleaved, see ef_oracle.c)."""
    xf = bits_to_f32(x_bits, x_bf16)
    wf = bits_to_f32(w_bits, w_bf16)
    T, H = xf.shape
    E = wf.shape[0]
    assert H % 8 == 0
    nch = H // 8
    xc = xf.reshape(T, nch, 8)
    wc = wf.reshape(E, nch, 8)
    acc = np.zeros((T, E, 128), dtype=np.float32)
    for r in range((nch + 127) // 128):
        c0 = r * 128
        c1 = min(nch, c0 + 128)
        nl = c1 - c0
        for i in range(8):
            prod = xc[:, None, c0:c1, i] * wc[None, :, c0:c1, i]
            acc[:, :, :nl] = (acc[:, :, :nl] + prod).astype(np.float32)
    G = _butterfly(acc.reshape(T, E, 4, 32))
    return ((G[..., 0] + G[..., 1]).astype(np.float32) + (G[..., 2] + G[..., 3]).astype(np.float32)).astype(np.float32)


def _topk_rank(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the top-k by (value desc, index asc), in rank order, per row."""
    order = np.argsort(-v, axis=-1, kind="stable")
    return order[..., :k].astype(np.int32)


def np_route_softmax(logits: np.ndarray, k: int, norm_topk: bool = True):
    logits = np.asarray(logits, dtype=np.float32)
    inds = _topk_rank(logits, k)
    sel = np.take_along_axis(logits, inds, axis=-1)
    m = sel[:, :1]
    if norm_topk:
        e = np_expf((sel - m).astype(np.float32))
        s = e[:, 0].copy()
        for j in range(1, k):
            s = (s + e[:, j]).astype(np.float32)
        w = (e / s[:, None]).astype(np.float32)
    else:
        ea = np_expf((logits - m).astype(np.float32))
        T, E = ea.shape
        pad = (-E) % 32
        lanes = np.zeros((T, 32), dtype=np.float32)
        eap = np.concatenate([ea, np.zeros((T, pad), np.float32)], axis=1).reshape(T, -1, 32)
        for r in range(eap.shape[1]):
            lanes = (lanes + eap[:, r, :]).astype(np.float32)
        z = _butterfly(lanes)
        w = (np_expf((sel - m).astype(np.float32)) / z[:, None]).astype(np.float32)
    return inds, w


def np_route_sigmoid_group(logits, e_bias, k, n_group, topk_group, norm=True, scaling=1.0):
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    s = np_sigmoidf(logits)
    c = s if e_bias is None else (s + np.asarray(e_bias, np.float32)[None, :]).astype(np.float32)
    c = c.copy()
    if n_group > 1:
        gsz = E // n_group
        cg = c.reshape(T, n_group, gsz)
        srt = -np.sort(-cg, axis=-1)
        gs = (srt[..., 0] + srt[..., 1]).astype(np.float32)
        keep = _topk_rank(gs, topk_group)
        mask = np.zeros((T, n_group), dtype=bool)
        np.put_along_axis(mask, keep, True, axis=1)
        cg = np.where(mask[..., None], cg, np.float32(0.0))
        c = cg.reshape(T, E).astype(np.float32)
    inds = _topk_rank(c, k)
    w = np.take_along_axis(s, inds, axis=-1).astype(np.float32)
    if norm and k > 1:
        tot = w[:, 0].copy()
        for j in range(1, k):
            tot = (tot + w[:, j]).astype(np.float32)
        w = (w / tot[:, None]).astype(np.float32)
    w = (w * np.float32(scaling)).astype(np.float32)
    return inds, w


# ---------------------------------------------------------------------------
# MLX affine quantisation (restated)
# ---------------------------------------------------------------------------
def np_unpack_codes(w: np.ndarray, bits: int) -> np.ndarray:
    """uint32 [..., cols*bits/32] -> codes [..., cols] (LSB-first)."""
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per)


def np_pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    q = q.astype(np.uint32).reshape(*q.shape[:-1], q.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def np_dequantize(w, s, b, bits: int, group: int, dtype=np.float32) -> np.ndarray:
    """dequant(w)[o, i] = s[o, i//g] * q[o, i] + b[o, i//g]  (fp32 by default)."""
    q = np_unpack_codes(w, bits).astype(dtype)
    sc = np.repeat(np.asarray(s, np.float16).astype(dtype), group, axis=-1)
    bi = np.repeat(np.asarray(b, np.float16).astype(dtype), group, axis=-1)
    return sc * q + bi


def np_moe_ffn(xf, inds, wts, gate, up, down, bits, group, shared=None, dtype=np.float64):
    """Dequantise-then-matmul MoE FFN in float64 (small cases)."""
    xf = np.asarray(xf, dtype)
    T, H = xf.shape
    k = inds.shape[1]
    y = np.zeros((T, H), dtype)

    def expert(mats, e, xin):
        (gw, gs, gb), (uw, us, ub), (dw, ds, db) = mats
        Wg = np_dequantize(gw[e], gs[e], gb[e], bits, group, dtype)
        Wu = np_dequantize(uw[e], us[e], ub[e], bits, group, dtype)
        Wd = np_dequantize(dw[e], ds[e], db[e], bits, group, dtype)
        g = xin @ Wg.T
        u = xin @ Wu.T
        h = g / (1.0 + np.exp(-g)) * u
        return h @ Wd.T

    for t in range(T):
        acc = None
        for j in range(k):
            o = expert((gate, up, down), int(inds[t, j]), xf[t:t + 1])[0] * dtype(wts[t, j])
            acc = o if acc is None else acc + o
        y[t] = acc
    if shared is not None:
        sg, su, sd = shared
        y = y + expert(((sg[0][None], sg[1][None], sg[2][None]),
                        (su[0][None], su[1][None], su[2][None]),
                        (sd[0][None], sd[1][None], sd[2][None])), 0, xf)
    return y


# ---------------------------------------------------------------------------
# C-library wrappers
# ---------------------------------------------------------------------------
def c_router_logits(x_bits, x_bf16, w_bits, w_bf16) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    w_bits = np.ascontiguousarray(w_bits, np.uint16)
    T, H = x_bits.shape
    E = w_bits.shape[0]
    out = np.empty((T, E), np.float32)
    lib().efo_router_logits(_ptr(x_bits), int(x_bf16), _ptr(w_bits), int(w_bf16), T, E, H, _ptr(out))
    return out


def c_route_softmax(logits, k, norm_topk=True):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    inds = np.empty((T, k), np.int32)
    wts = np.empty((T, k), np.float32)
    lib().efo_route_softmax(_ptr(logits), T, E, k, int(norm_topk), _ptr(inds), _ptr(wts))
    return inds, wts


def c_route_sigmoid_group(logits, e_bias, k, n_group, topk_group, norm=True, scaling=1.0):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    inds = np.empty((T, k), np.int32)
    wts = np.empty((T, k), np.float32)
    eb = None if e_bias is None else np.ascontiguousarray(e_bias, np.float32)
    lib().efo_route_sigmoid_group(_ptr(logits), None if eb is None else _ptr(eb), T, E, k,
                                  n_group, topk_group, int(norm), float(scaling), _ptr(inds), _ptr(wts))
    return inds, wts


def c_expf(x: float) -> float:
    return float(lib().efo_expf(float(x)))


def c_dequantize(w, s, b, bits, group) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint32)
    s = np.ascontiguousarray(s).view(np.uint16)
    b = np.ascontiguousarray(b).view(np.uint16)
    rows = w.shape[0]
    cols = w.shape[1] * 32 // bits
    out = np.empty((rows, cols), np.float32)
    lib().efo_dequantize(_ptr(w), _ptr(s), _ptr(b), rows, cols, bits, group, _ptr(out))
    return out


def _qm(w, s, b) -> _QMat:
    return _QMat(_ptr(w), _ptr(s), _ptr(b))


def c_moe_ffn(x_bits, x_bf16, inds, wts, gate, up, down, bits, group, shared=None) -> np.ndarray:
    """fp32 dequantise-then-matmul MoE FFN (C, OpenMP).  gate/up/down are
    (w uint32, s fp16, b fp16) stacks; shared is a tuple of three (w, s, b)
    single-expert triples or None."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    inds = np.ascontiguousarray(inds, np.int32)
    wts = np.ascontiguousarray(wts, np.float32)
    T, H = x_bits.shape
    k = inds.shape[1]
    E, I = gate[0].shape[0], gate[0].shape[1]
    keep = []

    def prep(m):
        w = np.ascontiguousarray(m[0], np.uint32)
        s = np.ascontiguousarray(m[1]).view(np.uint16)
        b = np.ascontiguousarray(m[2]).view(np.uint16)
        keep.extend([w, s, b])
        return _qm(w, s, b)

    g, u, d = prep(gate), prep(up), prep(down)
    shp = [None, None, None]
    if shared is not None:
        sh = [prep(m) for m in shared]
        shp = [ctypes.byref(q) for q in sh]
    y = np.empty((T, H), np.float32)
    rc = lib().efo_moe_ffn(_ptr(x_bits), int(x_bf16), T, H, I, E, k, bits, group, _ptr(inds), _ptr(wts),
                           g, u, d, shp[0], shp[1], shp[2], _ptr(y))
    if rc != 0:
        raise MemoryError("oracle efo_moe_ffn failed to allocate")
    return y


# ---------------------------------------------------------------------------
# whole layer
# ---------------------------------------------------------------------------
@dataclass
class RouterSpec:
    mode: str  # "softmax" | "sigmoid_group"
    k: int
    norm_topk: bool = True
    n_group: int = 1
    topk_group: int = 1
    scaling: float = 1.0


def route(logits, spec: RouterSpec, e_bias=None, use_c=True):
    if spec.mode == "softmax":
        if e_bias is not None:  # optional per-expert logit bias (fp32 add)
            logits = (np.asarray(logits, np.float32) + np.asarray(e_bias, np.float32)[None, :]).astype(np.float32)
        f = c_route_softmax if use_c else np_route_softmax
        return f(logits, spec.k, spec.norm_topk)
    f = c_route_sigmoid_group if use_c else np_route_sigmoid_group
    return f(logits, e_bias, spec.k, spec.n_group, spec.topk_group, spec.norm_topk, spec.scaling)


def moe_forward(x_bits, x_bf16, gate_w_bits, gate_w_bf16, spec: RouterSpec, e_bias, gate, up, down,
                bits, group, shared=None):
    """Full MoE layer on the CPU: (inds, wts, y fp32)."""
    logits = c_router_logits(x_bits, x_bf16, gate_w_bits, gate_w_bf16)
    inds, wts = route(logits, spec, e_bias)
    y = c_moe_ffn(x_bits, x_bf16, inds, wts, gate, up, down, bits, group, shared)
    return inds, wts, y


# ---------------------------------------------------------------- GGUF K-quants
# Block layouts and element orders as the reference's decoders read them
# (QK_K = 256 elements per block; value = d * sc * q - dmin * mn in fp32, then
# rounded to fp16):
#   Q2_K (84 B)  scales[16] @0 (lo nibble sc, hi nibble mn of group i/16),
#                qs[64] @16 (element i: bits 2(i%4).. of byte i/4), d @80, dmin @82
#                                                   ef_deepseek_mmap.py:330-378
#   Q3_K (110 B) hmask[32] @0, qs[64] @32, scales[12] @96, d @108; element
#                i = 32(4h + s) + b: q = ((qs[32h + b] >> 2s) & 3) - 4 * (1 - hmask bit
#                (4h + s) of byte b); 6-bit scale of group i/16 (low nibble from
#                bytes 0..7, high 2 bits from bytes 8..11) minus 32; no min
#                                                   ef_deepseek_mmap.py:717-773
#   Q4_K (144 B) d @0, dmin @2, scales[12] @4, qs[128] @16; elements 0..127 the
#                low nibbles of qs, 128..255 the high nibbles; sub-block i/32 has
#                sc = s[j] & 63 (j < 8), mn = s[8 + j] & 63 (j < 4) or
#                (s[j - 4] >> 6) | ((s[j + 4] >> 2) & 0x30) (j >= 4)
#                                                   ef_deepseek_mmap.py:655-714
KQ_BLOCK_BYTES = {10: 84, 11: 110, 12: 144}


def _f16_field(blocks: np.ndarray, off: int) -> np.ndarray:
    return blocks[:, off:off + 2].copy().view(np.float16).reshape(-1).astype(np.float32)


def np_kquant_codes(blocks: np.ndarray, dtype: int):
    """(q [n, 256] fp32, A [n, 256] fp32, B [n, 256] fp32) with value = A*q - B."""
    n = blocks.shape[0]
    if dtype == 10:
        sc = blocks[:, 0:16]
        qs = blocks[:, 16:80]
        d, dm = _f16_field(blocks, 80), _f16_field(blocks, 82)
        q = ((qs[:, :, None] >> (2 * np.arange(4, dtype=np.uint8))[None, None, :]) & 3).reshape(n, 256)
        A = np.repeat(d[:, None] * (sc & 15).astype(np.float32), 16, axis=1)
        B = np.repeat(dm[:, None] * (sc >> 4).astype(np.float32), 16, axis=1)
        return q.astype(np.float32), A, B
    if dtype == 11:
        hm, qs, sb = blocks[:, 0:32], blocks[:, 32:96], blocks[:, 96:108]
        d = _f16_field(blocks, 108)
        g = np.arange(16)
        lo = np.where(g < 8, sb[:, g % 8] & 15, sb[:, g % 8] >> 4)
        hi = (sb[:, 8 + g % 4] >> (2 * (g // 4)).astype(np.uint8)) & 3
        sc = (lo | (hi << 4)).astype(np.float32) - 32.0
        i = np.arange(256)
        h, sh, b = i // 128, (i // 32) % 4, i % 32
        q2 = (qs[:, 32 * h + b] >> (2 * sh).astype(np.uint8)) & 3
        hb = (hm[:, b] >> (4 * h + sh).astype(np.uint8)) & 1
        q = q2.astype(np.float32) - 4.0 * (1 - hb).astype(np.float32)
        A = np.repeat(d[:, None] * sc, 16, axis=1)
        return q, A, np.zeros_like(A)
    if dtype == 12:
        d, dm = _f16_field(blocks, 0), _f16_field(blocks, 2)
        s = blocks[:, 4:16]
        j = np.arange(8)
        sc = (s[:, j] & 63).astype(np.float32)
        mn = np.where(j < 4, s[:, 8 + j % 4] & 63, (s[:, j % 4] >> 6) | ((s[:, 8 + j % 4] >> 2) & 0x30))
        qs = blocks[:, 16:144]
        q = np.concatenate([qs & 15, qs >> 4], axis=1).astype(np.float32)
        A = np.repeat(d[:, None] * sc, 32, axis=1)
        B = np.repeat(dm[:, None] * mn.astype(np.float32), 32, axis=1)
        return q, A, B
    raise ValueError(f"not a K-quant type: {dtype}")


def np_dequant_kquant(raw, dtype: int) -> np.ndarray:
    """fp16 [n_blocks * 256] of raw K-quant blocks, as the reference decodes them."""
    bb = KQ_BLOCK_BYTES[dtype]
    blocks = np.frombuffer(bytes(raw), np.uint8)
    blocks = blocks[:len(blocks) // bb * bb].reshape(-1, bb)
    q, A, B = np_kquant_codes(blocks, dtype)
    with np.errstate(over="ignore", invalid="ignore"):
        v = (A * q - B).astype(np.float32)  # A*q is exact in fp32; one rounding at the subtraction
        return v.astype(np.float16).reshape(-1)


def np_kquant_matmul(x: np.ndarray, raw, dtype: int, N: int, K: int) -> np.ndarray:
    """y [T, N] fp64 = x [T, K] . W^T, W [N, K] the fp16 rows decoded from
    N * K / 256 K-quant blocks (row r = blocks [r K/256, (r+1) K/256))."""
    w = np_dequant_kquant(raw, dtype).astype(np.float64).reshape(N, K)
    return np.asarray(x, np.float64) @ w.T


def np_kquant_moe_ffn(xf, inds, wts, gate, up, down, shared=None) -> np.ndarray:
    """MoE FFN over K-quant experts: y [T, H] fp64 = sum_k wts[t, k] *
    E_{inds[t, k]}(x[t]) (+ shared(x[t])) with E(v) = (silu(v Wg^T) * (v Wu^T)) Wd^T
    on the fp16 matrices np_dequant_kquant decodes -- the reference's
    load_expert_dequantized (ef_deepseek_mmap.py:570-593) feeding its MoE
    forward (:1563-1660).  gate / up / down: (raw bytes of E stacked
    matrices, GGML type, n_rows, n_cols); shared: the same triple for one
    expert, or None."""
    xf = np.asarray(xf, np.float64)
    cache = {}

    def mat(p, e):
        raw, dt, rows, cols = p
        key = (id(raw), e)
        if key not in cache:
            per = rows * (cols // 256) * KQ_BLOCK_BYTES[dt]
            cache[key] = np_dequant_kquant(raw[e * per:(e + 1) * per], dt).astype(np.float64).reshape(rows, cols)
        return cache[key]

    def expert(mats, e, v):
        g = v @ mat(mats[0], e).T
        u = v @ mat(mats[1], e).T
        h = g / (1.0 + np.exp(-g)) * u
        return h @ mat(mats[2], e).T

    T, k = inds.shape
    y = np.zeros((T, xf.shape[1]), np.float64)
    for t in range(T):
        for j in range(k):
            y[t] += float(wts[t, j]) * expert((gate, up, down), int(inds[t, j]), xf[t:t + 1])[0]
        if shared is not None:
            y[t] += expert(shared, 0, xf[t:t + 1])[0]
    return y

