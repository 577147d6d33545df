"""numpy stand-in for the handful of MLX ops that the reference's
``streaming_moe_forward`` (ef_engine.py:598-706) and its expert cache call.

Used only by ``make_golden.py`` to execute the reference's own routing /
combine / cache code on this machine (mlx and mlx_lm are Apple-only and are
not vendored by the reference).  Each op restates MLX's documented meaning:

* ``argpartition(a, kth)``  -- MLX guarantees only a partition; the canonical
  rule used across this project is a full stable order, i.e. the first k of
  ``argpartition(-logits)`` are the top-k by (logit desc, index asc).
* ``softmax(..., precise=True)`` -- float32 softmax computed in float64.
* ``quantized_matmul(x, w, s, b, transpose=True, group_size, bits)`` --
  ``x @ dequant(w).T`` with MLX affine dequantisation
  ``s[o, i//g] * q[o, i] + b[o, i//g]``, codes LSB-first in uint32 words;
  evaluated in float64.
"""
from __future__ import annotations

import contextlib
import sys
import types

import numpy as np


def _argpartition(a, kth=None, axis=-1):
    return np.argsort(np.asarray(a), axis=axis, kind="stable")


def _softmax(a, axis=-1, precise=False):
    a64 = np.asarray(a, np.float64)
    m = a64.max(axis=axis, keepdims=True)
    e = np.exp(a64 - m)
    out = e / e.sum(axis=axis, keepdims=True)
    return out.astype(np.asarray(a).dtype if np.asarray(a).dtype != np.float64 else np.float64)


def _unpack(w, bits):
    per = 32 // bits
    shifts = np.arange(per, dtype=np.uint32) * bits
    q = (np.asarray(w, np.uint32)[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per)


def _dequantize(w, scales, biases=None, group_size=64, bits=4):
    q = _unpack(w, bits).astype(np.float64)
    s = np.repeat(np.asarray(scales, np.float16).astype(np.float64), group_size, axis=-1)
    out = s * q
    if biases is not None:
        out = out + np.repeat(np.asarray(biases, np.float16).astype(np.float64), group_size, axis=-1)
    return out


def _quantized_matmul(x, w, scales, biases=None, transpose=True, group_size=64, bits=4):
    W = _dequantize(w, scales, biases, group_size, bits)
    x64 = np.asarray(x, np.float64)
    return x64 @ (W.T if transpose else W)


def _silu(x):
    x = np.asarray(x, np.float64)
    return x / (1.0 + np.exp(-x))


def install() -> None:
    """Register ``mlx``, ``mlx.core`` and ``mlx.nn`` stand-ins in sys.modules."""
    core = types.ModuleType("mlx.core")
    core.argpartition = _argpartition
    core.take_along_axis = lambda a, i, axis=-1: np.take_along_axis(np.asarray(a), np.asarray(i), axis=axis)
    core.softmax = _softmax
    core.stop_gradient = lambda a: a
    core.eval = lambda *a, **k: None
    core.cpu = "cpu"
    core.gpu = "gpu"
    core.stream = lambda s: contextlib.nullcontext()
    core.concatenate = lambda arrs, axis=0: np.concatenate([np.asarray(a) for a in arrs], axis=axis)
    core.quantized_matmul = _quantized_matmul
    core.dequantize = _dequantize
    core.array = np.asarray
    core.zeros = lambda shape, dtype=None: np.zeros(shape, np.float64)
    core.set_default_device = lambda d: None
    nn = types.ModuleType("mlx.nn")
    nn.silu = _silu
    pkg = types.ModuleType("mlx")
    pkg.core = core
    pkg.nn = nn
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = core
    sys.modules["mlx.nn"] = nn
