"""GGUF K-quant weights on the GPU (``ef_kquant_*``).

``dequantize`` decodes Q2_K / Q3_K / Q4_K blocks to fp16 exactly as the
reference's ``dequant_q2_k_fast`` / ``dequant_q3_k_fast`` / ``dequant_q4_k_fast``
do (ef_deepseek_mmap.py:330-378, 655-773; they are what
``ExpertMmapLoader.load_expert_dequantized`` returns, :570-593).  ``matmul`` is
the decode GEMV over rows stored in those blocks, without materialising the
fp16 matrix.  ``load_expert`` reads one expert's blocks from a GGUF model
(``gguf.GGUFExperts``) onto the device.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L
from . import gguf as G
from .moe import _act_dt, _need_cuda, _stream_ptr, workspace

TYPES = G.KQUANT_TYPES


def _check_type(dtype: int) -> None:
    if dtype not in TYPES:
        raise ValueError(f"not a supported K-quant type: {dtype} (Q2_K=10, Q3_K=11, Q4_K=12)")


def dequantize(blocks: torch.Tensor, dtype: int, shape=None) -> torch.Tensor:
    """fp16 [n_blocks * 256] (or `shape`) of raw K-quant blocks (uint8 CUDA tensor)."""
    _check_type(dtype)
    _need_cuda(blocks)
    bb = G.GGML_BLOCK_SIZES[dtype][1]
    if blocks.dtype != torch.uint8 or blocks.numel() % bb:
        raise ValueError(f"blocks must be uint8 with a multiple of {bb} bytes")
    n = blocks.numel() // bb
    out = torch.empty(n * 256, dtype=torch.float16, device=blocks.device)
    L.check(L.lib().ef_kquant_dequantize(dtype, blocks.data_ptr(), n, out.data_ptr(), _stream_ptr(blocks.device)))
    return out if shape is None else out.reshape(shape)


def matmul(x: torch.Tensor, blocks: torch.Tensor, dtype: int, N: int, K: int) -> torch.Tensor:
    """y fp32 [..., N] = x [..., K] . W^T for W [N, K] stored as N rows of
    K/256 blocks (a GGML (K, N) tensor, or one expert of a stacked one).
    At most 32 rows of x (decode)."""
    _check_type(dtype)
    xf = x.reshape(-1, K).contiguous()
    _need_cuda(xf, blocks)
    T = xf.shape[0]
    y = torch.empty((T, N), dtype=torch.float32, device=xf.device)
    if T == 0:
        return y.reshape(*x.shape[:-1], N)
    ws = workspace(L.lib().ef_kquant_matmul_workspace_size(T, K), xf.device)
    L.check(L.lib().ef_kquant_matmul(xf.data_ptr(), _act_dt(xf), T, blocks.data_ptr(), dtype, N, K, y.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _stream_ptr(xf.device)))
    return y.reshape(*x.shape[:-1], N)


def load_expert(experts: G.GGUFExperts, layer: int, e: int, proj: str, device="cuda"):
    """(blocks uint8 CUDA tensor, GGML type, (K, N)) of one expert's matrix."""
    raw, dtype, shape = experts.load_expert_raw(layer, e, proj)
    t = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).to(device)
    return t, dtype, tuple(int(v) for v in shape)


def _main(argv=None) -> None:
    """Launch the GEMV on random blocks (for profiling):
    python -m expertflow_b200.kquant --type 10 --rows 32768 --cols 7168 --tokens 1 --reps 3"""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--type", type=int, default=G.GGML_TYPE_Q2_K)
    ap.add_argument("--rows", type=int, default=32768)
    ap.add_argument("--cols", type=int, default=7168)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    bb = G.GGML_BLOCK_SIZES[a.type][1]
    w = torch.randint(0, 256, (a.rows * (a.cols // 256) * bb,), dtype=torch.uint8, device="cuda")
    x = torch.randn((a.tokens, a.cols), device="cuda").to(torch.bfloat16)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(a.reps):
        if i == a.reps - 1:
            e0.record()
        matmul(x, w, a.type, a.rows, a.cols)
    e1.record()
    torch.cuda.synchronize()
    print(f"type {a.type}: {w.numel() / 1e6:.1f} MB of blocks, last launch {e0.elapsed_time(e1) * 1e3:.1f} us")


if __name__ == "__main__":
    _main()
