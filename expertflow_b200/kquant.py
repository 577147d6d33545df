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
from typing import Optional

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


class KQuantProj:
    """One stacked K-quant projection of a MoE layer: ``blocks`` (uint8 CUDA
    tensor) holds n_experts matrices of ``n_rows`` rows x ``n_cols`` columns
    back to back (a GGML (n_cols, n_rows, E) tensor such as
    ``blk.{i}.ffn_gate_exps``), ``expert_stride`` bytes apart."""

    def __init__(self, blocks: torch.Tensor, dtype: int, n_rows: int, n_cols: int, n_experts: int = 1):
        _check_type(dtype)
        if blocks.dtype != torch.uint8 or not blocks.is_cuda:
            raise ValueError("blocks must be a uint8 CUDA tensor")
        bb = G.GGML_BLOCK_SIZES[dtype][1]
        per = n_rows * (n_cols // 256) * bb
        if n_cols % 256 or blocks.numel() != per * n_experts:
            raise ValueError(f"{blocks.numel()} bytes are not {n_experts} x {n_rows} x {n_cols} {dtype} matrices")
        self.blocks, self.dtype, self.n_rows, self.n_cols, self.n_experts = blocks.contiguous(), dtype, n_rows, n_cols, n_experts
        self.expert_stride = per

    def kqweight(self) -> L.KQWeight:
        return L.KQWeight(self.blocks.data_ptr(), self.dtype, self.expert_stride)

    def dequantize_expert(self, e: int) -> torch.Tensor:
        """fp16 [n_rows, n_cols] of expert e (ExpertMmapLoader.load_expert_dequantized)."""
        s = self.expert_stride
        return dequantize(self.blocks[e * s:(e + 1) * s], self.dtype, (self.n_rows, self.n_cols))


class KQuantMoELayer:
    """MoE block over GGUF K-quant experts (``ef_kquant_moe_forward``): the
    router, permutation and combine of ``moe.MoELayer``; routed experts run
    silu(x Wg^T) * (x Wu^T) Wd^T on the fp16 weights the reference's decoders
    give (ef_deepseek_mmap.py:570-593, its MoE forward :1563-1660)."""

    def __init__(self, gate, gate_proj: KQuantProj, up_proj: KQuantProj, down_proj: KQuantProj, shared=None):
        self.gate = gate
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.shared = shared  # (gate, up, down) KQuantProj of one expert each, or None
        self.num_experts_per_tok = gate.top_k

    def cfg(self, act_dtype: int) -> L.MoECfg:
        c = L.MoECfg(hidden=self.gate_proj.n_cols, inter=self.gate_proj.n_rows, n_experts=self.gate_proj.n_experts,
                     top_k=self.gate.top_k, bits=4, group_size=64, n_shared=1 if self.shared else 0,
                     shared_inter=self.gate_proj.n_rows if self.shared else 0, act_dtype=act_dtype)
        self.gate.fill_cfg(c)
        return c

    def forward(self, x: torch.Tensor, inds_out: Optional[torch.Tensor] = None,
                wts_out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        H = self.gate_proj.n_cols
        xf = x.reshape(-1, H).contiguous()
        _need_cuda(xf)
        T = xf.shape[0]
        y = torch.empty(xf.shape, dtype=out_dtype or xf.dtype, device=xf.device)
        if T == 0:
            return y.reshape(x.shape)
        cfg = self.cfg(_act_dt(xf))
        cfg.out_f32 = int(y.dtype == torch.float32)
        ws = workspace(L.lib().ef_kquant_moe_workspace_size(ctypes.byref(cfg), T), xf.device)
        sq = [ctypes.byref(p.kqweight()) for p in self.shared] if self.shared else [None] * 3
        eb = self.gate.e_score_correction_bias
        L.check(L.lib().ef_kquant_moe_forward(
            ctypes.byref(cfg), xf.data_ptr(), T, self.gate.weight.data_ptr(), eb.data_ptr() if eb is not None else None,
            self.gate_proj.kqweight(), self.up_proj.kqweight(), self.down_proj.kqweight(), sq[0], sq[1], sq[2],
            y.data_ptr(), inds_out.data_ptr() if inds_out is not None else None,
            wts_out.data_ptr() if wts_out is not None else None, ws.data_ptr(), ws.numel(), _stream_ptr(xf.device)))
        return y.reshape(x.shape)

    __call__ = forward

    @staticmethod
    def from_gguf(experts: G.GGUFExperts, layer: int, gate, device="cuda") -> "KQuantMoELayer":
        """Layer `layer` of a GGUF model: the stacked ffn_{gate,up,down}_exps
        tensors (and the shared expert when the file has one) moved to `device`."""
        def read(sl, n_bytes):
            with open(sl.file, "rb") as f:
                f.seek(sl.offset)
                raw = f.read(n_bytes)
            if len(raw) != n_bytes:
                raise ValueError(f"{sl.file}: tensor past the end of the file")
            return torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).to(device)

        E = experts.n_experts
        projs = []
        for proj in ("gate", "up", "down"):
            sl = experts.stacked(layer, proj)
            cols, rows = int(sl.shape[0]), int(sl.shape[1])
            projs.append(KQuantProj(read(sl, sl.expert_bytes * E), sl.dtype, rows, cols, E))
        shared = None
        sls = [experts.shared_slice(layer, p) for p in ("gate", "up", "down")]
        if all(s is not None for s in sls):
            shared = tuple(KQuantProj(read(s, s.expert_bytes), s.dtype, int(s.shape[1]), int(s.shape[0]), 1)
                           for s in sls)
        return KQuantMoELayer(gate, *projs, shared=shared)


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
