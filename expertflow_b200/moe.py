"""Host-side mirror of the reference's MoE-layer interface, backed by libefmoe.

Reference call structure (paths relative to the reference checkout):

* ``streaming_moe_forward(moe_module, x, expert_cache=None)`` -- ef_engine.py:598-706.
  It reads ``moe_module.gate(x)`` (:610-618), ``num_experts_per_tok`` (:615),
  ``switch_mlp.{gate,up,down}_proj`` with ``["weight"]``, ``["scales"]``,
  ``.get("biases")``, ``.group_size``, ``.bits`` (:622-624, :661-667) and
  ``shared_experts`` (:628-631).  ``MoELayer`` carries exactly these
  attributes, and ``streaming_moe_forward`` accepts a ``MoELayer``.
* ``QuantizedSwitchLinear.__call__(x, indices)`` -- the gather_qmm contract
  ``x [B,S,1,1,in], indices [B,S,k] -> [B,S,k,1,out]`` (ef_engine_v4.py:52-64).
* ``mx.quantized_matmul(x, w, s, b, transpose=True, group_size, bits)``
  (ef_engine.py:689-694) and ``mx.dequantize`` (ef_cpu_fast.py:70-75).

All tensors live on a CUDA device; weights are int32 views of the uint32 MLX
words, fp16 scales and biases.  Everything runs on the current torch stream.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib as L
from .spec import MoESpec

_WS: dict = {}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Grow-only scratch buffer per (device, stream); the C ABI never allocates."""
    key = (device.index, _stream_ptr(device))
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def _act_dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return L.EF_DT_BF16
    if t.dtype == torch.float16:
        return L.EF_DT_F16
    raise TypeError(f"activations must be bfloat16 or float16, got {t.dtype}")


def _need_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("tensors must be contiguous CUDA tensors")


# ---------------------------------------------------------------------------
class QuantizedSwitchLinear:
    """A stack of quantised projections in the MLX affine layout.

    weight int32 [E, out, in*bits/32], scales/biases fp16 [E, out, in/64].
    Item access mirrors the mlx module parameters the reference reads
    (``proj["weight"]``, ``proj["scales"]``, ``proj.get("biases")``)."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
                 bits: int = 4):
        if weight.dim() == 2:
            weight, scales, biases = weight[None], scales[None], biases[None]
        if weight.dtype not in (torch.int32, torch.uint32):
            raise TypeError("weight must be int32/uint32 words")
        if scales.dtype != torch.float16 or biases.dtype != torch.float16:
            raise TypeError("scales/biases must be float16")
        _need_cuda(weight, scales, biases)
        self._p = {"weight": weight, "scales": scales, "biases": biases}
        self.group_size, self.bits = group_size, bits
        self.num_experts = weight.shape[0]
        self.output_dims = weight.shape[1]
        self.input_dims = weight.shape[2] * 32 // bits

    def __getitem__(self, key):
        return self._p[key]

    def get(self, key, default=None):
        return self._p.get(key, default)

    def __contains__(self, key):
        return key in self._p

    def qweight(self) -> L.QWeight:
        return L.QWeight(self._p["weight"].data_ptr(), self._p["scales"].data_ptr(), self._p["biases"].data_ptr())

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False) -> torch.Tensor:
        """gather_qmm: x [..., in] (e.g. [B,S,1,1,in]), indices [..., k] -> [..., k, 1, out]."""
        k = indices.shape[-1]
        lead = indices.shape[:-1]
        xf = x.reshape(-1, self.input_dims).contiguous()
        idx = indices.reshape(-1, k).to(torch.int32).contiguous()
        T = idx.shape[0]
        if xf.shape[0] != T:
            raise ValueError("x and indices disagree on the number of rows")
        y = torch.empty((T, k, self.output_dims), dtype=xf.dtype, device=xf.device)
        n = L.lib().ef_gather_qmm_workspace_size(T, k, self.num_experts, self.output_dims, self.input_dims)
        ws = workspace(n, xf.device)
        L.check(L.lib().ef_gather_qmm(xf.data_ptr(), _act_dt(xf), T, idx.data_ptr(), k, self.qweight(),
                                      self.num_experts, self.output_dims, self.input_dims, self.bits,
                                      self.group_size, y.data_ptr(), ws.data_ptr(), ws.numel(),
                                      _stream_ptr(xf.device)))
        return y.reshape(*lead, k, 1, self.output_dims)


class SwitchGLU:
    """mlx_lm SwitchGLU: ``down(silu(gate(x)) * up(x))`` per routed expert."""

    def __init__(self, gate_proj: QuantizedSwitchLinear, up_proj: QuantizedSwitchLinear,
                 down_proj: QuantizedSwitchLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def _cfg(self) -> L.MoECfg:
        g = self.gate_proj
        return L.MoECfg(hidden=g.input_dims, inter=g.output_dims, n_experts=g.num_experts, top_k=1, bits=g.bits,
                        group_size=g.group_size, router_mode=0, norm_topk=1, n_group=1, topk_group=1,
                        routed_scaling=1.0, n_shared=0, shared_inter=0, act_dtype=0, gate_dtype=1, path=0)

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """x [..., H], indices [..., k] -> fp32 [..., k, H] (unweighted expert outputs)."""
        H = self.gate_proj.input_dims
        k = indices.shape[-1]
        lead = indices.shape[:-1]
        xf = x.reshape(-1, H)
        rows = xf.repeat_interleave(k, dim=0).contiguous()
        ids = indices.reshape(-1).to(torch.int32).contiguous()
        return experts_forward(self, rows, ids).reshape(*lead, k, H)


def experts_forward(mlp: SwitchGLU, rows: torch.Tensor, row_expert: torch.Tensor) -> torch.Tensor:
    """y_rows[N, H] fp32 = SwiGLU_{row_expert[n]}(rows[n]) (ef_moe_experts_forward)."""
    _need_cuda(rows, row_expert)
    cfg = mlp._cfg()
    cfg.act_dtype = _act_dt(rows)
    N = rows.shape[0]
    H = mlp.gate_proj.input_dims
    y = torch.empty((N, H), dtype=torch.float32, device=rows.device)
    if N == 0:
        return y
    n = L.lib().ef_experts_workspace_size(ctypes.byref(cfg), N)
    ws = workspace(n, rows.device)
    L.check(L.lib().ef_moe_experts_forward(ctypes.byref(cfg), rows.data_ptr(), N, row_expert.data_ptr(),
                                           mlp.gate_proj.qweight(), mlp.up_proj.qweight(),
                                           mlp.down_proj.qweight(), None, None, None, y.data_ptr(),
                                           ws.data_ptr(), ws.numel(), _stream_ptr(rows.device)))
    return y


class QuantizedMLP(SwitchGLU):
    """Dense quantised SwiGLU (the shared expert): one-expert stacks."""

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        H = self.gate_proj.input_dims
        xf = x.reshape(-1, H).contiguous()
        ids = torch.zeros(xf.shape[0], dtype=torch.int32, device=x.device)
        return experts_forward(self, xf, ids).to(x.dtype).reshape(x.shape)


class MoEGate:
    """Router: fp16/bf16 weight [E, H]; softmax top-k or sigmoid group-limited."""

    def __init__(self, weight: torch.Tensor, top_k: int, mode: str = "softmax", norm_topk_prob: bool = True,
                 n_group: int = 1, topk_group: int = 1, routed_scaling_factor: float = 1.0,
                 e_score_correction_bias: Optional[torch.Tensor] = None):
        _need_cuda(weight, e_score_correction_bias)
        self.weight = weight
        self.top_k = top_k
        self.mode = mode
        self.norm_topk_prob = norm_topk_prob
        self.n_group, self.topk_group = n_group, topk_group
        self.routed_scaling_factor = routed_scaling_factor
        self.e_score_correction_bias = e_score_correction_bias

    @property
    def n_experts(self) -> int:
        return self.weight.shape[0]

    def fill_cfg(self, cfg: L.MoECfg) -> None:
        cfg.top_k = self.top_k
        cfg.router_mode = L.EF_ROUTER_SOFTMAX if self.mode == "softmax" else L.EF_ROUTER_SIGMOID_GROUP
        cfg.norm_topk = int(self.norm_topk_prob)
        cfg.n_group = self.n_group if self.mode != "softmax" else 1
        cfg.topk_group = self.topk_group if self.mode != "softmax" else 1
        cfg.routed_scaling = float(self.routed_scaling_factor if self.mode != "softmax" else 1.0)
        cfg.gate_dtype = L.EF_DT_F16 if self.weight.dtype == torch.float16 else L.EF_DT_BF16

    def __call__(self, x: torch.Tensor, logits_out: Optional[torch.Tensor] = None):
        """x [..., H] -> (inds int32 [..., k], scores fp32 [..., k])."""
        H = self.weight.shape[1]
        lead = x.shape[:-1]
        xf = x.reshape(-1, H).contiguous()
        T = xf.shape[0]
        cfg = L.MoECfg(hidden=H, inter=256, n_experts=self.n_experts, top_k=self.top_k, bits=4, group_size=64,
                       act_dtype=_act_dt(xf), n_shared=0, shared_inter=0, path=0)
        self.fill_cfg(cfg)
        inds = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        wts = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        n = L.lib().ef_router_workspace_size(ctypes.byref(cfg), T)
        ws = workspace(n, x.device)
        eb = self.e_score_correction_bias
        L.check(L.lib().ef_router_topk(ctypes.byref(cfg), xf.data_ptr(), T, self.weight.data_ptr(),
                                       eb.data_ptr() if eb is not None else None, inds.data_ptr(), wts.data_ptr(),
                                       logits_out.data_ptr() if logits_out is not None else None,
                                       ws.data_ptr(), ws.numel(), _stream_ptr(x.device)))
        return inds.reshape(*lead, self.top_k), wts.reshape(*lead, self.top_k)


class MoELayer(torch.nn.Module):
    """Drop-in MoE block: the attributes streaming_moe_forward reads, and a
    fused forward through ef_moe_forward (router, permute, quantised SwiGLU
    experts, weighted combine and the shared expert in one call)."""

    def __init__(self, gate: MoEGate, switch_mlp: SwitchGLU, shared_experts: Optional[QuantizedMLP] = None,
                 path: int = L.EF_PATH_AUTO):
        super().__init__()
        self.gate = gate
        self.switch_mlp = switch_mlp
        self.shared_experts = shared_experts
        self.num_experts_per_tok = gate.top_k
        self.path = path
        self._ef_layer_idx = -1

    def cfg(self, act_dtype: int) -> L.MoECfg:
        g = self.switch_mlp.gate_proj
        c = L.MoECfg(hidden=g.input_dims, inter=g.output_dims, n_experts=g.num_experts, top_k=self.gate.top_k,
                     bits=g.bits, group_size=g.group_size, n_shared=1 if self.shared_experts is not None else 0,
                     shared_inter=self.shared_experts.gate_proj.output_dims if self.shared_experts is not None else 0,
                     act_dtype=act_dtype, path=self.path)
        self.gate.fill_cfg(c)
        return c

    def forward(self, x: torch.Tensor, inds_out: Optional[torch.Tensor] = None,
                wts_out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                workspace_buf: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = MoE(x) in x's dtype, or fp32 (the un-rounded combine) with out_dtype=torch.float32.
        workspace_buf: caller-owned scratch (uint8, >= workspace_bytes(T)) instead of the shared one."""
        H = self.switch_mlp.gate_proj.input_dims
        xf = x.reshape(-1, H).contiguous()
        _need_cuda(xf)
        T = xf.shape[0]
        if out_dtype not in (None, xf.dtype, torch.float32):
            raise TypeError("out_dtype must be None, x.dtype or torch.float32")
        y = torch.empty(xf.shape, dtype=out_dtype or xf.dtype, device=xf.device)
        if T == 0:
            return y.reshape(x.shape)
        cfg = self.cfg(_act_dt(xf))
        cfg.out_f32 = int(y.dtype == torch.float32)
        n = L.lib().ef_moe_workspace_size(ctypes.byref(cfg), T)
        if workspace_buf is not None:
            if workspace_buf.numel() < n or workspace_buf.device != xf.device:
                raise ValueError(f"workspace_buf needs {n} bytes on {xf.device}")
            ws = workspace_buf
        else:
            ws = workspace(n, xf.device)
        sp = self.switch_mlp
        sh = self.shared_experts
        sq = [ctypes.byref(p.qweight()) for p in (sh.gate_proj, sh.up_proj, sh.down_proj)] if sh else [None] * 3
        eb = self.gate.e_score_correction_bias
        L.check(L.lib().ef_moe_forward(
            ctypes.byref(cfg), xf.data_ptr(), T, self.gate.weight.data_ptr(),
            eb.data_ptr() if eb is not None else None, sp.gate_proj.qweight(), sp.up_proj.qweight(),
            sp.down_proj.qweight(), sq[0], sq[1], sq[2], y.data_ptr(),
            inds_out.data_ptr() if inds_out is not None else None,
            wts_out.data_ptr() if wts_out is not None else None, ws.data_ptr(), ws.numel(),
            _stream_ptr(xf.device)))
        return y.reshape(x.shape)

    def workspace_bytes(self, T: int, act_dtype: torch.dtype = torch.bfloat16) -> int:
        cfg = self.cfg(L.EF_DT_BF16 if act_dtype == torch.bfloat16 else L.EF_DT_F16)
        return int(L.lib().ef_moe_workspace_size(ctypes.byref(cfg), T))

    def capture(self, T: int, dtype: torch.dtype = torch.bfloat16,
                out_dtype: Optional[torch.dtype] = None) -> "CapturedForward":
        """This layer's forward for T tokens captured in a CUDA graph."""
        return CapturedForward(self, T, dtype, out_dtype)

    # -- construction helpers -------------------------------------------------
    @staticmethod
    def from_arrays(spec: MoESpec, layer: dict, device="cuda", path: int = L.EF_PATH_AUTO) -> "MoELayer":
        """Build from a synthetic layer dict (numpy arrays or torch tensors)."""
        import numpy as np

        def T(a, dtype=None):
            if a is None:
                return None
            if isinstance(a, np.ndarray):
                if a.dtype == np.uint32:
                    a = a.view(np.int32)
                t = torch.from_numpy(np.ascontiguousarray(a))
            else:
                t = a
            t = t.to(device)
            return t.contiguous() if dtype is None else t.to(dtype).contiguous()

        def qlin(m):
            return QuantizedSwitchLinear(T(m[0]), T(m[1]), T(m[2]), spec.group_size, spec.bits)

        gate = MoEGate(T(layer["gate_w"]), spec.top_k, spec.router, spec.norm_topk, spec.n_group, spec.topk_group,
                       spec.routed_scaling, T(layer["e_bias"], torch.float32))
        mlp = SwitchGLU(qlin(layer["gate"]), qlin(layer["up"]), qlin(layer["down"]))
        shared = None
        if layer.get("shared") is not None:
            sg, su, sd = layer["shared"]
            shared = QuantizedMLP(qlin(sg), qlin(su), qlin(sd))
        return MoELayer(gate, mlp, shared, path)


class CapturedForward:
    """One MoELayer forward for a fixed token count captured in a CUDA graph:
    the layer's kernel launches (router, permute, gather, experts, combine)
    replay with one host call.  Write the input into ``.x`` (or pass it to
    ``__call__``), replay, read ``.y``.  The graph owns its input, output and
    workspace buffers, and keeps the layer's weight tensors alive."""

    def __init__(self, layer: MoELayer, T: int, dtype: torch.dtype = torch.bfloat16,
                 out_dtype: Optional[torch.dtype] = None):
        dev = layer.gate.weight.device
        H = layer.switch_mlp.gate_proj.input_dims
        self.layer = layer
        self.x = torch.zeros((T, H), dtype=dtype, device=dev)
        self.ws = torch.empty(max(layer.workspace_bytes(T, dtype), 1), dtype=torch.uint8, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # eager warm-up: sets kernel attributes outside the capture
            for _ in range(2):
                layer(self.x, out_dtype=out_dtype, workspace_buf=self.ws)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = layer(self.x, out_dtype=out_dtype, workspace_buf=self.ws)

    def __call__(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            self.x.copy_(x.reshape(self.x.shape), non_blocking=True)
        self.graph.replay()
        return self.y


def streaming_moe_forward(moe_module: MoELayer, x: torch.Tensor, expert_cache=None) -> torch.Tensor:
    """Drop-in for ef_engine.py:598 ``streaming_moe_forward``: x [B, S, H] -> [B, S, H].

    ``expert_cache`` (an ``ExpertSlotPool``) is consulted when the layer's
    experts are streamed from host memory; resident layers ignore it."""
    if expert_cache is not None and hasattr(expert_cache, "forward_layer"):
        return expert_cache.forward_layer(moe_module, x)
    return moe_module(x)


# ---------------------------------------------------------------------------
def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """``x @ dequant(w).T`` (mx.quantized_matmul with transpose=True)."""
    if not transpose:
        raise NotImplementedError("only transpose=True (the reference's call sites) is supported")
    out_dim = w.shape[-2]
    in_dim = w.shape[-1] * 32 // bits
    lead = x.shape[:-1]
    xf = x.reshape(-1, in_dim).contiguous()
    _need_cuda(xf, w, scales, biases)
    M = xf.shape[0]
    y = torch.empty((M, out_dim), dtype=xf.dtype, device=xf.device)
    n = L.lib().ef_quantized_matmul_workspace_size(M, out_dim, in_dim)
    ws = workspace(n, xf.device)
    L.check(L.lib().ef_quantized_matmul(xf.data_ptr(), _act_dt(xf), M, w.data_ptr(), scales.data_ptr(),
                                        biases.data_ptr(), out_dim, in_dim, bits, group_size, y.data_ptr(),
                                        ws.data_ptr(), ws.numel(), _stream_ptr(xf.device)))
    return y.reshape(*lead, out_dim)


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64, bits: int = 4,
               dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """mx.dequantize: [..., out, in*bits/32] words -> [..., out, in]."""
    _need_cuda(w, scales, biases)
    rows = w.numel() // w.shape[-1]
    cols = w.shape[-1] * 32 // bits
    out = torch.empty((*w.shape[:-1], cols), dtype=dtype, device=w.device)
    dt = {torch.float32: L.EF_DT_F32, torch.float16: L.EF_DT_F16, torch.bfloat16: L.EF_DT_BF16}[dtype]
    L.check(L.lib().ef_dequantize(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), rows, cols, bits, group_size,
                                  out.data_ptr(), dt, _stream_ptr(w.device)))
    return out


def permute(entries: torch.Tensor, k: int, n_experts: int, n_shared_rows: int = 0, seg_rows: int = 8) -> dict:
    """Stable counting sort of routed entries by expert (ef_permute): counts,
    offsets, row_src (token of each sorted row) and inv (sorted row of each
    entry), as the expert kernels consume them."""
    _need_cuda(entries)
    n = entries.numel()
    nb = n_experts + (1 if n_shared_rows > 0 else 0)
    dev = entries.device
    out = {"counts": torch.empty(nb, dtype=torch.int32, device=dev),
           "offsets": torch.empty(nb + 1, dtype=torch.int32, device=dev),
           "row_src": torch.empty(n + n_shared_rows, dtype=torch.int32, device=dev),
           "inv": torch.empty(n, dtype=torch.int32, device=dev)}
    nbytes = L.lib().ef_permute_workspace_size(n, n_experts, n_shared_rows, seg_rows)
    ws = workspace(nbytes, dev)
    L.check(L.lib().ef_permute(entries.data_ptr(), n, k, n_experts, n_shared_rows, seg_rows,
                               out["counts"].data_ptr(), out["offsets"].data_ptr(), out["row_src"].data_ptr(),
                               out["inv"].data_ptr(), ws.data_ptr(), ws.numel(), _stream_ptr(dev)))
    return out


def combine(rows: torch.Tensor, inv: torch.Tensor, wts: Optional[torch.Tensor], T: int, k: int,
            shared_base: int = -1, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """y[t] = sum_j wts[t, j] * rows[inv[t*k + j]] in j order (+ rows[shared_base + t]) (ef_combine)."""
    _need_cuda(rows, inv, wts)
    H = rows.shape[1]
    y = torch.empty((T, H), dtype=out_dtype, device=rows.device)
    dt = {torch.float32: L.EF_DT_F32, torch.float16: L.EF_DT_F16, torch.bfloat16: L.EF_DT_BF16}[out_dtype]
    L.check(L.lib().ef_combine(rows.data_ptr(), inv.data_ptr(), wts.data_ptr() if wts is not None else None, T, k,
                               H, shared_base, y.data_ptr(), dt, _stream_ptr(rows.device)))
    return y


def device_error(device=None) -> int:
    """Read and clear the device error word (0 = none)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = ctypes.c_int(0)
    L.lib().ef_get_device_error(_stream_ptr(dev), ctypes.byref(code))
    return code.value
