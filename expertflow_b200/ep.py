"""Expert parallelism: a MoE layer's experts sharded across the ranks of one
box, token rows exchanged with NCCL all-to-all over NVLink.

Expert e lives on rank e // (E / P); the router and the shared expert are
replicated and every rank routes its own tokens.  One forward:

1. ``ef_ep_dispatch``: route, sort the routed entries by expert (= by
   destination rank), pack the token rows and the destination's local expert
   ids, count the rows per destination;
2. all-to-all of the counts, then of the rows and ids (uneven splits);
3. ``ef_moe_experts_forward`` on the received rows (local experts);
4. all-to-all of the fp32 outputs back to their source ranks;
5. ``ef_ep_combine``: weighted sum over k in k order, + the shared expert.

The reference has no multi-device path (all experts run in one process,
ef_engine.py:678-703); the split above is the one the DeepSeek-V3-shaped
layer is served with across the 8 GPUs of a box.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib as L
from .moe import MoEGate, QuantizedMLP, SwitchGLU, _act_dt, _need_cuda, _stream_ptr, experts_forward, workspace
from .spec import MoESpec


class EpDeviceOps:
    """The device steps of one rank (C ABI)."""

    def __init__(self, spec: MoESpec, gate: MoEGate, local_mlp: SwitchGLU, shared: Optional[QuantizedMLP],
                 n_ranks: int):
        if spec.n_experts % n_ranks:
            raise ValueError("n_ranks must divide n_experts")
        self.spec, self.gate, self.local_mlp, self.shared_mlp = spec, gate, local_mlp, shared
        self.n_ranks = n_ranks
        self.e_local = spec.n_experts // n_ranks
        if local_mlp.gate_proj.num_experts != self.e_local:
            raise ValueError("local_mlp must hold E / n_ranks experts")

    def _cfg(self, act_dtype: int, out_f32: bool = False) -> L.MoECfg:
        s = self.spec
        c = L.MoECfg(hidden=s.hidden, inter=s.inter, n_experts=s.n_experts, top_k=s.top_k, bits=s.bits,
                     group_size=s.group_size, n_shared=0, shared_inter=0, act_dtype=act_dtype, path=L.EF_PATH_AUTO,
                     out_f32=int(out_f32))
        self.gate.fill_cfg(c)
        return c

    def dispatch(self, x: torch.Tensor) -> dict:
        _need_cuda(x)
        T, H = x.shape
        k = self.spec.top_k
        dev = x.device
        out = {"send_rows": torch.empty((T * k, H), dtype=x.dtype, device=dev),
               "send_eid": torch.empty((T * k,), dtype=torch.int32, device=dev),
               "send_counts": torch.empty((self.n_ranks,), dtype=torch.int32, device=dev),
               "inv": torch.empty((T * k,), dtype=torch.int32, device=dev),
               "wts": torch.empty((T * k,), dtype=torch.float32, device=dev),
               "inds": torch.empty((T, k), dtype=torch.int32, device=dev)}
        cfg = self._cfg(_act_dt(x))
        n = L.lib().ef_ep_dispatch_workspace_size(ctypes.byref(cfg), T)
        ws = workspace(n, dev)
        eb = self.gate.e_score_correction_bias
        L.check(L.lib().ef_ep_dispatch(
            ctypes.byref(cfg), self.n_ranks, x.data_ptr(), T, self.gate.weight.data_ptr(),
            eb.data_ptr() if eb is not None else None, out["send_rows"].data_ptr(), out["send_eid"].data_ptr(),
            out["send_counts"].data_ptr(), out["inv"].data_ptr(), out["wts"].data_ptr(), out["inds"].data_ptr(),
            ws.data_ptr(), ws.numel(), _stream_ptr(dev)))
        return out

    def experts(self, rows: torch.Tensor, eid: torch.Tensor) -> torch.Tensor:
        if rows.shape[0] == 0:
            return torch.empty((0, rows.shape[1]), dtype=torch.float32, device=rows.device)
        return experts_forward(self.local_mlp, rows, eid)

    def shared(self, x: torch.Tensor) -> Optional[torch.Tensor]:
        if self.shared_mlp is None:
            return None
        ids = torch.zeros(x.shape[0], dtype=torch.int32, device=x.device)
        return experts_forward(self.shared_mlp, x, ids)

    def combine(self, back: torch.Tensor, inv: torch.Tensor, wts: torch.Tensor, T: int, with_shared: bool,
                out_dtype: torch.dtype) -> torch.Tensor:
        H = back.shape[1]
        y = torch.empty((T, H), dtype=out_dtype, device=back.device)
        cfg = self._cfg(L.EF_DT_BF16 if out_dtype == torch.bfloat16 else L.EF_DT_F16,
                        out_f32=out_dtype == torch.float32)
        L.check(L.lib().ef_ep_combine(ctypes.byref(cfg), back.data_ptr(), inv.data_ptr(), wts.data_ptr(), T,
                                      int(with_shared), y.data_ptr(), _stream_ptr(back.device)))
        return y


def _rows_view(t: torch.Tensor) -> torch.Tensor:
    """Byte-preserving 2-byte float view for the exchange (NCCL has no int16)."""
    return t.view(torch.float16) if t.dtype == torch.bfloat16 else t


class ExpertParallelMoE:
    """One rank's MoE layer with its experts sharded across `group`."""

    def __init__(self, spec: MoESpec, ops, group=None):
        self.spec = spec
        self.ops = ops
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.last_counts = None

    def forward(self, x: torch.Tensor, inds_out: Optional[torch.Tensor] = None,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """y = MoE(x) for this rank's tokens; inds_out [T, k] receives the routing."""
        H, k = self.spec.hidden, self.spec.top_k
        xf = x.reshape(-1, H).contiguous()
        T = xf.shape[0]
        d = self.ops.dispatch(xf)
        if inds_out is not None:
            inds_out.copy_(d["inds"].reshape(inds_out.shape))
        recv_counts = torch.empty_like(d["send_counts"])
        dist.all_to_all_single(recv_counts, d["send_counts"], group=self.group)
        sc = d["send_counts"].tolist()
        rc = recv_counts.tolist()
        self.last_counts = (sc, rc)
        n_recv = sum(rc)
        recv_rows = torch.empty((n_recv, H), dtype=xf.dtype, device=xf.device)
        recv_eid = torch.empty((n_recv,), dtype=torch.int32, device=xf.device)
        dist.all_to_all_single(_rows_view(recv_rows), _rows_view(d["send_rows"]), rc, sc, group=self.group)
        dist.all_to_all_single(recv_eid, d["send_eid"], rc, sc, group=self.group)
        y_rows = self.ops.experts(recv_rows, recv_eid)
        sh = self.ops.shared(xf)
        back = torch.empty((T * k + (T if sh is not None else 0), H), dtype=torch.float32, device=xf.device)
        dist.all_to_all_single(back[:T * k], y_rows.contiguous(), sc, rc, group=self.group)
        if sh is not None:
            back[T * k:] = sh
        y = self.ops.combine(back, d["inv"], d["wts"], T, sh is not None, out_dtype or xf.dtype)
        return y.reshape(*x.shape[:-1], H)

    __call__ = forward


def shard_layer(spec: MoESpec, layer: dict, rank: int, n_ranks: int, device="cuda") -> EpDeviceOps:
    """This rank's EpDeviceOps from a full synthetic layer (numpy or torch):
    experts [rank * E/P, (rank + 1) * E/P), the replicated gate and shared expert."""
    from .moe import MoELayer

    e_loc = spec.n_experts // n_ranks
    sl = slice(rank * e_loc, (rank + 1) * e_loc)
    part = dict(layer)
    for kname in ("gate", "up", "down"):  # own copies, so the full layer can be freed
        part[kname] = tuple(a[sl].clone() if isinstance(a, torch.Tensor) else a[sl].copy() for a in layer[kname])
    # the gate keeps all E rows (routing is replicated); the experts are the shard
    local = MoELayer.from_arrays(spec.with_(n_experts=e_loc), part, device=device)
    return EpDeviceOps(spec, local.gate, local.switch_mlp, local.shared_experts, n_ranks)


def _dt_code(dt: torch.dtype) -> int:
    return {torch.bfloat16: L.EF_DT_BF16, torch.float16: L.EF_DT_F16, torch.float32: L.EF_DT_F32}[dt]


class PeerExpertParallelMoE:
    """One rank's MoE layer with its experts sharded across the ranks of
    `group`, exchanged by the library's own kernels through the peers' memory
    over NVLink (``ef_ep_forward``): no host synchronisation and no NCCL call
    in a forward, so a forward can be captured in a CUDA graph.

    Every rank must construct it (the exchange buffers' IPC handles are
    gathered once over `group`), run the same sequence of forwards (its own
    token count each, 0 allowed) and call ``close()`` together.  Without an
    initialised process group it is a single-rank layer (``ops`` holding all
    experts)."""

    def __init__(self, spec: MoESpec, ops: EpDeviceOps, group=None, max_tokens: int = 256, max_recv_rows: int = 0,
                 act_dtype: torch.dtype = torch.bfloat16, path: int = L.EF_PATH_AUTO):
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if ops.n_ranks != self.world:
            raise ValueError(f"ops shard the experts over {ops.n_ranks} ranks, the group has {self.world}")
        self.spec, self.ops, self.group = spec, ops, group
        self.max_tokens, self.act_dtype = max_tokens, act_dtype
        self.device = ops.gate.weight.device
        cfg = ops._cfg(_dt_code(act_dtype))
        if ops.shared_mlp is not None:
            cfg.n_shared, cfg.shared_inter = 1, ops.shared_mlp.gate_proj.output_dims
        cfg.path = path
        self._cfg = cfg
        g = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.check(L.lib().ef_ep_group_create(ctypes.byref(cfg), self.rank, self.world, max_tokens, max_recv_rows,
                                               ctypes.byref(g)))
        self._g = g
        try:
            h = (ctypes.c_uint8 * 64)()
            L.check(L.lib().ef_ep_group_handle(g, h))
            mine = bytes(h)
            if self.world > 1:
                on_gpu = dist.get_backend(group) == "nccl"
                t = torch.tensor(list(mine), dtype=torch.uint8, device=self.device if on_gpu else "cpu")
                parts = [torch.empty_like(t) for _ in range(self.world)]
                dist.all_gather(parts, t, group=group)
                handles = b"".join(bytes(p.cpu().tolist()) for p in parts)
            else:
                handles = mine
            buf = (ctypes.c_uint8 * len(handles)).from_buffer_copy(handles)
            with torch.cuda.device(self.device):
                L.check(L.lib().ef_ep_group_open(g, buf))
        except Exception:
            L.lib().ef_ep_group_destroy(g)
            self._g = None
            raise

    def workspace_bytes(self, T: int) -> int:
        return int(L.lib().ef_ep_workspace_size(self._g, T))

    def forward(self, x: torch.Tensor, inds_out: Optional[torch.Tensor] = None,
                wts_out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                workspace_buf: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = MoE(x) for this rank's tokens (x's dtype, or fp32 with out_dtype=torch.float32)."""
        if self._g is None:
            raise RuntimeError("the group is closed")
        H = self.spec.hidden
        xf = x.reshape(-1, H).contiguous()
        _need_cuda(xf)
        if xf.dtype != self.act_dtype:
            raise TypeError(f"activations must be {self.act_dtype} (the group's dtype)")
        T = xf.shape[0]
        od = out_dtype or xf.dtype
        y = torch.empty((T, H), dtype=od, device=xf.device)
        n = self.workspace_bytes(T)
        if workspace_buf is not None:
            if workspace_buf.numel() < n:
                raise ValueError(f"workspace_buf needs {n} bytes")
            ws = workspace_buf
        else:
            ws = workspace(n, xf.device)
        ops = self.ops
        sp, sh = ops.local_mlp, ops.shared_mlp
        sq = [ctypes.byref(p.qweight()) for p in (sh.gate_proj, sh.up_proj, sh.down_proj)] if sh else [None] * 3
        eb = ops.gate.e_score_correction_bias
        L.check(L.lib().ef_ep_forward(
            self._g, xf.data_ptr() if T else None, T, ops.gate.weight.data_ptr(),
            eb.data_ptr() if eb is not None else None, sp.gate_proj.qweight(), sp.up_proj.qweight(),
            sp.down_proj.qweight(), sq[0], sq[1], sq[2], y.data_ptr() if T else None, _dt_code(od),
            inds_out.data_ptr() if inds_out is not None else None,
            wts_out.data_ptr() if wts_out is not None else None, ws.data_ptr(), ws.numel(),
            _stream_ptr(xf.device)))
        return y.reshape(*x.shape[:-1], H)

    __call__ = forward

    def capture(self, T: int, out_dtype: Optional[torch.dtype] = None) -> "CapturedEpForward":
        """This rank's forward for T tokens captured in a CUDA graph (every
        rank captures, then replays the same number of times)."""
        return CapturedEpForward(self, T, out_dtype)

    def close(self) -> None:
        """Frees the exchange buffer after a barrier over the group (no rank
        may still be writing into it)."""
        if self._g is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        L.lib().ef_ep_group_destroy(self._g)
        self._g = None


class CapturedEpForward:
    """A PeerExpertParallelMoE forward for a fixed token count in a CUDA graph
    (own input, output and workspace buffers); two eager forwards first."""

    def __init__(self, layer: PeerExpertParallelMoE, T: int, out_dtype: Optional[torch.dtype] = None):
        dev = layer.device
        self.layer = layer
        self.x = torch.zeros((T, layer.spec.hidden), dtype=layer.act_dtype, device=dev)
        self.ws = torch.empty(max(layer.workspace_bytes(T), 1), dtype=torch.uint8, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
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


def _main(argv=None) -> None:
    """A one-rank peer-memory expert-parallel layer of the DeepSeek-V3 shape on
    cuda:0 (every exchange kernel runs; the peer stores land in this GPU's own
    buffer), for profiling:  python -m expertflow_b200.ep --tokens 32 --reps 5"""
    import argparse

    from . import synthetic
    from .spec import DEEPSEEK_V3

    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args(argv)
    spec = DEEPSEEK_V3
    layer = synthetic.make_layer_torch(spec, seed=1, device="cuda")
    m = PeerExpertParallelMoE(spec, shard_layer(spec, layer, 0, 1), max_tokens=a.tokens)
    del layer
    x = synthetic.make_x_torch(spec, a.tokens, seed=2, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(a.reps):
        if i == a.reps - 1:
            e0.record()
        m(x)
    e1.record()
    torch.cuda.synchronize()
    print(f"{a.tokens} tokens: last forward {e0.elapsed_time(e1) * 1e3:.1f} us")
    m.close()


if __name__ == "__main__":
    _main()
