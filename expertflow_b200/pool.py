"""Expert residency for streaming decode (the reference's expert cache).

* ``CachePolicy`` -- the reference's ``FrequencyWeightedCache``
  (ef_engine.py:48-104) over integer keys, via the C ABI (``ef_policy_*``).
* ``ExpertSlotPool`` -- the experts of many MoE layers in pinned host memory,
  streamed into HBM slots per layer (``ef_pool_*``); it is the
  ``expert_cache`` argument of ``streaming_moe_forward``
  (ef_engine.py:598, :650-675), and it runs the lookahead prediction of
  experiments/ef_v16_prefetch.py:92-113 (the next layer's gate on the
  current input) so the predicted experts' copies overlap this layer.
* ``ExpertStore`` -- expert weights read out of the model files by the
  library's reader threads (``ef_store_*``), the cold tier of a pool made
  with ``ExpertSlotPool.from_store``.
* ``zipf_layer_bias`` -- per-layer router logit bias log(p) for a shuffled
  Zipf popularity, the recipe of ef_integrated_engine.py:69-79.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from dataclasses import replace
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib as L
from .moe import MoEGate, _act_dt, _need_cuda, _stream_ptr, workspace
from .spec import MoESpec

_POLICIES = {"freq": L.EF_POLICY_FREQ, "lru": L.EF_POLICY_LRU, "belady": L.EF_POLICY_BELADY}
_NET = ("w1", "b1", "w2", "b2", "w3", "b3")


def load_predictor(src) -> dict:
    """Eviction-predictor weights: a dict, or the .npz that the reference's
    ``BeladyPredictor.save`` writes (ef_engine.py:143-148): w1 [3, H], b1 [H],
    w2 [H, H], b2 [H], w3 [H, 1], b3 [1], trained."""
    if isinstance(src, (str, os.PathLike)):
        z = np.load(src)
        src = {k: z[k] for k in z.files}
    out = {k: np.ascontiguousarray(np.asarray(src[k], np.float32)) for k in _NET}
    H = out["b1"].shape[0]
    if out["w1"].shape != (3, H) or out["w2"].shape != (H, H) or out["b2"].shape != (H,) or out["w3"].size != H \
            or out["b3"].size != 1:
        raise ValueError("predictor weights do not have the 3 -> H -> H -> 1 shapes")
    out["w3"] = out["w3"].reshape(H)
    out["trained"] = bool(np.asarray(src.get("trained", True)).reshape(-1)[0])
    return out


def _net_args(w: dict):
    H = w["b1"].shape[0]
    ptrs = [ctypes.c_void_p(w[k].ctypes.data) for k in _NET]
    return (H, *ptrs, int(w["trained"]))


class CachePolicy:
    """FrequencyWeightedCache(budget, decay) semantics: get / put / trim;
    ``kind="lru"``; ``kind="belady"``: BeladyExpertCache (learned eviction,
    ``set_predictor``; call ``trim()`` then ``end_token()`` once per token)."""

    def __init__(self, budget: int, decay: float = 0.95, kind: str = "freq", predictor=None):
        h = ctypes.c_void_p()
        L.check(L.lib().ef_policy_create(_POLICIES[kind], budget, decay, ctypes.byref(h)))
        self._h = h
        if predictor is not None:
            self.set_predictor(predictor)

    def set_predictor(self, predictor) -> None:
        w = load_predictor(predictor)
        self._net = w  # the library copies; kept for inspection
        L.check(L.lib().ef_policy_set_predictor(self._h, *_net_args(w)))

    def end_token(self) -> None:
        L.lib().ef_policy_end_token(self._h)

    def get(self, key: int) -> bool:
        return bool(L.lib().ef_policy_get(self._h, key))

    def put(self, key: int) -> None:
        L.lib().ef_policy_put(self._h, key)

    def trim(self) -> list:
        """Evict down to the budget, decay; returns the evicted keys in eviction order."""
        cap = max(len(self), 1)
        buf = (ctypes.c_longlong * cap)()
        n = L.lib().ef_policy_trim(self._h, ctypes.cast(buf, ctypes.c_void_p), cap)
        return [int(buf[i]) for i in range(n)]

    def keys(self) -> list:
        n = L.lib().ef_policy_keys(self._h, None, 0)
        buf = (ctypes.c_longlong * max(n, 1))()
        L.lib().ef_policy_keys(self._h, ctypes.cast(buf, ctypes.c_void_p), n)
        return [int(buf[i]) for i in range(n)]

    def score(self, key: int) -> float:
        return float(L.lib().ef_policy_score(self._h, key))

    def __len__(self) -> int:
        return int(L.lib().ef_policy_size(self._h))

    def close(self) -> None:
        if self._h:
            L.lib().ef_policy_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def zipf_layer_bias(n_layers: int, n_experts: int, skew: float = 1.1, seed: int = 42) -> np.ndarray:
    """[n_layers, n_experts] fp32 log-popularity: layer l's Zipf(skew) probabilities
    permuted by RandomState(seed).permutation per layer, as ef_integrated_engine.py:69-79."""
    rng = np.random.RandomState(seed)
    ranks = np.arange(1, n_experts + 1, dtype=np.float64)
    base = 1.0 / np.power(ranks, skew)
    out = np.empty((n_layers, n_experts), np.float32)
    for layer in range(n_layers):
        p = base[rng.permutation(n_experts)]
        p /= p.sum()
        out[layer] = np.log(p).astype(np.float32)
    return out


class StreamedMoELayer:
    """A MoE layer whose experts live in an ExpertSlotPool: the router (on the
    device) plus the attributes streaming_moe_forward reads."""

    def __init__(self, gate: MoEGate, layer_idx: int, spec: MoESpec):
        self.gate = gate
        self.num_experts_per_tok = gate.top_k
        self.shared_experts = None
        self._ef_layer_idx = layer_idx
        self.spec = spec


def _pool_moe_cfg(spec: MoESpec) -> L.MoECfg:
    return L.MoECfg(hidden=spec.hidden, inter=spec.inter, n_experts=spec.n_experts, top_k=spec.top_k,
                    bits=spec.bits, group_size=spec.group_size, n_shared=0, shared_inter=0,
                    act_dtype=L.EF_DT_BF16 if spec.act_dtype == "bfloat16" else L.EF_DT_F16,
                    path=L.EF_PATH_AUTO, router_mode=spec.router_mode, norm_topk=int(spec.norm_topk),
                    n_group=spec.n_group if spec.router != "softmax" else 1,
                    topk_group=spec.topk_group if spec.router != "softmax" else 1,
                    routed_scaling=spec.routed_scaling if spec.router != "softmax" else 1.0,
                    gate_dtype=L.EF_DT_F16 if spec.gate_dtype == "float16" else L.EF_DT_BF16)


_PROJS = ("gate", "up", "down")


class ExpertStore:
    """Expert weights read from model files by the library's reader threads
    (``ef_store_*``): the cold tier below the slot pool's pinned host blobs,
    standing in for the reference's memory-mapped expert reads and its
    page-cache prefetcher (ef_deepseek_mmap.py:431-570,
    experiments/ef_v18_prefetch2.py:76-200).

    ranges: per layer, 9 ``(file index, bf16, offset, stride)`` tuples in the
    order gate w, s, b, up w, s, b, down w, s, b -- expert e's copy of an
    array is ``size`` bytes at ``offset + e * stride`` (``size`` follows from
    the layer shape).  ``direct`` opens the files with O_DIRECT.  Host only:
    a store reads without a GPU.
    """

    def __init__(self, spec: MoESpec, paths: Sequence[str], ranges: Sequence[Sequence[tuple]], n_readers: int = 0,
                 direct: bool = False):
        if spec.n_shared:
            raise ValueError("the store holds routed experts only")
        self.spec = spec
        self.paths = [os.fspath(p) for p in paths]
        self.n_layers = len(ranges)
        arr = (L.FileArray * (9 * self.n_layers))()
        for li, rs in enumerate(ranges):
            if len(rs) != 9:
                raise ValueError(f"layer {li}: 9 arrays expected, got {len(rs)}")
            for a, (f, bf16, off, stride) in enumerate(rs):
                arr[9 * li + a] = L.FileArray(int(f), int(bool(bf16)), int(off), int(stride))
        self.cfg = _pool_moe_cfg(spec)
        cpaths = (ctypes.c_char_p * len(self.paths))(*[p.encode() for p in self.paths])
        h = ctypes.c_void_p()
        L.check(L.lib().ef_store_open(ctypes.byref(self.cfg), self.n_layers, ctypes.cast(cpaths, ctypes.c_void_p),
                                      len(self.paths), arr, int(n_readers), int(bool(direct)), ctypes.byref(h)))
        self._h = h
        self._pools = weakref.WeakSet()  # pools reading through this store (closed before it)

    @classmethod
    def from_safetensors(cls, path_or_index, layers: Optional[Sequence[int]] = None, spec: Optional[MoESpec] = None,
                         n_readers: int = 0, direct: bool = False) -> "ExpertStore":
        """A store over the switch_mlp experts of a safetensors checkpoint
        (layers: the checkpoint's MoE layer indices, in pool order; default
        every layer that has switch_mlp experts)."""
        from . import weights as W

        index = path_or_index if isinstance(path_or_index, W.SafetensorsIndex) else W.SafetensorsIndex(path_or_index)
        if layers is None:
            layers = W.moe_layers(index)
        if not layers:
            raise KeyError("no switch_mlp experts in the checkpoint")
        spec = spec or replace(W.infer_spec(index, layers[0]), n_shared=0)
        files, ranges = [], []
        for layer in layers:
            rs = []
            for fpath, bf16, off, stride in W.expert_ranges(index, layer, spec):
                if fpath not in files:
                    files.append(fpath)
                rs.append((files.index(fpath), bf16, off, stride))
            ranges.append(rs)
        return cls(spec, files, ranges, n_readers=n_readers, direct=direct)

    def info(self) -> dict:
        i = L.StoreInfo()
        L.check(L.lib().ef_store_get_info(self._h, ctypes.byref(i)))
        return {"blob_bytes": int(i.blob_bytes), "offsets": [int(v) for v in i.offsets], "n_layers": i.n_layers,
                "n_readers": i.n_readers, "direct": bool(i.direct), "reads": int(i.reads),
                "file_bytes": float(i.file_bytes)}

    def read(self, layers: Sequence[int], experts: Sequence[int]) -> list:
        """Expert blobs (numpy uint8, blob_bytes each) read in parallel."""
        n = len(layers)
        if len(experts) != n:
            raise ValueError("one expert per layer entry")
        nb = self.info()["blob_bytes"]
        bufs = [np.empty(nb, np.uint8) for _ in range(n)]
        li = (ctypes.c_int32 * max(n, 1))(*layers)
        ei = (ctypes.c_int32 * max(n, 1))(*experts)
        dst = (ctypes.c_void_p * max(n, 1))(*[b.ctypes.data for b in bufs])
        L.check(L.lib().ef_store_read(self._h, n, li, ei, dst))
        return bufs

    def split_blob(self, blob: np.ndarray) -> dict:
        """{"gate": (w uint32 [out, words], s fp16 [out, groups], b fp16), "up": ..., "down": ...} views of a blob."""
        off = self.info()["offsets"]
        H, I, bits = self.spec.hidden, self.spec.inter, self.spec.bits
        shapes = {"gate": (I, H), "up": (I, H), "down": (H, I)}
        out = {}
        for j, m in enumerate(_PROJS):
            rows, cols = shapes[m]
            w = blob[off[3 * j]:off[3 * j] + rows * cols * bits // 8].view(np.uint32).reshape(rows, cols * bits // 32)
            sb = rows * (cols // 64) * 2
            s = blob[off[3 * j + 1]:off[3 * j + 1] + sb].view(np.float16).reshape(rows, cols // 64)
            b = blob[off[3 * j + 2]:off[3 * j + 2] + sb].view(np.float16).reshape(rows, cols // 64)
            out[m] = (w, s, b)
        return out

    def close(self) -> None:
        """Close the store; pools still open over it are closed first (a pool
        reads through its store until it is destroyed)."""
        for pl in list(getattr(self, "_pools", ())):
            pl.close()
        if getattr(self, "_h", None):
            L.lib().ef_store_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertSlotPool:
    """HBM expert slots over a pinned-host expert pool (see module docstring).

    host_layers: per layer a dict {"gate": (w, s, b), "up": ..., "down": ...}
    of CPU tensors in the stacked MLX layout ([E, out, in*bits/32] int32
    words, [E, out, in/64] fp16 scales and biases).  The pool copies them into
    its own pinned store (one blob per expert) when it is created.

    ``ExpertSlotPool.from_store`` builds the pool over an ``ExpertStore``
    instead: only ``host_blobs`` experts stay in pinned host memory, and the
    rest are read from the model files when needed (or ahead, by the
    lookahead).
    """

    def __init__(self, spec: MoESpec, host_layers: Optional[Sequence[dict]], budget: int,
                 headroom: Optional[int] = None, policy: str = "freq", decay: float = 0.95, device=None,
                 store: Optional[ExpertStore] = None, host_blobs: int = 0):
        if spec.n_shared:
            raise ValueError("the slot pool streams routed experts only")
        self.spec = spec
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.cfg = _pool_moe_cfg(spec)
        self.store = store
        if store is not None:
            self.n_layers = store.n_layers
        else:
            self.n_layers = len(host_layers)
            host = list(host_layers)
            for hl in host:
                for k in _PROJS:
                    for a in hl[k]:
                        if a.is_cuda or not a.is_contiguous():
                            raise ValueError("host expert arrays must be contiguous CPU tensors")
            arr = L.QWeight * self.n_layers
            self._qw = {k: arr(*[L.QWeight(hl[k][0].data_ptr(), hl[k][1].data_ptr(), hl[k][2].data_ptr())
                                 for hl in host]) for k in _PROJS}
        self.pool_cfg = L.PoolCfg(n_layers=self.n_layers, budget=budget,
                                  headroom=spec.top_k if headroom is None else headroom,
                                  policy=_POLICIES[policy], decay=decay)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            if store is not None:
                if not getattr(store, "_h", None):
                    raise ValueError("the store is closed")
                L.check(L.lib().ef_pool_create_from_store(ctypes.byref(self.cfg), ctypes.byref(self.pool_cfg),
                                                          store._h, int(host_blobs), ctypes.byref(h)))
                store._pools.add(self)
            else:
                L.check(L.lib().ef_pool_create(ctypes.byref(self.cfg), ctypes.byref(self.pool_cfg), self._qw["gate"],
                                               self._qw["up"], self._qw["down"], ctypes.byref(h)))
        self._h = h

    @classmethod
    def from_store(cls, store: ExpertStore, budget: int, host_blobs: int, headroom: Optional[int] = None,
                   policy: str = "freq", decay: float = 0.95, device=None) -> "ExpertSlotPool":
        return cls(store.spec, None, budget, headroom=headroom, policy=policy, decay=decay, device=device,
                   store=store, host_blobs=host_blobs)

    # -- the reference's call -------------------------------------------------
    def forward_layer(self, moe_module: StreamedMoELayer, x: torch.Tensor, next_moe: Optional[StreamedMoELayer] = None,
                      inds_out: Optional[torch.Tensor] = None, wts_out: Optional[torch.Tensor] = None,
                      out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        return self.forward(moe_module._ef_layer_idx, x, moe_module.gate,
                            next_moe.gate if next_moe is not None else None, inds_out, wts_out, out_dtype)

    def forward(self, layer: int, x: torch.Tensor, gate: MoEGate, next_gate: Optional[MoEGate] = None,
                inds_out: Optional[torch.Tensor] = None, wts_out: Optional[torch.Tensor] = None,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        H = self.spec.hidden
        xf = x.reshape(-1, H).contiguous()
        _need_cuda(xf, gate.weight)
        T = xf.shape[0]
        if _act_dt(xf) != self.cfg.act_dtype:
            raise TypeError("x dtype does not match the pool's activation dtype")
        y = torch.empty(xf.shape, dtype=out_dtype or xf.dtype, device=xf.device)
        if T == 0:
            return y.reshape(x.shape)
        n = L.lib().ef_pool_workspace_size(self._h, T)
        ws = workspace(n, xf.device)
        eb = gate.e_score_correction_bias
        ng = next_gate.weight.data_ptr() if next_gate is not None else None
        neb = next_gate.e_score_correction_bias if next_gate is not None else None
        L.check(L.lib().ef_pool_moe_forward(
            self._h, layer, xf.data_ptr(), T, gate.weight.data_ptr(), eb.data_ptr() if eb is not None else None,
            ng, neb.data_ptr() if neb is not None else None, y.data_ptr(), int(y.dtype == torch.float32),
            inds_out.data_ptr() if inds_out is not None else None,
            wts_out.data_ptr() if wts_out is not None else None, ws.data_ptr(), ws.numel(), _stream_ptr(xf.device)))
        return y.reshape(x.shape)

    def decode_step(self, r: torch.Tensor, gates: Sequence[MoEGate], lookahead: int = 1,
                    eps: float = 1e-6) -> torch.Tensor:
        """One decode step through all layers in the library (ef_pool_decode_step):
        per layer r += y, x = rmsnorm(r), y = MoE_layer(x); then r += y and the
        per-token trim.  r: fp32 [T, H] residual stream, updated in place.
        lookahead: how many following layers (0, 1 or 2; True is 1) have their
        experts predicted from each layer's input and copied ahead."""
        lookahead = int(lookahead)
        if not 0 <= lookahead <= 2:
            raise ValueError("lookahead must be 0, 1 or 2 layers")
        if r.dtype != torch.float32 or not r.is_cuda or not r.is_contiguous():
            raise ValueError("r must be a contiguous fp32 CUDA tensor")
        if len(gates) != self.n_layers:
            raise ValueError("one gate per layer")
        T = r.reshape(-1, self.spec.hidden).shape[0]
        key = tuple(g.weight.data_ptr() for g in gates)
        if getattr(self, "_gate_key", None) != key:
            self._gate_ptrs = (ctypes.c_void_p * self.n_layers)(*[g.weight.data_ptr() for g in gates])
            self._bias_ptrs = (ctypes.c_void_p * self.n_layers)(
                *[g.e_score_correction_bias.data_ptr() if g.e_score_correction_bias is not None else None
                  for g in gates])
            self._gate_key = key
        n = L.lib().ef_pool_decode_workspace_size(self._h, T)
        ws = workspace(n, r.device)
        L.check(L.lib().ef_pool_decode_step(self._h, r.data_ptr(), T, self._gate_ptrs, self._bias_ptrs, int(lookahead),
                                            eps, ws.data_ptr(), ws.numel(), _stream_ptr(r.device)))
        return r

    def end_token(self) -> None:
        L.check(L.lib().ef_pool_end_token(self._h))

    def set_predictor(self, predictor) -> None:
        """Learned-eviction weights for every layer (pools made with policy="belady")."""
        L.check(L.lib().ef_pool_set_predictor(self._h, *_net_args(load_predictor(predictor))))

    def resident(self, layer: int) -> list:
        n = ctypes.c_int()
        buf = (ctypes.c_int32 * self.spec.n_experts)()
        L.check(L.lib().ef_pool_resident(self._h, layer, ctypes.cast(buf, ctypes.c_void_p), self.spec.n_experts,
                                         ctypes.byref(n)))
        return [int(buf[i]) for i in range(n.value)]

    def stats(self) -> dict:
        s = L.PoolStats()
        L.check(L.lib().ef_pool_get_stats(self._h, ctypes.byref(s)))
        d = s.as_dict()
        d["hit_rate"] = d["hits"] / d["accesses"] if d["accesses"] else 0.0
        d["copy_free_rate"] = 1.0 - d["copies_sync"] / d["accesses"] if d["accesses"] else 0.0
        return d

    def reset_stats(self) -> None:
        L.check(L.lib().ef_pool_reset_stats(self._h))

    def record_routing(self, on: bool = True) -> None:
        """Start (clearing the trace) or stop recording the routing trace."""
        L.check(L.lib().ef_pool_record_routing(self._h, int(on)))

    @property
    def routing_trace(self) -> list:
        """Per ended token, the (layer, expert) of every routed entry in
        routing order -- the reference's ``expert_cache.routing_trace``
        (ef_engine.py:222-229), the input of its Belady label computation."""
        n_p, n_t = ctypes.c_longlong(), ctypes.c_longlong()
        L.check(L.lib().ef_pool_routing_trace(self._h, None, 0, ctypes.byref(n_p), None, 0, ctypes.byref(n_t)))
        pairs = (ctypes.c_int32 * max(1, 2 * n_p.value))()
        ends = (ctypes.c_longlong * max(1, n_t.value))()
        L.check(L.lib().ef_pool_routing_trace(self._h, ctypes.cast(pairs, ctypes.c_void_p), n_p.value,
                                              ctypes.byref(n_p), ctypes.cast(ends, ctypes.c_void_p), n_t.value,
                                              ctypes.byref(n_t)))
        out, start = [], 0
        for i in range(n_t.value):
            end = int(ends[i])
            out.append([(int(pairs[2 * j]), int(pairs[2 * j + 1])) for j in range(start, end)])
            start = end
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            L.lib().ef_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def make_host_layers(spec: MoESpec, n_layers: int, seed: int = 0, device="cuda") -> list:
    """Seeded synthetic experts for n_layers layers in host memory (generated
    on the device one layer at a time, then copied out)."""
    from .synthetic import make_layer_torch

    out = []
    for layer in range(n_layers):
        d = make_layer_torch(spec, seed=seed + layer, device=device)
        out.append({k: tuple(a.cpu() for a in d[k]) for k in ("gate", "up", "down")})
        del d
    return out


def _main(argv=None) -> None:
    """A streamed decode for profiling: `layers` Qwen3-30B-A3B-shaped layers,
    25 % of each layer's experts in HBM, Zipf(1.1)-biased routing, lookahead
    over --lookahead layers (default 1); prints the time per token.
    python -m expertflow_b200.pool --layers 8 --steps 24"""
    import argparse

    from .moe import MoEGate
    from .spec import WORKLOADS
    from .synthetic import make_x_torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--lookahead", type=int, default=1)
    a = ap.parse_args(argv)
    spec = WORKLOADS["qwen3-30b-a3b-moe"]
    dev = torch.device("cuda", 0)
    host = make_host_layers(spec, a.layers, seed=3000, device=dev)
    bias = torch.from_numpy(zipf_layer_bias(a.layers, spec.n_experts, 1.1, seed=42)).to(dev)
    gates = []
    for layer in range(a.layers):
        g = torch.Generator(device=dev)
        g.manual_seed(77 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * spec.gate_std).to(torch.float16)
        gates.append(MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
    pl = ExpertSlotPool(spec, host, budget=spec.n_experts // 4, headroom=spec.top_k)
    rs = [make_x_torch(spec, 1, seed=5000 + t, device=dev).float().contiguous() for t in range(a.steps)]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for r in rs:
        pl.decode_step(r, gates, lookahead=a.lookahead)
    e1.record()
    torch.cuda.synchronize()
    st = pl.stats()
    print(f"{a.layers} layers x {a.steps} tokens: {e0.elapsed_time(e1) / a.steps:.3f} ms per token, "
          f"hit rate {st['hit_rate']:.3f}, {st['copies_prefetch']} prefetched, {st['copies_sync']} on demand")
    pl.close()


if __name__ == "__main__":
    _main()
