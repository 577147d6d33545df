"""Generate the golden fixtures in this directory by executing the REFERENCE's
own code (read from a reference checkout given by --reference or the
EF_REFERENCE environment variable).

* ``moe_*.npz`` -- ``streaming_moe_forward`` (ef_engine.py:598-706) run on
  seeded synthetic layers through ``mlx_shim`` (numpy stand-ins for the MLX ops
  it calls).  For the Mixtral-style cases the gate returns logits and the
  reference's own argpartition / take_along_axis / softmax code routes
  (ef_engine.py:613-618); for the DeepSeek/Qwen-style cases the gate returns
  ``(inds, scores)`` like mlx_lm's MoEGate and the reference code does the
  per-(token, k) quantized SwiGLU, the score-weighted sum and the shared add.
* ``cache_trace.npz`` -- ``FrequencyWeightedCache`` (ef_engine.py:48-104) driven
  by the reference's ``SimulatedMoERouter`` Zipf trace (ef_integrated_engine.py:44-118).

Run:  python tests/golden/make_golden.py --reference <reference checkout>
The fixtures store outputs plus a digest of the regenerated inputs; the inputs
themselves are regenerated from their seeds by expertflow_b200.synthetic.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from expertflow_b200.spec import MoESpec, MIXTRAL_SMALL  # noqa: E402
from expertflow_b200 import synthetic  # noqa: E402
from oracle import oracle as O  # noqa: E402

# Small cases that exercise every routing mode, both bit widths and the shared expert.
CASES = {
    "moe_mixtral_small_t1": (MIXTRAL_SMALL, 0, 1),
    "moe_mixtral_small_t5": (MIXTRAL_SMALL, 0, 5),
    "moe_qwen_small": (MoESpec(hidden=512, n_experts=32, top_k=4, inter=256, bits=4, router="softmax",
                               norm_topk=True, act_dtype="bfloat16"), 3, 6),
    "moe_qwen_small_nonorm": (MoESpec(hidden=256, n_experts=32, top_k=4, inter=128, bits=4, router="softmax",
                                      norm_topk=False, act_dtype="bfloat16"), 4, 5),
    "moe_deepseek_small": (MoESpec(hidden=512, n_experts=64, top_k=6, inter=256, bits=4,
                                   router="sigmoid_group", n_group=8, topk_group=4, routed_scaling=2.5,
                                   n_shared=1, act_dtype="bfloat16", e_bias_std=0.01), 5, 5),
    "moe_deepseek_small_8bit": (MoESpec(hidden=512, n_experts=64, top_k=8, inter=192, bits=8,
                                        router="sigmoid_group", n_group=8, topk_group=4, routed_scaling=2.5,
                                        n_shared=1, act_dtype="bfloat16", e_bias_std=0.01, gate_std=0.002), 6, 4),
}


class _Proj(dict):
    def __init__(self, w, s, b, group_size, bits):
        super().__init__(weight=w, scales=s, biases=b)
        self.group_size = group_size
        self.bits = bits


class _Switch:
    def __init__(self, layer, spec):
        g, u, d = layer["gate"], layer["up"], layer["down"]
        self.gate_proj = _Proj(*g, spec.group_size, spec.bits)
        self.up_proj = _Proj(*u, spec.group_size, spec.bits)
        self.down_proj = _Proj(*d, spec.group_size, spec.bits)


class _MoE:
    """Duck-typed mlx_lm MoE block: the attributes ef_engine.py:598-631 reads."""

    def __init__(self, spec, layer, mx, nn):
        self.spec, self.layer = spec, layer
        self.num_experts_per_tok = spec.top_k
        self.switch_mlp = _Switch(layer, spec)
        self._ef_layer_idx = 0
        self._mx, self._nn = mx, nn
        self.shared_experts = self._shared if layer["shared"] is not None else None

    def _logits(self, x):
        B, S, H = x.shape
        xb = synthetic.act_bits_np(x.reshape(B * S, H), self.spec.act_dtype)
        lg = O.np_router_logits(xb, self.spec.act_dtype == "bfloat16", self.layer["gate_w"].view(np.uint16), False)
        return lg.reshape(B, S, -1)

    def gate(self, x):
        lg = self._logits(x)
        B, S, E = lg.shape
        if self.spec.router == "softmax" and self.spec.norm_topk:
            return lg  # Mixtral style: the reference routes the logits itself
        spec = self.spec
        if spec.router == "softmax":
            inds, sc = O.np_route_softmax(lg.reshape(B * S, E), spec.top_k, spec.norm_topk)
        else:
            inds, sc = O.np_route_sigmoid_group(lg.reshape(B * S, E), self.layer["e_bias"], spec.top_k,
                                                spec.n_group, spec.topk_group, spec.norm_topk,
                                                spec.routed_scaling)
        return inds.reshape(B, S, -1), sc.reshape(B, S, -1)

    def _shared(self, x):
        mx, nn = self._mx, self._nn
        (gw, gs, gb), (uw, us, ub), (dw, ds, db) = self.layer["shared"]
        B, S, H = x.shape
        xf = x.reshape(B * S, H)
        g = mx.quantized_matmul(xf, gw, gs, gb, transpose=True, group_size=64, bits=self.spec.bits)
        u = mx.quantized_matmul(xf, uw, us, ub, transpose=True, group_size=64, bits=self.spec.bits)
        o = mx.quantized_matmul(nn.silu(g) * u, dw, ds, db, transpose=True, group_size=64, bits=self.spec.bits)
        return o.reshape(B, S, H)


def gen_moe(ef_engine, mx, nn, out_dir):
    for name, (spec, seed, T) in CASES.items():
        layer = synthetic.make_layer_np(spec, seed)
        xb = synthetic.make_x_np(spec, T, seed + 1000)
        xf = O.bits_to_f32(xb, spec.act_dtype == "bfloat16")
        moe = _MoE(spec, layer, mx, nn)
        # routing as the reference sees it (Mixtral path is recomputed inside)
        g = moe.gate(xf[None])
        if isinstance(g, tuple):
            inds, scores = g[0][0], g[1][0]
        else:
            k = spec.top_k
            inds = mx.argpartition(-g, kth=k - 1, axis=-1)[..., :k][0]
            scores = mx.softmax(np.take_along_axis(g[0], inds, axis=-1), axis=-1, precise=True)
        y = ef_engine.streaming_moe_forward(moe, xf[None].astype(np.float32), expert_cache=None)
        y = np.asarray(y, np.float64)[0]
        np.savez_compressed(
            os.path.join(out_dir, name + ".npz"),
            spec=json.dumps(spec.to_dict()), seed=seed, x_seed=seed + 1000, T=T,
            digest=synthetic.layer_digest(layer), inds=np.asarray(inds, np.int32),
            scores=np.asarray(scores, np.float32), y=y.astype(np.float32))
        print(f"{name}: T={T} y|max|={np.abs(y).max():.4f}")


def gen_cache(ef_engine, ef_integrated_engine, out_dir):
    n_layers, n_exp, k, tokens, budget = 4, 128, 8, 160, 96
    router = ef_integrated_engine.SimulatedMoERouter(n_experts=n_exp, n_active=k, n_moe_layers=n_layers,
                                                     zipf_skew=1.1, temporal_locality=0.4, seed=42)
    layer_probs = np.stack(router._layer_probs)
    cache = ef_engine.FrequencyWeightedCache(budget=budget, decay=0.95)
    accesses, hits, evicted_counts, resident = [], [], [], []
    for _ in range(tokens):
        for layer in range(n_layers):
            sel, _w = router.route(layer)
            for e in sorted(sel):
                key = (layer, int(e))
                accesses.append(layer * n_exp + int(e))
                if cache.get(key) is None:
                    cache.put(key, 1)
                    hits.append(0)
                else:
                    hits.append(1)
            accesses.append(-1)  # layer boundary marker
            hits.append(-1)
        evicted_counts.append(cache.trim())
        resident.append(sorted(l * n_exp + e for (l, e) in cache.cache.keys()))
        accesses.append(-2)  # end-of-token (trim) marker
        hits.append(-2)
    res = np.full((tokens, budget), -1, np.int32)
    for i, r in enumerate(resident):
        res[i, :len(r)] = r
    np.savez_compressed(os.path.join(out_dir, "cache_trace.npz"), n_layers=n_layers, n_experts=n_exp, k=k,
                        budget=budget, decay=0.95, accesses=np.asarray(accesses, np.int32),
                        hits=np.asarray(hits, np.int8), evicted=np.asarray(evicted_counts, np.int32),
                        resident=res, layer_probs=layer_probs, zipf_skew=1.1, seed=42)
    print(f"cache_trace: {len(accesses)} events, final hit rate {cache.total_hit_rate:.1f}%")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EF_REFERENCE"),
                    required="EF_REFERENCE" not in os.environ,
                    help="reference checkout to import (default: $EF_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    import mlx_shim

    mlx_shim.install()
    sys.path.insert(0, args.reference)
    import ef_engine  # noqa: E402  (reference module, imported read-only)
    import ef_integrated_engine  # noqa: E402
    import mlx.core as mx
    import mlx.nn as nn

    gen_moe(ef_engine, mx, nn, args.out)
    gen_cache(ef_engine, ef_integrated_engine, args.out)


if __name__ == "__main__":
    main()
