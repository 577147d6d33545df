"""MoE-layer benchmark: tokens/s and HBM GB/s (fraction of the measured roofline).

Default workload: one Qwen3-30B-A3B-shaped MoE layer (hidden 2048, 128 experts,
top-8 softmax, inter 768, 4-bit g64 affine weights, bf16 activations), a
decode batch of 64 tokens; the 1/8/32/64-token sweep is reported alongside.
A step is one MoE-layer forward (router, permute, gate/up+SwiGLU, down,
combine) over one batch with weights resident in HBM.  Several seeded layer
copies (each larger than L2) are rotated so every step reads cold weights.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--tokens T]

Multi-GPU (torchrun, one process per GPU): the line's workload becomes the
DeepSeek-V3-shaped layer (hidden 7168, 256 routed experts + 1 shared, top-8
sigmoid group-limited routing, inter 2048, 4-bit) with its experts sharded
across the GPUs (E/N each) and the token rows exchanged over NVLink peer
memory by the library's own kernels (ef_ep_forward, captured in a CUDA
graph).  Strong scaling: a global batch of --ep-tokens decode tokens split
evenly; value = that batch / the max-over-ranks step time.  The line also
carries the same run's single-GPU layer on the same batch (box_speedup),
weak scaling, per-phase kernel times, the EP output checked bit for bit
against the single-GPU layer (ep_parity) and the NCCL all-to-all version.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"
WORKLOAD = "qwen3-30b-a3b-moe"


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": float(p["hbm_gbs"]), "bf16": float(p["bf16_tflops"]),
                "bf16_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "kind": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "kind": "fallback"}


class ClockSampler:
    """nvidia-smi samples of SM clock / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
def algorithmic_bytes(spec, n_unique: int, T: int) -> dict:
    """Per-step algorithmic HBM bytes: packed codes + fp16 scales/biases of the
    distinct routed experts (+ shared), router weight, activations in/out."""
    per_expert = spec.expert_bytes()
    gate_up = per_expert * 2 // 3
    down = per_expert - gate_up
    shared = per_expert if spec.n_shared else 0
    act = T * spec.hidden * 2 * 2
    total = n_unique * per_expert + shared + spec.router_bytes() + act
    return {"total": total, "gate_up": (n_unique + (1 if spec.n_shared else 0)) * gate_up,
            "down": (n_unique + (1 if spec.n_shared else 0)) * down}


def run_cpu_reference(spec, T, budget_s, seed=0, layer=None, xb=None):
    """Time the oracle port (C, OpenMP, all host threads) on one batch of T tokens."""
    import numpy as np
    from expertflow_b200 import synthetic
    from oracle import oracle as O

    if layer is None:
        layer = synthetic.make_layer_np(spec, seed)
    if xb is None:
        xb = synthetic.make_x_np(spec, T, seed + 1)
    rs = O.RouterSpec(spec.router, spec.top_k, spec.norm_topk, spec.n_group, spec.topk_group, spec.routed_scaling)
    O.set_threads(os.cpu_count() or 1)
    O.moe_forward(xb[:1], spec.act_dtype == "bfloat16", layer["gate_w"].view(np.uint16), False, rs,
                  layer["e_bias"], layer["gate"], layer["up"], layer["down"], spec.bits, spec.group_size,
                  layer["shared"])  # warm-up (page-in, thread pool)
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        O.moe_forward(xb, spec.act_dtype == "bfloat16", layer["gate_w"].view(np.uint16), False, rs, layer["e_bias"],
                      layer["gate"], layer["up"], layer["down"], spec.bits, spec.group_size, layer["shared"])
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 50:
            break
    t = statistics.median(times)
    return {"tokens_per_s": T / t, "s_per_step": t, "steps": len(times), "cores": O.num_threads()}


# ---------------------------------------------------------------------------
def bench_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return 0
    from expertflow_b200.spec import WORKLOADS

    if ws > 1:  # the workload of our N > 1 line: DeepSeek-V3 layer, sampled to a few tokens per step
        wl = "deepseek-v3-moe"
        spec = WORKLOADS[wl]
        T = min(8, args.ep_tokens)
        cfg = {"workload": wl, "tokens_global": args.ep_tokens, "hidden": spec.hidden, "experts": spec.n_experts,
               "top_k": spec.top_k, "inter": spec.inter, "bits": spec.bits, "shared_experts": spec.n_shared}
        sample = f"{T}-token forwards of the {args.ep_tokens}-token workload's layer"
    else:
        wl = args.workload
        spec = WORKLOADS[wl]
        T = args.tokens
        cfg = {"workload": wl, "tokens": T, "hidden": spec.hidden, "experts": spec.n_experts, "top_k": spec.top_k,
               "inter": spec.inter, "bits": spec.bits}
        sample = f"full {T}-token layer forwards"
    budget = max(2.0, min(20.0, 2.0 * (args.steps + args.warmup)))
    r = run_cpu_reference(spec, T, budget)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["tokens_per_s"], 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": r["steps"], "warmup": 1, "ms_per_step": round(r["s_per_step"] * 1e3, 3),
        "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
        "dtype": "u4/u8 codes, f32 accumulate", "data": "synthetic (seeded)", "config": cfg,
        "cpu_baseline": {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": f"{r['steps']} {sample} (median), oracle/ef_oracle.c"},
        "e2e": {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class _Layers:
    """Seeded layer copies on one device, rotated per step so that every step
    reads weights that are not in L2 (each copy is larger than L2 or there
    are enough copies)."""

    def __init__(self, spec, dev, rank, path=None, min_bytes=1.5e9, seed0=1000):
        from expertflow_b200 import moe, synthetic, _lib

        self.spec = spec
        self.layer_bytes = spec.n_experts * spec.expert_bytes()
        self.n = max(2, math.ceil(min_bytes / self.layer_bytes))
        p = _lib.EF_PATH_AUTO if path is None else path
        self.layers = [moe.MoELayer.from_arrays(spec, synthetic.make_layer_torch(spec, seed=seed0 * (rank + 1) + i,
                                                                                 device=dev), device=dev, path=p)
                       for i in range(self.n)]


class _EpLayers:
    """Expert-parallel copies of one layer: this rank holds experts
    [rank * E/P, (rank + 1) * E/P) of each copy, the gate and shared expert
    replicated (experts exchanged with NCCL all-to-all)."""

    def __init__(self, spec, dev, rank, ws, min_bytes=1.5e9, seed0=1000):
        import torch
        from expertflow_b200 import synthetic
        from expertflow_b200.ep import ExpertParallelMoE, shard_layer

        self.spec = spec
        self.layer_bytes = spec.n_experts // ws * spec.expert_bytes()
        self.n = max(2, math.ceil(min_bytes / self.layer_bytes))
        self.layers = []
        for i in range(self.n):
            full = synthetic.make_layer_torch(spec, seed=seed0 + i, device=dev)
            ops = shard_layer(spec, full, rank, ws, device=dev)
            del full
            torch.cuda.empty_cache()
            self.layers.append(ExpertParallelMoE(spec, ops))


def _keep_loaded(fwd, n, e0, e1, steps, hold):
    """After the timed steps (e0..e1, already enqueued), keep replaying the same
    forwards, untimed, until about `hold` seconds have passed, so that a clock
    sampler running around the timed region sees the GPU under that load."""
    import torch

    if hold <= 0:
        torch.cuda.synchronize()
        return
    e1.synchronize()
    per = max(e0.elapsed_time(e1) / max(steps, 1), 1e-3)  # ms per step
    extra = int(min(20000, hold * 1e3 / per))
    for s in range(extra):
        fwd[s % n]()
    torch.cuda.synchronize()


def _time_layers(L, T, steps, warmup, pg, dev, trace=False, x_seed=7, graphs=False, hold=0.0):
    """CUDA-event time of `steps` forwards (max over ranks), the distinct
    experts per step (from the routing indices) and, with trace, the per-launch
    kernel times of a separate (eager) pass.  graphs: each layer copy's forward
    is captured in a CUDA graph (MoELayer.capture) and replayed."""
    import torch
    from expertflow_b200 import synthetic, _lib

    spec = L.spec
    xs = [synthetic.make_x_torch(spec, T, seed=x_seed + i, device=dev) for i in range(L.n)]
    uniq = []
    for i, m in enumerate(L.layers):
        inds = torch.empty((T, spec.top_k), dtype=torch.int32, device=dev)
        m(xs[i], inds_out=inds)
        uniq.append(int(torch.unique(inds).numel()))
    fwd = [(lambda m=m, x=x: m(x)) for m, x in zip(L.layers, xs)]
    if graphs:
        cfs = [m.capture(T, x.dtype) for m, x in zip(L.layers, xs)]
        for cf, x in zip(cfs, xs):
            cf.x.copy_(x)
        fwd = [cf.graph.replay for cf in cfs]
    for s in range(warmup):
        fwd[s % L.n]()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in range(steps):
        fwd[s % L.n]()
    e1.record(st)
    _keep_loaded(fwd, L.n, e0, e1, steps, hold)
    ms = e0.elapsed_time(e1) / steps
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    recs = []
    if trace:
        _lib.trace_enable(True)
        _lib.trace_read()
        for s in range(min(steps, 2 * L.n)):
            L.layers[s % L.n](xs[s % L.n])
        torch.cuda.synchronize()
        recs = _lib.trace_read()
        _lib.trace_enable(False)
    ub = [uniq[s % L.n] for s in range(steps)]
    return ms, ub, recs, xs


def _by_kernel(recs):
    by = {}
    for name, t in recs:
        by.setdefault(name, []).append(t)
    return by


def _cpu_sample(spec, m, x_dev, budget_s):
    """The oracle port on the host cores over a sample of the workload's tokens,
    with the weights of layer copy m (copied to host memory)."""
    import numpy as np
    import torch

    def q(p):
        return (p["weight"].cpu().numpy().view(np.uint32), p["scales"].cpu().numpy(), p["biases"].cpu().numpy())

    L0 = {"gate_w": m.gate.weight.cpu().numpy(),
          "e_bias": m.gate.e_score_correction_bias.cpu().numpy() if m.gate.e_score_correction_bias is not None else None,
          "gate": q(m.switch_mlp.gate_proj), "up": q(m.switch_mlp.up_proj), "down": q(m.switch_mlp.down_proj),
          "shared": None}
    if m.shared_experts is not None:
        sh = m.shared_experts
        L0["shared"] = tuple(q(pj) for pj in (sh.gate_proj, sh.up_proj, sh.down_proj))
    xb = x_dev.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return run_cpu_reference(spec, xb.shape[0], budget_s, layer=L0, xb=xb)


def section_decode(name, spec, Ts, args, pg, dev, rank, ws, peaks):
    """HBM-bound decode sweep on one layer shape (GEMV path); expert-parallel
    across the ranks when there are several."""
    L = _EpLayers(spec, dev, rank, ws) if ws > 1 else _Layers(spec, dev, rank)
    out = {"workload": name, "bound": "hbm", "layer_copies": L.n,
           "parallelism": f"ep{ws} (experts sharded, NCCL all-to-all)" if ws > 1 else "single",
           "l2": f"rotating {L.n} layer copies of {L.layer_bytes / 1e9:.2f} GB", "points": []}
    for T in Ts:
        ms, ub, recs, xs = _time_layers(L, T, args.steps, args.warmup, pg, dev, trace=True)
        ab = algorithmic_bytes(spec, statistics.mean(ub), T)
        by = _by_kernel(recs)
        kern = max(by, key=lambda k: sum(by[k])) if by else None
        k_ms = statistics.mean(by[kern]) if kern else None
        # algorithmic bytes are counted for one whole layer: meaningful on one GPU
        k_bytes = {"qmv_gate_up": ab["gate_up"], "qmv_down": ab["down"]}.get(kern) if ws == 1 else None
        gbs = ab["total"] / (ms * 1e-3) / 1e9
        pt = {"tokens": T, "tokens_per_s": round(ws * T / (ms * 1e-3), 1), "ms_per_step": round(ms, 5),
              "unique_experts": round(statistics.mean(ub), 2), "layer_gbs": round(gbs, 1),
              "layer_frac": round(gbs / peaks["hbm"], 4), "kernel": kern,
              "kernel_ms": round(k_ms, 5) if k_ms else None,
              "kernel_gbs": round(k_bytes / (k_ms * 1e-3) / 1e9, 1) if (k_ms and k_bytes) else None}
        if pt["kernel_gbs"]:
            pt["kernel_frac"] = round(pt["kernel_gbs"] / peaks["hbm"], 4)
        out["points"].append(pt)
    if rank == 0 and ws == 1 and not args.no_cpu:
        r = _cpu_sample(spec, L.layers[0], xs[0][:1], min(args.cpu_budget, 10.0))
        out["cpu_baseline"] = {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                               "sample": f"{r['steps']} single-token forwards of layer copy 0 (median)"}
    del L
    return out


def section_prefill(name, spec, T, args, pg, dev, rank, ws, peaks):
    """Tensor-bound prefill on the grouped-GEMM path."""
    from expertflow_b200 import _lib

    L = _EpLayers(spec, dev, rank, ws, min_bytes=1.0) if ws > 1 else _Layers(spec, dev, rank, path=_lib.EF_PATH_GEMM,
                                                                              min_bytes=1.0)
    steps = max(3, min(args.steps, 10))
    ms, ub, recs, xs = _time_layers(L, T, steps, args.warmup, pg, dev, trace=True)
    by = _by_kernel(recs)
    n_traced = min(steps, 2 * L.n)
    # per step: every launch of the kernel (routed and, expert-parallel, the
    # separate shared-expert launch) against all rows of the step
    rows = T * (spec.top_k + spec.n_shared)
    fl = {"qgemm_gate_up": 4.0 * spec.hidden * spec.inter * rows, "qgemm_down": 2.0 * spec.hidden * spec.inter * rows}
    kern = {}
    for k, f in fl.items():
        if k in by:
            t = sum(by[k]) / n_traced
            tf = f / (t * 1e-3) / 1e12
            kern[k] = {"ms": round(t, 4), "launches_per_step": len(by[k]) // n_traced, "tflops": round(tf, 1),
                       "frac_sustained": round(tf / peaks["bf16_sustained"], 4), "frac_burst": round(tf / peaks["bf16"], 4)}
    gemm_ms = sum(sum(by[k]) / n_traced for k in fl if k in by)
    gemm_tf = sum(fl.values()) / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    routed_tflop = 6.0 * spec.hidden * spec.inter * T * spec.top_k / 1e12
    out = {"workload": name, "bound": "tensor", "tokens": T, "tokens_per_s": round(ws * T / (ms * 1e-3), 1),
           "parallelism": f"ep{ws} (experts sharded, NCCL all-to-all)" if ws > 1 else "single",
           "ms_per_step": round(ms, 4), "steps": steps, "unique_experts": round(statistics.mean(ub), 2),
           "routed_tflop": round(routed_tflop, 4),
           "shared_tflop": round(6.0 * spec.hidden * spec.inter * T * spec.n_shared / 1e12, 4),
           "layer_tflops": round((routed_tflop + 6.0 * spec.hidden * spec.inter * T * spec.n_shared / 1e12) / (ms * 1e-3), 1),
           "gemm": kern, "gemm_tflops": round(gemm_tf, 1) if gemm_tf else None,
           "gemm_frac_sustained": round(gemm_tf / peaks["bf16_sustained"], 4) if gemm_tf else None,
           "peak_sustained": peaks["bf16_sustained"], "peak_burst": peaks["bf16"],
           "kernel_shares": {k: round(sum(v) / max(1e-9, sum(sum(x) for x in by.values())), 4) for k, v in by.items()},
           "l2": f"rotating {L.n} layer copies of {L.layer_bytes / 1e9:.2f} GB"}
    if rank == 0 and ws == 1 and not args.no_cpu:
        r = _cpu_sample(spec, L.layers[0], xs[0][:4], min(args.cpu_budget, 10.0))
        out["cpu_baseline"] = {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                               "sample": f"{r['steps']} 4-token forwards of layer copy 0 (median)"}
    del L
    return out


def section_stream(name, spec, args, dev):
    """48 stacked layers, experts streamed from pinned host memory into HBM
    slots (25% per layer) without lookahead and with one- and two-layer
    lookahead; single-token decode."""
    import numpy as np
    import torch
    from expertflow_b200 import moe, synthetic, pool as P

    NL, steps, budget = args.stream_layers, args.stream_steps, spec.n_experts // 4
    host = P.make_host_layers(spec, NL, seed=3000, device=dev)
    bias = torch.from_numpy(P.zipf_layer_bias(NL, spec.n_experts, 1.1, seed=42)).to(dev)
    gates = []
    for layer in range(NL):
        g = torch.Generator(device=dev)
        g.manual_seed(77 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * spec.gate_std).to(torch.float16)
        gates.append(moe.MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
    xs = [synthetic.make_x_torch(spec, 1, seed=5000 + t, device=dev) for t in range(steps)]

    def run(pl, lookahead, n):
        """n decode steps through all layers, in the library (ef_pool_decode_step)."""
        rs = [xs[t % steps].float().contiguous() for t in range(n)]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for t in range(n):
            pl.decode_step(rs[t], gates, lookahead=lookahead)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)

    res = P.ExpertSlotPool(spec, host, budget=spec.n_experts, headroom=spec.top_k)
    run(res, 0, steps)  # every expert the run touches becomes resident
    res.reset_stats()
    ms_res = run(res, 0, steps)
    st_res = res.stats()
    res.close()
    del res
    torch.cuda.empty_cache()
    out = {"workload": name, "layers": NL, "steps": steps, "slots_per_layer": budget + spec.top_k,
           "slots_note": f"the policy keeps {budget} of {spec.n_experts} experts per layer (25 %) across tokens; "
                         f"{spec.top_k} more slots hold one token's misses until the per-token trim, as the "
                         f"reference trims once per token",
           "loop": "ef_pool_decode_step (per layer: residual add + RMS norm, routed MoE on HBM slots)",
           "budget_per_layer": budget, "policy": "FrequencyWeightedCache (decay 0.95)",
           "resident_tokens_per_s": round(steps / (ms_res * 1e-3), 2),
           "resident_host_route_wait_ms_per_token": round(st_res["route_wait_ms"] / steps, 4),
           "resident_host_other_ms_per_token": round(st_res["host_ms"] / steps, 4)}
    for la in (0, 1, 2):
        pl = P.ExpertSlotPool(spec, host, budget=budget, headroom=spec.top_k)
        run(pl, la, min(16, steps))
        pl.reset_stats()
        ms = run(pl, la, steps)
        st = pl.stats()
        pl.close()
        exposed = max(0.0, ms - ms_res)
        d = {"tokens_per_s": round(steps / (ms * 1e-3), 2), "ms_per_token": round(ms / steps, 4),
             "hit_rate": round(st["hit_rate"], 4), "copy_free_rate": round(st["copy_free_rate"], 4),
             "h2d_bytes_per_token": round(st["h2d_bytes"] / steps), "copy_ms": round(st["copy_ms"], 1),
             "copy_gbs": round(st["h2d_bytes"] / max(st["copy_ms"], 1e-9) / 1e6, 1),
             "exposed_copy_ms": round(exposed, 1),
             "h2d_overlap": round(1.0 - exposed / st["copy_ms"], 4) if st["copy_ms"] > 0 else None,
             "copies_prefetch": st["copies_prefetch"], "prefetch_used": st["prefetch_used"],
             "copies_sync": st["copies_sync"],
             "stall_on_copies_ms_per_token": round(st["copy_wait_ms"] / steps, 4),
             "copy_hidden_frac_device": round(1.0 - st["copy_wait_ms"] / st["copy_ms"], 4) if st["copy_ms"] > 0 else None,
             "host_route_wait_ms_per_token": round(st["route_wait_ms"] / steps, 4),
             "host_other_ms_per_token": round(st["host_ms"] / steps, 4)}
        out[("no_lookahead", "lookahead", "lookahead2")[la]] = d
    if args.stream_files != "off":
        out["files"] = stream_from_files(spec, host, gates, run, steps, budget, ms_res, args)
    del host
    return out


def stream_from_files(spec, host, gates, run, steps, budget, ms_res, args):
    """The same decode with the experts in safetensors files on local disk
    (one shard per 8 layers, mlx_lm tensor names) under a pinned host tier of
    `--stream-host-frac` of all experts: misses in HBM and the host tier are
    read from the files by the library's reader threads (O_DIRECT unless the
    file system refuses it)."""
    import shutil
    import tempfile

    import numpy as np
    from expertflow_b200 import _lib as L, pool as P, weights as W

    NL, E = len(host), spec.n_experts
    need = NL * E * spec.expert_bytes()
    base = args.stream_dir or tempfile.gettempdir()
    free = shutil.disk_usage(base).free
    if free < 2 * need:
        return {"skipped": f"{free / 1e9:.1f} GB free under {base}, the model needs {need / 1e9:.1f} GB"}
    root = tempfile.mkdtemp(prefix="ef_stream_", dir=args.stream_dir or None)
    try:
        t0 = time.perf_counter()
        wm, per = {}, 8
        for k in range(0, NL, per):
            fn = f"model-{k // per + 1:05d}-of-{(NL + per - 1) // per:05d}.safetensors"
            t = {}
            for layer in range(k, min(NL, k + per)):
                for m, pn in zip(("gate", "up", "down"), ("gate_proj", "up_proj", "down_proj")):
                    w, sc, b = (a.numpy() for a in host[layer][m])
                    pre = f"model.layers.{layer}.mlp.switch_mlp.{pn}"
                    t[f"{pre}.weight"] = (w.view(np.uint32), "U32")
                    t[f"{pre}.scales"] = (sc, "F16")
                    t[f"{pre}.biases"] = (b, "F16")
            W.write_safetensors(os.path.join(root, fn), t)
            wm.update({n: fn for n in t})
        with open(os.path.join(root, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wm}, f)
        write_s = time.perf_counter() - t0
        direct = args.stream_files == "direct"
        try:
            store = P.ExpertStore.from_safetensors(root, spec=spec, direct=direct)
        except L.EfmoeError as ex:
            if not direct or ex.status != -9:
                raise
            direct = False
            store = P.ExpertStore.from_safetensors(root, spec=spec)
        host_blobs = max(2 * spec.top_k, int(args.stream_host_frac * NL * E))
        pl = P.ExpertSlotPool.from_store(store, budget=budget, host_blobs=host_blobs, headroom=spec.top_k)
        run(pl, 2, min(16, steps))  # file reads and copies two layers ahead
        pl.reset_stats()
        f0 = store.info()["file_bytes"]
        ms = run(pl, 2, steps)
        st = pl.stats()
        fb = store.info()["file_bytes"] - f0
        info = store.info()
        pl.close()
        store.close()
        asked = st["host_hits"] + st["host_reads"]
        return {"tokens_per_s": round(steps / (ms * 1e-3), 2), "ms_per_token": round(ms / steps, 4),
                "lookahead_layers": 2, "direct_io": bool(info["direct"]), "readers": info["n_readers"],
                "host_blobs": host_blobs, "host_frac": args.stream_host_frac,
                "model_bytes_on_disk": int(sum(os.path.getsize(os.path.join(root, n)) for n in os.listdir(root))),
                "write_s": round(write_s, 1),
                "hit_rate": round(st["hit_rate"], 4),
                "host_hit_rate": round(st["host_hits"] / asked, 4) if asked else None,
                "host_reads_per_token": round(st["host_reads"] / steps, 3),
                "host_reads_ahead": st["host_reads_ahead"],
                "file_bytes_per_token": round(fb / steps),
                "file_gbs": round(fb / (ms * 1e-3) / 1e9, 2),
                "read_wait_ms_per_token": round(st["read_wait_ms"] / steps, 4),
                "exposed_vs_resident_ms_per_token": round(max(0.0, ms - ms_res) / steps, 4)}
    finally:
        shutil.rmtree(root, ignore_errors=True)


def section_kquant(args, dev, peaks):
    """GGUF K-quant decode GEMV (ef_kquant_matmul) on a stack of 32
    DeepSeek-V3 gate projections (N = 32 x 2048 rows, K = 7168) per format:
    weights larger than L2, CUDA events around each launch.  Algorithmic bytes
    per launch = the blocks (N x K/256 x block bytes) + x + y."""
    import numpy as np
    import torch
    from expertflow_b200 import gguf as G, kquant as KQ

    N, K = 32 * 2048, 7168
    out = {"workload": "deepseek-v3 gate_proj x32 stacked, GGUF K-quant rows", "N": N, "K": K, "bound": "hbm",
           "points": []}
    for dtype, name in ((G.GGML_TYPE_Q2_K, "Q2_K"), (G.GGML_TYPE_Q3_K, "Q3_K"), (G.GGML_TYPE_Q4_K, "Q4_K")):
        bb = G.GGML_BLOCK_SIZES[dtype][1]
        nbytes = N * (K // 256) * bb
        w = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev)
        # fp16 super-block scales of the usual magnitude at the format's offsets
        wb = w.view(-1, bb)
        d = (torch.randn(wb.shape[0], device=dev).abs() * 0.01).to(torch.float16).view(torch.uint8).view(-1, 2)
        offs = {G.GGML_TYPE_Q2_K: (80, 82), G.GGML_TYPE_Q3_K: (108,), G.GGML_TYPE_Q4_K: (0, 2)}[dtype]
        for o in offs:
            wb[:, o:o + 2] = d
        for T in (1, 8, 32):
            x = torch.randn((T, K), device=dev).to(torch.bfloat16)
            for _ in range(max(3, args.warmup)):
                KQ.matmul(x, w, dtype, N, K)
            torch.cuda.synchronize()
            reps = max(10, args.steps)
            st = torch.cuda.current_stream()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for a, b in evs:
                a.record(st)
                KQ.matmul(x, w, dtype, N, K)
                b.record(st)
            torch.cuda.synchronize()
            ms = statistics.median(a.elapsed_time(b) for a, b in evs)
            alg = nbytes + T * K * 2 + T * N * 4
            gbs = alg / (ms * 1e-3) / 1e9
            out["points"].append({"format": name, "tokens": T, "us_per_launch": round(ms * 1e3, 2),
                                  "weight_bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm"], 4),
                                  "bits_per_weight": round(8 * bb / 256, 3)})
        del w, wb
        torch.cuda.empty_cache()
    out["moe"] = section_kquant_moe(args, dev, peaks)
    return out


def section_kquant_moe(args, dev, peaks):
    """The whole DeepSeek-V3-shaped MoE layer over GGUF K-quant experts
    (ef_kquant_moe_forward): 256 experts + shared, Q2_K gate/up and Q3_K down
    (a common mix in the reference's DeepSeek GGUF models), seeded blocks.
    Layer tokens/s (CUDA events around each forward) and the gate/up kernel's
    GB/s over the blocks of the distinct experts it ran."""
    import torch
    from expertflow_b200 import gguf as G, kquant as KQ, moe, synthetic, _lib
    from expertflow_b200.spec import DEEPSEEK_V3

    spec = DEEPSEEK_V3
    E, H, I = spec.n_experts, spec.hidden, spec.inter
    tg, td = G.GGML_TYPE_Q2_K, G.GGML_TYPE_Q3_K
    g = torch.Generator(device=dev)
    g.manual_seed(11)

    def proj(t, rows, cols, n, d_scale):
        bb = G.GGML_BLOCK_SIZES[t][1]
        raw = torch.randint(0, 256, (n * rows * (cols // 256), bb), dtype=torch.uint8, device=dev, generator=g)
        d = (torch.randn(raw.shape[0], device=dev, generator=g).abs() * d_scale).to(torch.float16)
        off = {G.GGML_TYPE_Q2_K: (80, 82), G.GGML_TYPE_Q3_K: (108,)}[t]
        for o in off:
            raw[:, o:o + 2] = d.view(torch.uint8).view(-1, 2)
        return KQ.KQuantProj(raw.reshape(-1), t, rows, cols, n)

    sc = {tg: 0.002, td: 0.0006}
    gate_w = (torch.randn((E, H), device=dev, generator=g) * spec.gate_std).to(torch.float16)
    e_bias = (torch.randn(E, device=dev, generator=g) * 0.01).float()
    gate = moe.MoEGate(gate_w, spec.top_k, spec.router, spec.norm_topk, spec.n_group, spec.topk_group,
                       spec.routed_scaling, e_bias)
    m = KQ.KQuantMoELayer(gate, proj(tg, I, H, E, sc[tg]), proj(tg, I, H, E, sc[tg]), proj(td, H, I, E, sc[td]),
                          shared=(proj(tg, I, H, 1, sc[tg]), proj(tg, I, H, 1, sc[tg]), proj(td, H, I, 1, sc[td])))
    gu_bytes = 2 * I * (H // 256) * G.GGML_BLOCK_SIZES[tg][1]
    out = {"workload": "deepseek-v3 layer over GGUF K-quant experts (Q2_K gate/up, Q3_K down), 256 experts + "
                       "shared", "layer_bytes": int(m.gate_proj.blocks.numel() * 2 + m.down_proj.blocks.numel()),
           "points": []}
    for T in (1, 8, 32):
        # eight batches in rotation route to different experts, so a forward
        # does not find the previous one's weights in L2
        xs = [synthetic.make_x_torch(spec, T, seed=5 + i, device=dev) for i in range(8)]
        x = xs[0]
        inds = torch.empty((T, spec.top_k), dtype=torch.int32, device=dev)
        m(x, inds_out=inds)
        n_u = int(torch.unique(inds).numel())
        for i in range(max(3, args.warmup)):
            m(xs[i % 8])
        torch.cuda.synchronize()
        reps = max(16, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            m(xs[i % 8])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        m(xs[1])
        _lib.trace_enable(True)
        _lib.trace_read()
        m(x)
        torch.cuda.synchronize()
        by = _by_kernel(_lib.trace_read())
        _lib.trace_enable(False)
        k_ms = by["kq_gate_up"][0]
        gbs = (n_u + 1) * gu_bytes / (k_ms * 1e-3) / 1e9
        out["points"].append({"tokens": T, "tokens_per_s": round(T / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
                              "unique_experts": n_u, "kq_gate_up_ms": round(k_ms, 4),
                              "kq_gate_up_gbs": round(gbs, 1), "kq_gate_up_frac": round(gbs / peaks["hbm"], 4),
                              "kernel_ms": {k: round(v[0], 4) for k, v in by.items()}})
    del m
    torch.cuda.empty_cache()
    return out


class _PeerEpLayers:
    """Expert-parallel copies of one layer over the peer-memory exchange
    (ef_ep_forward): this rank holds experts [rank * E/P, (rank + 1) * E/P)
    of each copy, the gate and shared expert replicated.  Copies are rotated
    per step so that every step reads weights that are not in L2."""

    def __init__(self, spec, dev, rank, ws, max_tokens, path=None, min_bytes=1.5e9, seed0=1000, keep_full=False):
        import torch
        from expertflow_b200 import moe, synthetic, _lib
        from expertflow_b200.ep import PeerExpertParallelMoE, shard_layer

        self.spec = spec
        self.layer_bytes = spec.n_experts // ws * spec.expert_bytes()
        self.n = max(2, math.ceil(min_bytes / self.layer_bytes))
        p = _lib.EF_PATH_AUTO if path is None else path
        self.layers, self.full = [], None
        for i in range(self.n):
            full = synthetic.make_layer_torch(spec, seed=seed0 + i, device=dev)
            ops = shard_layer(spec, full, rank, ws, device=dev)
            if keep_full and i == 0:  # copy 0 also as a whole single-GPU layer (parity and the 1-GPU number)
                self.full = moe.MoELayer.from_arrays(spec, full, device=dev, path=p)
            del full
            torch.cuda.empty_cache()
            self.layers.append(PeerExpertParallelMoE(spec, ops, max_tokens=max_tokens, path=p))

    def close(self):
        for m in self.layers:
            m.close()


def _time_ep(L, T, steps, warmup, pg, dev, x_seed, rank, graphs=True, trace=False, hold=0.0):
    """CUDA-event time per step (max over ranks) of T tokens per rank through
    the rotated expert-parallel copies; with trace, the per-launch times of a
    separate eager pass (kernel name -> mean ms, max over ranks)."""
    import torch
    from expertflow_b200 import synthetic, _lib

    spec = L.spec
    xs = [synthetic.make_x_torch(spec, T, seed=x_seed + 97 * rank + i, device=dev) for i in range(L.n)]
    if graphs:
        cfs = [m.capture(T) for m in L.layers]
        for cf, x in zip(cfs, xs):
            cf.x.copy_(x)
        fwd = [cf.graph.replay for cf in cfs]
    else:
        cfs = None
        fwd = [(lambda m=m, x=x: m(x)) for m, x in zip(L.layers, xs)]
    for s in range(warmup):
        fwd[s % L.n]()
    torch.cuda.synchronize()
    pg.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in range(steps):
        fwd[s % L.n]()
    e1.record(st)
    if hold > 0:
        # every rank replays the same number of extra forwards (the exchange pairs them up)
        e1.synchronize()
        per = torch.tensor([max(e0.elapsed_time(e1) / max(steps, 1), 1e-3)], device=dev)
        pg.all_reduce(per, op=pg.ReduceOp.MAX)
        for s in range(int(min(20000, hold * 1e3 / float(per.item())))):
            fwd[s % L.n]()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms = float(t.item())
    phases = {}
    if trace:
        n_tr = 2 * L.n
        _lib.trace_enable(True)
        _lib.trace_read()
        for s in range(n_tr):
            L.layers[s % L.n](xs[s % L.n])
        torch.cuda.synchronize()
        recs = _lib.trace_read()
        _lib.trace_enable(False)
        by = _by_kernel(recs)
        names = sorted(by)
        # every rank launches the same kernel sequence: reduce per name
        v = torch.tensor([sum(by[k]) / n_tr for k in names], device=dev, dtype=torch.float64)
        pg.all_reduce(v, op=pg.ReduceOp.MAX)
        phases = {k: round(float(x), 5) for k, x in zip(names, v.tolist())}
        phases["_launches_per_step"] = len(recs) // n_tr
    del cfs
    return ms, phases, xs


def bench_ep(args, pg, dev, rank, ws, local, peaks):
    """N > 1: the DeepSeek-V3-shaped layer with its experts sharded across the
    ranks (E/N per GPU), exchanged over NVLink peer memory by the library's
    kernels.  Headline: strong scaling, a fixed global batch split evenly over
    the ranks; alongside: weak scaling, the same-run single-GPU layer on the
    same global batch, per-phase kernel times, the EP output checked bit for
    bit against the single-GPU layer, and the NCCL all-to-all version."""
    import torch
    from expertflow_b200 import synthetic, _lib
    from expertflow_b200.ep import ExpertParallelMoE, shard_layer
    from expertflow_b200.spec import WORKLOADS

    name = "deepseek-v3-moe"
    spec = WORKLOADS[name]
    Tg = args.ep_tokens
    if Tg % ws:
        raise SystemExit(f"--ep-tokens {Tg} must be a multiple of the GPU count {ws}")
    Tl, Tw = Tg // ws, args.ep_weak_tokens
    L = _PeerEpLayers(spec, dev, rank, ws, max_tokens=max(Tl, Tw), keep_full=True)

    # parity: every rank's EP output equals the single-GPU layer on its tokens
    x0 = synthetic.make_x_torch(spec, Tl, seed=11 + rank, device=dev)
    inds = torch.empty((Tl, spec.top_k), dtype=torch.int32, device=dev)
    y_ep = L.layers[0](x0, inds_out=inds, out_dtype=torch.float32)
    y_1 = L.full(x0, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ok = torch.tensor([int(torch.equal(y_ep, y_1))], device=dev)
    pg.all_reduce(ok, op=pg.ReduceOp.MIN)
    ep_parity = bool(ok.item())
    # distinct local experts this rank runs per step (every rank's routing)
    allinds = [torch.empty_like(inds) for _ in range(ws)]
    pg.all_gather(allinds, inds)
    el = spec.n_experts // ws
    ai = torch.cat(allinds).reshape(-1)
    n_local = int(torch.unique(ai[(ai >= rank * el) & (ai < (rank + 1) * el)]).numel())

    with ClockSampler(local) as clk:
        ms, _, _ = _time_ep(L, Tl, args.steps, args.warmup, pg, dev, 7, rank, hold=0.3)
    clocks = clk.summary()
    value = Tg / (ms * 1e-3)
    _, phases, _ = _time_ep(L, Tl, 2, 1, pg, dev, 7, rank, graphs=False, trace=True)
    ms_w, phases_w, _ = _time_ep(L, Tw, max(5, args.steps // 2), args.warmup, pg, dev, 31, rank, trace=True)

    # the single-GPU layer on the same global batch (each rank its own, concurrently; max over ranks)
    xg = synthetic.make_x_torch(spec, Tg, seed=5, device=dev)
    cf1 = L.full.capture(Tg)
    cf1.x.copy_(xg)
    for _ in range(args.warmup):
        cf1.graph.replay()
    torch.cuda.synchronize()
    pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n1 = max(5, args.steps // 2)
    e0.record()
    for _ in range(n1):
        cf1.graph.replay()  # one layer copy: its weights (6.3 GB) are far larger than L2
    e1.record()
    torch.cuda.synchronize()
    t1 = torch.tensor([e0.elapsed_time(e1) / n1], device=dev)
    pg.all_reduce(t1, op=pg.ReduceOp.MAX)
    ms1 = float(t1.item())
    del cf1
    single = Tg / (ms1 * 1e-3)

    # roofline of the dominant kernel on this rank (algorithmic bytes of the
    # distinct local experts it ran, + the shared expert)
    kern = max((k for k in phases if not k.startswith("_")), key=lambda k: phases[k])
    per_e = spec.expert_bytes()
    k_bytes = {"qmv_gate_up": (n_local + 1) * per_e * 2 // 3, "qmv_down": (n_local + 1) * (per_e - per_e * 2 // 3)}
    kb = k_bytes.get(kern)
    achieved = kb / (phases[kern] * 1e-3) / 1e9 if kb else None

    # e2e: pinned host tokens -> captured EP forward -> pinned host output, copies in the timed region
    cfs = [m.capture(Tl) for m in L.layers]
    xh = [synthetic.make_x_torch(spec, Tl, seed=7 + 97 * rank + i, device=dev).cpu().pin_memory() for i in range(L.n)]
    yh = [torch.empty((Tl, spec.hidden), dtype=xh[0].dtype).pin_memory() for _ in range(L.n)]
    st = torch.cuda.current_stream()

    def serve(n):
        for s in range(n):
            i = s % L.n
            cfs[i].x.copy_(xh[i], non_blocking=True)
            cfs[i].graph.replay()
            yh[i].copy_(cfs[i].y, non_blocking=True)

    serve(args.warmup)
    torch.cuda.synchronize()
    pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    serve(args.steps)
    e1.record(st)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    pg.all_reduce(te, op=pg.ReduceOp.MAX)
    e2e_ms = float(te.item())
    del cfs

    # the same split exchanged with NCCL all-to-alls issued by the host (the baseline this path replaces)
    nccl = None
    if not args.no_nccl_baseline:
        full0 = synthetic.make_layer_torch(spec, seed=1000, device=dev)
        ops = shard_layer(spec, full0, rank, ws, device=dev)
        del full0
        torch.cuda.empty_cache()
        m = ExpertParallelMoE(spec, ops)
        for _ in range(2):
            m(x0)
        torch.cuda.synchronize()
        pg.barrier()
        e0.record()
        nn = 10
        for _ in range(nn):
            m(x0)
        e1.record()
        torch.cuda.synchronize()
        tn = torch.tensor([e0.elapsed_time(e1) / nn], device=dev)
        pg.all_reduce(tn, op=pg.ReduceOp.MAX)
        nccl = {"ms_per_step": round(float(tn.item()), 4), "tokens_per_s": round(Tg / (float(tn.item()) * 1e-3), 1),
                "what": "ExpertParallelMoE: host-issued NCCL all-to-alls of counts, rows, ids and fp32 outputs"}
        del m, ops
        torch.cuda.empty_cache()
    n_copies, layer_bytes = L.n, L.layer_bytes
    L.close()
    del L
    torch.cuda.empty_cache()
    return {
        "spec": spec, "value": value, "ms": ms, "clocks": clocks, "phases": phases, "Tg": Tg, "Tl": Tl, "Tw": Tw,
        "weak": {"tokens_per_rank": Tw, "tokens_per_s": round(ws * Tw / (ms_w * 1e-3), 1),
                 "ms_per_step": round(ms_w, 5), "phases_ms": phases_w},
        "single": {"tokens": Tg, "tokens_per_s": round(single, 1), "ms_per_step": round(ms1, 5),
                   "what": "the whole layer on one GPU (same run, CUDA graph)"},
        "ep_parity": ep_parity, "kern": kern, "k_ms": phases[kern], "k_bytes": kb, "achieved": achieved,
        "n_local": n_local, "e2e_ms": e2e_ms, "nccl": nccl, "n_copies": n_copies, "layer_bytes": layer_bytes,
    }


def section_prefill_ep(name, spec, Tg, args, pg, dev, rank, ws, peaks):
    """c4 at N > 1: the 8-bit DeepSeek-V3 prefill batch split over the ranks,
    experts sharded, exchanged over peer memory, grouped GEMM; the same-run
    single-GPU layer on the whole batch beside it."""
    import torch
    from expertflow_b200 import synthetic, _lib

    Tl = Tg // ws
    L = _PeerEpLayers(spec, dev, rank, ws, max_tokens=Tl, path=_lib.EF_PATH_GEMM, min_bytes=1.0, keep_full=True)
    steps = max(3, min(args.steps, 10))
    ms, phases, _ = _time_ep(L, Tl, steps, args.warmup, pg, dev, 51, rank, trace=True)
    x0 = synthetic.make_x_torch(spec, Tl, seed=13 + rank, device=dev)
    ok = torch.tensor([int(torch.equal(L.layers[0](x0, out_dtype=torch.float32),
                                       L.full(x0, out_dtype=torch.float32)))], device=dev)
    pg.all_reduce(ok, op=pg.ReduceOp.MIN)
    xg = synthetic.make_x_torch(spec, Tg, seed=5, device=dev)
    for _ in range(2):
        L.full(xg)
    torch.cuda.synchronize()
    pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        L.full(xg)
    e1.record()
    torch.cuda.synchronize()
    t1 = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    pg.all_reduce(t1, op=pg.ReduceOp.MAX)
    ms1 = float(t1.item())
    rows = Tg * (spec.top_k + spec.n_shared)  # whole box, per step
    gemm_ms = sum(v for k, v in phases.items() if k.startswith("qgemm"))
    # every rank runs about 1/ws of the rows: box TFLOP/s over the max-over-ranks kernel time
    gemm_tf = 6.0 * spec.hidden * spec.inter * rows / ws / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    out = {"workload": name, "tokens_global": Tg, "tokens_per_rank": Tl, "tokens_per_s": round(Tg / (ms * 1e-3), 1),
           "ms_per_step": round(ms, 4), "single_gpu_tokens_per_s": round(Tg / (ms1 * 1e-3), 1),
           "single_gpu_ms_per_step": round(ms1, 4), "box_speedup": round(ms1 / ms, 3),
           "ep_parity": bool(ok.item()), "phases_ms": phases,
           "gemm_tflops_per_gpu": round(gemm_tf, 1) if gemm_tf else None,
           "gemm_frac_sustained": round(gemm_tf / peaks["bf16_sustained"], 4) if gemm_tf else None,
           "parallelism": f"ep{ws} (experts sharded, peer-memory exchange over NVLink)"}
    L.close()
    del L
    torch.cuda.empty_cache()
    return out


def _ep_line(r, args, ws, peaks, sections):
    spec = r["spec"]
    hbm = peaks["hbm"]
    return {
        "metric": METRIC, "value": round(r["value"], 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(r["ms"], 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u4 codes x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; random-init weights of the named shape)",
        "config": {"workload": "deepseek-v3-moe", "tokens_global": r["Tg"], "tokens_per_rank": r["Tl"],
                   "hidden": spec.hidden, "experts": spec.n_experts, "experts_per_gpu": spec.n_experts // ws,
                   "top_k": spec.top_k, "inter": spec.inter, "bits": spec.bits, "shared_experts": spec.n_shared,
                   "parallelism": f"ep{ws} (experts sharded, peer-memory exchange over NVLink, no host sync)",
                   "launch": "CUDA graph per layer copy (PeerExpertParallelMoE.capture)",
                   "layer_copies": r["n_copies"],
                   "l2": f"rotating {r['n_copies']} shard copies of {r['layer_bytes'] / 1e6:.0f} MB per GPU"},
        "box_speedup": round(r["value"] / r["single"]["tokens_per_s"], 3),
        "single_gpu": r["single"],
        "weak": r["weak"],
        "ep_parity": r["ep_parity"],
        "nccl_alltoall": r["nccl"],
        "phases_ms": r["phases"],
        "roofline": {"kernel": r["kern"], "bound": "hbm",
                     "achieved": round(r["achieved"], 1) if r["achieved"] else None, "peak": hbm, "unit": "GB/s",
                     "frac": round(r["achieved"] / hbm, 4) if r["achieved"] else None, "traffic": None,
                     "peak_kind": peaks["kind"], "kernel_ms": r["k_ms"], "algorithmic_bytes": r["k_bytes"],
                     "local_experts_run": r["n_local"],
                     "timing": "CUDA events around each launch, eager traced pass, max over ranks"},
        "cpu_baseline": None,
        "e2e": {"value": round(r["Tg"] / (r["e2e_ms"] * 1e-3), 1), "unit": UNIT, "ms_per_step": round(r["e2e_ms"], 5),
                "h2d_bytes_per_step": r["Tg"] * spec.hidden * 2, "d2h_bytes_per_step": r["Tg"] * spec.hidden * 2,
                "api": "PeerExpertParallelMoE.capture (C ABI ef_ep_forward in a CUDA graph); pinned host tokens "
                       "copied in and the output read back on every rank every step"},
        "gpu_launches": r["phases"].get("_launches_per_step", 0) * args.steps,
        "clocks": r["clocks"],
        "workloads": sections,
    }


def _summary(line, sections):
    """The per-workload figures in a few keys, printed last in the line so
    that a tail of the output keeps them."""
    out = {"headline": {"workload": line["config"]["workload"], "tokens_per_s": line["value"],
                        "roofline_frac": (line.get("roofline") or {}).get("frac")}}
    if "box_speedup" in line:
        out["headline"]["box_speedup"] = line["box_speedup"]
        out["headline"]["ep_parity"] = line["ep_parity"]
    c2 = sections.get("c2")
    if c2:
        out["c2"] = {f"T{p['tokens']}": {"tok_s": p["tokens_per_s"], "kernel_frac": p.get("kernel_frac")}
                     for p in c2["points"]}
    c4 = sections.get("c4")
    if c4:
        if "gemm" in c4:
            g = c4["gemm"].get("qgemm_gate_up", {})
            out["c4"] = {"tok_s": c4["tokens_per_s"], "gemm_tflops": c4.get("gemm_tflops"),
                         "gate_up_frac_burst": g.get("frac_burst"), "gate_up_frac_sustained": g.get("frac_sustained"),
                         "frac_sustained": c4.get("gemm_frac_sustained")}
        else:
            out["c4"] = {"tok_s": c4["tokens_per_s"], "box_speedup": c4["box_speedup"],
                         "ep_parity": c4["ep_parity"], "gemm_frac_sustained": c4["gemm_frac_sustained"]}
    c3 = sections.get("c3")
    if c3:
        la = c3.get("lookahead", {})
        la2 = c3.get("lookahead2", {})
        out["c3"] = {"tok_s": la2.get("tokens_per_s"), "lookahead_layers": 2, "h2d_overlap": la2.get("h2d_overlap"),
                     "copy_hidden_frac_device": la2.get("copy_hidden_frac_device"),
                     "tok_s_lookahead1": la.get("tokens_per_s"), "resident_tok_s": c3.get("resident_tokens_per_s")}
    kq = sections.get("kq")
    if kq:
        out["kq"] = {f"{p['format']}_T{p['tokens']}": p["frac"] for p in kq["points"] if p["tokens"] == 1}
        if kq.get("moe"):
            out["kq_moe"] = {f"T{p['tokens']}": {"tok_s": p["tokens_per_s"], "gate_up_frac": p["kq_gate_up_frac"]}
                             for p in kq["moe"]["points"]}
    return out


def bench_ours(args):
    import torch
    from expertflow_b200 import build, moe, synthetic, _lib
    from expertflow_b200.spec import WORKLOADS

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    build.build()
    spec = WORKLOADS[args.workload]
    peaks = _peaks()
    hbm_peak = peaks["hbm"]
    if ws > 1:
        r = bench_ep(args, pg, dev, rank, ws, local, peaks)
        sections = {}
        if "c4" in args.sections:
            sections["c4"] = section_prefill_ep("deepseek-v3-moe-8bit", WORKLOADS["deepseek-v3-moe-8bit"], 4096,
                                                args, pg, dev, rank, ws, peaks)
            torch.cuda.empty_cache()
        line = _ep_line(r, args, ws, peaks, sections)
        line["workloads_summary"] = _summary(line, sections)
        if rank == 0:
            print(json.dumps(line), flush=True)
        pg.barrier()
        pg.destroy_process_group()
        return 0

    # ---- headline: T tokens through the configured workload (decode, GEMV)
    L = _Layers(spec, dev, rank)
    T = args.tokens
    with ClockSampler(local) as clk:
        ms, ub, _, _ = _time_layers(L, T, args.steps, args.warmup, pg, dev, graphs=True, hold=0.3)
    clocks = clk.summary()
    ms_eager, _, _, _ = _time_layers(L, T, args.steps, args.warmup, pg, dev)
    ms_tr, ub_tr, recs, _ = _time_layers(L, T, args.steps, 1, pg, dev, trace=True)
    n_u = statistics.mean(ub)
    ab = algorithmic_bytes(spec, n_u, T)
    value = ws * T / (ms * 1e-3)

    # dominant kernel (live CUDA events on the launching stream, traced pass)
    by = _by_kernel(recs)
    kern = max(by, key=lambda k: sum(by[k])) if by else None
    k_ms = statistics.mean(by[kern]) if kern else None
    k_bytes = {"qmv_gate_up": ab["gate_up"], "qmv_down": ab["down"]}.get(kern)
    achieved = (k_bytes / (k_ms * 1e-3) / 1e9) if (k_ms and k_bytes) else None
    traffic = None
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            traffic = json.load(f).get(f"{kern}@{args.workload}/T{T}")
    except Exception:
        pass
    shares = {k: round(sum(v) / max(1e-9, sum(sum(x) for x in by.values())), 4) for k, v in by.items()}

    # ---- sweep (same run)
    sweep = []
    for t_s in args.sweep:
        m_s, u_s, _, _ = _time_layers(L, t_s, args.steps, args.warmup, pg, dev, graphs=True)
        ab_s = algorithmic_bytes(spec, statistics.mean(u_s), t_s)
        gbs = ab_s["total"] / (m_s * 1e-3) / 1e9
        sweep.append({"tokens": t_s, "tokens_per_s": round(ws * t_s / (m_s * 1e-3), 1), "ms_per_step": round(m_s, 4),
                      "unique_experts": round(statistics.mean(u_s), 2), "layer_gbs": round(gbs, 1),
                      "layer_frac": round(gbs / hbm_peak, 4)})

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region
    # the public API's captured forward (MoELayer.capture) as a serving loop
    # would drive it: every step copies its pinned input into the graph's input
    # buffer and reads its output back to pinned memory on a copy stream, so
    # the copies of neighbouring steps overlap the replays; each layer copy's
    # buffers are reused only after the replay that last used them
    xh = [synthetic.make_x_torch(spec, T, seed=7 + i, device=dev).cpu().pin_memory() for i in range(L.n)]
    yh = [torch.empty((T, spec.hidden), dtype=xh[0].dtype).pin_memory() for _ in range(L.n)]
    cfs = [m.capture(T, xh[0].dtype) for m in L.layers]
    st = torch.cuda.current_stream()
    cs = torch.cuda.Stream(dev)

    def serve(n_steps):
        done = [None] * L.n  # per layer copy: its last replay
        h2d = [None] * L.n
        read = [None] * L.n  # per layer copy: the D2H of its last output

        def put(s):
            i = s % L.n
            with torch.cuda.stream(cs):
                if done[i] is not None:
                    cs.wait_event(done[i])  # the replay reading this input buffer is over
                cfs[i].x.copy_(xh[i], non_blocking=True)
                h2d[i] = torch.cuda.Event()
                h2d[i].record(cs)

        put(0)
        for s in range(n_steps):
            i = s % L.n
            if s + 1 < n_steps:
                put(s + 1)
            st.wait_event(h2d[i])
            if read[i] is not None:
                st.wait_event(read[i])  # the previous output of this copy has been read
            cfs[i].graph.replay()
            done[i] = torch.cuda.Event()
            done[i].record(st)
            with torch.cuda.stream(cs):
                cs.wait_event(done[i])
                yh[i].copy_(cfs[i].y, non_blocking=True)
                read[i] = torch.cuda.Event()
                read[i].record(cs)
        for ev in read:
            if ev is not None:
                st.wait_event(ev)

    serve(args.warmup)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    cs.wait_event(e0)
    serve(args.steps)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # ---- CPU baseline (rank 0, N = 1 only): the oracle on the same layer/batch
    cpu = None
    xs0 = synthetic.make_x_torch(spec, T, seed=7, device=dev)
    if rank == 0 and ws == 1 and not args.no_cpu:
        r = _cpu_sample(spec, L.layers[0], xs0, args.cpu_budget)
        cpu = {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
               "sample": f"{r['steps']} full {T}-token forwards of layer copy 0 (median), oracle/ef_oracle.c"}
    n_copies, layer_bytes = L.n, L.layer_bytes
    del L
    torch.cuda.empty_cache()

    # ---- the other workloads (each its own roofline)
    sections = {}
    want = set(args.sections)
    if "c2" in want:
        sections["c2"] = section_decode("deepseek-v3-moe", WORKLOADS["deepseek-v3-moe"], [1, 32, 256], args, pg, dev,
                                        rank, ws, peaks)
        torch.cuda.empty_cache()
    if "c4" in want:
        sections["c4"] = section_prefill("deepseek-v3-moe-8bit", WORKLOADS["deepseek-v3-moe-8bit"], 4096, args, pg,
                                         dev, rank, ws, peaks)
        torch.cuda.empty_cache()
    if "kq" in want and ws == 1:
        sections["kq"] = section_kquant(args, dev, peaks)
        torch.cuda.empty_cache()
    if "c3" in want and ws == 1:
        sections["c3"] = section_stream("qwen3-30b-a3b-moe x48 streamed", WORKLOADS["qwen3-30b-a3b-moe"], args, dev)
        torch.cuda.empty_cache()

    launches = len(recs) // max(1, min(args.steps, 2 * n_copies)) * args.steps if recs else 0
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 codes x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; random-init weights of the named shape)",
        "config": {"workload": args.workload, "tokens": T,
                   "hidden": spec.hidden, "experts": spec.n_experts, "top_k": spec.top_k, "inter": spec.inter,
                   "bits": spec.bits, "group": spec.group_size, "parallelism": "replicas" if ws > 1 else "single",
                   "launch": "CUDA graph per layer copy (MoELayer.capture)",
                   "layer_copies": n_copies, "l2": f"rotating {n_copies} layer copies of {layer_bytes/1e6:.0f} MB",
                   "unique_experts_per_step": round(n_u, 2)},
        "layer_gbs": round(ab["total"] / (ms * 1e-3) / 1e9, 1),
        "layer_frac": round(ab["total"] / (ms * 1e-3) / 1e9 / hbm_peak, 4),
        "roofline": {"kernel": kern, "bound": "hbm", "achieved": round(achieved, 1) if achieved else None,
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4) if achieved else None,
                     "traffic": traffic, "peak_kind": peaks["kind"], "kernel_ms": round(k_ms, 5) if k_ms else None,
                     "algorithmic_bytes": k_bytes, "timing": "CUDA events around each launch, traced pass",
                     "traced_ms_per_step": round(ms_tr, 5), "kernel_shares": shares},
        "cpu_baseline": cpu,
        "e2e": {"value": round(ws * T / (e2e_ms * 1e-3), 1), "unit": UNIT, "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": T * spec.hidden * 2, "d2h_bytes_per_step": T * spec.hidden * 2,
                "api": "MoELayer.capture (C ABI ef_moe_forward in a CUDA graph), pinned host x/y; each "
                       "step's H2D and D2H on a copy stream, overlapping neighbouring steps' replays"},
        "eager_ms_per_step": round(ms_eager, 5),
        "gpu_launches": launches,
        "sweep": sweep,
        "clocks": clocks,
        "workloads": sections,
    }
    line["workloads_summary"] = _summary(line, sections)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--sweep", type=int, nargs="*", default=[1, 8, 32, 64])
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sections", nargs="*", default=["c2", "c4", "c3", "kq"],
                    help="other workloads measured after the headline: c2 (DeepSeek-V3 decode), "
                         "c4 (DeepSeek-V3 8-bit prefill), c3 (48-layer streamed decode), "
                         "kq (GGUF K-quant decode GEMV)")
    ap.add_argument("--stream-layers", type=int, default=48)
    ap.add_argument("--stream-steps", type=int, default=512)
    ap.add_argument("--stream-files", default="direct", choices=["direct", "buffered", "off"],
                    help="c3 again with the experts in safetensors files under a bounded pinned host tier")
    ap.add_argument("--stream-host-frac", type=float, default=0.25)
    ap.add_argument("--stream-dir", default=None, help="where the c3 model files go (default: the temp dir)")
    ap.add_argument("--ep-tokens", type=int, default=256,
                    help="N > 1: global decode batch of the DeepSeek-V3 layer, split over the GPUs (strong scaling)")
    ap.add_argument("--ep-weak-tokens", type=int, default=256, help="N > 1: tokens per GPU of the weak-scaling run")
    ap.add_argument("--no-nccl-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    # stdout carries exactly one JSON line: NCCL's log lines (its version banner
    # included) go to stderr unless the caller chose a log file
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    if args.impl == "reference":
        return bench_reference(args)
    return bench_ours(args)


if __name__ == "__main__":
    sys.exit(main())
