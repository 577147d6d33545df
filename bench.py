"""MoE-layer benchmark: tokens/s and HBM GB/s (fraction of the measured roofline).

Default workload: one Qwen3-30B-A3B-shaped MoE layer (hidden 2048, 128 experts,
top-8 softmax, inter 768, 4-bit g64 affine weights, bf16 activations), a
decode batch of 64 tokens; the 1/8/32/64-token sweep is reported alongside.
A step is one MoE-layer forward (router, permute, gate/up+SwiGLU, down,
combine) over one batch with weights resident in HBM.  Several seeded layer
copies (each larger than L2) are rotated so every step reads cold weights.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--tokens T]

Multi-GPU (torchrun, one process per GPU): the decode layer does not shard,
so every rank runs an independent replica (no collective in the data path);
time is the max over ranks, value = all ranks' tokens / that time.
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
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


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
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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

    spec = WORKLOADS[args.workload]
    T = args.tokens
    budget = max(2.0, min(20.0, 2.0 * (args.steps + args.warmup)))
    r = run_cpu_reference(spec, T, budget)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["tokens_per_s"], 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": r["steps"], "warmup": 1, "ms_per_step": round(r["s_per_step"] * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4/u8 codes, f32 accumulate",
        "data": "synthetic (seeded)", "config": {"workload": args.workload, "tokens": T, "hidden": spec.hidden,
                                                 "experts": spec.n_experts, "top_k": spec.top_k,
                                                 "inter": spec.inter, "bits": spec.bits},
        "cpu_baseline": {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": f"{r['steps']} full {T}-token layer forwards (median), oracle/ef_oracle.c"},
        "e2e": {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_ours(args):
    import torch
    import numpy as np
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
    hbm_peak, tf_peak, peak_kind = _peaks()

    # rotate over layer copies so that the weights touched per step exceed L2
    layer_bytes = spec.n_experts * spec.expert_bytes()
    n_copies = max(2, math.ceil(1.5e9 / layer_bytes))
    layers = [moe.MoELayer.from_arrays(spec, synthetic.make_layer_torch(spec, seed=1000 * rank + i, device=dev),
                                       device=dev) for i in range(n_copies)]

    def measure(T, steps, warmup, trace=False):
        xs = [synthetic.make_x_torch(spec, T, seed=7 + i, device=dev) for i in range(n_copies)]
        # distinct experts per (copy, batch), counted from the routing indices
        uniq = []
        for i, m in enumerate(layers):
            inds = torch.empty((T, spec.top_k), dtype=torch.int32, device=dev)
            m(xs[i], inds_out=inds)
            uniq.append(int(torch.unique(inds).numel()))
        for s in range(warmup):
            layers[s % n_copies](xs[s % n_copies])
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if trace:
            _lib.trace_enable(True)
            _lib.trace_read()
        e0.record(st)
        for s in range(steps):
            layers[s % n_copies](xs[s % n_copies])
        e1.record(st)
        torch.cuda.synchronize()
        recs = []
        if trace:
            recs = _lib.trace_read()
            _lib.trace_enable(False)
        ms = e0.elapsed_time(e1) / steps
        if pg:
            t = torch.tensor([ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        ub = [uniq[s % n_copies] for s in range(steps)]
        return ms, ub, recs

    # ---- headline: T tokens
    T = args.tokens
    with ClockSampler(local) as clk:
        ms, ub, _ = measure(T, args.steps, args.warmup)
    clocks = clk.summary()
    ms_tr, ub_tr, recs = measure(T, args.steps, 1, trace=True)
    n_u = statistics.mean(ub)
    ab = algorithmic_bytes(spec, n_u, T)
    value = ws * T / (ms * 1e-3)

    # dominant kernel (live CUDA events on the launching stream, traced pass)
    by = {}
    for name, t in recs:
        by.setdefault(name, []).append(t)
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
        m_s, u_s, _ = measure(t_s, args.steps, args.warmup)
        ab_s = algorithmic_bytes(spec, statistics.mean(u_s), t_s)
        gbs = ab_s["total"] / (m_s * 1e-3) / 1e9
        sweep.append({"tokens": t_s, "tokens_per_s": round(ws * t_s / (m_s * 1e-3), 1), "ms_per_step": round(m_s, 4),
                      "unique_experts": round(statistics.mean(u_s), 2), "layer_gbs": round(gbs, 1),
                      "layer_frac": round(gbs / hbm_peak, 4)})

    # ---- e2e through the public API with host buffers (pinned), copies inside the timed region
    m0 = layers[0]
    xh = [synthetic.make_x_torch(spec, T, seed=7 + i, device=dev).cpu().pin_memory() for i in range(n_copies)]
    yh = torch.empty((T, spec.hidden), dtype=xh[0].dtype).pin_memory()
    st = torch.cuda.current_stream()
    for s in range(args.warmup):
        xd = xh[s % n_copies].to(dev, non_blocking=True)
        yh.copy_(moe.streaming_moe_forward(layers[s % n_copies], xd[None])[0], non_blocking=True)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in range(args.steps):
        xd = xh[s % n_copies].to(dev, non_blocking=True)
        yh.copy_(moe.streaming_moe_forward(layers[s % n_copies], xd[None])[0], non_blocking=True)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    del m0

    # ---- CPU baseline (rank 0, N = 1 only): the oracle on the same layer/batch
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        L0 = {"gate_w": layers[0].gate.weight.cpu().numpy(), "e_bias": None, "shared": None}
        for n in ("gate", "up", "down"):
            p = getattr(layers[0].switch_mlp, f"{n}_proj")
            L0[n] = (p["weight"].cpu().numpy().view(np.uint32), p["scales"].cpu().numpy(),
                     p["biases"].cpu().numpy())
        xb = synthetic.make_x_torch(spec, T, seed=7, device=dev).contiguous().view(torch.int16).cpu().numpy()
        r = run_cpu_reference(spec, T, args.cpu_budget, layer=L0, xb=xb.view(np.uint16))
        cpu = {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
               "sample": f"{r['steps']} full {T}-token forwards of layer copy 0 (median), oracle/ef_oracle.c"}

    launches = len(recs)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 codes x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; random-init weights of the named shape)",
        "config": {"workload": WORKLOAD if args.workload == WORKLOAD else args.workload, "tokens": T,
                   "hidden": spec.hidden, "experts": spec.n_experts, "top_k": spec.top_k, "inter": spec.inter,
                   "bits": spec.bits, "group": spec.group_size, "parallelism": "replicas" if ws > 1 else "single",
                   "layer_copies": n_copies, "l2": f"rotating {n_copies} layer copies of {layer_bytes/1e6:.0f} MB",
                   "unique_experts_per_step": round(n_u, 2)},
        "layer_gbs": round(ab["total"] / (ms * 1e-3) / 1e9, 1),
        "layer_frac": round(ab["total"] / (ms * 1e-3) / 1e9 / hbm_peak, 4),
        "roofline": {"kernel": kern, "bound": "hbm", "achieved": round(achieved, 1) if achieved else None,
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4) if achieved else None,
                     "traffic": traffic, "peak_kind": peak_kind, "kernel_ms": round(k_ms, 5) if k_ms else None,
                     "algorithmic_bytes": k_bytes, "timing": "CUDA events around each launch, traced pass",
                     "traced_ms_per_step": round(ms_tr, 5), "kernel_shares": shares},
        "cpu_baseline": cpu,
        "e2e": {"value": round(ws * T / (e2e_ms * 1e-3), 1), "unit": UNIT, "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": T * spec.hidden * 2, "d2h_bytes_per_step": T * spec.hidden * 2,
                "api": "streaming_moe_forward (C ABI ef_moe_forward), pinned host x/y"},
        "gpu_launches": launches,
        "sweep": sweep,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return bench_reference(args)
    return bench_ours(args)


if __name__ == "__main__":
    sys.exit(main())
