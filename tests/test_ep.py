"""Expert parallelism: the exchange choreography of ExpertParallelMoE.

* CPU (gloo, world size 2): the rank-local device steps are replaced by the
  oracle (routing, per-row SwiGLU, weighted combine in numpy / the C
  restatement), so the test checks the host logic -- splits, the three
  all-to-alls, row order, the shared expert, the combine -- against the
  single-process oracle forward.
* GPU (NCCL, 2 GPUs, skipped with fewer): the real device steps against the
  single-GPU layer forward and the oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import assert_ffn_close


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spec(shared=True):
    from expertflow_b200.spec import MoESpec

    if shared:
        return MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=4, router="sigmoid_group", n_group=4,
                       topk_group=2, routed_scaling=2.5, n_shared=1, act_dtype="bfloat16", e_bias_std=0.01)
    return MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=8, router="softmax", act_dtype="bfloat16")


def _router_spec(spec):
    from oracle import oracle as O

    return O.RouterSpec(spec.router, spec.top_k, spec.norm_topk, spec.n_group, spec.topk_group, spec.routed_scaling)


class CpuOracleOps:
    """The rank-local steps restated with the oracle (test double for EpDeviceOps)."""

    def __init__(self, spec, layer, rank, n_ranks):
        self.spec, self.layer, self.n_ranks = spec, layer, n_ranks
        self.e_loc = spec.n_experts // n_ranks
        sl = slice(rank * self.e_loc, (rank + 1) * self.e_loc)
        self.local = {k: tuple(a[sl] for a in layer[k]) for k in ("gate", "up", "down")}

    def _bits(self, x):
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)

    def dispatch(self, x):
        from oracle import oracle as O

        spec = self.spec
        T, k = x.shape[0], spec.top_k
        lg = O.np_router_logits(self._bits(x), True, self.layer["gate_w"].view(np.uint16), False)
        inds, wts = O.route(lg, _router_spec(spec), self.layer["e_bias"], use_c=False)
        ent = inds.reshape(-1)
        order = np.argsort(ent, kind="stable")  # by expert, then entry index
        inv = np.empty_like(order)
        inv[order] = np.arange(order.size)
        send_rows = x[torch.from_numpy(order // k)]
        counts = np.bincount(ent // self.e_loc, minlength=self.n_ranks)
        return {"send_rows": send_rows.contiguous(), "send_eid": torch.from_numpy((ent[order] % self.e_loc).astype(np.int32)),
                "send_counts": torch.from_numpy(counts.astype(np.int32)), "inv": torch.from_numpy(inv.astype(np.int32)),
                "wts": torch.from_numpy(wts.reshape(-1).astype(np.float32)), "inds": torch.from_numpy(inds)}

    def _rows(self, rows, eid, mats):
        from oracle import oracle as O

        xf = O.bits_to_f32(self._bits(rows), True)
        ids = eid.numpy().astype(np.int64)[:, None]
        y = O.np_moe_ffn(xf, ids, np.ones(ids.shape, np.float32), *mats, self.spec.bits, self.spec.group_size)
        return torch.from_numpy(np.asarray(y, np.float32))

    def experts(self, rows, eid):
        if rows.shape[0] == 0:
            return torch.empty((0, rows.shape[1]), dtype=torch.float32)
        return self._rows(rows, eid, (self.local["gate"], self.local["up"], self.local["down"]))

    def shared(self, x):
        if self.layer["shared"] is None:
            return None
        sg, su, sd = self.layer["shared"]
        mats = tuple(tuple(a[None] for a in m) for m in (sg, su, sd))
        return self._rows(x, torch.zeros(x.shape[0], dtype=torch.int32), mats)

    def combine(self, back, inv, wts, T, with_shared, out_dtype):
        k = self.spec.top_k
        b = back.double().numpy()
        r = b[inv.numpy().astype(np.int64)].reshape(T, k, -1)
        y = (r * wts.double().numpy().reshape(T, k, 1)).sum(1)
        if with_shared:
            y = y + b[T * k:]
        return torch.from_numpy(y.astype(np.float32))


def _cpu_rank(rank, world, port, shared, out_q):
    import torch.distributed as dist
    from expertflow_b200 import synthetic
    from expertflow_b200.ep import ExpertParallelMoE

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        spec = _spec(shared)
        layer = synthetic.make_layer_np(spec, 11)
        xb = synthetic.make_x_np(spec, 9, 5)  # 9 tokens: rank 0 takes 5, rank 1 takes 4
        xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
        lo, hi = (0, 5) if rank == 0 else (5, 9)
        ep = ExpertParallelMoE(spec, CpuOracleOps(spec, layer, rank, world))
        y = ep(xt[lo:hi], out_dtype=torch.float32)
        out_q.put((rank, y.numpy(), ep.last_counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shared", [True, False])
def test_ep_exchange_matches_oracle_on_gloo(shared):
    import torch.multiprocessing as mp
    from expertflow_b200 import synthetic
    from oracle import oracle as O

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_rank, args=(r, 2, port, shared, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (y, c)) for r, y, c in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    spec = _spec(shared)
    layer = synthetic.make_layer_np(spec, 11)
    xb = synthetic.make_x_np(spec, 9, 5)
    _, _, y_ref = O.moe_forward(xb, True, layer["gate_w"].view(np.uint16), False, _router_spec(spec),
                                layer["e_bias"], layer["gate"], layer["up"], layer["down"], spec.bits,
                                spec.group_size, layer["shared"])
    y = np.concatenate([res[0][0], res[1][0]])
    assert_ffn_close(y, y_ref, max_abs=1e-4, rel=1e-5, what="EP over gloo")
    # what rank r sent to rank s is what rank s received from rank r
    (s0, r0), (s1, r1) = res[0][1], res[1][1]
    assert s0[1] == r1[0] and s1[0] == r0[1] and sum(s0) == 5 * spec.top_k and sum(s1) == 4 * spec.top_k


# ---------------------------------------------------------------- GPU (NCCL)
def _gpu_rank(rank, world, port, T, bits, out_q):
    import datetime

    import torch.distributed as dist
    from expertflow_b200 import build, moe, synthetic
    from expertflow_b200.ep import ExpertParallelMoE, shard_layer
    from expertflow_b200.spec import DEEPSEEK_V3

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        build.build()
        spec = DEEPSEEK_V3.with_(hidden=1024, inter=512, n_experts=32, n_group=8, topk_group=4, bits=bits)
        layer = synthetic.make_layer_torch(spec, seed=21, device=dev)
        ops = shard_layer(spec, layer, rank, world, device=dev)
        ep = ExpertParallelMoE(spec, ops)
        x = synthetic.make_x_torch(spec, T * world, seed=3, device=dev)
        mine = x[rank * T:(rank + 1) * T].contiguous()
        y = ep(mine, out_dtype=torch.float32)
        full = moe.MoELayer.from_arrays(spec, layer, device=dev)
        y1 = full(mine, out_dtype=torch.float32)
        torch.cuda.synchronize()
        out_q.put((rank, y.cpu().numpy(), y1.cpu().numpy(), moe.device_error(dev)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("T,bits", [(3, 4), (40, 8)])
def test_ep_nccl_two_gpus_matches_single_gpu(T, bits):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, 2, port, T, bits, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, y, y1, err in res:
        assert err == 0
        # same kernels on the same rows: identical to the single-GPU layer
        np.testing.assert_array_equal(y, y1)
