"""Expert parallelism over NVLink peer memory (ef_ep_forward).

The exchange runs inside the library's kernels (rows stored into the
destination rank's buffer, flags released at system scope, bounded waits), so
the result must equal the single-GPU layer's bit for bit whenever both run the
same expert kernels: the combine reads the same fp32 expert rows in the same k
order.

* 1 GPU: a single-rank group (every expert local; dispatch and return go
  through this rank's own buffer), several forwards in a row with changing
  token counts (0 included), and a CUDA-graph-captured forward.
* 2 GPUs (skipped with fewer): two processes, experts split in half, each
  rank's output against the single-GPU layer on the same tokens, over several
  forwards with per-rank token counts that differ (one rank with none), then
  captured replays.
"""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import assert_ffn_close

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _small_spec(bits=4):
    from expertflow_b200.spec import DEEPSEEK_V3

    return DEEPSEEK_V3.with_(hidden=1024, inter=512, n_experts=32, n_group=8, topk_group=4, bits=bits)


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build

    build.build()


@pytest.mark.parametrize("which,path,Ts", [("small", "gemv", (5, 1, 0, 17, 64)),
                                          ("small", "gemm", (300, 129, 0, 300)),
                                          ("deepseek-v3", "gemv", (1, 32, 7))])
def test_single_rank_group_equals_layer(which, path, Ts):
    from expertflow_b200 import moe, synthetic, _lib as L
    from expertflow_b200.ep import PeerExpertParallelMoE, shard_layer
    from expertflow_b200.spec import DEEPSEEK_V3

    spec = _small_spec() if which == "small" else DEEPSEEK_V3
    p = {"gemv": L.EF_PATH_GEMV, "gemm": L.EF_PATH_GEMM}[path]
    layer = synthetic.make_layer_torch(spec, seed=5)
    full = moe.MoELayer.from_arrays(spec, layer, path=p)
    ep = PeerExpertParallelMoE(spec, shard_layer(spec, layer, 0, 1), max_tokens=max(Ts), path=p)
    try:
        for i, T in enumerate(Ts):
            x = synthetic.make_x_torch(spec, T, seed=40 + i)
            inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
            inds1 = torch.empty_like(inds)
            y = ep(x, inds_out=inds, out_dtype=torch.float32)
            y1 = full(x, inds_out=inds1, out_dtype=torch.float32)
            yb = ep(x)
            torch.cuda.synchronize()
            assert torch.equal(inds, inds1), f"forward {i}: routing differs"
            assert torch.equal(y, y1), f"forward {i} (T={T}): differs from the single-GPU layer"
            assert torch.equal(yb, y1.to(x.dtype))
        assert moe.device_error() == 0
    finally:
        ep.close()


def test_single_rank_group_oracle_and_capture():
    """Against the oracle, then a captured forward replayed with new inputs."""
    from expertflow_b200 import moe, synthetic
    from expertflow_b200.ep import PeerExpertParallelMoE, shard_layer
    from oracle import oracle as O

    spec = _small_spec()
    layer = synthetic.make_layer_np(spec, 9)
    ep = PeerExpertParallelMoE(spec, shard_layer(spec, layer, 0, 1), max_tokens=16)
    try:
        xb = synthetic.make_x_np(spec, 16, 2)
        x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
        y = ep(x, out_dtype=torch.float32)
        rs = O.RouterSpec(spec.router, spec.top_k, spec.norm_topk, spec.n_group, spec.topk_group,
                          spec.routed_scaling)
        _, _, y_ref = O.moe_forward(xb, True, layer["gate_w"].view(np.uint16), False, rs, layer["e_bias"],
                                    layer["gate"], layer["up"], layer["down"], spec.bits, spec.group_size,
                                    layer["shared"])
        assert_ffn_close(y.cpu().numpy(), y_ref, what="peer EP, one rank")
        cf = ep.capture(16, out_dtype=torch.float32)
        for seed in (3, 4):
            x2 = synthetic.make_x_torch(spec, 16, seed=seed)
            yg = cf(x2).clone()
            ye = ep(x2, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(yg, ye)
        assert moe.device_error() == 0
    finally:
        ep.close()


# ---------------------------------------------------------------- 2 GPUs
def _rank(rank, world, port, bits, out_q):
    import datetime

    import torch.distributed as dist
    from expertflow_b200 import build, moe, synthetic, _lib as L
    from expertflow_b200.ep import PeerExpertParallelMoE, shard_layer

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    ep = None
    try:
        build.build()
        spec = _small_spec(bits)
        layer = synthetic.make_layer_torch(spec, seed=21, device=dev)
        full = moe.MoELayer.from_arrays(spec, layer, device=dev, path=L.EF_PATH_GEMV)
        ep = PeerExpertParallelMoE(spec, shard_layer(spec, layer, rank, world, device=dev), max_tokens=48,
                                   path=L.EF_PATH_GEMV)
        results = []
        # per-step token counts of (rank 0, rank 1); rank 1 has none in step 2
        for step, counts in enumerate(((3, 5), (48, 1), (7, 0), (16, 16))):
            T = counts[rank]
            x = synthetic.make_x_torch(spec, T, seed=100 * step + rank, device=dev)
            y = ep(x, out_dtype=torch.float32)
            y1 = full(x, out_dtype=torch.float32)
            torch.cuda.synchronize()
            results.append(bool(torch.equal(y, y1)))
        cf = ep.capture(16, out_dtype=torch.float32)
        for seed in (7, 8):
            x = synthetic.make_x_torch(spec, 16, seed=1000 * seed + rank, device=dev)
            yg = cf(x).clone()
            y1 = full(x, out_dtype=torch.float32)
            torch.cuda.synchronize()
            results.append(bool(torch.equal(yg, y1)))
        out_q.put((rank, results, moe.device_error(dev)))
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("bits", [4, 8])
def test_two_gpus_equal_single_gpu_layer(bits):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, bits, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, results, err in res:
        assert err == 0, f"rank {rank}: device error {err}"
        assert all(results), f"rank {rank}: {results}"
