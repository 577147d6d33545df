"""The cold tier: expert blobs read out of safetensors files by the library's
reader threads (ef_store_*), and slot pools over it.

CPU: blobs read from a sharded checkpoint (buffered and O_DIRECT) hold exactly
the checkpoint's arrays; bf16 scales become fp16 by the exact rule of
``weights._bf16_to_f16`` for every one of the 65,536 bf16 bit patterns; bad
ranges and truncated files are rejected when the store opens.
GPU: a pool over the store, with a host tier far smaller than the model,
gives bit-identical outputs and the same HBM residency as a pool holding every
expert in pinned memory; a failed read leaves the pool usable.
"""
import json
import os

import numpy as np
import pytest

from expertflow_b200 import synthetic
from expertflow_b200 import weights as W
from expertflow_b200.spec import MoESpec

SPEC = MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=4, router="softmax", act_dtype="bfloat16")
SPEC8 = MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=8, router="softmax", act_dtype="bfloat16")


@pytest.fixture(scope="module")
def P():
    from expertflow_b200 import build

    build.build()
    from expertflow_b200 import pool

    return pool


def _write_model(d, spec, n_layers, seed=0, n_shards=2, bf16_scales=False):
    layers = [synthetic.make_layer_np(spec, seed + i) for i in range(n_layers)]
    t = {}
    for i, lay in enumerate(layers):
        t.update(W.layer_tensors(lay, i))
    if bf16_scales:  # scales as bf16 patterns of values fp16 holds exactly
        for name in list(t):
            if name.endswith((".scales", ".biases")) and "switch_mlp" in name:
                a = t[name][0].astype(np.float32)
                t[name] = ((a.view(np.uint32) >> 16).astype(np.uint16), "BF16")
    names = sorted(t)
    per = (len(names) + n_shards - 1) // n_shards
    wm = {}
    for k in range(n_shards):
        fn = f"model-{k + 1:05d}-of-{n_shards:05d}.safetensors"
        part = names[k * per:(k + 1) * per]
        W.write_safetensors(os.path.join(d, fn), {n: t[n] for n in part})
        wm.update({n: fn for n in part})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": wm}, f)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump({"num_experts_per_tok": spec.top_k, "quantization": {"group_size": 64, "bits": spec.bits}}, f)
    return layers, t


def _check_blob(store, blob, layer, e):
    got = store.split_blob(blob)
    for m in ("gate", "up", "down"):
        w, s, b = layer[m]
        np.testing.assert_array_equal(got[m][0], np.asarray(w)[e].view(np.uint32))
        np.testing.assert_array_equal(got[m][1].view(np.uint16), np.asarray(s, np.float16)[e].view(np.uint16))
        np.testing.assert_array_equal(got[m][2].view(np.uint16), np.asarray(b, np.float16)[e].view(np.uint16))


@pytest.mark.parametrize("spec", [SPEC, SPEC8])
def test_store_reads_checkpoint_experts(P, tmp_path, spec):
    layers, _ = _write_model(str(tmp_path), spec, 3, seed=5)
    store = P.ExpertStore.from_safetensors(str(tmp_path), n_readers=4)
    info = store.info()
    assert info["n_layers"] == 3 and info["n_readers"] == 4 and not info["direct"]
    assert info["blob_bytes"] >= spec.expert_bytes() and info["offsets"][9] <= info["blob_bytes"]
    assert all(o % 16 == 0 for o in info["offsets"])
    rng = np.random.default_rng(0)
    ls = [int(v) for v in rng.integers(0, 3, 40)]
    es = [int(v) for v in rng.integers(0, spec.n_experts, 40)]
    blobs = store.read(ls, es)
    for blob, l, e in zip(blobs, ls, es):
        _check_blob(store, blob, layers[l], e)
    info = store.info()
    assert info["reads"] == 40 and info["file_bytes"] == 40 * spec.expert_bytes()
    store.close()


def test_store_direct_io(P, tmp_path):
    from expertflow_b200 import _lib as L

    layers, _ = _write_model(str(tmp_path), SPEC, 2, seed=8, n_shards=3)
    try:
        store = P.ExpertStore.from_safetensors(str(tmp_path), direct=True, n_readers=3)
    except L.EfmoeError as ex:  # a file system without O_DIRECT (tmpfs before Linux 6.6, overlays)
        assert ex.status == -9 and "O_DIRECT" in str(ex)
        pytest.skip(f"O_DIRECT not supported here: {ex}")
    assert store.info()["direct"]
    ls, es = [0, 1, 1, 0, 1], [0, 15, 7, 3, 0]
    for blob, l, e in zip(store.read(ls, es), ls, es):
        _check_blob(store, blob, layers[l], e)
    store.close()


def test_store_layer_subset_and_order(P, tmp_path):
    layers, _ = _write_model(str(tmp_path), SPEC, 4, seed=2)
    idx = W.SafetensorsIndex(str(tmp_path))
    assert W.moe_layers(idx) == [0, 1, 2, 3]
    store = P.ExpertStore.from_safetensors(idx, layers=[3, 1])
    b = store.read([0, 1], [9, 2])
    _check_blob(store, b[0], layers[3], 9)
    _check_blob(store, b[1], layers[1], 2)
    store.close()


def test_store_bf16_scales_converted(P, tmp_path):
    layers, _ = _write_model(str(tmp_path), SPEC, 2, seed=3, bf16_scales=True)
    store = P.ExpertStore.from_safetensors(str(tmp_path))
    for blob, (l, e) in zip(store.read([0, 1], [4, 11]), [(0, 4), (1, 11)]):
        got = store.split_blob(blob)
        for m in ("gate", "up", "down"):
            for a, want in ((1, layers[l][m][1]), (2, layers[l][m][2])):
                bits = (np.asarray(want, np.float16)[e].astype(np.float32).view(np.uint32) >> 16).astype(np.uint32)
                np.testing.assert_array_equal(got[m][a].astype(np.float32), (bits << 16).view(np.float32))
    store.close()


def _bf16_exact_mask(pat: np.ndarray):
    f32 = (pat.astype(np.uint32) << 16).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        f16 = f32.astype(np.float16)
    return (f16.astype(np.float32) == f32) | ~np.isfinite(f32), f16


def _bf16_store(P, d, values):
    """A one-layer checkpoint whose gate scales hold `values` (bf16 bits) in
    expert 0 and exact fillers elsewhere; returns the store."""
    lay = synthetic.make_layer_np(SPEC, 1)
    t = W.layer_tensors(lay, 0)
    for name in list(t):
        if name.endswith((".scales", ".biases")) and "switch_mlp" in name:
            a = t[name][0].astype(np.float32)
            t[name] = ((a.view(np.uint32) >> 16).astype(np.uint16), "BF16")
    name = "model.layers.0.mlp.switch_mlp.gate_proj.scales"
    arr = t[name][0].copy()
    flat = arr.reshape(arr.shape[0], -1)
    flat[0, :len(values)] = values
    t[name] = (arr, "BF16")
    p = os.path.join(d, "m.safetensors")
    W.write_safetensors(p, t)
    return P.ExpertStore.from_safetensors(p, n_readers=2)


def test_bf16_to_fp16_every_pattern(P, tmp_path):
    """All 65,536 bf16 bit patterns: every exact one converts to numpy's fp16
    (NaNs stay NaN), and a read holding an inexact one fails with EF_ERR_IO."""
    from expertflow_b200 import _lib as L

    pat = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    exact, f16 = _bf16_exact_mask(pat)
    n_per = SPEC.inter * SPEC.hidden // 64  # gate scales of one expert
    good = pat[exact]
    for k in range(0, len(good), n_per):
        chunk = good[k:k + n_per]
        d = tmp_path / f"g{k}"
        d.mkdir()
        store = _bf16_store(P, str(d), chunk)
        got = store.split_blob(store.read([0], [0])[0])["gate"][1].reshape(-1)[:len(chunk)]
        want = f16[exact][k:k + n_per]
        nan = np.isnan(want)
        assert np.isnan(got[nan]).all()
        np.testing.assert_array_equal(got[~nan].view(np.uint16), want[~nan].view(np.uint16))
        store.close()
    bad = pat[~exact]
    # every inexact exponent class: bf16 subnormals, too large, and fp16
    # subnormal magnitudes with too many significant bits
    rng = np.random.default_rng(1)
    picks = np.unique(np.concatenate([bad[:4], bad[-4:], rng.choice(bad, 24, replace=False),
                                      bad[(bad & 0x7f80) == (0x7f80 & (103 << 7))][:2]]))
    for v in picks:
        d = tmp_path / f"b{int(v)}"
        d.mkdir()
        store = _bf16_store(P, str(d), np.array([v], np.uint16))
        with pytest.raises(L.EfmoeError) as ei:
            store.read([0], [0])
        assert ei.value.status == -9
        store.read([0], [1])  # other experts of the same array still read
        store.close()


def test_store_rejects_bad_ranges(P, tmp_path):
    from expertflow_b200 import _lib as L

    _write_model(str(tmp_path), SPEC, 1, n_shards=1)
    idx = W.SafetensorsIndex(str(tmp_path))
    rs = W.expert_ranges(idx, 0, SPEC)
    files = [rs[0][0]]
    base = [(0, bf, off, st) for _, bf, off, st in rs]
    P.ExpertStore(SPEC, files, [base]).close()
    size = os.path.getsize(files[0])
    cases = {
        "past the end": [(0, False, size - 10, base[0][3])] + base[1:],
        "stride below size": [(0, False, base[0][2], base[0][3] - 4)] + base[1:],
        "codes as bf16": [(0, True, base[0][2], base[0][3])] + base[1:],
        "file index": [(1, False, base[0][2], base[0][3])] + base[1:],
    }
    for why, r in cases.items():
        with pytest.raises(L.EfmoeError) as ei:
            P.ExpertStore(SPEC, files, [r])
        assert ei.value.status == -1, why
    with pytest.raises(L.EfmoeError) as ei:
        P.ExpertStore(SPEC, [str(tmp_path / "missing.safetensors")], [base])
    assert ei.value.status == -9
    # a checkpoint tensor with the wrong shape is refused before the library sees it
    with pytest.raises(ValueError):
        W.expert_ranges(idx, 0, SPEC8)


def test_store_read_range_errors(P, tmp_path):
    from expertflow_b200 import _lib as L

    _write_model(str(tmp_path), SPEC, 1, n_shards=1)
    store = P.ExpertStore.from_safetensors(str(tmp_path))
    with pytest.raises(L.EfmoeError):
        store.read([1], [0])
    with pytest.raises(L.EfmoeError):
        store.read([0], [16])
    assert store.read([], []) == []
    store.close()


# ---------------------------------------------------------------- GPU
def _gates(spec, n_layers, seed):
    import torch
    from expertflow_b200 import moe, pool

    dev = torch.device("cuda")
    bias = torch.from_numpy(pool.zipf_layer_bias(n_layers, spec.n_experts, 1.1, seed=seed)).to(dev)
    gates = []
    for layer in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 100 + layer)
        gw = (torch.randn((spec.n_experts, spec.hidden), generator=g, device=dev) * 0.02).to(torch.float16)
        gates.append(moe.MoEGate(gw, spec.top_k, "softmax", True, e_score_correction_bias=bias[layer].contiguous()))
    return gates


def _host_layers(layers):
    import torch

    return [{m: tuple(torch.from_numpy(np.ascontiguousarray(np.asarray(a)).view(np.int16 if a.dtype == np.float16
                                                                                   else np.int32)) for a in lay[m])
             for m in ("gate", "up", "down")} for lay in layers]


@pytest.mark.gpu
@pytest.mark.parametrize("direct", [False, True])
def test_pool_over_store_matches_pinned_pool(P, tmp_path, direct):
    import torch
    from expertflow_b200 import _lib as L, moe

    spec = MoESpec(hidden=1024, n_experts=32, top_k=4, inter=256, bits=4, router="softmax", act_dtype="bfloat16")
    n_layers, steps = 4, 8
    layers, _ = _write_model(str(tmp_path), spec, n_layers, seed=40, n_shards=3)
    try:
        store = P.ExpertStore.from_safetensors(str(tmp_path), n_readers=4, direct=direct)
    except L.EfmoeError as ex:
        if direct and ex.status == -9:
            pytest.skip(f"O_DIRECT not supported here: {ex}")
        raise
    gates = _gates(spec, n_layers, 7)
    pinned = P.ExpertSlotPool(spec, _host_layers(layers), budget=6, headroom=spec.top_k)
    cold = P.ExpertSlotPool.from_store(store, budget=6, host_blobs=12, headroom=spec.top_k)
    for t in range(steps):
        ra = synthetic.make_x_torch(spec, 2, seed=60 + t).float().contiguous()
        rb = ra.clone()
        pinned.decode_step(ra, gates, lookahead=True)
        cold.decode_step(rb, gates, lookahead=True)
        torch.cuda.synchronize()
        assert torch.equal(ra, rb), t
        for layer in range(n_layers):
            assert pinned.resident(layer) == cold.resident(layer), (t, layer)
    sa, sb = pinned.stats(), cold.stats()
    for k in ("accesses", "hits", "misses", "evictions", "tokens"):
        assert sa[k] == sb[k], k
    assert sb["host_reads"] > 12 and sb["host_evictions"] > 0 and sb["host_reads_ahead"] > 0
    assert sa["host_reads"] == 0 and sa["host_hits"] == 0
    assert store.info()["file_bytes"] == sb["host_reads"] * spec.expert_bytes()
    assert moe.device_error() == 0
    cold.close()
    pinned.close()
    store.close()


@pytest.mark.gpu
def test_pool_over_store_failed_read_leaves_pool_usable(P, tmp_path):
    """Layer 1's scales hold a bf16 value fp16 cannot carry: its forward fails
    with EF_ERR_IO every time (no half-updated residency), layer 0 keeps working."""
    import torch
    from expertflow_b200 import _lib as L, moe

    spec = SPEC
    d = tmp_path / "m"
    d.mkdir()
    layers = [synthetic.make_layer_np(spec, 70 + i) for i in range(2)]
    tens = {}
    for i, lay in enumerate(layers):
        tens.update(W.layer_tensors(lay, i))
    name = "model.layers.1.mlp.switch_mlp.up_proj.scales"
    a = (tens[name][0].astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    a.reshape(a.shape[0], -1)[:, 0] = 0x4780  # 65536.0: above fp16's range, in every expert
    tens[name] = (a, "BF16")
    W.write_safetensors(str(d / "model.safetensors"), tens)
    store = P.ExpertStore.from_safetensors(str(d / "model.safetensors"), spec=spec)
    gates = _gates(spec, 2, 3)
    pool = P.ExpertSlotPool.from_store(store, budget=4, host_blobs=8)
    x = synthetic.make_x_torch(spec, 1, seed=1)
    y0 = pool.forward(0, x, gates[0], out_dtype=torch.float32)
    for _ in range(2):
        with pytest.raises(L.EfmoeError) as ei:
            pool.forward(1, x, gates[1])
        assert ei.value.status == -9
    assert pool.resident(1) == []
    y0b = pool.forward(0, x, gates[0], out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y0, y0b)
    assert moe.device_error() == 0
    pool.close()
    store.close()


def test_store_close_closes_its_pools_first(P, tmp_path):
    """A pool reads through its store until it is destroyed, so closing the
    store closes the pools still open over it first."""
    _write_model(str(tmp_path), SPEC, 1, n_shards=1)
    store = P.ExpertStore.from_safetensors(str(tmp_path))
    order = []

    class FakePool:  # stands in for an ExpertSlotPool (creating one needs a GPU)
        def close(self):
            order.append(("pool", bool(store._h)))

    fake = FakePool()
    store._pools.add(fake)
    store.close()
    assert order == [("pool", True)] and store._h is None
    store.close()  # idempotent
