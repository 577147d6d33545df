"""MLX safetensors import (expertflow_b200.weights).

CPU: a synthetic layer written under mlx_lm tensor names (one file, a sharded
directory with model.safetensors.index.json and config.json, the Mixtral
prefix) reads back bit-identical with the spec the tensors and config imply;
bf16 scales convert exactly or are rejected; a quantised router is dequantised
like the oracle's dequantise.  GPU: a layer loaded from a file runs the same
forward as the same layer built from arrays.
"""
import json
import os

import numpy as np
import pytest

from expertflow_b200 import synthetic, weights as W
from expertflow_b200.spec import MoESpec

DS = MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=4, router="sigmoid_group", n_group=4, topk_group=2,
             routed_scaling=2.5, n_shared=1, act_dtype="bfloat16", e_bias_std=0.01)
QW = MoESpec(hidden=512, n_experts=16, top_k=4, inter=256, bits=8, router="softmax", act_dtype="bfloat16")

DS_CONFIG = {"num_experts_per_tok": 4, "n_group": 4, "topk_group": 2, "routed_scaling_factor": 2.5,
             "norm_topk_prob": True, "scoring_func": "sigmoid", "torch_dtype": "bfloat16",
             "quantization": {"group_size": 64, "bits": 4}}


def _same_layer(a, b):
    np.testing.assert_array_equal(np.asarray(a["gate_w"]).view(np.uint16), np.asarray(b["gate_w"]).view(np.uint16))
    if a["e_bias"] is None:
        assert b["e_bias"] is None
    else:
        np.testing.assert_array_equal(a["e_bias"], b["e_bias"])
    for m in ("gate", "up", "down"):
        for x, y in zip(a[m], b[m]):
            np.testing.assert_array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8))
    if a["shared"] is None:
        assert b["shared"] is None
    else:
        for tx, ty in zip(a["shared"], b["shared"]):
            for x, y in zip(tx, ty):
                np.testing.assert_array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8))


def test_single_file_round_trip(tmp_path):
    layer = synthetic.make_layer_np(QW, 3)
    p = str(tmp_path / "model.safetensors")
    W.write_safetensors(p, W.layer_tensors(layer, 5))
    got, spec = W.load_layer_arrays(p, 5)
    _same_layer(layer, got)
    assert (spec.hidden, spec.inter, spec.n_experts, spec.bits, spec.group_size) == (512, 256, 16, 8, 64)
    assert spec.router == "softmax" and spec.n_shared == 0 and spec.gate_dtype == "float16"


def test_sharded_directory_with_config(tmp_path):
    layer = synthetic.make_layer_np(DS, 4)
    t = W.layer_tensors(layer, 2)
    names = sorted(t)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    weight_map = {}
    for fn, ns in shards.items():
        W.write_safetensors(str(tmp_path / fn), {n: t[n] for n in ns})
        weight_map.update({n: fn for n in ns})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    (tmp_path / "config.json").write_text(json.dumps(DS_CONFIG))
    got, spec = W.load_layer_arrays(str(tmp_path), 2)
    _same_layer(layer, got)
    assert spec.router == "sigmoid_group" and (spec.n_group, spec.topk_group, spec.routed_scaling) == (4, 2, 2.5)
    assert spec.n_shared == 1 and spec.top_k == 4 and spec.bits == 4


def test_mixtral_prefix(tmp_path):
    layer = synthetic.make_layer_np(QW, 1)
    p = str(tmp_path / "m.safetensors")
    W.write_safetensors(p, W.layer_tensors(layer, 0, prefix="model.layers.{i}.block_sparse_moe"))
    got, _ = W.load_layer_arrays(p, 0)
    _same_layer(layer, got)
    with pytest.raises(KeyError):
        W.load_layer_arrays(p, 1)


def test_bf16_scales_exact_or_rejected(tmp_path):
    layer = synthetic.make_layer_np(QW, 2)
    t = W.layer_tensors(layer, 0)
    name = "model.layers.0.mlp.switch_mlp.up_proj.scales"
    s = t[name][0].astype(np.float32)
    # bf16 patterns of values fp16 holds exactly (7-bit mantissas in fp16's normal range)
    bf = (s.view(np.uint32) >> 16).astype(np.uint16)
    t[name] = (bf, "BF16")
    p = str(tmp_path / "bf.safetensors")
    W.write_safetensors(p, t)
    got, _ = W.load_layer_arrays(p, 0)
    want = (bf.astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(got["up"][1].astype(np.float32), want)
    # a value below fp16's normal range cannot be carried exactly
    bad = bf.copy()
    bad.flat[5] = (np.array([1e-9], np.float32).view(np.uint32)[0] >> 16).astype(np.uint16)
    t[name] = (bad, "BF16")
    W.write_safetensors(p, t)
    with pytest.raises(ValueError):
        W.load_layer_arrays(p, 0)


def test_quantised_router_dequantised(tmp_path):
    from oracle import oracle as O

    layer = synthetic.make_layer_np(QW, 6)
    t = W.layer_tensors(layer, 0)
    rng = np.random.default_rng(0)
    E, H = QW.n_experts, QW.hidden
    gw = rng.integers(0, 2 ** 32, size=(E, H * 4 // 32), dtype=np.uint64).astype(np.uint32)
    gs = (rng.random((E, H // 64), dtype=np.float32) * 0.01 + 0.001).astype(np.float16)
    gb = (-(gs.astype(np.float32) * 7.5)).astype(np.float16)
    t["model.layers.0.mlp.gate.weight"] = (gw, "U32")
    t["model.layers.0.mlp.gate.scales"] = (gs, "F16")
    t["model.layers.0.mlp.gate.biases"] = (gb, "F16")
    d = tmp_path / "q"
    d.mkdir()
    W.write_safetensors(str(d / "model.safetensors"), t)
    (d / "config.json").write_text(json.dumps({"num_experts_per_tok": 4, "quantization": {"group_size": 64, "bits": 4}}))
    got, spec = W.load_layer_arrays(str(d), 0)
    ref = O.c_dequantize(gw, gs, gb, 4, 64).astype(np.float16)
    np.testing.assert_array_equal(got["gate_w"], ref)
    assert spec.bits == 8 and spec.gate_dtype == "float16"  # experts stay 8-bit


def test_truncated_file_rejected(tmp_path):
    layer = synthetic.make_layer_np(QW, 2)
    p = str(tmp_path / "t.safetensors")
    W.write_safetensors(p, W.layer_tensors(layer, 0))
    with open(p, "r+b") as f:
        f.truncate(os.path.getsize(p) - 100)
    with pytest.raises(ValueError):
        W.SafetensorsIndex(p)


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [DS, QW])
def test_loaded_layer_forward_matches_arrays(tmp_path, spec):
    import torch
    from expertflow_b200 import moe

    layer = synthetic.make_layer_np(spec, 9)
    p = str(tmp_path / "model.safetensors")
    W.write_safetensors(p, W.layer_tensors(layer, 0))
    (tmp_path / "config.json").write_text(json.dumps(DS_CONFIG if spec is DS else {"num_experts_per_tok": 4}))
    m_file = W.load_moe_layer(str(tmp_path), 0, spec=spec)
    m_arr = moe.MoELayer.from_arrays(spec, layer)
    x = synthetic.make_x_torch(spec, 37, seed=4)
    torch.testing.assert_close(m_file(x, out_dtype=torch.float32), m_arr(x, out_dtype=torch.float32), rtol=0, atol=0)
