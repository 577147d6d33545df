"""Pins the CPU oracle: against the golden fixtures produced by the reference's
own code (tests/golden/make_golden.py), and C restatement vs numpy twin."""
import glob
import json
import math
import os

import numpy as np
import pytest

from conftest import assert_ffn_close
from expertflow_b200 import synthetic
from expertflow_b200.spec import MoESpec
from oracle import oracle as O


def _cases(golden_dir):
    return sorted(glob.glob(os.path.join(golden_dir, "moe_*.npz")))


def _load(path):
    z = np.load(path)
    spec = MoESpec(**json.loads(str(z["spec"])))
    return spec, z


def _layer_and_x(spec, z):
    layer = synthetic.make_layer_np(spec, int(z["seed"]))
    assert synthetic.layer_digest(layer) == str(z["digest"]), "synthetic generator drifted"
    x = synthetic.make_x_np(spec, int(z["T"]), int(z["x_seed"]))
    return layer, x


def _spec_router(spec):
    return O.RouterSpec(mode=spec.router, k=spec.top_k, norm_topk=spec.norm_topk, n_group=spec.n_group,
                        topk_group=spec.topk_group, scaling=spec.routed_scaling)


def test_golden_files_present(golden_dir):
    assert len(_cases(golden_dir)) >= 6
    assert os.path.exists(os.path.join(golden_dir, "cache_trace.npz"))


@pytest.mark.parametrize("name", ["moe_mixtral_small_t1", "moe_mixtral_small_t5", "moe_qwen_small",
                                  "moe_qwen_small_nonorm", "moe_deepseek_small", "moe_deepseek_small_8bit"])
def test_oracle_matches_reference_golden(golden_dir, name):
    spec, z = _load(os.path.join(golden_dir, name + ".npz"))
    layer, x = _layer_and_x(spec, z)
    bf = spec.act_dtype == "bfloat16"
    inds, wts, y = O.moe_forward(x, bf, layer["gate_w"].view(np.uint16), False, _spec_router(spec),
                                 layer["e_bias"], layer["gate"], layer["up"], layer["down"], spec.bits,
                                 spec.group_size, layer["shared"])
    # routing indices: bit-exact, in the same (rank) order as the reference run
    np.testing.assert_array_equal(inds, z["inds"])
    np.testing.assert_allclose(wts, z["scores"], rtol=2e-6, atol=1e-7)
    # fp32 oracle vs float64 reference execution: far inside the product tolerance
    assert_ffn_close(y, z["y"], max_abs=1e-5, rel=1e-5, what=name)
    # the numpy twin routes identically
    lg = O.np_router_logits(x, bf, layer["gate_w"].view(np.uint16), False)
    i2, w2 = O.route(lg, _spec_router(spec), layer["e_bias"], use_c=False)
    np.testing.assert_array_equal(i2, inds)
    np.testing.assert_array_equal(w2.view(np.uint32), wts.view(np.uint32))


def test_oracle_float64_twin_small(golden_dir):
    spec, z = _load(os.path.join(golden_dir, "moe_deepseek_small.npz"))
    layer, x = _layer_and_x(spec, z)
    xf = O.bits_to_f32(x, True)
    y64 = O.np_moe_ffn(xf, z["inds"], z["scores"], layer["gate"], layer["up"], layer["down"], spec.bits,
                       spec.group_size, layer["shared"])
    assert_ffn_close(y64, z["y"], max_abs=1e-6, rel=1e-6, what="np float64 twin")


def test_expf_accuracy_and_twins():
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.uniform(-104, 89, 20000).astype(np.float32),
                         np.float32([0.0, -0.0, 1.0, -1.0, 88.72, -87.33, -100.0, -103.9, 1e-30, -1e-30])])
    v = O.np_expf(xs)
    cv = np.array([O.c_expf(float(t)) for t in xs[:2000]], np.float32)
    np.testing.assert_array_equal(cv.view(np.uint32), v[:2000].view(np.uint32))
    ref = np.exp(xs.astype(np.float64))
    ok = (ref > 1.2e-38) & (ref < 3e38)
    rel = np.abs(v[ok] - ref[ok]) / ref[ok]
    assert rel.max() < 2.5 * 2.0 ** -24
    assert O.np_expf(np.float32(100.0)) == np.inf
    assert O.np_expf(np.float32(-200.0)) == 0.0
    assert math.isnan(float(O.np_expf(np.float32(np.nan))))


@pytest.mark.parametrize("T,E,H", [(1, 16, 1024), (3, 7, 264), (4, 256, 7168), (2, 128, 2048)])
def test_router_logits_c_equals_numpy(T, E, H):
    rng = np.random.default_rng(T * 100 + E)
    x = synthetic.act_bits_np(rng.standard_normal((T, H), dtype=np.float32), "bfloat16")
    w = rng.normal(0, 0.02, (E, H)).astype(np.float16).view(np.uint16)
    a = O.np_router_logits(x, True, w, False)
    b = O.c_router_logits(x, True, w, False)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    ref = O.bits_to_f32(x, True).astype(np.float64) @ O.bits_to_f32(w, False).astype(np.float64).T
    assert np.abs(a - ref).max() < 1e-5


def test_router_ties_break_to_lowest_index():
    lg = np.zeros((2, 16), np.float32)
    lg[0, [3, 5, 9]] = 1.0  # three-way tie for top-2 -> 3, 5
    lg[1, :] = 0.5          # all tied -> 0, 1
    for use_c in (True, False):
        inds, w = O.route(lg, O.RouterSpec("softmax", 2), use_c=use_c)
        np.testing.assert_array_equal(inds, [[3, 5], [0, 1]])
        np.testing.assert_allclose(w, 0.5)
    # sigmoid-group: equal group scores keep the lowest groups; masked experts are 0.0
    lg = np.zeros((1, 64), np.float32)
    inds, w = O.route(lg, O.RouterSpec("sigmoid_group", 4, True, 8, 2, 2.5), np.zeros(64, np.float32))
    np.testing.assert_array_equal(inds, [[0, 1, 2, 3]])
    np.testing.assert_allclose(w, 2.5 / 4)


def test_sigmoid_group_masked_zero_beats_negative():
    # experts outside the kept groups score exactly 0.0 (mlx_lm / DeepSeek-V3
    # masked_fill(0.0)); a kept expert with a negative corrected score ranks below them.
    E, G = 16, 4
    lg = np.full((1, E), -30.0, np.float32)   # sigmoid ~ 0
    lg[0, 0:4] = 5.0                          # group 0 strong
    eb = np.zeros(E, np.float32)
    eb[4:8] = 0.5                             # group 1 kept by bias
    eb[5] = -1.0                              # kept expert with negative corrected score
    for use_c in (True, False):
        inds, _ = O.route(lg, O.RouterSpec("sigmoid_group", 8, True, G, 2, 1.0), eb, use_c=use_c)
        assert 5 not in inds[0, :7].tolist()
        assert inds[0, -1] == 8  # first masked expert (0.0) beats expert 5 (-0.5)


def test_dequantize_format_lsb_first():
    # one row, 64 columns, codes 0..15 repeating: word j holds codes 8j..8j+7 LSB-first
    q = (np.arange(64) % 16).astype(np.uint32)[None]
    w = O.np_pack_codes(q, 4)
    assert w[0, 0] == sum(int(c) << (4 * i) for i, c in enumerate(range(8)))
    s = np.array([[0.5]], np.float16)
    b = np.array([[-4.0]], np.float16)
    d = O.c_dequantize(w, s, b, 4, 64)
    np.testing.assert_array_equal(d[0], 0.5 * q[0] - 4.0)
    q8 = (np.arange(64) * 3 % 256).astype(np.uint32)[None]
    w8 = O.np_pack_codes(q8, 8)
    d8 = O.c_dequantize(w8, s, b, 8, 64)
    np.testing.assert_array_equal(d8[0], 0.5 * q8[0] - 4.0)
    np.testing.assert_array_equal(O.np_unpack_codes(w8, 8), q8)
