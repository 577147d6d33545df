"""MoE layer over GGUF K-quant experts (ef_kquant_moe_forward).

CPU: the oracle's K-quant FFN slices stacked experts the way the GGUF
layout stores them (one expert's FFN equals the single-matrix K-quant GEMV of
its slices).
GPU: the layer against the oracle (routing bit for bit, FFN output within the
fp tolerance) for every format pairing of gate/up and down, with and without
a shared expert, at token counts whose experts take one and several 8-row
segments; the layer loaded from a GGUF file equals the one built from the
same blocks.
"""
import os

import numpy as np
import pytest

from conftest import assert_ffn_close
from expertflow_b200 import gguf as G
from expertflow_b200.spec import MoESpec
from oracle import oracle as O

Q2, Q3, Q4 = G.GGML_TYPE_Q2_K, G.GGML_TYPE_Q3_K, G.GGML_TYPE_Q4_K


def _spec(shared):
    if shared:
        return MoESpec(hidden=1024, n_experts=16, top_k=4, inter=512, bits=4, router="sigmoid_group", n_group=4,
                       topk_group=2, routed_scaling=2.5, n_shared=1, act_dtype="bfloat16", e_bias_std=0.01)
    return MoESpec(hidden=1024, n_experts=16, top_k=4, inter=512, bits=4, router="softmax", act_dtype="bfloat16")


def _kq_layer(spec, tg, td, seed):
    """Random stacked K-quant projections (raw bytes, type, rows, cols) and a router."""
    rng = np.random.default_rng(seed)
    E, H, I = spec.n_experts, spec.hidden, spec.inter

    # super-block scales that give weights of about 0.02 in magnitude, as in
    # real checkpoints (the code and sub-scale ranges differ per format)
    d_scale = {Q2: 0.002, Q3: 0.0006, Q4: 0.0001}

    def proj(t, rows, cols, n):
        return (G.random_kquant_blocks(t, n * rows * cols // 256, rng, d_scale=d_scale[t]), t, rows, cols)

    layer = {"gate": proj(tg, I, H, E), "up": proj(tg, I, H, E), "down": proj(td, H, I, E),
             "gate_w": rng.normal(0, spec.gate_std, (E, H)).astype(np.float16),
             "e_bias": rng.normal(0, 0.01, E).astype(np.float32) if spec.router == "sigmoid_group" else None,
             "shared": None}
    if spec.n_shared:
        layer["shared"] = (proj(tg, I, H, 1), proj(tg, I, H, 1), proj(td, H, I, 1))
    return layer


def test_oracle_stacked_slices_match_single_matrix_gemv():
    spec = _spec(False)
    layer = _kq_layer(spec, Q2, Q4, 1)
    x = np.random.default_rng(2).standard_normal((1, spec.hidden)).astype(np.float32)
    e = 5
    y = O.np_kquant_moe_ffn(x, np.array([[e]]), np.ones((1, 1), np.float32), layer["gate"], layer["up"],
                            layer["down"])

    def sl(p, e):
        raw, t, rows, cols = p
        per = rows * (cols // 256) * O.KQ_BLOCK_BYTES[t]
        return raw[e * per:(e + 1) * per], t, rows, cols

    g = O.np_kquant_matmul(x, *[sl(layer["gate"], e)[i] for i in (0, 1)], spec.inter, spec.hidden)
    u = O.np_kquant_matmul(x, *[sl(layer["up"], e)[i] for i in (0, 1)], spec.inter, spec.hidden)
    h = g / (1.0 + np.exp(-g)) * u
    ref = O.np_kquant_matmul(h, *[sl(layer["down"], e)[i] for i in (0, 1)], spec.hidden, spec.inter)
    np.testing.assert_allclose(y, ref, rtol=1e-12, atol=1e-12)


def _device_layer(spec, layer):
    import torch
    from expertflow_b200 import kquant as KQ, moe

    def P(p, n):
        raw, t, rows, cols = p
        return KQ.KQuantProj(torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda(), t, rows, cols, n)

    gate = moe.MoEGate(torch.from_numpy(layer["gate_w"]).cuda(), spec.top_k, spec.router, spec.norm_topk,
                       spec.n_group, spec.topk_group, spec.routed_scaling,
                       None if layer["e_bias"] is None else torch.from_numpy(layer["e_bias"]).cuda())
    E = spec.n_experts
    shared = tuple(P(p, 1) for p in layer["shared"]) if layer["shared"] else None
    return KQ.KQuantMoELayer(gate, P(layer["gate"], E), P(layer["up"], E), P(layer["down"], E), shared)


@pytest.mark.gpu
@pytest.mark.parametrize("tg,td,shared", [(Q2, Q2, True), (Q3, Q4, False), (Q4, Q3, True), (Q2, Q4, False)])
@pytest.mark.parametrize("T", [1, 5, 37])
def test_layer_matches_oracle(tg, td, shared, T):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build, moe, synthetic

    build.build()
    spec = _spec(shared)
    layer = _kq_layer(spec, tg, td, 10 * tg + td + T)
    m = _device_layer(spec, layer)
    xb = synthetic.make_x_np(spec, T, 3)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
    y = m(x, inds_out=inds, wts_out=wts, out_dtype=torch.float32)
    yb = m(x)
    torch.cuda.synchronize()
    rs = O.RouterSpec(spec.router, spec.top_k, spec.norm_topk, spec.n_group, spec.topk_group, spec.routed_scaling)
    lg = O.c_router_logits(xb, True, layer["gate_w"].view(np.uint16), False)
    i_ref, w_ref = O.route(lg, rs, layer["e_bias"])
    np.testing.assert_array_equal(inds.cpu().numpy(), i_ref)
    np.testing.assert_array_equal(wts.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))
    y_ref = O.np_kquant_moe_ffn(O.bits_to_f32(xb, True), i_ref, w_ref, layer["gate"], layer["up"], layer["down"],
                                layer["shared"])
    assert_ffn_close(y.cpu().numpy(), y_ref, what=f"K-quant layer {tg}/{td} T={T}")
    assert torch.equal(yb, y.to(torch.bfloat16))
    assert moe.device_error() == 0


@pytest.mark.gpu
def test_layer_from_gguf_file_equals_arrays(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build, kquant as KQ, synthetic

    build.build()
    spec = _spec(True)
    layer = _kq_layer(spec, Q2, Q3, 77)
    E, H, I = spec.n_experts, spec.hidden, spec.inter
    tensors = {}
    for proj, (raw, t, rows, cols) in zip(("gate", "up", "down"), (layer["gate"], layer["up"], layer["down"])):
        tensors[f"blk.3.ffn_{proj}_exps.weight"] = ((cols, rows, E), t, raw)
    for proj, (raw, t, rows, cols) in zip(("gate", "up", "down"), layer["shared"]):
        tensors[f"blk.3.ffn_{proj}_shexp.weight"] = ((cols, rows), t, raw)
    path = os.path.join(tmp_path, "model.gguf")
    G.write_gguf(path, tensors, {"deepseek2.expert_count": E})
    ref = _device_layer(spec, layer)
    m = KQ.KQuantMoELayer.from_gguf(G.GGUFExperts(path), 3, ref.gate)
    assert m.shared is not None and m.down_proj.dtype == Q3
    x = synthetic.make_x_torch(spec, 9, seed=4)
    y = m(x, out_dtype=torch.float32)
    y_ref = ref(x, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    # expert e's dequantised slice is the reference decoder's output for its bytes
    e = 11
    per = I * (H // 256) * O.KQ_BLOCK_BYTES[Q2]
    want = O.np_dequant_kquant(layer["gate"][0][e * per:(e + 1) * per], Q2).reshape(I, H)
    np.testing.assert_array_equal(m.gate_proj.dequantize_expert(e).cpu().numpy().view(np.uint16),
                                  want.view(np.uint16))
