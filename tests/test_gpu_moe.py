"""GPU parity of the MoE-layer hot path against the CPU oracle and the golden
fixtures produced by the reference's own code.  All calls go through the C ABI
(libefmoe.so) via the package's host layer."""
import glob
import json
import os

import numpy as np
import pytest

from conftest import assert_ffn_close
from expertflow_b200 import synthetic
from expertflow_b200.spec import MoESpec
from expertflow_b200.spec import QWEN3_30B_A3B, DEEPSEEK_V3, DEEPSEEK_V3_PREFILL_8BIT, MIXTRAL_SMALL
from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build

    build.build()
    yield
    from expertflow_b200 import moe

    assert moe.device_error() == 0, "a kernel reported a device-side error"


def _moe():
    from expertflow_b200 import moe

    return moe


def _spec_router(spec):
    return O.RouterSpec(mode=spec.router, k=spec.top_k, norm_topk=spec.norm_topk, n_group=spec.n_group,
                        topk_group=spec.topk_group, scaling=spec.routed_scaling)


def _x_tensor(bits_np, spec):
    dt = torch.bfloat16 if spec.act_dtype == "bfloat16" else torch.float16
    return torch.from_numpy(bits_np.view(np.int16)).cuda().view(dt)


def _bits_of(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# ---------------------------------------------------------------- golden fixtures
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "moe_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_layer_matches_reference_golden(path):
    moe = _moe()
    z = np.load(path)
    spec = MoESpec(**json.loads(str(z["spec"])))
    layer = synthetic.make_layer_np(spec, int(z["seed"]))
    assert synthetic.layer_digest(layer) == str(z["digest"])
    xb = synthetic.make_x_np(spec, int(z["T"]), int(z["x_seed"]))
    m = moe.MoELayer.from_arrays(spec, layer)
    x = _x_tensor(xb, spec)
    T, k = x.shape[0], spec.top_k
    inds = torch.empty((T, k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, k), dtype=torch.float32, device="cuda")
    y = m(x, inds_out=inds, wts_out=wts, out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(inds.cpu().numpy(), z["inds"])
    np.testing.assert_allclose(wts.cpu().numpy(), z["scores"], rtol=2e-6, atol=1e-7)
    assert_ffn_close(y.cpu().numpy(), z["y"], what=os.path.basename(path))
    # the act-dtype output is exactly the rounding of the fp32 combine, and the
    # drop-in entry point gives the same result
    y16 = moe.streaming_moe_forward(m, x[None])[0]
    assert y16.dtype == x.dtype and torch.equal(y16, y.to(x.dtype))


# ---------------------------------------------------------------- router bit-exactness
@pytest.mark.parametrize("spec,T", [(QWEN3_30B_A3B, 1), (QWEN3_30B_A3B, 64), (DEEPSEEK_V3, 1), (DEEPSEEK_V3, 256),
                                    (DEEPSEEK_V3_PREFILL_8BIT, 4096), (MIXTRAL_SMALL, 3),
                                    (QWEN3_30B_A3B.with_(norm_topk=False), 33)])
def test_router_indices_bit_exact(spec, T):
    moe = _moe()
    rng = np.random.default_rng(T)
    gate = rng.normal(0, spec.gate_std, (spec.n_experts, spec.hidden)).astype(np.float16)
    eb = rng.normal(0, 0.01, spec.n_experts).astype(np.float32) if spec.router == "sigmoid_group" else None
    xb = synthetic.act_bits_np(rng.standard_normal((T, spec.hidden), dtype=np.float32), spec.act_dtype)
    g = moe.MoEGate(torch.from_numpy(gate).cuda(), spec.top_k, spec.router, spec.norm_topk, spec.n_group,
                    spec.topk_group, spec.routed_scaling, None if eb is None else torch.from_numpy(eb).cuda())
    logits = torch.empty((T, spec.n_experts), dtype=torch.float32, device="cuda")
    inds, wts = g(_x_tensor(xb, spec), logits_out=logits)
    lg_ref = O.c_router_logits(xb, spec.act_dtype == "bfloat16", gate.view(np.uint16), False)
    np.testing.assert_array_equal(logits.cpu().numpy().view(np.uint32), lg_ref.view(np.uint32))
    i_ref, w_ref = O.route(lg_ref, _spec_router(spec), eb)
    np.testing.assert_array_equal(inds.cpu().numpy(), i_ref)
    np.testing.assert_array_equal(wts.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))


def test_router_ties_and_masking():
    moe = _moe()
    E, H = 64, 256
    gate = np.zeros((E, H), np.float16)
    gate[[3, 5, 9], 0] = 1.0  # three-way tie
    x = np.zeros((2, H), np.float32)
    x[:, 0] = 1.0
    xb = synthetic.act_bits_np(x, "bfloat16")
    g = moe.MoEGate(torch.from_numpy(gate).cuda(), 2)
    inds, wts = g(_x_tensor(xb, QWEN3_30B_A3B))
    assert inds.cpu().tolist() == [[3, 5], [3, 5]]
    # all tied -> lowest indices; sigmoid groups tied -> lowest groups
    g2 = moe.MoEGate(torch.zeros((E, H), dtype=torch.float16, device="cuda"), 4, "sigmoid_group", True, 8, 2, 2.5,
                     torch.zeros(E, dtype=torch.float32, device="cuda"))
    inds, wts = g2(_x_tensor(xb, QWEN3_30B_A3B))
    assert inds.cpu().tolist() == [[0, 1, 2, 3]] * 2
    np.testing.assert_allclose(wts.cpu().numpy(), 2.5 / 4)


# ---------------------------------------------------------------- full-size layers
def _torch_layer(spec, seed=0):
    return synthetic.make_layer_torch(spec, seed)


def _to_np_qmat(m):
    w, s, b = m
    return (w.cpu().numpy().view(np.uint32), s.cpu().numpy(), b.cpu().numpy())


def _oracle_sampled(spec, layer_t, xb, inds, wts, tokens):
    """Oracle FFN output for a subset of tokens (independent per token)."""
    sub_inds = inds[tokens]
    needed = sorted(set(sub_inds.reshape(-1).tolist()))
    remap = {e: i for i, e in enumerate(needed)}
    sel = torch.tensor(needed, dtype=torch.long, device="cuda")

    def take(m):
        return tuple(a.index_select(0, sel) for a in m)

    g, u, d = (_to_np_qmat(take(layer_t[n])) for n in ("gate", "up", "down"))
    sh = None
    if layer_t["shared"] is not None:
        sh = tuple(tuple(a.cpu().numpy().view(np.uint32) if a.dtype == torch.int32 else a.cpu().numpy() for a in m)
                   for m in layer_t["shared"])
    ri = np.vectorize(remap.get)(sub_inds).astype(np.int32)
    return O.c_moe_ffn(xb[tokens], spec.act_dtype == "bfloat16", ri, wts[tokens], g, u, d, spec.bits,
                       spec.group_size, sh)


@pytest.mark.parametrize("spec,T", [(QWEN3_30B_A3B, 1), (QWEN3_30B_A3B, 8), (QWEN3_30B_A3B, 32),
                                    (QWEN3_30B_A3B, 64), (DEEPSEEK_V3, 1), (DEEPSEEK_V3, 32), (DEEPSEEK_V3, 64),
                                    (DEEPSEEK_V3, 256), (MIXTRAL_SMALL, 1)])
def test_full_size_layer_parity(spec, T):
    """Every token of a full-size decode batch against the oracle (routing bit
    for bit, FFN output within the tolerance)."""
    moe = _moe()
    layer = _torch_layer(spec, seed=11)
    m = moe.MoELayer.from_arrays(spec, layer)
    x = synthetic.make_x_torch(spec, T, seed=5)
    inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
    y = m(x, inds_out=inds, wts_out=wts, out_dtype=torch.float32)
    torch.cuda.synchronize()
    xb = _bits_of(x)
    gate = layer["gate_w"].cpu().numpy()
    eb = layer["e_bias"].cpu().numpy() if layer["e_bias"] is not None else None
    lg = O.c_router_logits(xb, spec.act_dtype == "bfloat16", gate.view(np.uint16), False)
    i_ref, w_ref = O.route(lg, _spec_router(spec), eb)
    np.testing.assert_array_equal(inds.cpu().numpy(), i_ref)
    np.testing.assert_array_equal(wts.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))
    tokens = np.arange(T)
    y_ref = _oracle_sampled(spec, layer, xb, i_ref, w_ref, tokens)
    assert_ffn_close(y.cpu().numpy(), y_ref, what=f"{spec.hidden}/{T}")
    del m, layer
    torch.cuda.empty_cache()


def test_permute_matches_numpy_counting_sort():
    """ef_permute against a numpy stable sort, with ragged expert counts, empty
    experts, a shared bin and a maximal-size histogram."""
    moe = _moe()
    rng = np.random.default_rng(3)
    for T, k, E, n_sh, seg in ((1, 1, 1, 0, 8), (37, 8, 128, 0, 8), (256, 8, 256, 256, 8), (4096, 8, 256, 0, 192),
                               (1000, 4, 512, 1000, 192), (5, 2, 16, 5, 8)):
        # skewed ids: a few hot experts, most empty
        p = rng.zipf(1.3, size=T * k) % E
        ents = p.astype(np.int32)
        got = moe.permute(torch.from_numpy(ents).cuda(), k, E, n_sh, seg)
        order = np.argsort(ents, kind="stable")
        counts = np.bincount(ents, minlength=E)
        nb = E + (1 if n_sh else 0)
        c_ref = np.concatenate([counts, [n_sh]]) if n_sh else counts
        off = np.concatenate([[0], np.cumsum(c_ref)])
        inv = np.empty(T * k, np.int64)
        inv[order] = np.arange(T * k)
        row_src = np.concatenate([order // k, np.arange(n_sh)]) if n_sh else order // k
        np.testing.assert_array_equal(got["counts"].cpu().numpy(), c_ref[:nb])
        np.testing.assert_array_equal(got["offsets"].cpu().numpy(), off)
        np.testing.assert_array_equal(got["inv"].cpu().numpy(), inv)
        np.testing.assert_array_equal(got["row_src"].cpu().numpy(), row_src)


def test_combine_matches_numpy_weighted_sum():
    """ef_combine: the k-order weighted sum with a shared row, fp32 and bf16 out."""
    moe = _moe()
    rng = np.random.default_rng(4)
    for T, k, H, sh in ((1, 8, 2048, False), (33, 8, 7168, True), (300, 2, 1024, False)):
        n = T * k + (T if sh else 0)
        rows = rng.standard_normal((n, H)).astype(np.float32)
        inv = rng.permutation(T * k).astype(np.int32)
        w = rng.random(T * k).astype(np.float32)
        r = torch.from_numpy(rows).cuda()
        y = moe.combine(r, torch.from_numpy(inv).cuda(), torch.from_numpy(w).cuda(), T, k,
                        T * k if sh else -1).cpu().numpy()
        acc = rows[inv].reshape(T, k, H) * w.reshape(T, k, 1)
        ref = acc[:, 0].astype(np.float32)
        for j in range(1, k):
            ref = ref + acc[:, j]
        if sh:
            ref = ref + rows[T * k:]
        # the kernel contracts each multiply-add (one rounding), numpy rounds twice
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
        yb = moe.combine(r, torch.from_numpy(inv).cuda(), torch.from_numpy(w).cuda(), T, k,
                         T * k if sh else -1, out_dtype=torch.bfloat16)
        assert torch.equal(yb, torch.from_numpy(y).cuda().to(torch.bfloat16))


def test_layer_deterministic_and_repeatable():
    moe = _moe()
    spec = QWEN3_30B_A3B
    m = moe.MoELayer.from_arrays(spec, _torch_layer(spec, 3))
    x = synthetic.make_x_torch(spec, 40, seed=9)
    a = m(x)
    b = m(x)
    assert torch.equal(a, b)
    # a token's output does not depend on the other tokens in the batch
    c = m(x[7:8].contiguous())
    assert torch.equal(a[7:8], c)


# ---------------------------------------------------------------- MLX op equivalents
@pytest.mark.parametrize("bits", [4, 8])
def test_dequantize_bit_exact(bits):
    moe = _moe()
    spec = MoESpec(hidden=512, n_experts=2, top_k=1, inter=256, bits=bits)
    layer = synthetic.make_layer_np(spec, 2)
    w, s, b = (a[1] for a in layer["gate"])
    got = moe.dequantize(torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
                         torch.from_numpy(b).cuda(), 64, bits)
    ref = O.c_dequantize(w, s, b, bits, 64)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    got16 = moe.dequantize(torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
                           torch.from_numpy(b).cuda(), 64, bits, torch.float16)
    np.testing.assert_array_equal(got16.cpu().numpy(), ref.astype(np.float16))


@pytest.mark.parametrize("bits,M", [(4, 1), (4, 5), (8, 3), (4, 70)])
def test_quantized_matmul(bits, M):
    moe = _moe()
    spec = MoESpec(hidden=1024, n_experts=1, top_k=1, inter=512, bits=bits)
    layer = synthetic.make_layer_np(spec, 4)
    w, s, b = (a[0] for a in layer["gate"])  # [512, 1024]
    xb = synthetic.make_x_np(spec, M, 8)
    x = _x_tensor(xb, spec)
    y = moe.quantized_matmul(x, torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
                             torch.from_numpy(b).cuda(), True, 64, bits)
    ref = O.bits_to_f32(xb, True).astype(np.float64) @ O.np_dequantize(w, s, b, bits, 64, np.float64).T
    assert_ffn_close(y.float().cpu().numpy(), ref, max_abs=2e-2, rel=4e-3, what="qmm (bf16 output)")


def test_gather_qmm_contract():
    moe = _moe()
    spec = MoESpec(hidden=512, n_experts=6, top_k=2, inter=256, bits=4)
    layer = synthetic.make_layer_np(spec, 6)
    w, s, b = layer["up"]
    lin = moe.QuantizedSwitchLinear(torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(s).cuda(),
                                    torch.from_numpy(b).cuda(), 64, 4)
    xb = synthetic.make_x_np(spec, 6, 3)
    x = _x_tensor(xb, spec).reshape(2, 3, 1, 1, 512)
    idx = torch.tensor([[[0, 5], [2, 2], [1, 3]], [[4, 0], [5, 5], [3, 1]]], dtype=torch.int32, device="cuda")
    y = lin(x, idx)
    assert tuple(y.shape) == (2, 3, 2, 1, 256)
    xf = O.bits_to_f32(xb, True).astype(np.float64)
    ii = idx.cpu().numpy().reshape(6, 2)
    for t in range(6):
        for j in range(2):
            ref = xf[t] @ O.np_dequantize(w[ii[t, j]], s[ii[t, j]], b[ii[t, j]], 4, 64, np.float64).T
            assert_ffn_close(y.reshape(6, 2, 256)[t, j].float().cpu().numpy(), ref, max_abs=2e-2, rel=4e-3)


def test_experts_forward_rows():
    moe = _moe()
    spec = MoESpec(hidden=512, n_experts=8, top_k=1, inter=256, bits=4)
    layer = synthetic.make_layer_np(spec, 12)
    m = moe.MoELayer.from_arrays(spec, layer)
    xb = synthetic.make_x_np(spec, 37, 1)
    ids = np.random.default_rng(0).integers(0, 8, 37).astype(np.int32)
    y = moe.experts_forward(m.switch_mlp, _x_tensor(xb, spec), torch.from_numpy(ids).cuda())
    ref = O.c_moe_ffn(xb, True, ids[:, None], np.ones((37, 1), np.float32), layer["gate"], layer["up"],
                      layer["down"], 4, 64, None)
    assert_ffn_close(y.cpu().numpy(), ref, what="experts_forward")


def test_empty_and_single_token_edges():
    moe = _moe()
    spec = QWEN3_30B_A3B
    m = moe.MoELayer.from_arrays(spec, _torch_layer(spec, 1))
    x = synthetic.make_x_torch(spec, 0)
    assert m(x).shape == (0, spec.hidden)
    # every token routed to the same experts: a full 32-row segment plus a ragged one
    gate = m.gate.weight.clone()
    m.gate.weight = torch.zeros_like(gate)
    x = synthetic.make_x_torch(spec, 45, seed=2)
    inds = torch.empty((45, spec.top_k), dtype=torch.int32, device="cuda")
    y = m(x, inds_out=inds)
    assert (inds.cpu().numpy() == np.arange(spec.top_k)[None]).all()
    m.gate.weight = gate
    assert torch.isfinite(y.float()).all()


# ---------------------------------------------------------------- grouped GEMM (tcgen05) path
@pytest.mark.parametrize("bits,shared,T,H,I", [(4, False, 160, 1024, 256), (8, False, 128, 1024, 256),
                                               (4, True, 200, 1024, 256), (8, True, 300, 1024, 256),
                                               # partial weight tiles (I % 128, H % 256 != 0) and experts
                                               # with more rows than one segment holds
                                               (8, True, 900, 1152, 192), (4, False, 1000, 1088, 320)])
def test_gemm_path_matches_oracle(bits, shared, T, H, I):
    moe = _moe()
    from expertflow_b200 import _lib as L

    spec = MoESpec(hidden=H, n_experts=16, top_k=4, inter=I, bits=bits, router="sigmoid_group" if shared else
                   "softmax", n_group=4 if shared else 1, topk_group=2 if shared else 1,
                   routed_scaling=2.5 if shared else 1.0, n_shared=1 if shared else 0, act_dtype="bfloat16",
                   e_bias_std=0.01)
    layer = synthetic.make_layer_np(spec, 31 + bits)
    xb = synthetic.make_x_np(spec, T, 7)
    x = _x_tensor(xb, spec)
    out = {}
    for path in (L.EF_PATH_GEMM, L.EF_PATH_GEMM_PAIR, L.EF_PATH_GEMV):
        m = moe.MoELayer.from_arrays(spec, layer, path=path)
        inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
        out[path] = (m(x, inds_out=inds, out_dtype=torch.float32), inds)
    torch.cuda.synchronize()
    i_ref, w_ref, y_ref = O.moe_forward(xb, True, layer["gate_w"].view(np.uint16), False, _spec_router(spec),
                                        layer["e_bias"], layer["gate"], layer["up"], layer["down"], bits, 64,
                                        layer["shared"])
    for path, (y, inds) in out.items():
        np.testing.assert_array_equal(inds.cpu().numpy(), i_ref)
        assert_ffn_close(y.cpu().numpy(), y_ref, what=f"path {path}")
    # the SM-pair kernel accumulates the same products in the same k order
    assert torch.equal(out[L.EF_PATH_GEMM][0], out[L.EF_PATH_GEMM_PAIR][0])


def test_prefill_deepseek_v3_8bit_sampled():
    """DeepSeek-V3-shaped prefill: 4096 tokens, 8-bit, grouped GEMM path."""
    moe = _moe()
    from expertflow_b200 import _lib as L

    spec = DEEPSEEK_V3_PREFILL_8BIT
    T = 4096
    layer = _torch_layer(spec, seed=41)
    m = moe.MoELayer.from_arrays(spec, layer, path=L.EF_PATH_GEMM)
    x = synthetic.make_x_torch(spec, T, seed=9)
    inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
    y = m(x, inds_out=inds, wts_out=wts, out_dtype=torch.float32)
    torch.cuda.synchronize()
    xb = _bits_of(x)
    lg = O.c_router_logits(xb, True, layer["gate_w"].cpu().numpy().view(np.uint16), False)
    i_ref, w_ref = O.route(lg, _spec_router(spec), layer["e_bias"].cpu().numpy())
    np.testing.assert_array_equal(inds.cpu().numpy(), i_ref)
    # every token routed to the two most-loaded experts (more rows than one
    # 192-row GEMM segment holds, so each spans two segments), plus the first
    # and last token of eight other experts and the batch's first and last
    ent = i_ref.reshape(-1)
    counts = np.bincount(ent, minlength=spec.n_experts)
    top2 = np.argsort(-counts, kind="stable")[:2]
    assert (counts[top2] > 192).all(), counts[top2]
    toks = set()
    for e in top2:
        toks.update((np.nonzero(ent == e)[0] // spec.top_k).tolist())
    for e in np.nonzero(counts)[0][:: max(1, len(np.nonzero(counts)[0]) // 8)][:8]:
        te = np.nonzero(ent == e)[0] // spec.top_k
        toks.update((int(te[0]), int(te[-1])))
    toks.update((0, T - 1))
    tokens = np.array(sorted(toks))
    y_ref = _oracle_sampled(spec, layer, xb, i_ref, w_ref, tokens)
    assert_ffn_close(y.cpu().numpy()[tokens], y_ref, what="prefill 8-bit")
    del m, layer
    torch.cuda.empty_cache()


@pytest.mark.parametrize("spec_name,T", [("qwen3-30b-a3b-moe", 1), ("qwen3-30b-a3b-moe", 64),
                                         ("mixtral-small-h1024-e16", 300)])
def test_captured_forward_equals_eager(spec_name, T):
    """The CUDA-graph-captured layer forward replays exactly the eager forward
    (decode GEMV and grouped-GEMM paths), with new inputs written into .x."""
    moe = _moe()
    from expertflow_b200 import _lib as L
    from expertflow_b200.spec import WORKLOADS

    spec = WORKLOADS[spec_name]
    layer = _torch_layer(spec, seed=8)
    m = moe.MoELayer.from_arrays(spec, layer, path=L.EF_PATH_GEMM if T >= 256 else L.EF_PATH_AUTO)
    dt = torch.bfloat16 if spec.act_dtype == "bfloat16" else torch.float16
    cf = m.capture(T, dt, out_dtype=torch.float32)
    for seed in (1, 2):
        x = synthetic.make_x_torch(spec, T, seed=seed)
        y_graph = cf(x).clone()
        y_eager = m(x, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(y_graph, y_eager)
    assert moe.device_error() == 0
