"""GGUF K-quants: the reader, the oracle and the GPU kernels against the
reference's own decoders (tests/golden/kquant_gguf.npz, made by
tests/golden/make_gguf_golden.py from ef_deepseek_mmap.py).

CPU: the oracle's Q2_K / Q3_K / Q4_K decode equals the reference's output bit
for bit (including blocks with arbitrary fp16 super-block scales); the scalar
and vectorised Q2_K decoders agree as the reference's own test asks
(tests/test_gguf_loader.py:139-151); tensor byte sizes, the parse of a
two-file model and every expert's byte range match the reference; the
reader's error behaviour follows the reference's parser tests
(tests/test_gguf_loader.py:94-136).
GPU: ef_kquant_dequantize is bit-exact with the reference; ef_kquant_matmul
is within the fp tolerance of the oracle over every format, token count and
both activation dtypes (Q4_K within the bound of the reference's fp16 rounding
of each weight, since its GEMV contracts the exact weights).
"""
import hashlib
import importlib.util
import json
import os
import struct

import numpy as np
import pytest

from conftest import REPO
from expertflow_b200 import gguf as G
from oracle import oracle as O

GOLDEN = os.path.join(REPO, "tests", "golden", "kquant_gguf.npz")
TYPES = (G.GGML_TYPE_Q2_K, G.GGML_TYPE_Q3_K, G.GGML_TYPE_Q4_K)


def _gen():
    spec = importlib.util.spec_from_file_location("make_gguf_golden",
                                                  os.path.join(REPO, "tests", "golden", "make_gguf_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _same_f16(got_bits, want_bits):
    got, want = np.asarray(got_bits, np.uint16), np.asarray(want_bits, np.uint16)
    nan = np.isnan(want.view(np.float16))
    assert np.isnan(got.view(np.float16)[nan]).all()
    np.testing.assert_array_equal(got[~nan], want[~nan])


@pytest.fixture(scope="module")
def Z():
    return np.load(GOLDEN)


@pytest.mark.parametrize("dtype", TYPES)
def test_oracle_matches_reference_decoders(Z, dtype):
    _same_f16(O.np_dequant_kquant(Z[f"blocks_{dtype}"].tobytes(), dtype).view(np.uint16), Z[f"dequant_{dtype}"])


def test_q2k_scalar_and_fast_agree(Z):
    scalar = Z["q2k_scalar"].view(np.float16).astype(np.float32)
    fast = Z[f"dequant_{G.GGML_TYPE_Q2_K}"][:1024].view(np.float16).astype(np.float32)
    np.testing.assert_allclose(scalar, fast, atol=1e-2)
    ours = O.np_dequant_kquant(Z[f"blocks_{G.GGML_TYPE_Q2_K}"][:4 * 84].tobytes(), G.GGML_TYPE_Q2_K)
    np.testing.assert_allclose(ours.astype(np.float32), scalar, atol=1e-2)


def test_tensor_byte_sizes(Z):
    for row in Z["byte_sizes"]:
        dt, a, b, c, nd, want = (int(v) for v in row)
        shape = (a, b, c)[:nd]
        assert G.tensor_byte_size(shape, dt) == want, (dt, shape)
    with pytest.raises(ValueError, match="Unsupported GGML type"):
        G.tensor_byte_size((256,), 999)
    assert G.tensor_byte_size((257,), G.GGML_TYPE_F16) == 514


def test_parse_and_expert_ranges_match_reference(Z, tmp_path):
    gen = _gen()
    paths = gen.write_model(str(tmp_path))
    assert [hashlib.sha256(open(p, "rb").read()).hexdigest() for p in paths] == list(Z["model_file_sha"])
    infos, tensors, meta = G.parse_split_gguf(str(tmp_path))
    want = json.loads(str(Z["parsed_json"]))
    assert [i.data_offset for i in infos] == want["data_offsets"]
    assert [i.alignment for i in infos] == want["alignments"]
    assert [i.version for i in infos] == want["versions"]
    assert json.loads(json.dumps(meta)) == want["metadata"]
    got = {n: [list(t.shape), t.dtype, t.offset, t.file_idx, t.total_bytes] for n, t in sorted(tensors.items())}
    assert got == want["tensors"]
    ex = G.GGUFExperts(str(tmp_path))
    assert ex.layers() == [1, 2] and ex.n_experts == 4
    for layer, e, proj, dt, shape, raw_sha, deq_sha in Z["experts"]:
        raw, dtype, shp = ex.load_expert_raw(int(layer), int(e), str(proj))
        assert dtype == int(dt) and list(shp) == json.loads(str(shape))
        assert hashlib.sha256(raw).hexdigest() == raw_sha
        deq = O.np_dequant_kquant(raw, dtype)
        assert hashlib.sha256(deq.view(np.uint16).tobytes()).hexdigest() == deq_sha, (layer, e, proj)
    raw, dt, _ = ex.load_expert_raw(1, 2, "down")
    _same_f16(O.np_dequant_kquant(raw, dt).view(np.uint16)[:8192], Z["expert_1_2_down"])
    with pytest.raises(KeyError):
        ex.expert(1, 4, "gate")
    with pytest.raises(KeyError):
        ex.expert(3, 0, "gate")


def test_per_expert_tensors(tmp_path):
    """Mixtral-style files name each expert's tensor (blk.{i}.ffn_{proj}.{e}.weight)."""
    rng = np.random.default_rng(3)
    t = {}
    for e in range(3):
        for proj in ("gate", "up", "down"):
            t[f"blk.0.ffn_{proj}.{e}.weight"] = ((256, 32), G.GGML_TYPE_Q4_K,
                                                 G.random_kquant_blocks(G.GGML_TYPE_Q4_K, 32, rng))
    p = str(tmp_path / "mixtral.gguf")
    G.write_gguf(p, t, {"llama.expert_count": 3})
    ex = G.GGUFExperts(p)
    for e in range(3):
        raw, dt, shape = ex.load_expert_raw(0, e, "up")
        assert raw == t[f"blk.0.ffn_up.{e}.weight"][2] and dt == G.GGML_TYPE_Q4_K and shape == (256, 32)


def test_parser_errors_follow_reference(tmp_path):
    with pytest.raises(FileNotFoundError):
        G.parse_gguf("/nonexistent/path/model.gguf")
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"\x00" * 104)
    with pytest.raises(ValueError, match="Not a GGUF file"):
        G.parse_gguf(str(bad))
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(struct.pack("<I", G.GGUF_MAGIC))
    with pytest.raises(struct.error):
        G.parse_gguf(str(trunc))
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    with pytest.raises(struct.error):
        G.parse_gguf(str(empty))
    minimal = tmp_path / "minimal.gguf"
    minimal.write_bytes(struct.pack("<IIQQ", G.GGUF_MAGIC, 3, 0, 0))
    info = G.parse_gguf(str(minimal))
    assert info.n_tensors == 0 and info.version == 3 and info.metadata == {} and info.tensors == {}
    d = tmp_path / "empty_dir"
    d.mkdir()
    with pytest.raises(FileNotFoundError, match="No .gguf files"):
        G.parse_split_gguf(str(d))
    with pytest.raises(FileNotFoundError):
        G.parse_split_gguf("/nonexistent/model_dir")


def test_writer_rejects_wrong_sizes(tmp_path):
    with pytest.raises(ValueError):
        G.write_gguf(str(tmp_path / "x.gguf"), {"t": ((256,), G.GGML_TYPE_Q2_K, b"\0" * 83)})


# ---------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def K():
    from expertflow_b200 import build

    build.build()
    from expertflow_b200 import kquant

    return kquant


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", TYPES)
def test_gpu_dequantize_bit_exact(K, Z, dtype):
    import torch

    raw = torch.from_numpy(Z[f"blocks_{dtype}"].copy()).cuda()
    got = K.dequantize(raw, dtype).cpu().numpy().view(np.uint16)
    _same_f16(got, Z[f"dequant_{dtype}"])
    rng = np.random.default_rng(dtype)
    big = G.random_kquant_blocks(dtype, 4096 + 7, rng)  # a ragged count of blocks
    got = K.dequantize(torch.from_numpy(np.frombuffer(big, np.uint8).copy()).cuda(), dtype).cpu().numpy()
    _same_f16(got.view(np.uint16), O.np_dequant_kquant(big, dtype).view(np.uint16))


@pytest.mark.gpu
def test_gpu_dequantize_model_experts(K, Z, tmp_path):
    gen = _gen()
    gen.write_model(str(tmp_path))
    ex = G.GGUFExperts(str(tmp_path))
    for layer, e, proj, dt, shape, raw_sha, deq_sha in Z["experts"]:
        blocks, dtype, _ = K.load_expert(ex, int(layer), int(e), str(proj))
        got = K.dequantize(blocks, dtype).cpu().numpy().view(np.uint16)
        assert hashlib.sha256(got.tobytes()).hexdigest() == deq_sha, (layer, e, proj)


def _check_close(y, ref, bound=None):
    """Within 2e-2 absolute (or, with `bound`, within it elementwise) and 1e-3
    relative L2 of the oracle."""
    y = np.asarray(y, np.float64)
    err = np.abs(y - ref)
    rel_l2 = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    ok = (err <= bound).all() if bound is not None else err.max() <= 2e-2
    assert ok and rel_l2 <= 1e-3, (float(err.max()), float(rel_l2))


def _q4_bound(x, raw, dtype, N, K):
    """Q4_K: the kernel contracts the exact weights A q - B (codes on the tensor
    cores, scale and min folded in fp32), the oracle the reference's fp16
    weights RN16(A q - B); they differ by at most half an fp16 ulp per weight,
    2^-11 |w|, so |y - ref| <= 2^-10 sum |x| |w| (twice that, for the fp32
    accumulation) + 1e-5.  Other formats: None (the 2e-2 bar)."""
    if dtype != G.GGML_TYPE_Q4_K:
        return None
    w = np.abs(O.np_dequant_kquant(raw, dtype).astype(np.float64).reshape(N, K))
    return 2.0 ** -10 * (np.abs(np.asarray(x, np.float64)) @ w.T) + 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", TYPES)
@pytest.mark.parametrize("T", [1, 3, 8, 13, 24, 32])
def test_gpu_matmul_matches_oracle(K, dtype, T):
    import torch

    rng = np.random.default_rng(10 * dtype + T)
    for N, Kd in ((2048, 2048), (64, 768), (16, 256)):  # split-K tiles, odd block counts, one block per row
        raw = G.random_kquant_blocks(dtype, N * Kd // 256, rng)
        x = rng.standard_normal((T, Kd)).astype(np.float32)
        for act in (torch.bfloat16, torch.float16):
            xt = torch.from_numpy(x).to(act).cuda()
            xf = xt.float().cpu().numpy()
            ref = O.np_kquant_matmul(xf, raw, dtype, N, Kd)
            y = K.matmul(xt, torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda(), dtype, N, Kd)
            _check_close(y.cpu().numpy(), ref, _q4_bound(xf, raw, dtype, N, Kd))
    from expertflow_b200.moe import device_error
    assert device_error() == 0


@pytest.mark.gpu
def test_gpu_matmul_large_and_deterministic(K):
    """A matrix far larger than the SMs' tiles (no split), run twice: identical."""
    import torch

    rng = np.random.default_rng(5)
    N, Kd, dtype = 8192, 7168, G.GGML_TYPE_Q4_K
    raw = G.random_kquant_blocks(dtype, N * Kd // 256, rng)
    w = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda()
    x = torch.from_numpy(rng.standard_normal((4, Kd)).astype(np.float32)).to(torch.bfloat16).cuda()
    y1, y2 = K.matmul(x, w, dtype, N, Kd), K.matmul(x, w, dtype, N, Kd)
    assert torch.equal(y1, y2)
    xf = x.float().cpu().numpy()
    _check_close(y1.cpu().numpy(), O.np_kquant_matmul(xf, raw, dtype, N, Kd), _q4_bound(xf, raw, dtype, N, Kd))


@pytest.mark.gpu
def test_gpu_matmul_rejects_and_flags(K):
    import torch
    from expertflow_b200 import _lib as L
    from expertflow_b200.moe import device_error

    w = torch.zeros(16 * 84, dtype=torch.uint8, device="cuda")
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        K.matmul(x, w, 13, 16, 256)            # Q5_K: refused by the wrapper ...
    y = torch.empty((1, 16), dtype=torch.float32, device="cuda")
    ws = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    st = L.lib().ef_kquant_matmul(x.data_ptr(), L.EF_DT_BF16, 1, w.data_ptr(), 13, 16, 256, y.data_ptr(),
                                  ws.data_ptr(), ws.numel(), None)
    assert st == -2                            # ... and by the C ABI (EF_ERR_UNSUPPORTED)
    with pytest.raises(L.EfmoeError):
        K.matmul(torch.zeros((1, 200), dtype=torch.bfloat16, device="cuda"), w, 10, 16, 200)  # K % 256
    with pytest.raises(L.EfmoeError):
        K.matmul(torch.zeros((33, 256), dtype=torch.bfloat16, device="cuda"), w, 10, 16, 256)  # T > 32
    x[0, 5] = float("inf")                     # outside fp16: flagged on the device, not silently clipped
    K.matmul(x, w, 10, 16, 256)
    torch.cuda.synchronize()
    assert device_error() != 0
    assert device_error() == 0
