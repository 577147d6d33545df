"""ef_moe_forward_noalloc: the layer forward for callers that cannot allocate
device memory (an FFI host without a CUDA allocator of its own, or a decode
loop that must not call cudaMalloc).  It must give the same output as
ef_moe_forward with a caller workspace, on consecutive calls that reuse the
library's fixed scratch array.  Collected last so that a failure here comes
after every other test has run."""
import ctypes

import numpy as np
import pytest

from conftest import assert_ffn_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _call_noalloc(L, m, x, y, inds, wts):
    cfg = m.cfg(L.EF_DT_BF16 if x.dtype == torch.bfloat16 else L.EF_DT_F16)
    cfg.out_f32 = int(y.dtype == torch.float32)
    sp = m.switch_mlp
    sh = m.shared_experts
    sq = [ctypes.byref(p.qweight()) for p in (sh.gate_proj, sh.up_proj, sh.down_proj)] if sh else [None] * 3
    eb = m.gate.e_score_correction_bias
    return L.lib().ef_moe_forward_noalloc(
        ctypes.byref(cfg), x.data_ptr(), x.shape[0], m.gate.weight.data_ptr(),
        eb.data_ptr() if eb is not None else None, sp.gate_proj.qweight(), sp.up_proj.qweight(),
        sp.down_proj.qweight(), sq[0], sq[1], sq[2], y.data_ptr(), inds.data_ptr(), wts.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("which", ["qwen3", "deepseek"])
def test_noalloc_matches_workspace_entry_point_twice(which):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build, moe, synthetic, _lib as L
    from expertflow_b200.spec import QWEN3_30B_A3B, DEEPSEEK_V3

    build.build()
    spec = QWEN3_30B_A3B if which == "qwen3" else DEEPSEEK_V3
    m = moe.MoELayer.from_arrays(spec, synthetic.make_layer_torch(spec, seed=21))
    for call, T in enumerate((48, 5)):  # two calls in a row with different batches
        x = synthetic.make_x_torch(spec, T, seed=100 + call)
        y_ref = m(x, out_dtype=torch.float32)
        y = torch.full((T, spec.hidden), float("nan"), dtype=torch.float32, device="cuda")
        inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
        wts = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
        rc = _call_noalloc(L, m, x, y, inds, wts)
        assert rc == 0, L.lib().ef_last_error_message()
        torch.cuda.synchronize()
        # the same kernels on the same inputs: identical, not merely close
        assert torch.equal(y, y_ref), f"noalloc call {call} differs from ef_moe_forward"
        assert_ffn_close(y.cpu().numpy(), y_ref.cpu().numpy(), what=f"noalloc call {call}")
        inds2 = torch.empty_like(inds)
        m(x, inds_out=inds2)
        assert torch.equal(inds, inds2)
    assert moe.device_error() == 0


def test_noalloc_rejects_batches_beyond_the_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from expertflow_b200 import build, moe, synthetic, _lib as L
    from expertflow_b200.spec import QWEN3_30B_A3B

    build.build()
    spec = QWEN3_30B_A3B
    m = moe.MoELayer.from_arrays(spec, synthetic.make_layer_torch(spec, seed=22))
    cfg = m.cfg(L.EF_DT_BF16)
    T = 1
    while L.lib().ef_moe_workspace_size(ctypes.byref(cfg), T) <= (64 << 20):
        T *= 2
    x = synthetic.make_x_torch(spec, T, seed=3)
    y = torch.empty((T, spec.hidden), dtype=torch.bfloat16, device="cuda")
    inds = torch.empty((T, spec.top_k), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, spec.top_k), dtype=torch.float32, device="cuda")
    rc = _call_noalloc(L, m, x, y, inds, wts)
    assert rc == -4  # EF_ERR_WORKSPACE
    assert b"scratch" in L.lib().ef_last_error_message()
