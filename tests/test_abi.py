"""C-ABI library checks that need no GPU: it loads, exports every symbol the
public header declares, and rejects bad arguments on the host."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "efmoe.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ef_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    from expertflow_b200 import build, _lib

    build.build()
    return _lib


def test_header_declares_entry_points():
    names = _declared()
    for n in ("ef_moe_forward", "ef_router_topk", "ef_quantized_matmul", "ef_dequantize", "ef_gather_qmm",
              "ef_moe_experts_forward", "ef_moe_workspace_size"):
        assert n in names


def test_library_exports_every_declared_symbol(L):
    lib = L.lib()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes signature table covers the header
    assert set(_declared()) <= set(L.SIGNATURES), set(_declared()) - set(L.SIGNATURES)


def test_version_and_status_strings(L):
    assert "sm_100a" in L.version()
    assert L.lib().ef_status_string(-4).decode() == "workspace too small"


def _cfg(L, **kw):
    base = dict(hidden=2048, inter=768, n_experts=128, top_k=8, bits=4, group_size=64, router_mode=0, norm_topk=1,
                n_group=1, topk_group=1, routed_scaling=1.0, n_shared=0, shared_inter=0, act_dtype=0,
                gate_dtype=1, path=0)
    base.update(kw)
    return L.MoECfg(**base)


def test_workspace_sizes_grow_with_tokens(L):
    lib = L.lib()
    c = _cfg(L)
    sizes = [lib.ef_moe_workspace_size(ctypes.byref(c), T) for T in (1, 8, 64, 512)]
    assert all(s > 0 for s in sizes) and sizes == sorted(sizes)
    c2 = _cfg(L, hidden=7168, inter=2048, n_experts=256, router_mode=1, n_group=8, topk_group=4,
              routed_scaling=2.5, n_shared=1, shared_inter=2048)
    assert lib.ef_moe_workspace_size(ctypes.byref(c2), 256) > lib.ef_moe_workspace_size(ctypes.byref(c), 256)


@pytest.mark.parametrize("kw,status", [
    (dict(bits=3), -2), (dict(group_size=32), -2), (dict(hidden=1000), -2), (dict(inter=96), -2), (dict(top_k=0), -2),
    (dict(n_experts=0), -2), (dict(router_mode=7), -1), (dict(router_mode=1, n_group=3), -2),
    (dict(router_mode=1, n_group=8, topk_group=9), -1), (dict(n_shared=1, shared_inter=512), -2),
    (dict(act_dtype=2), -2),
])
def test_forward_rejects_bad_config_on_host(L, kw, status):
    lib = L.lib()
    c = _cfg(L, **kw)
    q = L.QWeight(16, 16, 16)
    rc = lib.ef_moe_forward(ctypes.byref(c), 16, 1, 16, None, q, q, q, None, None, None, 16, None, None, 16,
                            1 << 30, None)
    assert rc == status, (kw, rc, lib.ef_last_error_message())


def test_forward_rejects_null_and_misaligned_pointers(L):
    lib = L.lib()
    c = _cfg(L)
    q = L.QWeight(16, 16, 16)
    assert lib.ef_moe_forward(ctypes.byref(c), None, 1, 16, None, q, q, q, None, None, None, 16, None, None, 16,
                              1 << 30, None) == -1
    bad = L.QWeight(18, 16, 16)
    assert lib.ef_moe_forward(ctypes.byref(c), 16, 1, 16, None, bad, q, q, None, None, None, 16, None, None, 16,
                              1 << 30, None) == -1
    assert lib.ef_moe_forward(ctypes.byref(c), 16, 1, 16, None, q, q, q, None, None, None, 16, None, None, 16,
                              8, None) == -4
    # zero tokens is a no-op
    assert lib.ef_moe_forward(ctypes.byref(c), 16, 0, 16, None, q, q, q, None, None, None, 16, None, None, 16,
                              8, None) == 0


def test_qmm_and_dequant_validation(L):
    lib = L.lib()
    assert lib.ef_quantized_matmul(16, 0, 4, 16, 16, 16, 64, 100, 4, 64, 16, 16, 1 << 30, None) == -2
    assert lib.ef_quantized_matmul(16, 0, 4, 16, 16, 16, 64, 96, 4, 64, 16, 16, 1 << 30, None) == -2
    assert lib.ef_quantized_matmul(16, 0, 4, 16, 16, 16, 60, 256, 4, 64, 16, 16, 1 << 30, None) == -2
    assert lib.ef_dequantize(16, 16, 16, 4, 64, 5, 64, 16, 2, None) == -2
    assert lib.ef_dequantize(16, 16, 16, 0, 64, 4, 64, 16, 2, None) == 0
    assert lib.ef_gather_qmm(16, 0, 2, 16, 0, L.QWeight(16, 16, 16), 4, 64, 256, 4, 64, 16, 16, 1 << 30,
                             None) == -1
