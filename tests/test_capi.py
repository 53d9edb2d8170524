"""The C-ABI library loads, exports every symbol include/sbb200.h declares, and
its host-side validation answers without touching a GPU."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "sbb200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(sbb200_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol(sbb):
    lib_path = sbb.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (sbb200_\w+)", out))
    declared = declared_symbols()
    assert declared, "no declarations parsed"
    assert declared <= exported, f"missing exports: {sorted(declared - exported)}"
    lib = sbb.lib()
    for name in declared:
        assert hasattr(lib, name)


def test_abi_version(sbb):
    assert sbb.lib().sbb200_abi_version() == 1


def test_workspace_query_is_host_only(sbb):
    n1 = sbb.nvfp4_moe_workspace_bytes(64, 170, 8, 4096, 1280)
    n2 = sbb.nvfp4_moe_workspace_bytes(128, 170, 8, 4096, 1280)
    assert 0 < n1 < n2
    assert n1 % 256 == 0


def _call(lib, M=4, E=8, top_k=2, K=256, I=64, act=2, out_dt=0, ptr=1, ws_bytes=1 << 40):
    P = ctypes.c_void_p(ptr) if ptr else None
    return lib.sbb200_nvfp4_moe(None, P, P, P, P, P, P, P, P, P, P, ws_bytes, P, out_dt, M, E,
                                top_k, K, I, act, 1)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(K=48), -1, "multiples of 32"),
    (dict(I=40), -1, "multiples of 32"),
    (dict(M=0), -1, "nonzero"),
    (dict(act=7), -1, "dtypes"),
    (dict(out_dt=9), -1, "dtypes"),
    (dict(E=513), -4, "E above"),
    (dict(top_k=65), -4, "top_k above"),
    (dict(ptr=0), -1, "null pointer"),
    (dict(ws_bytes=16), -2, "workspace"),
])
def test_nvfp4_moe_validation(sbb, kw, code, msg):
    lib = sbb.lib()
    assert _call(lib, **kw) == code
    assert msg in sbb.last_error()


def test_last_error_truncation(sbb):
    lib = sbb.lib()
    _call(lib, K=48)
    n = lib.sbb200_last_error(None, 0)
    assert n > 8
    buf = ctypes.create_string_buffer(8)
    assert lib.sbb200_last_error(buf, 8) == n
    assert len(buf.value) == 7


def test_create_rejects_bad_shape_without_device(sbb):
    lib = sbb.lib()
    assert not lib.sbb200_create(0, 0, 8, 170, 4096, 1280)
    assert "max_tokens" in sbb.last_error()
    assert not lib.sbb200_create(0, 16, 8, 170, 4095, 1280)


def test_codec_validation(sbb):
    lib = sbb.lib()
    P = ctypes.c_void_p(1)
    assert lib.sbb200_nvfp4_dequant(None, P, P, P, 1, P, 4, 24) == -1
    assert "multiple of 16" in sbb.last_error()
    assert lib.sbb200_nvfp4_quantize(None, P, 5, P, 1, P, P, 4, 32) == -1
    assert lib.sbb200_route_plan(None, P, 4, 2, 0, P, P, P, P, P, None) == -1


def test_health_rejects_null(sbb):
    assert sbb.lib().sbb200_health(None, None, None, 0) == -1


def test_router_topk_validation(sbb):
    L = sbb.lib()
    assert L.sbb200_router_topk(None, None, 7, 4, 8, 2, None, None) == -1  # dtype
    assert "dtype" in sbb.last_error()
    assert L.sbb200_router_topk(None, None, 0, 4, 8, 9, None, None) == -1  # top_k > E
    assert "top_k" in sbb.last_error()
    assert L.sbb200_router_topk(None, None, 0, 4, 600, 2, None, None) == -1  # E > 512
    assert L.sbb200_router_topk(None, None, 0, 0, 8, 2, None, None) == 0    # no tokens: no work
    assert L.sbb200_router_topk(None, None, 0, 4, 8, 2, None, None) == -1  # null pointers
    assert "null" in sbb.last_error()


def test_w4a4_static_scales_come_together(sbb):
    import ctypes
    L = sbb.lib()
    dummy = ctypes.c_void_p(16)
    args = [None, dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy, dummy,
            dummy, None, None, None,   # a13_gscale only: incomplete static set
            dummy, 1 << 30, dummy, 2, 4, 8, 2, 512, 256, 2, 1, None, 0]
    assert L.sbb200_nvfp4_moe_w4a4(*args) == -1
    assert "together" in sbb.last_error()


def test_from_logits_validation(sbb):
    import ctypes
    L = sbb.lib()
    d = ctypes.c_void_p(16)
    base = [None, d, d, 2, d, d, d, d, d, d, d, d, d, 1 << 30, d, 2, 4, 8, 2, 512, 256, 2, 1]
    bad_dt = list(base)
    bad_dt[3] = 9
    assert L.sbb200_nvfp4_moe_from_logits(*bad_dt) == -1
    assert "dtype" in sbb.last_error()
    big_k = list(base)
    big_k[18] = 9  # top_k > E
    assert L.sbb200_nvfp4_moe_from_logits(*big_k) == -1
    assert "top_k" in sbb.last_error()
