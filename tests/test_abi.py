"""The C-ABI library: it loads, exports every function include/laya_b200.h
declares (engine, front end, HTTP service), and fails with a status code (never an abort) when there is no GPU
or the arguments are bad.  No compute runs here."""
import ctypes
import os
import re

import pytest

from laya_rust_b200 import engine as E

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("laya_b200.h", "laya_frontend.h", "laya_serve.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(laya_[a-z0-9_]+)\s*\(", text))
    return sorted(names - {"laya_tap_fn"})


def test_header_declares_the_engine_seam():
    names = declared_functions()
    for n in ["laya_open", "laya_forward", "laya_info", "laya_close", "laya_last_error",
              "laya_upload_weight_f16", "laya_upload_weight_f32", "laya_finalize"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = E.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_open_without_a_usable_device_reports_an_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(E.LayaError) as ei:
        E.Engine(gguf_path=os.path.join(ROOT, "nope.gguf"))
    assert ei.value.code in (E.LAYA_E_CUDA, E.LAYA_E_INVALID)
    assert E.lib().laya_last_error().decode()


def test_null_arguments_are_rejected_with_a_status():
    lib = E.lib()
    assert lib.laya_open(0, None, None) == E.LAYA_E_INVALID
    assert lib.laya_forward(None, None, None, None) == E.LAYA_E_INVALID
    assert lib.laya_plan_stats(None, None, None, None) == E.LAYA_E_INVALID
    assert "null" in lib.laya_last_error().decode()
    lib.laya_close(None)  # no-op


def test_front_end_and_service_reject_bad_arguments_with_a_status():
    """The front-end and HTTP-service entry points: null or out-of-range
    arguments come back as LAYA_E_INVALID with a message, never an abort."""
    from laya_rust_b200 import frontend as FE, serve as S
    L = S.lib()
    FE.lib()
    out = ctypes.c_void_p()
    n = ctypes.c_int64()
    assert L.laya_serve_open(None, ctypes.byref(out)) == E.LAYA_E_INVALID
    assert L.laya_serve_stop(None) == E.LAYA_E_INVALID
    assert L.laya_serve_wait(None) == E.LAYA_E_INVALID
    assert L.laya_serve_stats(None, None, 0) == E.LAYA_E_INVALID
    L.laya_serve_close(None)  # no-op
    assert L.laya_requests_merge(None, 2, ctypes.byref(out)) == E.LAYA_E_INVALID
    assert L.laya_requests_merge(None, 0, None) == E.LAYA_E_INVALID
    assert L.laya_requests_pack_windows(None, 16384, 4, ctypes.byref(n)) == E.LAYA_E_INVALID
    assert L.laya_requests_pack(None, 16384, 0, ctypes.byref(n)) == E.LAYA_E_INVALID
    assert E.lib().laya_last_error().decode()
