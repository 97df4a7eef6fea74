"""CPU tests of the C ABI: the library loads, exports every declared entry
point, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "navsampler.h")).read()
    return re.findall(r"NCB_API\s+[\w\s\*]+?\b(ncb_\w+)\s*\(", text)


def test_header_declares_the_boundary():
    names = declared_symbols()
    assert len(names) >= 12
    for must in ("ncb_sampler_create", "ncb_sample_rows_device", "ncb_sample_rows",
                 "ncb_logits_filter_top_p_device", "ncb_sampler_last_status"):
        assert must in names


def test_library_exports_every_declared_symbol(navlib):
    from neuraval_b200 import native
    for name in declared_symbols():
        assert hasattr(navlib, name), name
        assert name in native.SIGNATURES, name


def test_status_messages(navlib):
    for st in range(9):
        assert navlib.ncb_sampler_status_message(st)
    assert navlib.ncb_sampler_status_message(7) == b"invalid argument"


def test_null_and_invalid_arguments_are_rejected(navlib):
    from neuraval_b200 import native
    p = native.make_params(temperature=0.7, top_p=0.9, top_k=40)
    st = navlib.ncb_sample_rows_device(None, None, 1, 10, None, None, None, ctypes.byref(p),
                                       None, None, None, None)
    assert st == native.NCB_ERROR_NOT_INITIALIZED
    assert navlib.ncb_sampler_last_status() == st
    assert navlib.ncb_sampler_create(0, 0, 10, 10, ctypes.byref(ctypes.c_void_p())) == 7
    assert navlib.ncb_sampler_create(0, 1, 10, 10, None) == 7
    assert navlib.ncb_sampler_destroy(None) == 7


def test_create_without_a_device_reports_no_device(navlib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    st = navlib.ncb_sampler_create(0, 4, 1000, 16, ctypes.byref(h))
    assert st in (1, 2) and not h.value
