"""The C ABI library loads, exports every function include/*.h declares, and
applies the reference's argument checks (src/api/c/mlipcpp_api.cpp) without
touching a GPU."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT
import mlipcpp_b200 as mb

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(mlipcpp_\w+)\s*\(", text))
    return sorted(names)


def test_headers_declare_reference_api():
    names = set(declared_functions())
    reference_api = {  # include/mlipcpp/mlipcpp.h:36-463 of the reference
        "mlipcpp_version", "mlipcpp_error_string", "mlipcpp_get_last_error", "mlipcpp_set_backend",
        "mlipcpp_get_backend_name", "mlipcpp_backend_is_gpu", "mlipcpp_is_backend_available",
        "mlipcpp_suppress_logging", "mlipcpp_model_options_default", "mlipcpp_model_create",
        "mlipcpp_model_load", "mlipcpp_model_free", "mlipcpp_model_get_cutoff",
        "mlipcpp_predict_options_default", "mlipcpp_predict", "mlipcpp_predict_ptr",
        "mlipcpp_predict_with_options", "mlipcpp_predict_ptr_with_options",
        "mlipcpp_result_get_energy", "mlipcpp_result_get_forces", "mlipcpp_result_get_stress",
        "mlipcpp_result_n_atoms", "mlipcpp_result_has_forces", "mlipcpp_result_has_stress",
        "mlipcpp_result_free"}
    assert reference_api <= names


@pytest.mark.parametrize("name", declared_functions())
def test_symbol_exported(name):
    lib = ctypes.CDLL(mb.LIB_PATH)
    assert hasattr(lib, name)


def test_struct_layouts():
    # mlipcpp_system_t / options must keep the reference's C layout
    assert ctypes.sizeof(mb._System) == 40
    assert ctypes.sizeof(mb._ModelOptions) == 12
    assert ctypes.sizeof(mb._PredictOptions) == 3


def test_basic_calls_without_gpu():
    L = mb.lib()
    assert mb.version().count(".") == 2
    assert L.mlipcpp_error_string(0) == b"Success"
    assert L.mlipcpp_error_string(9) == b"Operation not supported"
    assert L.mlipcpp_error_string(1234) == b"Unknown error"
    o = mb._ModelOptions()
    assert L.mlipcpp_model_options_default(ctypes.byref(o)) == 0
    assert (o.backend, o.precision, o.cutoff_override) == (0, 0, 0.0)
    p = mb._PredictOptions()
    assert L.mlipcpp_predict_options_default(ctypes.byref(p)) == 0
    assert (p.compute_forces, p.compute_stress, p.use_nc_forces) == (True, False, False)
    assert L.mlipcpp_model_options_default(None) == mb.NULL_POINTER
    assert L.mlipcpp_get_last_error() == b"NULL pointer for options"
    c = ctypes.c_float()
    assert L.mlipcpp_model_get_cutoff(None, ctypes.byref(c)) == mb.INVALID_HANDLE
    r = ctypes.c_void_p()
    assert L.mlipcpp_predict(None, None, True, ctypes.byref(r)) == mb.INVALID_HANDLE
    e = ctypes.c_float()
    assert L.mlipcpp_result_get_energy(None, ctypes.byref(e)) == mb.INVALID_HANDLE
    L.mlipcpp_result_free(None)
    L.mlipcpp_model_free(None)
    h = L.mlipcpp_model_create(None)
    assert h
    assert L.mlipcpp_model_get_cutoff(h, ctypes.byref(c)) == mb.MODEL_NOT_LOADED
    assert L.mlipcpp_model_load(h, None) == mb.NULL_POINTER
    L.mlipcpp_model_free(h)
    assert not L.mlipcpp_is_backend_available(mb.Backend.CPU)


def test_load_without_gpu_fails_loudly(model_file):
    if mb.lib().mlipcpp_backend_is_gpu():
        pytest.skip("a GPU is present")
    with pytest.raises(mb.MLIPError) as ei:
        mb.Predictor(model_file("tiny"))
    assert ei.value.code == mb.BACKEND


def test_python_api_surface():
    for name in ("predict", "predict_with_options", "predict_batch", "predict_device", "cutoff",
                 "model_type", "set_timing", "last_timings", "last_shape"):
        assert hasattr(mb.Predictor, name)


def test_neighbor_list_rejects_bad_cutoff_before_device_work():
    L = mb.lib()
    fn = L.mlipcpp_b200_neighbor_list
    pos = (ctypes.c_float * 3)(0.0, 0.0, 0.0)
    cell = (ctypes.c_float * 9)(10, 0, 0, 0, 10, 0, 0, 0, 10)
    for bad in (0.0, -2.0, float("nan"), float("inf")):
        rc = fn(1, pos, cell, None, ctypes.c_float(bad), 0, None, None, None, None, None)
        assert rc == -mb.INVALID_PARAMETER, bad
        assert b"cutoff" in L.mlipcpp_get_last_error()


def test_device_allocation_counter_exported():
    assert mb.lib().mlipcpp_b200_device_allocations() >= 0
