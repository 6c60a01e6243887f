"""The C ABI library loads, exports every entry point declared in
include/swiftlet_cuda.h, and reports errors without a GPU."""
import ctypes as C
import os
import re

import pytest

import swiftlet_b200 as swl
from conftest import ROOT, REF_FIXTURES


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "swiftlet_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(swl_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("swl_model_open", "swl_model_close", "swl_model_config", "swl_state_new", "swl_state_free",
              "swl_state_position", "swl_step", "swl_step_batch", "swl_pool_stats", "swl_pool_resize", "swl_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = C.CDLL(swl.library_path() if os.path.exists(swl.library_path()) else swl.lib()._name)
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert set(declared_symbols()) == set(swl._SIGNATURES)


def test_open_missing_dir_is_an_io_error(tmp_path):
    h = C.c_void_p()
    rc = swl.lib().swl_model_open(str(tmp_path / "nope").encode(), 0.0, 0, C.byref(h))
    assert rc == swl.SWL_ERR_IO
    assert b"config.json" in swl.lib().swl_last_error()


def test_open_malformed_config_is_a_format_error(tmp_path):
    (tmp_path / "config.json").write_text("{ not json")
    h = C.c_void_p()
    assert swl.lib().swl_model_open(str(tmp_path).encode(), 0.0, 0, C.byref(h)) == swl.SWL_ERR_FORMAT


def test_null_arguments_are_rejected():
    assert swl.lib().swl_model_open(None, 0.0, 0, None) == swl.SWL_ERR_INVALID
    assert swl.lib().swl_step(None, None, None, 0, None) == swl.SWL_ERR_INVALID
    assert swl.lib().swl_state_position(None) == -1
    out = (C.c_double * 4)()
    assert swl.lib().swl_ep_timing(None, 0, out) == swl.SWL_ERR_INVALID


def test_python_mirror_raises_without_gpu_or_loads_with_one():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: covered by the gpu tests")
    with pytest.raises(swl.SwiftletError) as e:
        swl.QwenCUDAModel(os.path.join(REF_FIXTURES, "tiny-model-q4"))
    assert e.value.code == swl.SWL_ERR_CUDA
