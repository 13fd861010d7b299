"""The C-ABI library loads and exports every symbol include/qlinear.h declares (CPU only:
no compute call is made without a GPU)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qlinear.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"QLINEAR_API\s+[\w\s\*]*?\b(qlinear_\w+)\s*\(", text)))


def test_header_declares_the_api():
    syms = declared_symbols()
    for name in ("qlinear_backend_create", "qlinear_weights_create", "qlinear_run_f32",
                 "qlinear_run_swiglu_f32", "qlinear_run_device", "qlinear_strerror"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from open_rknpu2_lm_infer_b200 import _lib
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\b(qlinear_\w+)\b", out))
    assert set(declared_symbols()) <= exported
    # nothing else leaks out under the qlinear_ prefix
    assert exported <= set(declared_symbols())


def test_python_signatures_cover_the_header():
    from open_rknpu2_lm_infer_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_only_calls():
    from open_rknpu2_lm_infer_b200 import _lib
    lib = _lib.load()
    assert lib.qlinear_strerror(0) == b"ok"
    assert lib.qlinear_strerror(-5) == b"device wait timed out"
    assert lib.qlinear_version().startswith(b"qlinear-b200")


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from open_rknpu2_lm_infer_b200 import Backend, NpuError
    with pytest.raises(NpuError):
        Backend(device=0)


def test_no_cpu_fallback_when_library_missing(tmp_path):
    from open_rknpu2_lm_infer_b200 import _lib
    with pytest.raises(_lib.QLinearUnavailable):
        _lib.load(str(tmp_path / "libqlinear_b200.so"))


def test_noalloc_limits_match_the_header():
    """The Python constants of the allocation-free call's limits are the header's."""
    from open_rknpu2_lm_infer_b200 import _lib
    text = open(HEADER).read()
    defs = dict(re.findall(r"#define\s+(QLINEAR_NOALLOC_\w+)\s+(\d+)", text))
    assert int(defs["QLINEAR_NOALLOC_MAX_ROWS"]) == _lib.NOALLOC_MAX_ROWS
    assert int(defs["QLINEAR_NOALLOC_MAX_K"]) == _lib.NOALLOC_MAX_K
