"""The allocation-free decode call (qlinear_run_device_noalloc), through the C ABI.

It serves callers that cannot allocate device memory while they run a layer (a process
whose device memory is reserved up front by its own pool allocator, or a latency-critical
decode loop that must not call cudaMalloc/cudaFree).  Its activation codes live in a fixed
scratch array compiled into the library, shared by every call on the device; so the test
makes two calls in a row, with different inputs and weights, and checks each against the
regular entry point (qlinear_run_device) with the tolerance the other parity tests use for
these outputs: bit-exact.  This file is collected last and runs alone as well.
"""
import ctypes

import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def noalloc(lib, lin, a, out, rows, ldc=None, stream=None):
    c_type = {torch.float16: L.F16, torch.float32: L.F32, torch.int32: L.I32}[out.dtype]
    a_type = {torch.float16: L.F16, torch.float32: L.F32}[a.dtype]
    return lib.qlinear_run_device_noalloc(lin._raw, a.data_ptr(), a_type, out.data_ptr(), c_type,
                                          ldc if ldc is not None else out.shape[1], rows, stream)


def test_noalloc_matches_regular_call_twice():
    lib = L.load()
    backend = Backend(device=0)
    cases = [(4, 2560, 1024, 1, torch.float16), (8, 2560, 768, 8, torch.float16),
             (4, 4096, 512, 5, torch.float32), (8, 9728, 256, 3, torch.int32)]
    for bits, k, n, rows, out_dtype in cases:
        lin = backend.load(QuantMatrix(bits, k, n, W.weight_codes(bits, k, n, stream=k + n),
                                       W.weight_scales(n, stream=k + n)))
        for call in range(2):  # two calls in a row: the shared scratch keeps the last call's data
            x = torch.from_numpy(W.activations(rows, k, stream=100 * call + rows)).cuda()
            want = torch.zeros((rows, n), dtype=out_dtype, device="cuda")
            got = torch.full((rows, n), 7, dtype=out_dtype, device="cuda")
            lin.run_device(x, want, rows)
            assert noalloc(lib, lin, x, got, rows) == L.QLINEAR_OK
            torch.cuda.synchronize()
            assert torch.equal(got, want), (bits, k, n, rows, call)
        lin.close()
    backend.close()


def test_noalloc_allocates_nothing_and_honours_ldc():
    """After a first call (which looks up the scratch's address), further calls leave the
    device's free memory and the backend's workspaces as they were; an output of row stride
    ldc > N receives exactly its N columns per row."""
    lib = L.load()
    backend = Backend(device=0)
    bits, k, n, rows, ldc = 4, 2560, 640, 6, 700
    lin = backend.load(QuantMatrix(bits, k, n, W.weight_codes(bits, k, n, stream=77),
                                   W.weight_scales(n, stream=77)))
    xs = [torch.from_numpy(W.activations(rows, k, stream=s)).cuda() for s in (78, 79)]
    want = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
    got = torch.full((rows, ldc), -3.0, dtype=torch.float16, device="cuda")
    assert noalloc(lib, lin, xs[0], got, rows, ldc=ldc) == L.QLINEAR_OK  # first call: set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    ws0 = backend.stats()["workspace_payload_bytes"]
    for i in range(6):
        assert noalloc(lib, lin, xs[i % 2], got, rows, ldc=ldc) == L.QLINEAR_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert backend.stats()["workspace_payload_bytes"] == ws0
    lin.run_device(xs[1], want, rows)
    torch.cuda.synchronize()
    assert torch.equal(got[:, :n], want)
    assert torch.all(got[:, n:] == -3.0)
    lin.close()
    backend.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = L.load()
    backend = Backend(device=0)
    lin = backend.load(QuantMatrix(8, 256, 128, W.weight_codes(8, 256, 128), W.weight_scales(128)))
    rows = L.NOALLOC_MAX_ROWS + 1
    x = torch.zeros((rows, 256), dtype=torch.float16, device="cuda")
    out = torch.zeros((rows, 128), dtype=torch.float16, device="cuda")
    assert noalloc(lib, lin, x, out, rows) == L.QLINEAR_ERR_LIMIT
    assert b"limit" in lib.qlinear_strerror(L.QLINEAR_ERR_LIMIT)
    big_k = L.NOALLOC_MAX_K + 128
    wide = backend.load(QuantMatrix(8, big_k, 128, np.ones((big_k, 128), np.int8),
                                    np.full(128, 1e-3, np.float32)))
    xw = torch.zeros((1, big_k), dtype=torch.float16, device="cuda")
    assert noalloc(lib, wide, xw, out, 1) == L.QLINEAR_ERR_LIMIT
    lin.close()
    wide.close()
    backend.close()
