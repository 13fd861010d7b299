"""Failure detection on the GPU without a fault: a kernel wait that nothing satisfies gives
up after a short limit, the kernel records the timeout and returns, the host call reports
QLINEAR_ERR_TIMEOUT, and the backend and its context stay usable (the next call is
bit-exact).  The same bounded-wait path guards every pipeline wait of the GEMM."""
import time

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_backend_recovers(backend, golden):
    assert backend.selftest_wait_timeout(limit_s=5.0) == L.QLINEAR_ERR_PARAM  # > 2 s refused
    t0 = time.perf_counter()
    rc = backend.selftest_wait_timeout(limit_s=0.2)
    dt = time.perf_counter() - t0
    assert rc == L.QLINEAR_ERR_TIMEOUT
    assert 0.2 <= dt < 5.0
    backend.check()  # the error word was cleared
    codes, scales = W.kat_matrix(8)
    lin = backend.load(QuantMatrix(8, 256, 256, codes, scales))
    x = W.kat_input(256, 256)
    out = np.zeros((33, 256), np.float32)
    lin.run(x, out, 33)
    np.testing.assert_array_equal(out, golden["kat_w8_y"][:33])
    lin.close()
