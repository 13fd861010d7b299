"""Failure detection on the GPU without a fault: a kernel wait that nothing satisfies gives
up after a short limit, the kernel records the timeout and returns, the host call reports
QLINEAR_ERR_TIMEOUT, and the backend and its context stay usable (the next call is
bit-exact).  The same bounded-wait path guards every pipeline wait of the GEMM."""
import time

import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200.npu import NpuError
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


def test_peer_signal_wait(backend):
    """The split-N exchange's completion signal on one GPU: flags a rank raises satisfy the
    wait; a rank that never signals makes it give up after its limit with a timeout status,
    and the backend stays usable.  (The other rank is emulated by writing its flag from the
    host: two waiting kernels never run on one GPU.)"""
    import torch
    from open_rknpu2_lm_infer_b200.sharded import _DeviceArray
    dev = torch.device("cuda", backend.device)
    a, _ = backend.peer_buffer_create(16)
    b, _ = backend.peer_buffer_create(16)
    try:
        va = torch.as_tensor(_DeviceArray(a, (2,), "<i8"), device=dev)
        vb = torch.as_tensor(_DeviceArray(b, (2,), "<i8"), device=dev)
        assert va.tolist() == [0, 0] and vb.tolist() == [0, 0]  # zero at creation
        backend.peer_signal_wait([a], 0, 1)  # one rank: its own flag satisfies the wait
        backend.check()
        assert va.tolist() == [1, 0]
        va[1] = 2  # rank 1 signalled epoch 2
        torch.cuda.synchronize(dev)
        backend.peer_signal_wait([a, b], 0, 2)
        backend.check()
        assert va.tolist() == [2, 2] and vb.tolist() == [2, 0]
        t0 = time.perf_counter()
        backend.peer_signal_wait([a, b], 0, 3, limit_s=0.1)  # rank 1 never signals epoch 3
        with pytest.raises(NpuError) as e:
            backend.check()
        assert e.value.rc == L.QLINEAR_ERR_TIMEOUT
        assert time.perf_counter() - t0 >= 0.1
        assert va.tolist() == [3, 2] and vb.tolist() == [3, 0]
        backend.check()  # cleared
        for sig, rank in (([a, b], 2), ([a, b], -1), ([a] * 9, 0), ([], 0)):
            with pytest.raises(NpuError) as e:
                backend.peer_signal_wait(sig, rank, 4)
            assert e.value.rc == L.QLINEAR_ERR_PARAM
    finally:
        torch.cuda.synchronize(dev)
        backend.peer_buffer_free(a, False)
        backend.peer_buffer_free(b, False)
