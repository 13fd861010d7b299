"""The reference's host call (Linear::run, src/npu.rs:1006) with page-locked host buffers:
the library copies them by DMA directly instead of staging them; the results must be bit
for bit those of the staged path (ordinary numpy arrays) and of the oracle, including an
output of row stride ldc > N (one part of a fused projection, qlinear_run_f32_ex) and the
SwiGLU call."""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def pinned(shape):
    return torch.zeros(shape, dtype=torch.float32).pin_memory().numpy()


@pytest.mark.parametrize("bits,k,n,rows", [(4, 2560, 1024, 300), (8, 4096, 2560, 5),
                                           (4, 1000, 200, 1)])
def test_pinned_host_buffers_match_staged(backend, coracle, bits, k, n, rows):
    w = W.weight_codes(bits, k, n, stream=500 + n)
    sw = W.weight_scales(n, stream=500 + n)
    lin = backend.load(QuantMatrix(bits, k, n, w, sw))
    x = W.activations(rows, k, stream=501).astype(np.float32)
    xp = pinned((rows, k))
    xp[:] = x
    out_staged = np.zeros((rows, n), np.float32)
    out_pinned = pinned((rows, n))
    lin.run(x, out_staged, rows)
    lin.run(xp, out_pinned, rows)
    np.testing.assert_array_equal(out_pinned, out_staged)
    np.testing.assert_array_equal(out_pinned, coracle.linear(w, sw, x))
    # a column range of a wider pinned output (row stride ldc)
    ldc, col = n + 96, 40
    wide = pinned((rows, ldc))
    wide[:] = -1.0
    lin.run_columns(xp, wide, rows, ldc=ldc, col=col)
    np.testing.assert_array_equal(wide[:, col:col + n], out_staged)
    assert np.all(wide[:, :col] == -1.0) and np.all(wide[:, col + n:] == -1.0)
    # SwiGLU on a pinned output
    if n % 2 == 0:
        mid_staged = np.zeros((rows, n // 2), np.float32)
        mid_pinned = pinned((rows, n // 2))
        assert lin.run_swiglu(x, mid_staged, rows)
        assert lin.run_swiglu(xp, mid_pinned, rows)
        np.testing.assert_array_equal(mid_pinned, mid_staged)
    lin.close()
