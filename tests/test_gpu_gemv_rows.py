"""Decode GEMV (rows <= 8) against the oracle, bit-exact, at the row counts and shapes that
exercise its layouts: W4 activation codes interleaved in shared memory (16-byte halves of
each 32-code unit grouped per block of 32 units, a row's last block partial), tasks of two
weight rows (W4 at 3..8 rows, W8 at 5..8: the CTA's rows split in halves, the second one row
shorter when the count is odd), rows cut into several chunks, the balanced mode at one or
two rows ((row, chunk) tasks dealt round-robin to the warps, int32 sums added in shared
memory), and the path that reads codes quantised by the separate kernel (K not a multiple
of the fused prologue's vector)."""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu

CASES = [
    # bits, K, N, rows
    (4, 2560, 1000, 5),     # 7 rows per CTA: halves of 4 and 3
    (4, 2560, 1000, 8),
    (4, 3200, 2048, 4),     # 100 units per row: blocks of 32, 32, 32, 4
    (4, 8192, 4096, 7),
    (4, 203, 300, 6),       # K not a multiple of 8: codes from the act-quant kernel
    (4, 203, 300, 2),
    (4, 9728, 2560, 1),     # 304 units per row: a last block of 16 units
    (8, 9728, 2560, 8),     # W8 paired, three chunks per row
    (8, 2560, 9728, 6),
    (8, 2560, 1000, 3),     # W8 unpaired at four rows
    (8, 203, 300, 8),
    # balanced (row, chunk) tasks at one or two rows, sums added in shared memory
    (8, 2560, 9728, 1),     # cfg1: whole rows (66 per CTA)
    (8, 9728, 2560, 1),     # balanced: 18 rows per CTA in one-unit tasks
    (4, 9728, 2560, 2),     # two-unit tasks
    (8, 4096, 2560, 2),
    (4, 8192, 7168, 1),
]


@pytest.mark.parametrize("bits,k,n,rows", CASES)
def test_gemv_rows_bit_exact(backend, coracle, bits, k, n, rows):
    w = W.weight_codes(bits, k, n, stream=900 + k)
    sw = W.weight_scales(n, stream=900 + n)
    xh = W.activations(rows, k, stream=900 + rows)
    lin = backend.load(QuantMatrix(bits, k, n, w, sw))
    y, acc = coracle.linear(w, sw, xh, want_acc=True)
    a = torch.from_numpy(np.ascontiguousarray(xh)).cuda()
    before = backend.stats()["gemv_calls"]
    out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
    acc_gpu = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
    lin.run_device(a, out, rows)
    lin.run_device(a, acc_gpu, rows)
    backend.check()
    assert backend.stats()["gemv_calls"] - before == 2
    np.testing.assert_array_equal(acc_gpu.cpu().numpy(), acc)
    np.testing.assert_array_equal(out.cpu().numpy(), y.astype(np.float16))
    # the host f32 path (src/npu.rs:1006) on the same rows
    out32 = np.zeros((rows, n), np.float32)
    lin.run(xh.astype(np.float32), out32, rows)
    np.testing.assert_array_equal(out32, y)
    lin.close()
