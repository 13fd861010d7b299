"""The GEMM's stream-K schedule (csrc/gemm_sm100.cu, QLINEAR_BACKEND_GEMM_STREAM_K): shapes
whose whole tiles would leave most CTA pairs idle run with every pair taking an equal share
of the k-blocks and split tiles summed in a workspace.  Accumulators and fp16 outputs must equal the oracle's
bit for bit, on the first call and on a repeat call (the kernel zeroes the workspace it
used), for W8, W4 (int8 expansion) and W4 unpacked in shared memory."""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu

SHAPES = [
    (8, 1024, 2560, 64),     # 10 tiles over all pairs: every tile cut into several segments
    (4, 2560, 9728, 512),    # cfg0: 76 tiles, one pair's worth past a full wave
    (4, 8192, 3584, 512),    # cfg4 at 8 GPUs (one rank's columns): 28 tiles
    (8, 8192, 7168, 300),    # cfg4 at 4 GPUs, ragged token tiles
    (4, 9728, 2560, 33),     # long k-loop, few tiles
]


def _run(b, coracle, bits, k, n, rows):
    w = W.weight_codes(bits, k, n, stream=k + n)
    sw = W.weight_scales(n, stream=k + n)
    xh = W.activations(rows, k, stream=rows + 3)
    lin = b.load(QuantMatrix(bits, k, n, w, sw))
    y, acc = coracle.linear(w, sw, xh, want_acc=True)
    a = torch.from_numpy(np.ascontiguousarray(xh)).cuda()
    before = b.stats()["gemm_stream_k_calls"]
    for _ in range(2):
        out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
        acc_gpu = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
        lin.run_device(a, acc_gpu, rows)
        lin.run_device(a, out, rows)
        b.check()
        np.testing.assert_array_equal(acc_gpu.cpu().numpy(), acc)
        np.testing.assert_array_equal(out.cpu().numpy(), y.astype(np.float16))
    assert b.stats()["gemm_stream_k_calls"] - before == 4
    lin.close()


@pytest.fixture(scope="module")
def sk_backend():
    b = Backend(device=0, gemm_stream_k=True)
    yield b
    b.close()


@pytest.mark.parametrize("bits,k,n,rows", SHAPES)
def test_stream_k_bit_exact(sk_backend, coracle, bits, k, n, rows):
    _run(sk_backend, coracle, bits, k, n, rows)


def test_default_backend_uses_whole_tiles(backend, coracle):
    before = backend.stats()["gemm_stream_k_calls"]
    w = W.weight_codes(4, 2560, 9728, stream=3)
    lin = backend.load(QuantMatrix(4, 2560, 9728, w, W.weight_scales(9728, stream=3)))
    x = torch.from_numpy(np.ascontiguousarray(W.activations(512, 2560, stream=4))).cuda()
    out = torch.zeros((512, 9728), dtype=torch.float16, device="cuda")
    lin.run_device(x, out, 512)
    backend.check()
    assert backend.stats()["gemm_stream_k_calls"] == before
    lin.close()


def test_stream_k_w4_packed_only(coracle):
    b = Backend(device=0, w4_packed_only=True, gemm_stream_k=True)
    try:
        _run(b, coracle, 4, 2560, 9728, 512)
        _run(b, coracle, 4, 8192, 3584, 100)
    finally:
        b.close()
