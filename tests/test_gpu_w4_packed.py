"""The prefill GEMM on packed W4 weights (no int8 copy): the converter warps unpack the
nibbles of each stage into tensor memory and the MMA reads its weight operand from there.

Checked against the oracle (src/npu.rs:1097-1121) the way the default path is: int32
accumulators and fp16 outputs bit-exact against f16(oracle); SwiGLU in the epilogue within
1e-3 relative (fp16) of the oracle's SwiGLU and bit for bit the default mode's fused
result; the MLP block bit for bit the default mode's.  Shapes cover token tiles of 32..128,
ragged rows, K and N that are not multiples of the tile, several waves with the tail split,
the full cfg4 layer, and the split-N exchange kernels (several local destinations).
"""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
from open_rknpu2_lm_infer_b200 import _lib as L
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def packed():
    b = Backend(device=0, w4_packed_only=True)
    assert b.stats()["w4_prefill"] == "packed"
    yield b
    b.close()


def f16_bits(a):
    return np.asarray(a, np.float16).view(np.uint16)


@pytest.mark.parametrize("k,n,rows", [
    (2560, 9728, 512),    # cfg0
    (2560, 1024, 9),      # the smallest GEMM row count
    (2560, 1024, 100),    # ragged token tile
    (8192, 1024, 300),
    (4096, 2560, 77),
    (1000, 200, 40),      # K and N not multiples of the tiles
    (512, 3584, 512),     # a narrow shard: halved token tiles
    (2560, 9728, 2000),   # several waves, tail split
])
def test_packed_gemm_matches_oracle(packed, coracle, k, n, rows):
    w = W.weight_codes(4, k, n, stream=400 + n)
    sw = W.weight_scales(n, stream=400 + n)
    xh = W.activations(rows, k, stream=401 + rows)
    lin = packed.load(QuantMatrix(4, k, n, w, sw))
    assert lin.device_bytes < k * n  # 0.5 byte per weight (+ scales)
    y, acc = coracle.linear(w, sw, xh, want_acc=True)
    a = torch.from_numpy(xh).cuda()
    out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
    acc_gpu = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
    out32 = torch.zeros((rows, n), dtype=torch.float32, device="cuda")
    lin.run_device(a, out, rows)
    lin.run_device(a, acc_gpu, rows)
    lin.run_device(a, out32, rows)
    packed.check()
    np.testing.assert_array_equal(acc_gpu.cpu().numpy(), acc)
    np.testing.assert_array_equal(f16_bits(out.cpu().numpy()), f16_bits(y))
    np.testing.assert_array_equal(out32.cpu().numpy(), y)
    lin.close()


def test_packed_cfg4_full_width(packed, coracle):
    k, n = 8192, 28672
    w, sw = W.weight_codes(4, k, n), W.weight_scales(n)
    lin = packed.load(QuantMatrix(4, k, n, w, sw))
    for rows, sample in ((512, None), (8192, 256)):
        xh = W.activations(rows, k)
        out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
        lin.run_device(torch.from_numpy(xh).cuda(), out, rows)
        packed.check()
        idx = np.arange(rows) if sample is None else \
            np.unique(np.linspace(0, rows - 1, sample).round().astype(np.int64))
        y = coracle.linear(w, sw, np.ascontiguousarray(xh[idx]))
        got = out[torch.from_numpy(idx).cuda()].cpu().numpy()
        np.testing.assert_array_equal(f16_bits(got), f16_bits(y), err_msg=f"rows={rows}")
    lin.close()


@pytest.mark.parametrize("n,rows", [(2 * 1024, 64), (2 * 1000, 200), (2 * 9728, 512)])
def test_packed_swiglu_epilogue(packed, backend, coracle, n, rows):
    k = 2560
    w = W.weight_codes(4, k, n, stream=410 + rows)
    sw = W.weight_scales(n, stream=410 + rows)
    xh = W.activations(rows, k, stream=411)
    a = torch.from_numpy(xh).cuda()
    lp = packed.load(QuantMatrix(4, k, n, w, sw))
    ld = backend.load(QuantMatrix(4, k, n, w, sw))  # the default mode (int8 copy)
    for dtype in (torch.float16, torch.float32):
        got = torch.zeros((rows, n // 2), dtype=dtype, device="cuda")
        want = torch.zeros((rows, n // 2), dtype=dtype, device="cuda")
        before = packed.stats()["gemm_swiglu_fused_calls"]
        lp.run_device(a, got, rows, swiglu=True)
        ld.run_device(a, want, rows, swiglu=True)
        packed.check()
        backend.check()
        assert packed.stats()["gemm_swiglu_fused_calls"] == before + 1
        assert torch.equal(got, want)
    ref = coracle.swiglu(coracle.linear(w, sw, xh))
    g = got.cpu().numpy()
    assert (np.abs(g - ref) / np.maximum(np.abs(ref), 1.0)).max() <= 1e-3
    lp.close()
    ld.close()


def test_packed_mlp_block_matches_default(packed, backend):
    hidden, f, rows = 2560, 9728, 128
    gc, gs = W.weight_codes(4, hidden, 2 * f, stream=420), W.weight_scales(2 * f, stream=420)
    dc, ds = W.weight_codes(4, f, hidden, stream=421), W.weight_scales(hidden, stream=421)
    a = torch.from_numpy(W.activations(rows, hidden, stream=422)).cuda()
    outs = []
    for b in (packed, backend):
        gu = b.load(QuantMatrix(4, hidden, 2 * f, gc, gs))
        dn = b.load(QuantMatrix(4, f, hidden, dc, ds))
        out = torch.zeros((rows, hidden), dtype=torch.float16, device="cuda")
        b.run_mlp_device(gu, dn, a, out, rows)
        b.check()
        outs.append(out.cpu().numpy())
        gu.close()
        dn.close()
    np.testing.assert_array_equal(f16_bits(outs[0]), f16_bits(outs[1]))


@pytest.mark.parametrize("ndst", [2, 4])
def test_packed_scatter_kernels(packed, coracle, ndst):
    """The split-N exchange's GEMM (every element stored to each destination) with local
    buffers standing in for the peers'."""
    k, n, rows, ldc, col0 = 2560, 1024, 200, 4096, 1024
    w = W.weight_codes(4, k, n, stream=430)
    sw = W.weight_scales(n, stream=430)
    xh = W.activations(rows, k, stream=431)
    lin = packed.load(QuantMatrix(4, k, n, w, sw))
    bufs = [torch.zeros((rows, ldc), dtype=torch.float16, device="cuda") for _ in range(ndst)]
    lin.run_device_scatter(torch.from_numpy(xh).cuda(), [b.data_ptr() for b in bufs], L.F16,
                           ldc, col0, rows)
    packed.check()
    want = f16_bits(coracle.linear(w, sw, xh))
    for b in bufs:
        got = b.cpu().numpy()
        np.testing.assert_array_equal(f16_bits(got[:, col0:col0 + n]), want)
        assert not got[:, :col0].any() and not got[:, col0 + n:].any()
    lin.close()
