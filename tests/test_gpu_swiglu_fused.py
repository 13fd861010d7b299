"""SwiGLU computed in the prefill GEMM's epilogue (Linear::run_swiglu, src/npu.rs:1009-1024).

The fused kernel stages each output channel's gate and up weight rows side by side and
forms silu(g) * u from the exact f32 dequantised values, so no [rows][N] intermediate is
written.  Bar: bit-identical to the unfused path (GEMM into f32, then the SwiGLU pass; the
same f32 expression with the same expf), and within the reference's tolerance of the
oracle (3e-5 relative for f32, src/npu.rs:1199-1210; 1e-3 for fp16).
"""
import json

import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def compare(actual, expected, tol):
    """The reference's comparison (src/npu.rs:1124-1131)."""
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    assert np.all(np.isfinite(actual))
    bad = np.abs(actual - expected) > tol * np.maximum(np.abs(expected), 1.0)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, first {np.argwhere(bad)[:3]}"


@pytest.fixture(scope="module")
def backends():
    fused = Backend(device=0)
    unfused = Backend(device=0, swiglu_unfused=True)
    yield fused, unfused
    fused.close()
    unfused.close()


def fused_calls(b):
    return b.stats()["gemm_swiglu_fused_calls"]


def run_both(backends, bits, k, n, rows, dtype, stream_id, ldc=None):
    fused, unfused = backends
    w = W.weight_codes(bits, k, n, stream=stream_id)
    sw = W.weight_scales(n, stream=stream_id)
    xh = W.activations(rows, k, stream=stream_id + 1)
    a = torch.from_numpy(xh).cuda()
    h = n // 2
    ldc = ldc or h
    outs = []
    for b in (fused, unfused):
        lin = b.load(QuantMatrix(bits, k, n, w, sw))
        out = torch.full((rows, ldc), 7.0, dtype=dtype, device="cuda")
        before = fused_calls(b)
        lin.run_device(a, out, rows, swiglu=True, ldc=ldc)
        b.check()
        outs.append((out.cpu().numpy(), fused_calls(b) - before))
        lin.close()
    (got, n_fused), (ref, n_unfused) = outs
    assert n_fused == 1 and n_unfused == 0  # each backend took the path under test
    return w, sw, xh, got, ref


@pytest.mark.parametrize("bits,k,n,rows", [
    (4, 2560, 2 * 1024, 64),
    (8, 2560, 2 * 1024, 200),
    (4, 256, 2 * 200, 300),     # h = 200: a partial channel tile, gate boxes cross into up rows
    (8, 512, 2 * 136, 9),       # h = 136: 16-channel boxes past the gate half
    (4, 1024, 2 * 3584, 1000),  # ragged token tiles
])
def test_fused_matches_unfused_and_oracle(backends, coracle, bits, k, n, rows):
    w, sw, xh, got, ref = run_both(backends, bits, k, n, rows, torch.float16, 300 + rows)
    np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))
    want = coracle.swiglu(coracle.linear(w, sw, xh))
    compare(got.astype(np.float32), want, 1e-3)


@pytest.mark.parametrize("bits,rows", [(4, 33), (8, 256)])
def test_fused_f32_within_reference_tolerance(backends, coracle, bits, rows):
    k, n = 768, 2 * 640
    w, sw, xh, got, ref = run_both(backends, bits, k, n, rows, torch.float32, 400 + rows)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    want = coracle.swiglu(coracle.linear(w, sw, xh))
    compare(got, want, 3e-5)


def test_fused_strided_output_leaves_other_columns(backends):
    k, n, rows, ldc = 512, 2 * 256, 40, 300
    *_, got, ref = run_both(backends, 4, k, n, rows, torch.float16, 500, ldc=ldc)
    np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))
    assert np.all(got[:, n // 2:] == np.float16(7.0))


def test_cfg2_gate_up_shape_tail_split(backends):
    """cfg2's gate/up matrix (2560 -> 2 x 9728) at M=512: 152 tiles on the pairs, the last
    partial wave cut into token sub-tiles; bit-identical to the unfused path."""
    *_, got, ref = run_both(backends, 4, 2560, 2 * 9728, 512, torch.float16, 600)
    np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_host_f32_swiglu_uses_fused_kernel(backends, coracle):
    """Linear::run_swiglu through the host f32 call (src/npu.rs:1009): the reference's own
    test data (src/npu.rs:1161-1224) at the row counts it checks."""
    fused, _ = backends
    codes, scales = W.kat_matrix(4)
    x = W.kat_input(256, 256)
    lin = fused.load(QuantMatrix(4, 256, 256, codes, scales))
    want = coracle.swiglu(coracle.linear(codes, scales, x))
    before = fused_calls(fused)
    for rows in (32, 33, 65, 128, 129, 256):
        mid = np.zeros((rows, 128), np.float32)
        assert lin.run_swiglu(x, mid, rows)
        compare(mid, want[:rows], 3e-5)
    assert fused_calls(fused) - before == 6
    lin.close()
    json.dumps(fused.stats())


@pytest.mark.parametrize("bits,k,n,rows", [
    (4, 2560, 2 * 9728, 16),   # cfg2 gate/up at 16 tokens: 76 tiles cut over every pair
    (8, 1024, 2 * 1280, 64),   # 10 tiles, each cut into several segments
    (4, 4096, 2 * 3584, 300),  # ragged token tiles
])
def test_fused_stream_k_matches_unfused(coracle, bits, k, n, rows):
    """The SwiGLU epilogue on split tiles (stream-K): the tile's partial sums are summed in
    the workspace and the finishing warp forms silu(g) * u; bit-identical to the unfused
    path, repeatable (the workspace counters are left at zero)."""
    fused = Backend(device=0, gemm_stream_k=True)
    unfused = Backend(device=0, gemm_stream_k=True, swiglu_unfused=True)
    try:
        w = W.weight_codes(bits, k, n, stream=700 + rows)
        sw = W.weight_scales(n, stream=700 + rows)
        xh = W.activations(rows, k, stream=701 + rows)
        a = torch.from_numpy(xh).cuda()
        outs = []
        for b in (fused, unfused):
            lin = b.load(QuantMatrix(bits, k, n, w, sw))
            sk0, f0 = b.stats()["gemm_stream_k_calls"], fused_calls(b)
            res = []
            for _ in range(2):
                out = torch.zeros((rows, n // 2), dtype=torch.float16, device="cuda")
                lin.run_device(a, out, rows, swiglu=True)
                b.check()
                res.append(out.cpu().numpy())
            np.testing.assert_array_equal(res[0].view(np.uint16), res[1].view(np.uint16))
            assert b.stats()["gemm_stream_k_calls"] - sk0 == 2
            outs.append((res[0], fused_calls(b) - f0))
            lin.close()
        (got, nf), (ref, nu) = outs
        assert nf == 2 and nu == 0
        np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))
        compare(got.astype(np.float32), coracle.swiglu(coracle.linear(w, sw, xh)), 1e-3)
    finally:
        fused.close()
        unfused.close()
