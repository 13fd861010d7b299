"""The MLP block of a decoder layer (src/model/dense.rs:499-530: gate_up.run_swiglu into an
f32 middle, then down.run) through qlinear_run_mlp_device, decode and prefill shapes.

Bar: bit for bit the two separate device calls with an f32 middle, and within 1e-3 relative
of the
oracle chain in f32 (the middle's exp differs from numpy's in the last bits, which can move
a code of the down projection's quantisation by one).
"""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def compare(actual, expected, tol):
    """The reference's comparison (src/npu.rs:1124-1131)."""
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    assert np.all(np.isfinite(actual))
    bad = np.abs(actual - expected) > tol * np.maximum(np.abs(expected), 1.0)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, first {np.argwhere(bad)[:3]}"


def load_block(backend, b1, b2, hidden, f, seed):
    gu_codes = W.weight_codes(b1, hidden, 2 * f, stream=seed)
    gu_scales = W.weight_scales(2 * f, stream=seed)
    dn_codes = W.weight_codes(b2, f, hidden, stream=seed + 1)
    dn_scales = W.weight_scales(hidden, stream=seed + 1)
    gu = backend.load(QuantMatrix(b1, hidden, 2 * f, gu_codes, gu_scales))
    dn = backend.load(QuantMatrix(b2, f, hidden, dn_codes, dn_scales))
    return gu, dn, (gu_codes, gu_scales, dn_codes, dn_scales)


def two_calls(gu, dn, a, rows, out_dtype):
    f = gu.n() // 2
    mid = torch.zeros((rows, f), dtype=torch.float32, device="cuda")
    gu.run_device(a, mid, rows, swiglu=True)
    out = torch.zeros((rows, dn.n()), dtype=out_dtype, device="cuda")
    dn.run_device(mid, out, rows)
    return out


def mlp_calls(backend):
    return backend.stats()["mlp_calls"]


@pytest.mark.parametrize("b1,b2", [(4, 8), (4, 4), (8, 8), (8, 4)])
def test_mlp_one_row_matches_two_calls(backend, coracle, b1, b2):
    hidden, f = 2560, 9728  # the Qwen3-4B MLP of the cfg2 block
    gu, dn, (gc, gs, dc, ds) = load_block(backend, b1, b2, hidden, f, 40 + 2 * b1 + b2)
    xh = W.activations(1, hidden, stream=41)
    a = torch.from_numpy(xh).cuda()
    want = two_calls(gu, dn, a, 1, torch.float16).cpu().numpy()
    before = mlp_calls(backend)
    for _ in range(3):  # repeated calls: the barrier's epochs advance
        out = torch.zeros((1, hidden), dtype=torch.float16, device="cuda")
        backend.run_mlp_device(gu, dn, a, out, 1)
        backend.check()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))
    assert mlp_calls(backend) - before == 3
    # against the oracle chain in f32 (W8 gate/up can push the fp16 output past 65504)
    want32 = two_calls(gu, dn, a, 1, torch.float32).cpu().numpy()
    out32 = torch.zeros((1, hidden), dtype=torch.float32, device="cuda")
    backend.run_mlp_device(gu, dn, a, out32, 1)
    backend.check()
    np.testing.assert_array_equal(out32.cpu().numpy().view(np.uint32), want32.view(np.uint32))
    mid = coracle.swiglu(coracle.linear(gc, gs, xh))
    compare(out32.cpu().numpy(), coracle.linear(dc, ds, mid), 1e-3)
    gu.close()
    dn.close()


def test_mlp_f32_in_out_and_ragged_widths(backend, coracle):
    hidden, f = 1000, 600  # partial weight units and a short last CTA in both phases
    gu, dn, (gc, gs, dc, ds) = load_block(backend, 4, 8, hidden, f, 50)
    x = W.activations(1, hidden, stream=51).astype(np.float32)
    a = torch.from_numpy(x).cuda()
    want = two_calls(gu, dn, a, 1, torch.float32).cpu().numpy()
    before = mlp_calls(backend)
    out = torch.zeros((1, hidden), dtype=torch.float32, device="cuda")
    backend.run_mlp_device(gu, dn, a, out, 1)
    backend.check()
    assert mlp_calls(backend) - before == 1
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    mid = coracle.swiglu(coracle.linear(gc, gs, x))
    compare(out.cpu().numpy(), coracle.linear(dc, ds, mid), 3e-5)
    gu.close()
    dn.close()


@pytest.mark.parametrize("rows,f", [(3, 1024), (64, 1024), (1, 602)])
def test_mlp_rows_and_odd_middle_width(backend, rows, f):
    """Several rows (decode GEMV with paired rows; prefill GEMM with the SwiGLU epilogue) and a
    middle width that is not a multiple of 4 (the down call then reads act-quant codes)."""
    hidden = 512
    gu, dn, _ = load_block(backend, 4, 8, hidden, f, 60 + rows)
    a = torch.from_numpy(W.activations(rows, hidden, stream=61)).cuda()
    want = two_calls(gu, dn, a, rows, torch.float16).cpu().numpy()
    before = mlp_calls(backend)
    out = torch.zeros((rows, hidden), dtype=torch.float16, device="cuda")
    backend.run_mlp_device(gu, dn, a, out, rows)
    backend.check()
    assert mlp_calls(backend) - before == 1
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))
    gu.close()
    dn.close()


def test_mlp_rejects_mismatched_shapes(backend):
    from open_rknpu2_lm_infer_b200 import NpuError
    gu, dn, _ = load_block(backend, 4, 8, 512, 256, 70)
    other = backend.load(QuantMatrix(8, 300, 512, W.weight_codes(8, 300, 512),
                                     W.weight_scales(512)))
    a = torch.zeros((1, 512), dtype=torch.float16, device="cuda")
    out = torch.zeros((1, 512), dtype=torch.float16, device="cuda")
    with pytest.raises(NpuError):
        backend.run_mlp_device(gu, other, a, out, 1)  # down K != gate_up N/2
    with pytest.raises(NpuError):
        backend.run_mlp_device(gu, dn, a, out, 1, ldc=100)
    for lin in (gu, dn, other):
        lin.close()
