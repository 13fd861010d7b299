"""Projection orchestration on the CUDA library (src/model/projection.rs:142-243): mixed-bit
q/k/v run as two linears writing their column ranges in place, compared bit-exactly with
the oracle per module; host f32 path (qlinear_run_f32_ex) and device fp16 path (output
stride), GEMV (rows <= 8) and GEMM (rows > 8)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from open_rknpu2_lm_infer_b200 import MatrixLoader, Projection, QuantMatrix

pytestmark = pytest.mark.gpu

K = 320  # not a multiple of 128: padded in the device layout


def matrix(bits, k, n, seed):
    rng = np.random.default_rng(seed)
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    codes = rng.integers(lo, hi + 1, size=(k, n), dtype=np.int8)
    scales = np.exp(rng.uniform(np.log(1e-3), np.log(1e-2), n)).astype(np.float32)
    return QuantMatrix(bits, k, n, codes.reshape(-1), scales)


MODULES = [("q", 192, 4), ("k", 64, 4), ("v", 64, 8)]


@pytest.fixture(scope="module")
def setup(backend):
    ld = MatrixLoader({name: matrix(bits, K, n, 100 + i) for i, (name, n, bits) in enumerate(MODULES)})
    p = Projection.load(backend, ld, [(n, c) for n, c, _ in MODULES], K)
    yield p, ld
    p.close()


def expected(ld, x, names):
    return np.concatenate([O.linear(np.asarray(ld.matrices[n].codes, np.int8).reshape(K, -1),
                                    ld.matrices[n].scales, x) for n in names], axis=1)


@pytest.mark.parametrize("rows", [1, 4, 33, 300])
def test_mixed_bit_projection_host_path(setup, rows):
    p, ld = setup
    assert [(lin.bits, lin.n(), off) for lin, off in p.parts] == [(4, 256, 0), (8, 64, 256)]
    x = np.random.default_rng(rows).standard_normal((rows, K)).astype(np.float32)
    out = np.full((rows, p.width), np.nan, np.float32)
    p.run(x, out, rows)
    np.testing.assert_array_equal(out, expected(ld, x, ["q", "k", "v"]))
    kv = np.full((rows, 64), np.nan, np.float32)
    p.run_from(1, x, kv, rows)
    np.testing.assert_array_equal(kv, expected(ld, x, ["v"]))


@pytest.mark.parametrize("rows", [1, 5, 40])
def test_mixed_bit_projection_device_path(setup, rows):
    p, ld = setup
    x16 = (np.random.default_rng(50 + rows).standard_normal((rows, K))).astype(np.float16)
    out = torch.full((rows, p.width), float("nan"), dtype=torch.float16, device="cuda")
    p.run_device(torch.from_numpy(x16).cuda(), out, rows)
    torch.cuda.synchronize()
    want = expected(ld, x16.astype(np.float32), ["q", "k", "v"]).astype(np.float16)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_single_matrix_gate_up_swiglu(backend):
    ld = MatrixLoader({"gate": matrix(4, K, 128, 7), "up": matrix(4, K, 128, 8)})
    p = Projection.load(backend, ld, [("gate", 128), ("up", 128)], K)
    try:
        assert len(p.parts) == 1
        x = np.random.default_rng(9).standard_normal((6, K)).astype(np.float32)
        mid = np.zeros((6, 128), np.float32)
        assert p.run_swiglu(x, mid, 6)
        y = expected(ld, x, ["gate", "up"])
        want = O.swiglu(y)
        bad = np.abs(mid - want) > 3e-5 * np.maximum(np.abs(want), 1.0)
        assert not bad.any()
    finally:
        p.close()
