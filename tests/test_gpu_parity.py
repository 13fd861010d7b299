"""Parity of the CUDA path (through the C ABI) with the reference's arithmetic.

Bar: int8 codes, int32 accumulators and f32 outputs bit-exact; fp16 outputs equal to the
oracle's f32 value rounded once to fp16 (bit-exact); SwiGLU within the reference's own
tolerance (3e-5 relative, src/npu.rs:1199-1210) for f32 and 1e-3 relative for fp16.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from open_rknpu2_lm_infer_b200 import NpuError, QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu

KAT_ROWS = [1, 2, 3, 5, 9, 17, 32, 33, 65, 127, 128, 129, 191, 192, 193, 255, 256]


def compare(actual, expected, tol):
    """The reference's comparison (src/npu.rs:1124-1131)."""
    actual = np.asarray(actual, np.float32)
    expected = np.asarray(expected, np.float32)
    assert np.all(np.isfinite(actual))
    bad = np.abs(actual - expected) > tol * np.maximum(np.abs(expected), 1.0)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, first {np.argwhere(bad)[:3]}"


def swiglu_expected(y):
    h = y.shape[1] // 2
    gate, up = y[:, :h], y[:, h:]
    return (gate / (np.float32(1) + np.exp(-gate)) * up).astype(np.float32)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_linear_padding_and_swiglu(backend, golden, bits):
    """src/npu.rs:1161-1224 restated: the same generators and row counts, tightened to
    bit-exact f32 for the plain output."""
    codes, scales = W.kat_matrix(bits)
    x = W.kat_input(256, 256)
    ref = golden[f"kat_w{bits}_y"]
    lin = backend.load(QuantMatrix(bits, 256, 256, codes, scales),
                       reload=lambda: (_ for _ in ()).throw(RuntimeError("reloaded")))
    for rows in KAT_ROWS:
        out = np.zeros((rows, 256), np.float32)
        lin.run(x, out, rows)
        np.testing.assert_array_equal(out, ref[:rows], err_msg=f"rows={rows}")
        compare(out, ref[:rows], 2e-5)
        if rows >= 32 or bits == 8:
            mid = np.zeros((rows, 128), np.float32)
            assert lin.run_swiglu(x, mid, rows)
            compare(mid, swiglu_expected(ref[:rows]), 3e-5)
    backend.retain_workspaces([1, 64])
    backend.prepare(3)
    assert backend.tune_operations() == 0
    s = backend.stats()
    assert s["tune_calls"] == 0 and s["weight_reload_calls"] == 0
    assert s["backend"] == "cuda-sm100a"


@pytest.mark.parametrize("n", [32, 64])
def test_narrow_w8_gdn_gates_match_integer_oracle(backend, golden, n):
    """src/npu/narrow_projection.rs:3-68 restated (W8, K=2560, rows 1,2,3,5,7)."""
    w, sw, x = W.narrow_kat(n)
    lin = backend.load(QuantMatrix(8, 2560, n, w, sw))
    for rows in (1, 2, 3, 5, 7):
        backend.prepare(rows)
        out = np.zeros((rows, n), np.float32)
        lin.run(x, out, rows)
        np.testing.assert_array_equal(out, golden[f"narrow_n{n}_y"][:rows])


@pytest.mark.parametrize("name", ["seed_k2560", "seed_k9728", "seed_k8192", "seed_k100"])
def test_act_quant_codes_bit_exact(backend, golden, name):
    xh = golden[f"{name}_x"]
    rows, k = xh.shape
    codes = torch.zeros((rows, k), dtype=torch.int8, device="cuda")
    scales = torch.zeros(rows, dtype=torch.float32, device="cuda")
    sums = torch.zeros(rows, dtype=torch.int32, device="cuda")
    backend.act_quant_device(dev(xh), rows, k, codes, scales, sums)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), golden[f"{name}_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden[f"{name}_scales"])
    np.testing.assert_array_equal(sums.cpu().numpy(),
                                  golden[f"{name}_codes"].astype(np.int64).sum(1))


def test_act_quant_edge_cases(backend, golden):
    x = golden["edge_x"]
    rows, k = x.shape
    codes = torch.zeros((rows, k), dtype=torch.int8, device="cuda")
    scales = torch.zeros(rows, dtype=torch.float32, device="cuda")
    backend.act_quant_device(dev(x), rows, k, codes, scales)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), golden["edge_codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), golden["edge_scales"])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("rows", [1, 3, 8, 9, 40, 256])
def test_int32_accumulators_bit_exact(backend, golden, bits, rows):
    codes, scales = W.kat_matrix(bits)
    lin = backend.load(QuantMatrix(bits, 256, 256, codes, scales))
    x = W.kat_input(256, 256)[:rows]
    acc = torch.zeros((rows, 256), dtype=torch.int32, device="cuda")
    lin.run_device(dev(x), acc, rows)
    backend.check()
    np.testing.assert_array_equal(acc.cpu().numpy(), golden[f"kat_w{bits}_acc"][:rows])


def test_odd_shape(backend, golden):
    lin = backend.load(QuantMatrix(4, 100, 72, golden["odd_w"], golden["odd_sw"]))
    x = golden["odd_x"].astype(np.float32)
    out = np.zeros((3, 72), np.float32)
    lin.run(x, out, 3)
    np.testing.assert_array_equal(out, golden["odd_y"])


@pytest.mark.parametrize("bits,k,n,rows", [
    (4, 2560, 9728, 512),   # cfg0
    (8, 2560, 9728, 1),     # cfg1
    (8, 2560, 9728, 4),     # cfg1
    (4, 2560, 9728, 16),
    (8, 9728, 2560, 128),   # cfg2 down
    (4, 8192, 1024, 8),     # cfg4 K, N slice (decode)
    (4, 8192, 1024, 300),   # cfg4 K, N slice, ragged token tiles
    (8, 4096, 2560, 77),    # o_proj shape, odd rows
    (8, 1024, 3584, 512),   # cfg4's N/8 shard width: 256-token tiles halved to 128
    (4, 512, 1024, 512),    # narrower still: halved twice, 64-token tiles
])
def test_seeded_config_shapes_fp16(backend, coracle, bits, k, n, rows):
    w = W.weight_codes(bits, k, n, stream=bits)
    sw = W.weight_scales(n, stream=bits)
    xh = W.activations(rows, k, stream=rows)
    lin = backend.load(QuantMatrix(bits, k, n, w, sw))
    y, acc = coracle.linear(w, sw, xh, want_acc=True)
    out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
    a = dev(xh)
    lin.run_device(a, out, rows)
    acc_gpu = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
    lin.run_device(a, acc_gpu, rows)
    backend.check()
    np.testing.assert_array_equal(acc_gpu.cpu().numpy(), acc)
    np.testing.assert_array_equal(out.cpu().numpy(), y.astype(np.float16))
    rel = np.abs(out.cpu().numpy().astype(np.float32) - y) / np.maximum(np.abs(y), 1e-3)
    assert rel.max() <= 1e-3


@pytest.mark.parametrize("bits,rows", [(4, 1), (4, 4), (4, 64), (8, 2), (8, 200)])
def test_swiglu_device_fp16(backend, coracle, bits, rows):
    k, n = 2560, 2 * 1024
    w = W.weight_codes(bits, k, n, stream=20 + bits)
    sw = W.weight_scales(n, stream=20 + bits)
    xh = W.activations(rows, k, stream=30 + rows)
    lin = backend.load(QuantMatrix(bits, k, n, w, sw))
    y = coracle.linear(w, sw, xh)
    want = coracle.swiglu(y)
    out = torch.zeros((rows, n // 2), dtype=torch.float16, device="cuda")
    lin.run_device(dev(xh), out, rows, swiglu=True)
    backend.check()
    got = out.cpu().numpy().astype(np.float32)
    compare(got, want, 1e-3)


def test_large_rows_ragged(backend, coracle):
    bits, k, n, rows = 4, 256, 384, 1000
    w = W.weight_codes(bits, k, n, stream=99)
    sw = W.weight_scales(n, stream=99)
    x = W.activations(rows, k, stream=99).astype(np.float32)
    lin = backend.load(QuantMatrix(bits, k, n, w, sw))
    out = np.zeros((rows, n), np.float32)
    lin.run(x, out, rows)
    np.testing.assert_array_equal(out, coracle.linear(w, sw, x))


@pytest.mark.parametrize("bits", [4, 8])
def test_checkpoint_storage_upload(backend, bits):
    """Upload from compressed-tensors storage (src/model/checkpoint.rs:352-378) gives the
    same results as the QuantMatrix [K][N] upload."""
    k, n, rows = 200, 130, 20
    w = W.weight_codes(bits, k, n, stream=50 + bits)
    sw = W.weight_scales(n, stream=50 + bits)
    if bits == 4:
        kw = (k + 7) // 8
        u = np.zeros((n, kw * 8), np.uint32)
        u[:, :k] = (w.T.astype(np.int32) + 8).astype(np.uint32)
        words = np.zeros((n, kw), np.uint32)
        for j in range(8):
            words |= u[:, j::8] << np.uint32(4 * j)
        storage = words.view(np.int32)
    else:
        storage = np.ascontiguousarray(w.T)
    lin_a = backend.load(QuantMatrix(bits, k, n, w, sw))
    lin_b = backend.load_checkpoint(bits, k, n, storage, sw)
    x = W.activations(rows, k, stream=51).astype(np.float32)
    oa = np.zeros((rows, n), np.float32)
    ob = np.zeros((rows, n), np.float32)
    lin_a.run(x, oa, rows)
    lin_b.run(x, ob, rows)
    np.testing.assert_array_equal(oa, ob)


def test_shard_columns_match_full(backend, coracle):
    bits, k, n, rows = 4, 512, 1024, 24
    w = W.weight_codes(bits, k, n, stream=60)
    sw = W.weight_scales(n, stream=60)
    x = W.activations(rows, k, stream=60).astype(np.float32)
    full = coracle.linear(w, sw, x)
    qm = QuantMatrix(bits, k, n, w, sw)
    for g in (2, 4, 8):
        for r in range(g):
            lo, hi = r * n // g, (r + 1) * n // g
            lin = backend.load_shard(qm, lo, hi)
            out = np.zeros((rows, hi - lo), np.float32)
            lin.run(x, out, rows)
            np.testing.assert_array_equal(out, full[:, lo:hi])


def test_errors_are_status_codes(backend):
    codes, scales = W.kat_matrix(8)
    lin = backend.load(QuantMatrix(8, 256, 256, codes, scales))
    x = W.kat_input(4, 256)
    with pytest.raises(ValueError):
        lin.run(x, np.zeros((4, 255), np.float32), 4)
    with pytest.raises(ValueError):
        lin.run(x, np.zeros((4, 256), np.float32), 0)
    with pytest.raises(ValueError):
        backend.load(QuantMatrix(3, 256, 256, codes, scales))
    bad = scales.copy()
    bad[3] = 0.0
    with pytest.raises(NpuError):
        backend.load(QuantMatrix(8, 256, 256, codes, bad))
    out = torch.zeros((4, 256), dtype=torch.float16, device="cuda")
    with pytest.raises(NpuError):
        lin.run_device(dev(x), out, 4, ldc=100)


@pytest.mark.parametrize("rows", [9, 40, 300, 512])
def test_w4_packed_only_backend(coracle, rows):
    """The memory-lean mode (QLINEAR_BACKEND_W4_PACKED_ONLY): the prefill GEMM unpacks the
    nibbles in shared memory; results must be identical to the oracle (and therefore to
    the default mode, which reads an int8 expansion)."""
    from open_rknpu2_lm_infer_b200 import Backend
    b = Backend(device=0, w4_packed_only=True)
    k, n = 2560, 1024
    w = W.weight_codes(4, k, n, stream=70)
    sw = W.weight_scales(n, stream=70)
    xh = W.activations(rows, k, stream=71)
    lin = b.load(QuantMatrix(4, k, n, w, sw))
    assert lin.device_bytes < k * n  # packed only: 0.5 byte per weight (+ scales)
    y, acc = coracle.linear(w, sw, xh, want_acc=True)
    out = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
    acc_gpu = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
    a = dev(xh)
    lin.run_device(a, out, rows)
    lin.run_device(a, acc_gpu, rows)
    b.check()
    np.testing.assert_array_equal(acc_gpu.cpu().numpy(), acc)
    np.testing.assert_array_equal(out.cpu().numpy(), y.astype(np.float16))
    lin.close()
    b.close()


def test_w4_default_keeps_int8_copy(backend):
    k, n = 512, 256
    lin = backend.load(QuantMatrix(4, k, n, W.weight_codes(4, k, n), W.weight_scales(n)))
    assert lin.device_bytes >= k * n + k * n // 2


def test_weights_outlive_backend_handle():
    """Weights keep their backend alive (src/npu.rs:252-260): freeing the backend handle first
    and the weights afterwards -- or leaving the weights to interpreter exit -- is safe."""
    import subprocess
    import sys
    from open_rknpu2_lm_infer_b200 import Backend
    b = Backend(device=0)
    codes, scales = W.kat_matrix(8)
    lin = b.load(QuantMatrix(8, 256, 256, codes, scales))
    b.close()
    lin.close()
    script = (
        "from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix\n"
        "from open_rknpu2_lm_infer_b200 import workloads as W\n"
        "b = Backend(device=0)\n"
        "c, s = W.kat_matrix(4)\n"
        "keep = b.load(QuantMatrix(4, 256, 256, c, s))\n"
        "b.close()\n")
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", script], cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
