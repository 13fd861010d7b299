"""Host-side models of the device data layouts and warp algorithms (CPU only).

These restate, in numpy, what the kernels do with indices -- the W4 nibble layout written
by pack.cu and read by gemv.cu / gemm_sm100.cu, the offset-binary correction, the
128-byte swizzle the converter writes, and the GEMV's halving butterfly -- so that an
index error shows up here before any GPU run."""
import numpy as np
import pytest

from open_rknpu2_lm_infer_b200 import workloads as W


def pack_w4(codes_kn: np.ndarray, kp: int, np_: int) -> np.ndarray:
    """Device W4 layout: word w of row n = codes k = 8w..8w+7, byte j = u(8w+j) |
    u(8w+j+4) << 4, u = code + 8, padding code 0."""
    k, n = codes_kn.shape
    u = np.full((np_, kp), 8, np.uint8)
    u[:n, :k] = (codes_kn.T.astype(np.int16) + 8).astype(np.uint8)
    u = u.reshape(np_, kp // 8, 8)
    b = (u[:, :, 0:4] | (u[:, :, 4:8] << 4)).astype(np.uint8)  # [np, words, 4]
    return b.reshape(np_, kp // 2)


def unpack_words(packed_row: np.ndarray) -> np.ndarray:
    """What gemv.cu / the converter compute: for each 32-bit word, lo = w & 0x0F0F0F0F
    gives codes 8w..8w+3, hi = (w >> 4) & 0x0F0F0F0F gives 8w+4..8w+7 (as u = code+8)."""
    words = packed_row.view(np.uint32)
    lo = (words & np.uint32(0x0F0F0F0F)).view(np.uint8).reshape(-1, 4)
    hi = ((words >> np.uint32(4)) & np.uint32(0x0F0F0F0F)).view(np.uint8).reshape(-1, 4)
    return np.concatenate([lo, hi], axis=1).reshape(-1)


def test_w4_layout_roundtrip_and_correction():
    k, n, kp, np_ = 200, 70, 256, 128
    codes = W.weight_codes(4, k, n, stream=5)
    packed = pack_w4(codes, kp, np_)
    x = np.random.default_rng(1).integers(-127, 128, size=(3, kp)).astype(np.int8)
    x[:, k:] = 0
    for row in range(np_):
        u = unpack_words(packed[row]).astype(np.int32)
        want_codes = np.zeros(kp, np.int32)
        if row < n:
            want_codes[:k] = codes[:, row]
        np.testing.assert_array_equal(u - 8, want_codes)
        # dp4a(u, x) then subtract 8 * sum(x): the exact signed dot product
        for m in range(3):
            acc_u = int((u * x[m].astype(np.int32)).sum())
            assert acc_u - 8 * int(x[m].astype(np.int32).sum()) == \
                int((want_codes * x[m].astype(np.int32)).sum())


def test_converter_swizzle_is_a_permutation_of_16_byte_chunks():
    """The W4 converter writes logical chunk c of row r at physical chunk c ^ (r % 8):
    the 128-byte swizzle TMA uses for the activation tile, so both MMA operands share one
    descriptor format.  Each thread owns packed chunk cp (codes 32cp..32cp+31) of its row
    and writes output chunks 2cp and 2cp+1."""
    seen = np.zeros((128, 8), bool)
    for ct in range(128):
        cp = ct & 3
        for j in range(4):
            row = (ct >> 2) + 32 * j
            for c in (2 * cp, 2 * cp + 1):
                phys = c ^ (row & 7)
                assert not seen[row, phys]
                seen[row, phys] = True
    assert seen.all()
    # bank check: the 8 threads of one 128-bit store phase hit 8 distinct 16-byte bank groups
    for phase in range(16):
        groups = set()
        for ct in range(phase * 8, phase * 8 + 8):
            row = (ct >> 2)
            groups.add((2 * (ct & 3)) ^ (row & 7))
        assert len(groups) == 8


@pytest.mark.parametrize("v", [1, 2, 4, 8, 16, 32])
def test_gemv_halving_butterfly(v):
    """warp_reduce_spread<V> in gemv.cu: after it, lane l holds the warp-wide sum of value
    index l // (32 // V)."""
    rng = np.random.default_rng(v)
    vals = rng.integers(-1000, 1000, size=(32, v))
    want = vals.sum(0)
    lanes = [list(vals[l]) for l in range(32)]
    off = 16
    n = v
    while n > 1:
        new = []
        for l in range(32):
            upper = (l & off) != 0
            p = l ^ off
            cur = lanes[l][:]
            for i in range(n // 2):
                send_p = lanes[p][i] if ((p & off) != 0) else lanes[p][i + n // 2]
                keep = cur[i + n // 2] if upper else cur[i]
                cur[i] = keep + send_p
            new.append(cur)
        lanes = new
        n //= 2
        off >>= 1
    while off >= 1:
        lanes = [[lanes[l][0] + lanes[l ^ off][0]] + lanes[l][1:] for l in range(32)]
        off >>= 1
    for l in range(32):
        assert lanes[l][0] == want[l // (32 // v)]


def test_kat_generators_match_reference_formulas():
    codes, scales = W.kat_matrix(4)
    assert codes[0, 0] == -8 and codes[0, 1] == (13 % 16) - 8
    assert codes[1, 0] == ((256 * 13 + 7) % 16) - 8
    assert scales[11] == np.float32(0.002)
    x = W.kat_input(2, 256)
    assert x[0, 0] == np.float32(-1.0)
    assert x[1, 0] == np.float32(((256 * 17 + 3) % 127) / np.float32(63.0) - np.float32(1.0))


def test_workload_distributions():
    x = W.activations(64, 2560)
    assert x.dtype == np.float16
    col_amax = np.abs(x.astype(np.float32)).max(0)
    assert (col_amax > 15).sum() >= 20          # ~26 outlier channels x20
    w4 = W.weight_codes(4, 64, 64)
    assert w4.min() == -8 and w4.max() == 7
    w8 = W.weight_codes(8, 256, 256)
    assert w8.min() == -127 and w8.max() == 127
    s = W.weight_scales(1000)
    assert s.min() >= 1e-3 and s.max() <= 1e-2
    bits = W.layer_bits()
    frac = np.mean([b == 4 for row in bits for b in row])
    assert 0.6 < frac < 0.8
