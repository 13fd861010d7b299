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


# ---------------------------------------------------------------------------------------
# Stream-K schedule of the GEMM (csrc/gemm_sm100.cu: plan_gemm, Sched, sk_split), restated
# with the same integer formulas: a split region of sk_tiles tiles walked by groups of pairs
# (one group per token tile), then whole tiles strided over the pairs.  Every (tile,
# k-block) is covered exactly once, every pair gets the same work (+-1 k-block), the segment
# count of a split tile equals sk_split's nseg, and split tiles get distinct workspace slots.

def _sk_plan(ch_tiles, ntt, nkb, maxp):
    tiles = ch_tiles * ntt
    group = min(maxp // ntt, ch_tiles * nkb)
    P = group * ntt
    whole = max(0, tiles // P - 1)
    return P, tiles - whole * P


def _sk_segments(ch_tiles, ntt, nkb, P, sk_tiles, cid):
    base = ch_tiles * ntt - sk_tiles  # whole tiles first, then the split region
    t = cid
    while t < base:
        yield t, 0, nkb
        t += P
    pg, i, g = P // ntt, cid // ntt, cid % ntt
    units = (sk_tiles // ntt) * nkb
    u, end = units * i // pg, units * (i + 1) // pg
    while u < end:
        tc = u // nkb
        kb0 = u - tc * nkb
        kb1 = kb0 + (end - u) if end - u < nkb - kb0 else nkb
        yield base + tc * ntt + g, kb0, kb1
        u += kb1 - kb0


def _sk_split(t, sk_tiles, ntt, nkb, P, tiles):
    t -= tiles - sk_tiles
    g, tc, pg = t % ntt, t // ntt, P // ntt
    units = (sk_tiles // ntt) * nkb
    s0, e0 = tc * nkb, tc * nkb + nkb
    bf = ((s0 + 1) * pg + units - 1) // units
    bl = min((e0 * pg + units - 1) // units - 1, pg - 1)
    return g * pg + bf, (bl - bf + 1 if bl >= bf else 0) + 1


def test_stream_k_schedule_covers_every_iteration_once():
    import random
    rng = random.Random(5)
    cases = [(112, 2, 64, 74), (38, 2, 20, 74), (10, 1, 8, 74), (3, 1, 8, 24), (1, 1, 8, 8),
             (112, 4, 64, 74), (112, 3, 64, 74), (14, 2, 64, 74), (38, 1, 20, 74)]
    cases += [(rng.randint(1, 200), rng.randint(1, 6), rng.randint(8, 80), rng.randint(1, 74))
              for _ in range(3000)]
    for ch_tiles, ntt, nkb, maxp in cases:
        if maxp // ntt < 1:
            continue
        P, sk_tiles = _sk_plan(ch_tiles, ntt, nkb, maxp)
        tiles = ch_tiles * ntt
        assert sk_tiles % ntt == 0 and (tiles - sk_tiles) % P == 0
        seen, work = {}, []
        for cid in range(P):
            segs = list(_sk_segments(ch_tiles, ntt, nkb, P, sk_tiles, cid))
            assert segs, (ch_tiles, ntt, nkb, P, cid)      # no pair is idle
            work.append(sum(b - a for _, a, b in segs))
            for t, kb0, kb1 in segs:
                assert 0 <= t < tiles and 0 <= kb0 < kb1 <= nkb
                assert t < tiles - sk_tiles or (t - (tiles - sk_tiles)) % ntt == cid % ntt
                seen.setdefault(t, []).append((kb0, kb1))
        assert max(work) - min(work) <= 1
        slots = set()
        for t in range(tiles):
            segs = sorted(seen[t])
            assert segs[0][0] == 0 and segs[-1][1] == nkb
            assert all(a[1] == b[0] for a, b in zip(segs, segs[1:]))
            if t < tiles - sk_tiles:
                assert len(segs) == 1
                continue
            slot, nseg = _sk_split(t, sk_tiles, ntt, nkb, P, tiles)
            assert nseg == len(segs), (ch_tiles, ntt, nkb, P, t)
            if nseg > 1:
                assert 0 <= slot < P and slot not in slots
                slots.add(slot)


# Restatement of the GEMM's token-tile choice and tail split (csrc/gemm_sm100.cu plan_gemm,
# csrc/gemm_impl.cuh Sched / tile_geom), with the same integer formulas: the token tile from
# the row count, halved for narrow shards while twice the tiles fit in one wave; whole tiles
# strided over the pairs; the R tiles of a last partial wave (at most half the pairs) each cut
# into S sub-tiles of tok / S tokens, sub-tile j on pair j.  Every (channel tile, token) is
# computed exactly once, over the whole k-loop, and every sub-tile is >= 32 tokens.

def _plan_tok(rows, np_, maxp):
    tiles_m = max(1, (rows + 255) // 256)
    tok = (rows + tiles_m - 1) // tiles_m
    tok = max(32, (tok + 31) // 32 * 32)
    ch_tiles = (np_ + 255) // 256
    while tok >= 128 and tok % 64 == 0 and ch_tiles * ((rows + tok // 2 - 1) // (tok // 2)) <= maxp:
        tok //= 2
    ntt = (rows + tok - 1) // tok
    tiles = ch_tiles * ntt
    R, S = 0, 1
    if tiles > maxp:
        R = tiles % maxp
        while R > 0 and 2 * S * R <= maxp and tok // (2 * S) >= 32 and (tok // (2 * S)) % 32 == 0:
            S *= 2
    return tok, ntt, tiles, (R if S > 1 else 0), S


def _tail_items(tiles, sk_tiles, split, P, cid):
    t = cid
    while t < tiles - sk_tiles:
        yield t
        t += P
    if cid < sk_tiles * split:
        yield tiles + cid


def _tile_geom(t, tiles, ntt, tok, sk_tiles, split):
    if t < tiles:
        tc = t // ntt
        return tc, (t - tc * ntt) * tok, tok
    j = t - tiles
    tile = tiles - sk_tiles + j // split
    tc = tile // ntt
    ntok = tok // split
    return tc, (tile - tc * ntt) * tok + (j % split) * ntok, ntok


def test_token_tile_and_tail_split_cover_every_token_once():
    import random
    rng = random.Random(11)
    # (rows, Np, pairs): cfg4 M=512 on 1 and 8 GPUs, cfg0, ragged and small shapes
    cases = [(512, 28672, 74), (512, 3584, 74), (512, 7168, 74), (512, 14336, 74),
             (512, 9728, 74), (500, 9728, 74), (300, 1024, 74), (9, 256, 74), (8192, 28672, 74)]
    cases += [(rng.randint(9, 3000), rng.randint(1, 150) * 128, rng.randint(1, 74))
              for _ in range(400)]
    hit = {}
    for rows, np_, maxp in cases:
        tok, ntt, tiles, sk_tiles, split = _plan_tok(rows, np_, maxp)
        if (rows, np_, maxp) == (512, 28672, 74):
            assert (tok, tiles, sk_tiles, split) == (256, 224, 2, 8)
        if (rows, np_, maxp) == (512, 3584, 74):
            assert (tok, tiles, sk_tiles, split) == (128, 56, 0, 1)
        P = min(tiles, maxp)
        assert (tiles - sk_tiles) % P == 0 or sk_tiles == 0
        cover = np.zeros(((np_ + 255) // 256, ntt * tok), np.int32)
        for cid in range(P):
            for t in _tail_items(tiles, sk_tiles, split, P, cid):
                tc, tok0, ntok = _tile_geom(t, tiles, ntt, tok, sk_tiles, split)
                assert ntok >= 32 and ntok % 32 == 0 and ntok <= tok
                cover[tc, tok0:tok0 + ntok] += 1
        assert (cover == 1).all(), (rows, np_, maxp)
        hit[split > 1] = True
    assert hit.get(True) and hit.get(False)


# The decode GEMV's skewed row split (csrc/gemv_impl.cuh: gemv_row_start, gemv_skew_q10 and
# the rows_per_cta bound plan() sizes the shared memory for), restated in exact integers.
def _skew_q10(nrows, row_bytes, nseg, grid, mt):
    if mt > 2 or grid < 2:
        return 0
    ramp = 68 * 1024
    cta_bytes = nrows * row_bytes * nseg // grid
    if cta_bytes <= 0:
        return 0
    q = min(410, ramp * 1024 // cta_bytes)
    return q if q >= 16 else 0


def _row_start(j, G, n, q):
    return n * ((1024 + q) * j * G - q * j * j) // (1024 * G * G)


@pytest.mark.parametrize("nrows,row_bytes,nseg,mt", [
    (9728, 2560, 1, 1), (9728, 2560, 1, 2), (6144, 1280, 1, 1), (2560, 4096, 1, 1),
    (9728, 1280, 2, 1), (2560, 9728, 1, 2), (28672, 4096, 1, 1), (151936, 2560, 1, 1),
    (200, 512, 1, 1), (149, 128, 1, 1), (148, 128, 2, 2), (5000, 64, 1, 1)])
@pytest.mark.parametrize("sms", [148, 132, 7])
def test_gemv_skewed_rows_cover_every_row_once(nrows, row_bytes, nseg, mt, sms):
    g = min(sms, nrows)
    q = _skew_q10(nrows, row_bytes, nseg, g, mt)
    if not q:
        return
    pmax = (nrows * (1024 + q) + 1024 * g - 1) // (1024 * g) + 2
    starts = [_row_start(j, g, nrows, q) for j in range(g + 1)]
    assert starts[0] == 0 and starts[-1] == nrows
    counts = np.diff(starts)
    assert counts.min() >= 0 and counts.max() <= pmax  # the kernel's clamp never bites
    # a ramp: non-increasing up to the rounding of one row
    assert np.all(np.diff(counts) <= 1)
    # the int64 products of the kernel's formula stay far below 2^63
    assert nrows * (1024 + q) * g * g < 2 ** 62


def test_gemv_skew_only_at_one_or_two_rows():
    assert _skew_q10(9728, 2560, 1, 148, 4) == 0 and _skew_q10(9728, 2560, 1, 148, 8) == 0
    assert _skew_q10(9728, 2560, 1, 148, 1) == 410
    assert _skew_q10(151936, 2560, 1, 148, 1) == 27  # the lm_head: a 2.6% ramp
