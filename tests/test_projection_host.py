"""Projection orchestration (src/model/projection.rs:142-243, src/model/checkpoint.rs:392-423)
on the CPU: grouping of adjacent same-bit modules, concatenation layout, column offsets,
suffix runs, the swiglu rule.  The linears are the numpy oracle behind a fake backend, so
this checks the host logic only; tests/test_gpu_projection.py runs the same orchestration
on the CUDA library."""
import numpy as np
import pytest

from oracle import oracle as O
from open_rknpu2_lm_infer_b200 import MatrixLoader, Projection, QuantMatrix, concatenate


def matrix(bits, k, n, seed):
    rng = np.random.default_rng(seed)
    lo, hi = (-8, 7) if bits == 4 else (-127, 127)
    codes = rng.integers(lo, hi + 1, size=(k, n), dtype=np.int8)
    scales = np.exp(rng.uniform(np.log(1e-3), np.log(1e-2), n)).astype(np.float32)
    return QuantMatrix(bits, k, n, codes.reshape(-1), scales)


class FakeLinear:
    """Linear with the oracle's arithmetic and the CUDA Linear's host methods."""

    def __init__(self, m: QuantMatrix):
        self.m, self.bits = m, m.bits
        self.w = np.asarray(m.codes, np.int8).reshape(m.k, m.n)

    def n(self):
        return self.m.n

    def k(self):
        return self.m.k

    def _y(self, x, rows):
        return O.linear(self.w, self.m.scales, np.asarray(x, np.float32).reshape(-1, self.m.k)[:rows])

    def run(self, x, out, rows):
        out.reshape(rows, self.m.n)[:] = self._y(x, rows)

    def run_columns(self, x, out, rows, ldc, col=0, swiglu=False):
        assert not swiglu
        flat = out.reshape(-1)
        y = self._y(x, rows)
        for r in range(rows):
            flat[r * ldc + col:r * ldc + col + self.m.n] = y[r]

    def run_swiglu(self, x, out, rows):
        out.reshape(rows, self.m.n // 2)[:] = O.swiglu(self._y(x, rows))
        return True

    def close(self):
        pass


class FakeBackend:
    def __init__(self):
        self.loaded = []

    def load(self, m, reload=None):
        self.loaded.append((m, reload))
        return FakeLinear(m)


K = 96
MODULES = [("q", 48, 4), ("k", 16, 4), ("v", 16, 8), ("o", 32, 4)]


def loader():
    return MatrixLoader({name: matrix(bits, K, n, i) for i, (name, n, bits) in enumerate(MODULES)})


def test_concatenate_layout_and_errors():
    a, b = matrix(4, 16, 3, 1), matrix(4, 16, 5, 2)
    c = concatenate([a, b])
    assert (c.bits, c.k, c.n) == (4, 16, 8)
    full = np.asarray(c.codes).reshape(16, 8)
    np.testing.assert_array_equal(full[:, :3], np.asarray(a.codes).reshape(16, 3))
    np.testing.assert_array_equal(full[:, 3:], np.asarray(b.codes).reshape(16, 5))
    np.testing.assert_array_equal(c.scales, np.concatenate([a.scales, b.scales]))
    assert concatenate([a]) is a
    with pytest.raises(ValueError, match="empty"):
        concatenate([])
    with pytest.raises(ValueError, match="identical bit widths and K"):
        concatenate([a, matrix(8, 16, 3, 3)])
    with pytest.raises(ValueError, match="identical bit widths and K"):
        concatenate([a, matrix(4, 32, 3, 4)])


def test_grouping_offsets_and_reload():
    be, ld = FakeBackend(), loader()
    p = Projection.load(be, ld, [(n, c) for n, c, _ in MODULES], K)
    # q,k share W4 -> one matrix; v is W8; o is W4 again but not adjacent to q,k
    assert [(lin.m.bits, lin.m.n, off) for lin, off in p.parts] == [(4, 64, 0), (8, 16, 64),
                                                                   (4, 32, 80)]
    assert p.width == 112 and p.scratch_width() == 64
    first, reload = be.loaded[0]
    again = reload()
    np.testing.assert_array_equal(again.codes, first.codes)
    np.testing.assert_array_equal(again.scales, first.scales)


@pytest.mark.parametrize("rows", [1, 3, 17])
def test_run_and_suffix_match_per_module_oracle(rows):
    be, ld = FakeBackend(), loader()
    p = Projection.load(be, ld, [(n, c) for n, c, _ in MODULES], K)
    x = np.random.default_rng(7).standard_normal((rows, K)).astype(np.float32)
    per = {name: O.linear(np.asarray(ld.matrices[name].codes, np.int8).reshape(K, n),
                          ld.matrices[name].scales, x) for name, n, _ in MODULES}
    out = np.full((rows, p.width), np.nan, np.float32)
    p.run(x, out, rows)
    np.testing.assert_array_equal(out, np.concatenate([per[n] for n, _, _ in MODULES], axis=1))
    # suffix from the W8 part (KV-only style): [v | o]
    tail = np.full((rows, 48), np.nan, np.float32)
    p.run_from(1, x, tail, rows)
    np.testing.assert_array_equal(tail, np.concatenate([per["v"], per["o"]], axis=1))
    # single-part suffix runs the linear directly
    last = np.zeros((rows, 32), np.float32)
    p.run_from(2, x, last, rows)
    np.testing.assert_array_equal(last, per["o"])
    with pytest.raises(ValueError, match="suffix shape"):
        p.run_from(1, x, np.zeros((rows, 47), np.float32), rows)
    with pytest.raises(ValueError, match="invalid projection suffix"):
        p.run_from(3, x, tail, rows)


def test_swiglu_only_for_a_single_matrix():
    ld = MatrixLoader({"gate": matrix(4, K, 32, 11), "up": matrix(4, K, 32, 12),
                       "down": matrix(8, K, 32, 13)})
    fused = Projection.load(FakeBackend(), ld, [("gate", 32), ("up", 32)], K)
    assert len(fused.parts) == 1
    x = np.random.default_rng(3).standard_normal((2, K)).astype(np.float32)
    mid = np.zeros((2, 32), np.float32)
    assert fused.run_swiglu(x, mid, 2)
    split = Projection.load(FakeBackend(), ld, [("gate", 32), ("down", 32)], K)
    assert len(split.parts) == 2
    assert not split.run_swiglu(x, mid, 2)
