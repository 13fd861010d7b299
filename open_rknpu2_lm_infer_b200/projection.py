"""Projection orchestration over the quantized linears (the quantized part of the
reference's src/model/projection.rs and the fused-matrix concatenation of
src/model/checkpoint.rs:392-423).

A decoder projection is a list of modules that read the same input row and whose outputs
sit side by side in one fused row (q/k/v, gate/up).  ``Projection.load`` walks the modules
in order, groups adjacent modules that share a bit width, concatenates each group into one
``QuantMatrix`` (codes [K][N_1 + N_2 + ...], scales in the same order) and uploads it as one
linear, remembering its column offset (src/model/projection.rs:142-189).  ``run_from``
runs a suffix of the parts (src/model/projection.rs:200-232): one part writes the output
directly; several parts each write their column range of the fused [rows][width] output.
The reference routes every part but the first row through a scratch buffer and a
row-by-row copy; here each part's call writes its columns in place
(``qlinear_run_f32_ex`` / the device path's output stride), so there is no scratch and no
copy.  ``run_swiglu`` fuses only when the projection is one matrix
(src/model/projection.rs:233-243).

Floating-point projections (``Linear::Floating`` / ``SplitK``) are not part of the
quantized path and are not mirrored.
"""
from __future__ import annotations

from typing import Protocol

import numpy as np

from . import _lib as L
from .npu import Backend, Linear, QuantMatrix


class QuantLoader(Protocol):
    """What Projection.load needs from a checkpoint (src/model/checkpoint.rs:320-389)."""

    def bits(self, name: str) -> int: ...

    def load(self, name: str, n: int, k: int) -> QuantMatrix: ...


class MatrixLoader:
    """In-memory QuantLoader: module name -> QuantMatrix."""

    def __init__(self, matrices: dict[str, QuantMatrix]):
        self.matrices = dict(matrices)

    def bits(self, name: str) -> int:
        return self.matrices[name].bits

    def load(self, name: str, n: int, k: int) -> QuantMatrix:
        m = self.matrices[name]
        if (m.n, m.k) != (n, k):
            raise ValueError(f"{name}: expected [{k}][{n}], found [{m.k}][{m.n}]")
        return m


def concatenate(matrices: list[QuantMatrix]) -> QuantMatrix:
    """src/model/checkpoint.rs:392-423: one [K][sum N] matrix, columns in module order."""
    if not matrices:
        raise ValueError("empty fused projection")
    if len(matrices) == 1:
        return matrices[0]
    bits, k = matrices[0].bits, matrices[0].k
    if any(m.bits != bits or m.k != k for m in matrices):
        raise ValueError("fused projections require identical bit widths and K")
    codes = np.concatenate(
        [np.asarray(m.codes, dtype=np.int8).reshape(k, m.n) for m in matrices], axis=1)
    scales = np.concatenate([np.asarray(m.scales, dtype=np.float32).reshape(-1)
                             for m in matrices])
    return QuantMatrix(bits, k, int(codes.shape[1]), np.ascontiguousarray(codes).reshape(-1),
                       scales)


class Projection:
    def __init__(self):
        self.parts: list[tuple[Linear, int]] = []  # (linear, column offset)
        self.width = 0

    @classmethod
    def load(cls, backend: Backend, loader: QuantLoader, modules: list[tuple[str, int]],
             k: int, cpu=None) -> "Projection":
        """src/model/projection.rs:142-189.  `modules`: (name, n) in fused column order;
        `cpu` (the reference's thread pool) is accepted and unused."""
        result = cls()
        first = 0
        while first < len(modules):
            bits = loader.bits(modules[first][0])
            last = first + 1
            while last < len(modules) and loader.bits(modules[last][0]) == bits:
                last += 1
            group = list(modules[first:last])

            def reload(group=group):
                return concatenate([loader.load(name, n, k) for name, n in group])

            matrix = reload()
            linear = backend.load(matrix, reload)
            result.parts.append((linear, result.width))
            result.width += matrix.n
            first = last
        return result

    def close(self) -> None:
        for linear, _ in self.parts:
            linear.close()
        self.parts = []

    def scratch_width(self) -> int:
        """src/model/projection.rs:131-141 (kept for API parity: no scratch is used)."""
        if len(self.parts) <= 1:
            return 0
        return max(linear.n() for linear, _ in self.parts)

    def run(self, input: np.ndarray, output: np.ndarray, rows: int, scratch=None) -> None:
        self.run_from(0, input, output, rows, scratch)

    def run_from(self, first: int, input: np.ndarray, output: np.ndarray, rows: int,
                 scratch=None) -> None:
        """src/model/projection.rs:200-232: run parts[first:] into output [rows][width - base]
        (base = the first part's column offset)."""
        if not 0 <= first < len(self.parts):
            raise ValueError("invalid projection suffix")
        base = self.parts[first][1]
        width = self.width - base
        if output.size != rows * width:
            raise ValueError("projection suffix shape mismatch")
        if len(self.parts) - first == 1:
            self.parts[first][0].run(input, output, rows)
            return
        for linear, offset in self.parts[first:]:
            linear.run_columns(input, output, rows, ldc=width, col=offset - base)

    def run_swiglu(self, input: np.ndarray, output: np.ndarray, rows: int) -> bool:
        """src/model/projection.rs:233-243: fused only when the projection is one matrix."""
        if len(self.parts) != 1:
            return False
        return self.parts[0][0].run_swiglu(input, output, rows)

    def run_device(self, a, out, rows: int, first: int = 0, stream=None) -> None:
        """Device-resident run_from: `a` [rows][K] fp16/f32 and `out` [rows][width - base]
        (fp16 or f32) device tensors; each part writes its columns with the output stride."""
        if not 0 <= first < len(self.parts):
            raise ValueError("invalid projection suffix")
        base = self.parts[first][1]
        width = self.width - base
        if tuple(out.shape) != (rows, width) or not out.is_contiguous():
            raise ValueError("projection suffix shape mismatch")
        s = str(out.dtype)
        out_type, elem = (L.F16, 2) if "float16" in s else (L.F32, 4) if "float32" in s else (None, 0)
        if out_type is None:
            raise TypeError(s)
        for linear, offset in self.parts[first:]:
            linear.run_device(a, out.data_ptr() + elem * (offset - base), rows, ldc=width,
                              stream=stream, out_type=out_type)
