"""CPU oracle for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` /
``--impl reference`` legs import this module, and only as the checker or as the
timed CPU baseline.  The product package never imports it.

Two restatements of the reference's CPU implementation of the path live here, both
following the ``oracle`` function of src/npu.rs:1097-1121 of open_rknpu2_lm_infer:

* ``NumpyOracle`` -- vectorised numpy, for small and medium cases;
* ``COracle``     -- ctypes binding of ``oracle/qlinear_ref.c`` (OpenMP), used for large
  shapes and as the CPU baseline that bench.py times.

Arithmetic (per activation row):
  amax = max |x| (NaN ignored, src/npu.rs:1101); scale = 1 if amax == 0 else
  max(amax/127, FLT_MIN) (:1102-1106); q = clamp(round_away(x * (1/scale)), -127, 127),
  NaN -> 0 (:1107-1110); acc = sum q*w in i32 (:1111-1116); y = (f32(acc)*scale)*s_w (:1117).

Parity is pinned by tests/golden/ (see tests/golden/make_golden.py), whose act-quant
vectors come from the reference's own numpy ``quantize`` in
scripts/qwen35/audit_batch_attention_trace.py:17-23.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ROUND_AWAY = 0  # f32::round, the reference's rounding (src/npu.rs:1109)
ROUND_EVEN = 1  # round-half-even, opt-in only

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqlinear_oracle.so")

F32_MIN = np.float32(np.finfo(np.float32).tiny)


# ----------------------------------------------------------------------------- numpy port
def round_away(v: np.ndarray) -> np.ndarray:
    """f32::round: nearest integer, halfway cases away from zero (exact in f32).

    Implemented as trunc(v) + sign(v) when |v - trunc(v)| >= 0.5; the fractional part
    v - trunc(v) is exact in binary floating point, so there is no double rounding
    (unlike floor(|v| + 0.5), which maps 0.49999997 to 1).
    """
    v = np.asarray(v, dtype=np.float32)
    t = np.trunc(v)
    frac = np.abs(v - t)
    return np.where(frac >= np.float32(0.5), t + np.sign(v), t).astype(np.float32)


def act_quant(x: np.ndarray, round_mode: int = ROUND_AWAY):
    """Per-row dynamic int8 quantisation (src/npu.rs:1099-1110).

    x: [rows, K] float32 (fp16 inputs must be widened with ``.astype(np.float32)``,
    which is exact).  Returns (codes int8 [rows, K], scales float32 [rows]).
    """
    x = np.asarray(x, dtype=np.float32)
    assert x.ndim == 2
    with np.errstate(invalid="ignore", over="ignore"):
        ax = np.abs(x)
        amax = np.where(np.isnan(ax), np.float32(0), ax).max(axis=1) if x.shape[1] else \
            np.zeros(x.shape[0], np.float32)
        amax = amax.astype(np.float32)
        scale = np.where(amax == 0, np.float32(1),
                         np.maximum(amax / np.float32(127), F32_MIN)).astype(np.float32)
        inv = (np.float32(1) / scale).astype(np.float32)
        scaled = (x * inv[:, None]).astype(np.float32)
        r = round_away(scaled) if round_mode == ROUND_AWAY else np.rint(scaled).astype(np.float32)
        r = np.where(np.isnan(r), np.float32(0), np.clip(r, -127, 127))
    return r.astype(np.int8), scale


def int_gemm(codes: np.ndarray, w_kn: np.ndarray) -> np.ndarray:
    """acc[m, n] = sum_k codes[m, k] * w[k, n], exact (src/npu.rs:1111-1116)."""
    acc = codes.astype(np.int64) @ w_kn.astype(np.int64)
    assert np.all(np.abs(acc) < 2**31)
    return acc.astype(np.int32)


def dequant(acc: np.ndarray, sa: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """y = (f32(acc) * s_a) * s_w with two RN f32 products (src/npu.rs:1117)."""
    t = (acc.astype(np.float32) * sa.astype(np.float32)[:, None]).astype(np.float32)
    return (t * sw.astype(np.float32)[None, :]).astype(np.float32)


def linear(w_kn: np.ndarray, w_scales: np.ndarray, x: np.ndarray, round_mode: int = ROUND_AWAY,
           return_parts: bool = False):
    """The whole oracle of src/npu.rs:1097-1121 on f32 input [rows, K]."""
    codes, sa = act_quant(x, round_mode)
    acc = int_gemm(codes, w_kn)
    y = dequant(acc, sa, w_scales)
    if return_parts:
        return y, codes, sa, acc
    return y


def swiglu(y: np.ndarray) -> np.ndarray:
    """mid = gate / (1 + exp(-gate)) * up, gate = y[:, :N/2], up = y[:, N/2:]
    (expectation of src/npu.rs:1202-1208), evaluated in f32."""
    y = np.asarray(y, dtype=np.float32)
    h = y.shape[1] // 2
    gate, up = y[:, :h], y[:, h:]
    with np.errstate(over="ignore"):
        return (gate / (np.float32(1) + np.exp(-gate)) * up).astype(np.float32)


def count_ties(x: np.ndarray) -> int:
    """How many elements of x land exactly on a .5 after scaling (the only inputs where
    ties-away and half-even differ)."""
    x = np.asarray(x, dtype=np.float32)
    _, sa = act_quant(x)
    with np.errstate(invalid="ignore", over="ignore"):
        scaled = (x * (np.float32(1) / sa)[:, None]).astype(np.float32)
        return int(np.count_nonzero(np.abs(scaled - np.trunc(scaled)) == np.float32(0.5)))


# ----------------------------------------------------------------------------- C oracle
def build(force: bool = False) -> str:
    """Compile oracle/qlinear_ref.c (gcc, OpenMP) into oracle/_build/."""
    if force or not os.path.exists(_LIB_PATH) or \
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "qlinear_ref.c")):
        subprocess.run(["make", "-s", "-C", _HERE] + (["-B"] if force else []), check=True)
    return _LIB_PATH


class COracle:
    """ctypes binding of oracle/qlinear_ref.c."""

    def __init__(self, path: str | None = None):
        path = path or _LIB_PATH
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        for name, args in {
            "qref_act_quant_f32": [P, I64, I64, I, P, P, P],
            "qref_act_quant_f16": [P, I64, I64, I, P, P, P],
            "qref_int_gemm": [P, I64, I64, P, I64, P],
            "qref_dequant": [P, I64, I64, P, P, P],
            "qref_linear_f32": [P, P, I64, I64, P, I64, I, P, P],
            "qref_linear_f16": [P, P, I64, I64, P, I64, I, P, P],
            "qref_swiglu": [P, I64, I64, P],
        }.items():
            fn = getattr(self.lib, name)
            fn.argtypes = args
            fn.restype = I
        self.lib.qref_max_threads.restype = I
        self.lib.qref_set_threads.argtypes = [I]

    @staticmethod
    def _p(a: np.ndarray):
        assert a.flags.c_contiguous
        return a.ctypes.data_as(ctypes.c_void_p)

    def max_threads(self) -> int:
        return self.lib.qref_max_threads()

    def set_threads(self, n: int) -> None:
        self.lib.qref_set_threads(int(n))

    def act_quant(self, x: np.ndarray, round_mode: int = ROUND_AWAY):
        x = np.ascontiguousarray(x)
        rows, k = x.shape
        codes = np.empty((rows, k), np.int8)
        scales = np.empty(rows, np.float32)
        rowsums = np.empty(rows, np.int32)
        fn = self.lib.qref_act_quant_f16 if x.dtype == np.float16 else self.lib.qref_act_quant_f32
        if x.dtype not in (np.float16, np.float32):
            raise TypeError(x.dtype)
        rc = fn(self._p(x), rows, k, round_mode, self._p(codes), self._p(scales), self._p(rowsums))
        assert rc == 0
        return codes, scales, rowsums

    def linear(self, w_kn: np.ndarray, w_scales: np.ndarray, x: np.ndarray,
               round_mode: int = ROUND_AWAY, want_acc: bool = False):
        w_kn = np.ascontiguousarray(w_kn, dtype=np.int8)
        w_scales = np.ascontiguousarray(w_scales, dtype=np.float32)
        x = np.ascontiguousarray(x)
        rows, k = x.shape
        n = w_kn.shape[1]
        assert w_kn.shape[0] == k and w_scales.shape == (n,)
        y = np.empty((rows, n), np.float32)
        acc = np.empty((rows, n), np.int32) if want_acc else None
        fn = self.lib.qref_linear_f16 if x.dtype == np.float16 else self.lib.qref_linear_f32
        rc = fn(self._p(w_kn), self._p(w_scales), k, n, self._p(x), rows, round_mode, self._p(y),
                self._p(acc) if acc is not None else None)
        assert rc == 0
        return (y, acc) if want_acc else y

    def swiglu(self, y: np.ndarray) -> np.ndarray:
        y = np.ascontiguousarray(y, dtype=np.float32)
        rows, n = y.shape
        mid = np.empty((rows, n // 2), np.float32)
        assert self.lib.qref_swiglu(self._p(y), rows, n, self._p(mid)) == 0
        return mid
