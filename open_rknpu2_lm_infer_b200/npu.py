"""Host-side mirror of the reference's quantized-linear backend API.

Same names, argument meaning and error behaviour as ``crate::npu`` of
open_rknpu2_lm_infer (src/npu.rs), with the RK3588 NPU replaced by the sm_100a CUDA
library behind include/qlinear.h:

=====================================  =============================================
reference (src/npu.rs)                 here
=====================================  =============================================
``QuantMatrix`` :112-118               ``QuantMatrix`` (codes [K][N] int8, scales [N])
``Backend::new(options, domain)`` :310 ``Backend(device=..)``
``Backend::load(matrix, reload)`` :368 ``Backend.load(matrix, reload=None)``
``Backend::prepare(rows)`` :595        ``Backend.prepare(rows)``
``Backend::retain_workspaces`` :616    ``Backend.retain_workspaces(rows)``
``Backend::weight_bytes`` :624         ``Backend.weight_bytes()``
``Backend::tune_operations`` :627      ``Backend.tune_operations()`` (always 0)
``Backend::stats`` :631                ``Backend.stats()`` (dict)
``Linear::k / n`` :1000-1005           ``Linear.k() / n()``
``Linear::run`` :1006                  ``Linear.run(input, output, rows)``
``Linear::run_swiglu`` :1009           ``Linear.run_swiglu(input, output, rows)``
=====================================  =============================================

Errors raise ``NpuError`` with the message shape of ``check()`` (src/npu.rs:138-144):
``"{op}: {detail} ({rc})"``.  ``run``'s shape check is the one of src/npu.rs:1028-1031.
Differences: rows may exceed 256 (no M-bucket cap), ``run_swiglu`` returns True for any
bits and rows (the CUDA path always fuses), no tuning material is kept (``reload`` is
accepted and never called).  The device-resident entry point ``Linear.run_device``
(fp16 in / fp16 out, caller stream) has no reference counterpart.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass

import numpy as np

from . import _lib as L


def _dtype_code(t) -> int:
    s = str(getattr(t, "dtype", ""))
    if "float16" in s:
        return L.F16
    if "float32" in s:
        return L.F32
    if "int32" in s:
        return L.I32
    raise TypeError(s)


class NpuError(RuntimeError):
    def __init__(self, op: str, rc: int):
        self.op, self.rc = op, rc
        super().__init__(f"{op}: {L.strerror(rc)} ({rc})")


def _check(rc: int, op: str) -> None:
    if rc != 0:
        raise NpuError(op, rc)


def _ptr(a) -> int:
    """Address of a numpy array (host) or torch tensor (device or host)."""
    if isinstance(a, np.ndarray):
        assert a.flags.c_contiguous, "buffers must be C-contiguous"
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        assert a.is_contiguous(), "tensors must be contiguous"
        return a.data_ptr()
    if isinstance(a, int):
        return a
    raise TypeError(type(a))


@dataclass
class QuantMatrix:
    """Weight container of src/npu.rs:112-118: codes int8 in [K][N] order (k*N + n),
    W4 codes in [-8, 7] one per byte, W8 codes in [-127, 127]; scales f32 [N] > 0."""
    bits: int
    k: int
    n: int
    codes: np.ndarray
    scales: np.ndarray


class Backend:
    """Owns the CUDA device context, a host-path stream and the per-call workspaces
    (src/npu.rs:230-254).  Single-threaded, like the reference's Rc<RefCell<..>>."""

    def __init__(self, device: int = 0, round_mode: int = L.ROUND_AWAY, max_rows: int = 256,
                 w4_packed_only: bool = False, gemm_stream_k: bool = False,
                 swiglu_unfused: bool = False):
        self._lib = L.load()
        cfg = L.BackendConfig()
        self._lib.qlinear_backend_config_init(ctypes.byref(cfg))
        cfg.device, cfg.round_mode, cfg.max_rows = device, round_mode, max_rows
        cfg.flags = ((L.BACKEND_W4_PACKED_ONLY if w4_packed_only else 0) |
                     (L.BACKEND_GEMM_STREAM_K if gemm_stream_k else 0) |
                     (L.BACKEND_SWIGLU_UNFUSED if swiglu_unfused else 0))
        raw = self._lib.qlinear_backend_create(ctypes.byref(cfg))
        if not raw:
            raise NpuError("create CUDA backend", self._lib.qlinear_last_status())
        self._raw = raw
        self.device = device
        self._tune_calls = 0

    # -- lifetime -----------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_raw", None):
            self._lib.qlinear_backend_free(self._raw)
            self._raw = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def raw(self):
        if not self._raw:
            raise NpuError("backend", L.QLINEAR_ERR_STATE)
        return self._raw

    # -- Backend API (src/npu.rs:368-661) -----------------------------------------
    def load(self, matrix: QuantMatrix, reload=None) -> "Linear":
        """Backend::load (src/npu.rs:368-484): validates and uploads one QuantMatrix."""
        if matrix.bits not in (4, 8):
            raise ValueError("linear weights must use 4 or 8 bits")
        if not (0 < matrix.k <= 2**31 - 1 and 0 < matrix.n <= 2**31 - 1):
            raise ValueError("invalid linear dimensions")
        codes = np.ascontiguousarray(matrix.codes, dtype=np.int8).reshape(-1)
        scales = np.ascontiguousarray(matrix.scales, dtype=np.float32).reshape(-1)
        if codes.size != matrix.k * matrix.n or scales.size != matrix.n:
            raise ValueError("linear weight shape mismatch")
        return Linear._create(self, matrix.bits, matrix.k, matrix.n, codes, scales)

    def load_shard(self, matrix: QuantMatrix, n_begin: int, n_end: int) -> "Linear":
        """Column slice [n_begin, n_end) of a QuantMatrix (split-N rank shard)."""
        codes = np.ascontiguousarray(matrix.codes, dtype=np.int8).reshape(-1)
        scales = np.ascontiguousarray(matrix.scales, dtype=np.float32).reshape(-1)
        if codes.size != matrix.k * matrix.n or scales.size != matrix.n:
            raise ValueError("linear weight shape mismatch")
        return Linear._create(self, matrix.bits, matrix.k, matrix.n, codes, scales,
                              shard=(n_begin, n_end))

    def load_checkpoint(self, bits: int, k: int, n: int, storage: np.ndarray,
                        scales: np.ndarray) -> "Linear":
        """Upload straight from compressed-tensors storage (src/model/checkpoint.rs:352-378):
        W4 ``weight_packed`` int32 [N][ceil(K/8)], W8 ``weight`` int8 [N][K]."""
        storage = np.ascontiguousarray(storage)
        scales = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        return Linear._create(self, bits, k, n, storage, scales, checkpoint=True)

    def prepare(self, rows: int) -> None:
        """Backend::prepare (src/npu.rs:595-615): size the workspaces for `rows`."""
        if rows < 1:
            raise ValueError("linear batch must be >= 1")
        _check(self._lib.qlinear_backend_prepare(self.raw, rows), "prepare workspaces")

    def retain_workspaces(self, rows) -> None:
        """Backend::retain_workspaces (src/npu.rs:616-623).  The CUDA backend keeps one
        workspace sized for the largest call, so there is nothing per bucket to drop."""
        for r in rows:
            if r < 1:
                raise ValueError("linear batch must be >= 1")

    def weight_bytes(self) -> int:
        return int(self.stats()["weight_payload_bytes"])

    def tune_operations(self) -> int:
        return 0

    def stats(self) -> dict:
        n = self._lib.qlinear_backend_stats(self.raw, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        self._lib.qlinear_backend_stats(self.raw, buf, n + 1)
        return json.loads(buf.value.decode())

    def launches(self) -> int:
        return int(self._lib.qlinear_backend_launches(self.raw))

    def profile(self, enable: bool) -> None:
        """Per-kernel device timing (the reference's `timings` argument, src/npu.rs:1047)."""
        _check(self._lib.qlinear_backend_profile(self.raw, 1 if enable else 0), "profile")

    def profile_collect(self):
        """(quant_ms_total, main_ms_total, calls) since the last collect."""
        q, m, c = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
        _check(self._lib.qlinear_backend_profile_collect(self.raw, ctypes.byref(q),
                                                         ctypes.byref(m), ctypes.byref(c)),
               "profile collect")
        return q.value, m.value, c.value

    def interleave_columns(self, src, dst, shards: int, rows: int, shard_cols: int,
                           elem_bytes: int, stream=None) -> None:
        """dst[m][s*shard_cols + j] = src[s][m][j] (split-N output assembly)."""
        _check(self._lib.qlinear_interleave_columns(self.raw, _ptr(src), _ptr(dst), shards, rows,
                                                    shard_cols, elem_bytes, stream),
               "interleave columns")

    def check(self, stream=None) -> None:
        _check(self._lib.qlinear_backend_check(self.raw, stream), "device check")

    # -- split-N exchange buffers (qlinear_peer_buffer_*) -----------------------------
    def peer_buffer_create(self, nbytes: int) -> tuple[int, bytes]:
        """Device buffer on this backend's GPU + its CUDA IPC handle (for the peers)."""
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * L.IPC_HANDLE_BYTES)()
        _check(self._lib.qlinear_peer_buffer_create(self.raw, nbytes, ctypes.byref(ptr), handle),
               "peer buffer create")
        return int(ptr.value), bytes(handle)

    def peer_buffer_open(self, handle: bytes) -> int:
        """Map a peer's exchange buffer (its IPC handle) into this process."""
        ptr = ctypes.c_void_p()
        h = (ctypes.c_ubyte * L.IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _check(self._lib.qlinear_peer_buffer_open(self.raw, h, ctypes.byref(ptr)), "peer buffer open")
        return int(ptr.value)

    def peer_buffer_free(self, ptr: int, opened: bool) -> None:
        _check(self._lib.qlinear_peer_buffer_free(self.raw, ptr, 1 if opened else 0),
               "peer buffer free")

    def peer_signal_wait(self, sig, rank: int, epoch: int, limit_s: float = 0.0,
                         stream=None) -> None:
        """qlinear_peer_signal_wait: raise this rank's flag to `epoch` in every rank's signal
        array (`sig`: device addresses in rank order, this GPU's own at `rank`) and wait on
        `stream` until every rank's flag here has reached it (0 s limit: the default 2 s)."""
        arr = (ctypes.c_void_p * len(sig))(*[int(p) for p in sig])
        _check(self._lib.qlinear_peer_signal_wait(self.raw, arr, len(sig), rank, epoch,
                                                  int(limit_s * 1e9), stream),
               "peer signal wait")

    def selftest_wait_timeout(self, limit_s: float = 0.2) -> int:
        """Run the failure-path self-test (a bounded wait that nothing satisfies); returns the
        status, QLINEAR_ERR_TIMEOUT when the path works."""
        return int(self._lib.qlinear_selftest_wait_timeout(self.raw, int(limit_s * 1e9)))

    def run_mlp_device(self, gate_up: "Linear", down: "Linear", a, out, rows: int,
                       ldc: int | None = None, stream=None) -> None:
        """The MLP block of src/model/dense.rs:499-530 on device buffers: out = down(silu(g) *
        u), [g | u] = gate_up(a), with the reference's f32 middle; one fused launch for a
        single row (qlinear_run_mlp_device)."""
        _check(self._lib.qlinear_run_mlp_device(
            self.raw, gate_up._raw, down._raw, _ptr(a), _dtype_code(a), _ptr(out), _dtype_code(out),
            down.n() if ldc is None else ldc, rows, stream), "MLP device run")

    def swiglu_device(self, y, out, rows: int, n: int, ldc: int | None = None,
                      stream=None) -> None:
        """out[m][j] = silu(y[m][j]) * y[m][n/2 + j] for an f32 [rows][n] gate/up output on the
        device (the reference's Cpu::swiglu fallback, src/model/dense.rs:509-523, for a
        gate/up projection of two matrices)."""
        _check(self._lib.qlinear_swiglu_device(self.raw, _ptr(y), rows, n, _ptr(out),
                                               _dtype_code(out), n // 2 if ldc is None else ldc,
                                               stream), "swiglu device")

    def row_amax_device(self, a, rows: int, k: int, amax, stream=None) -> None:
        """amax[m] = max |a[m][:k]| (device buffers; NaN ignored like Rust's f32::max)."""
        _check(self._lib.qlinear_row_amax_device(self.raw, _ptr(a), _dtype_code(a), rows, k,
                                                 _ptr(amax), stream), "row amax")

    def act_quant_device(self, a, rows: int, k: int, codes, scales, rowsums=None,
                         stream=None) -> None:
        """Activation quantisation alone (device buffers); exports the int8 codes."""
        a_type = L.F16 if str(getattr(a, "dtype", "")) in ("torch.float16", "float16") else L.F32
        _check(self._lib.qlinear_act_quant_device(
            self.raw, _ptr(a), a_type, rows, k, _ptr(codes), _ptr(scales),
            _ptr(rowsums) if rowsums is not None else None, stream), "act quant")


class Linear:
    """One uploaded QuantMatrix (src/npu.rs:255-260)."""

    def __init__(self):
        raise TypeError("use Backend.load")

    @classmethod
    def _create(cls, backend: Backend, bits: int, k: int, n: int, data: np.ndarray,
                scales: np.ndarray, shard=None, checkpoint=False) -> "Linear":
        self = object.__new__(cls)
        self._backend = backend
        self._lib = backend._lib
        cfg = L.WeightConfig(bits, k, n, 0)
        if checkpoint:
            raw = self._lib.qlinear_weights_create_checkpoint(
                backend.raw, ctypes.byref(cfg), _ptr(data), _ptr(scales))
        elif shard is not None:
            raw = self._lib.qlinear_weights_create_shard(
                backend.raw, ctypes.byref(cfg), _ptr(data), _ptr(scales), shard[0], shard[1])
        else:
            raw = self._lib.qlinear_weights_create(backend.raw, ctypes.byref(cfg), _ptr(data),
                                                   _ptr(scales))
        if not raw:
            raise NpuError(f"W{bits} weights", self._lib.qlinear_last_status())
        self._raw = raw
        info = L.WeightInfo()
        _check(self._lib.qlinear_weights_query(raw, ctypes.byref(info)), "weight query")
        self.bits, self._k, self._n = info.bits, info.K, info.N
        self.k_padded, self.n_padded = info.K_padded, info.N_padded
        self.device_bytes = int(info.device_bytes)
        return self

    def close(self) -> None:
        if getattr(self, "_raw", None):
            self._lib.qlinear_weights_free(self._raw)
            self._raw = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def k(self) -> int:
        return self._k

    def n(self) -> int:
        return self._n

    def _host(self, input, output, rows: int, swiglu: bool) -> None:
        if rows < 1:
            raise ValueError("linear batch must be >= 1")
        width = self._n // 2 if swiglu else self._n
        input = np.asarray(input)
        if input.dtype != np.float32 or output.dtype != np.float32:
            raise TypeError("Linear.run takes f32 buffers (src/npu.rs:1006)")
        if input.size < rows * self._k or output.size < rows * width:
            raise ValueError("linear input/output shape mismatch")
        if not (input.flags.c_contiguous and output.flags.c_contiguous):
            raise ValueError("buffers must be C-contiguous")
        fn = self._lib.qlinear_run_swiglu_f32 if swiglu else self._lib.qlinear_run_f32
        _check(fn(self._backend.raw, self._raw, input.ctypes.data, output.ctypes.data, rows),
               f"W{self.bits} SwiGLU run" if swiglu else f"W{self.bits} run")

    def run(self, input: np.ndarray, output: np.ndarray, rows: int) -> None:
        """Linear::run (src/npu.rs:1006): f32 [rows][K] -> f32 [rows][N], synchronous."""
        self._host(input, output, rows, False)

    def run_swiglu(self, input: np.ndarray, output: np.ndarray, rows: int) -> bool:
        """Linear::run_swiglu (src/npu.rs:1009-1024): f32 [rows][N/2]; always fused here."""
        if self._n % 2:
            return False
        self._host(input, output, rows, True)
        return True

    def run_columns(self, input: np.ndarray, output: np.ndarray, rows: int, ldc: int,
                    col: int = 0, swiglu: bool = False) -> None:
        """f32 [rows][K] -> columns [col, col + width) of the f32 rows of stride `ldc` in
        `output` (width = N, or N/2 with swiglu); the rest of each row is untouched.  One
        part of a fused projection (src/model/projection.rs:215-228) written in place."""
        if rows < 1:
            raise ValueError("linear batch must be >= 1")
        width = self._n // 2 if swiglu else self._n
        input = np.asarray(input)
        if input.dtype != np.float32 or output.dtype != np.float32:
            raise TypeError("Linear.run_columns takes f32 buffers")
        if not (input.flags.c_contiguous and output.flags.c_contiguous):
            raise ValueError("buffers must be C-contiguous")
        if (col < 0 or ldc < col + width or input.size < rows * self._k
                or output.size < (rows - 1) * ldc + col + width):
            raise ValueError("linear input/output shape mismatch")
        _check(self._lib.qlinear_run_f32_ex(
            self._backend.raw, self._raw, input.ctypes.data, output.ctypes.data + 4 * col, ldc,
            rows, L.RUN_SWIGLU if swiglu else 0), f"W{self.bits} run")

    def run_device(self, a, out, rows: int, swiglu: bool = False, ldc: int | None = None,
                   stream=None, out_type: int | None = None) -> None:
        """Device-resident call: `a` [rows][K] fp16/f32 and `out` [rows][ldc] (fp16, f32 or
        int32 accumulators) are device buffers (torch tensors or raw pointers); async on
        `stream` (a cudaStream_t value; None = legacy default stream)."""
        a_type = _dtype_code(a)
        c_type = _dtype_code(out) if out_type is None else out_type
        width = self._n // 2 if swiglu else self._n
        if ldc is None:
            ldc = width
        _check(self._lib.qlinear_run_device(
            self._backend.raw, self._raw, _ptr(a), a_type, _ptr(out), c_type, ldc, rows,
            L.RUN_SWIGLU if swiglu else 0, stream), f"W{self.bits} device run")

    def run_device_amax(self, a, row_amax, out, rows: int, stream=None) -> None:
        """This K slice of a split-K linear: `a` [rows][K_slice] quantised with the scale of
        the given whole-row maxima `row_amax` [rows]; `out` int32 receives the exact partial
        accumulators (fp16/f32: this slice's dequantised partial)."""
        _check(self._lib.qlinear_run_device_amax(
            self._backend.raw, self._raw, _ptr(a), _dtype_code(a), _ptr(row_amax), _ptr(out),
            _dtype_code(out), self._n, rows, stream), f"W{self.bits} split-K run")

    def dequant_device(self, acc, row_amax, out, rows: int, stream=None) -> None:
        """out = (f32(acc) * s_a) * s_w for int32 accumulators summed over the K slices."""
        _check(self._lib.qlinear_dequant_device(
            self._backend.raw, self._raw, _ptr(acc), self._n, _ptr(row_amax), _ptr(out),
            _dtype_code(out), self._n, rows, stream), "dequant")

    def run_device_multicast(self, a, outs, mc: int, out_type: int, ldc: int, col_offset: int,
                             rows: int, stream=None) -> None:
        """qlinear_run_device_multicast: as run_device_scatter, but the tensor-core GEMM stores
        each output element once through `mc`, the NVSwitch multicast address bound to every
        rank's exchange buffer (`outs`: their unicast addresses, this GPU's first, used by the
        decode GEMV)."""
        s = str(getattr(a, "dtype", ""))
        a_type = L.F16 if "float16" in s else L.F32 if "float32" in s else None
        if a_type is None:
            raise TypeError(s)
        arr = (ctypes.c_void_p * len(outs))(*[int(p) for p in outs])
        _check(self._lib.qlinear_run_device_multicast(
            self._backend.raw, self._raw, _ptr(a), a_type, arr, len(outs), int(mc), out_type,
            ldc, col_offset, rows, stream), f"W{self.bits} device multicast run")

    def run_device_scatter(self, a, outs, out_type: int, ldc: int, col_offset: int, rows: int,
                           swiglu: bool = False, stream=None) -> None:
        """qlinear_run_device_scatter: the output columns go to column col_offset of every
        buffer in `outs` (device addresses: this GPU's and the peers' exchange buffers)."""
        s = str(getattr(a, "dtype", ""))
        a_type = L.F16 if "float16" in s else L.F32 if "float32" in s else None
        if a_type is None:
            raise TypeError(s)
        arr = (ctypes.c_void_p * len(outs))(*[int(p) for p in outs])
        _check(self._lib.qlinear_run_device_scatter(
            self._backend.raw, self._raw, _ptr(a), a_type, arr, len(outs), out_type, ldc,
            col_offset, rows, L.RUN_SWIGLU if swiglu else 0, stream),
               f"W{self.bits} device scatter run")
