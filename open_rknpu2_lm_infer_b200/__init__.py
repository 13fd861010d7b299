"""B200 (sm_100a) quantized-linear hot path of open_rknpu2_lm_infer.

dynamic per-token int8 activation quantisation -> W4/W8 x int8 GEMM/GEMV with exact int32
accumulation -> per-token x per-channel dequant epilogue, behind a mirror of the
reference's ``npu::Backend / Linear / QuantMatrix`` API (``open_rknpu2_lm_infer_b200.npu``)
and the C ABI of ``include/qlinear.h`` (``lib/libqlinear_b200.so``).
"""
from .npu import Backend, Linear, NpuError, QuantMatrix  # noqa: F401
from .projection import MatrixLoader, Projection, concatenate  # noqa: F401
from .layers import DenseLayerLinears, OutputHead  # noqa: F401
from ._lib import LIB_PATH, QLinearUnavailable, ROUND_AWAY, ROUND_EVEN  # noqa: F401

__all__ = ["Backend", "Linear", "NpuError", "QuantMatrix", "LIB_PATH", "QLinearUnavailable",
           "ROUND_AWAY", "ROUND_EVEN", "MatrixLoader", "Projection", "concatenate",
           "DenseLayerLinears", "OutputHead"]
