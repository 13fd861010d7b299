"""Seeded synthetic workloads with the shapes and value distributions of the benchmark
configurations of the quantized-linear path.

The reference publishes no dataset for this path; every input is synthetic and seeded
(numpy PCG64, seed 42 by default, one sub-stream per tensor).  Distributions:

* activations: fp16 from N(0, 1); 1% of the K channels (``round(0.01*K)`` distinct
  indices, the same for every row) multiplied by 20 as outlier channels;
* W4 codes: uniform integers in [-8, 7]; W8 codes: uniform integers in [-127, 127];
* per-output-channel scales: exp(U(ln 1e-3, ln 1e-2)) in f32 (log-uniform).

Weight codes are produced in the reference's ``QuantMatrix`` layout: int8 ``[K][N]``
row-major, element (k, n) at ``k*N + n`` (src/npu.rs:112-118, :1115).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

SEED = 42


def _rng(seed: int, stream: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, stream])))


def activations(rows: int, k: int, seed: int = SEED, stream: int = 0,
                outlier_frac: float = 0.01, outlier_gain: float = 20.0) -> np.ndarray:
    """fp16 [rows, k]: N(0,1) with round(outlier_frac*k) channels scaled by outlier_gain."""
    g = _rng(seed, 1000 + stream)
    x = g.standard_normal((rows, k), dtype=np.float32)
    n_out = int(round(outlier_frac * k))
    if n_out:
        idx = g.choice(k, size=n_out, replace=False)
        x[:, idx] *= np.float32(outlier_gain)
    return x.astype(np.float16)


def weight_codes(bits: int, k: int, n: int, seed: int = SEED, stream: int = 0) -> np.ndarray:
    """int8 codes in the QuantMatrix layout [k][n]."""
    g = _rng(seed, 2000 + stream)
    if bits == 4:
        return g.integers(-8, 8, size=(k, n), dtype=np.int8)
    if bits == 8:
        return g.integers(-127, 128, size=(k, n), dtype=np.int8)
    raise ValueError("bits must be 4 or 8")


def weight_scales(n: int, seed: int = SEED, stream: int = 0) -> np.ndarray:
    g = _rng(seed, 3000 + stream)
    return np.exp(g.uniform(np.log(1e-3), np.log(1e-2), size=n)).astype(np.float32)


@dataclass(frozen=True)
class Shape:
    name: str
    bits: int
    k: int
    n: int


# Benchmark configurations (shapes only; row counts are swept by the callers).
CFG0 = Shape("cfg0 W4A8 gate_proj", 4, 2560, 9728)          # M = 512
CFG1 = Shape("cfg1 W8A8 decode", 8, 2560, 9728)              # M in {1, 4}
CFG2_GATE_UP = Shape("cfg2 W4A8 gate/up fused", 4, 2560, 19456)
CFG2_DOWN = Shape("cfg2 W8A8 down", 8, 9728, 2560)
CFG4 = Shape("cfg4 W4A8 large", 4, 8192, 28672)              # M in {1, 8, 512, 8192}

QWEN3_4B_LAYER = (  # (name, k, n) of the four linear groups of one decoder layer
    ("qkv", 2560, 6144), ("o", 4096, 2560), ("gate_up", 2560, 19456), ("down", 9728, 2560))


def layer_bits(layers: int = 36, seed: int = SEED, p_w4: float = 0.7) -> list[list[int]]:
    """Per-layer, per-linear W4/W8 draw (Bernoulli p_w4 for W4) of the 36-layer config."""
    g = _rng(seed, 4000)
    draw = g.random((layers, len(QWEN3_4B_LAYER)))
    return [[4 if v < p_w4 else 8 for v in row] for row in draw]


def kat_matrix(bits: int, k: int = 256, n: int = 256):
    """Deterministic QuantMatrix of the reference's quantized_linear_padding_and_swiglu
    test (src/npu.rs:1172-1184): codes ((i*13 + i/256*7) % (16|255)) - (8|127) with
    i = k*n_index flat index, scales 0.002 + (n % 11) * 1e-4."""
    i = np.arange(k * n, dtype=np.int64)
    mod, off = (16, 8) if bits == 4 else (255, 127)
    codes = (((i * 13 + i // 256 * 7) % mod) - off).astype(np.int8).reshape(k, n)
    scales = (np.float32(0.002) + (np.arange(n) % 11).astype(np.float32) * np.float32(0.0001))
    return codes, scales.astype(np.float32)


def kat_input(rows: int = 256, k: int = 256) -> np.ndarray:
    """Input of the same test (src/npu.rs:1185-1187): ((i*17 + i/256*3) % 127)/63 - 1."""
    i = np.arange(rows * k, dtype=np.int64)
    return (((i * 17 + i // 256 * 3) % 127).astype(np.float32) / np.float32(63.0)
            - np.float32(1.0)).reshape(rows, k)


def narrow_kat(n: int, k: int = 2560, rows: int = 7):
    """W8 narrow-projection test data (src/npu/narrow_projection.rs:24-31, :40-42)."""
    i = np.arange(k * n, dtype=np.int64)
    codes = (((i * 13 + i // n * 7) % 255) - 127).astype(np.int8).reshape(k, n)
    scales = (np.float32(0.001) + (np.arange(n) % 11).astype(np.float32) * np.float32(0.0001))
    j = np.arange(rows * k, dtype=np.int64)
    x = (((j * 17 + j // k * 3) % 127).astype(np.float32) / np.float32(63.0)
         - np.float32(1.0)).reshape(rows, k)
    return codes, scales.astype(np.float32), x


# The Qwen3-4B-shaped dense model of the 36-layer configuration.
QWEN3_4B = {"hidden": 2560, "q_heads": 32, "kv_heads": 8, "head_dim": 128,
            "intermediate": 9728, "vocab": 151936, "layers": 36}


def cfg3_module_bits(layers: int = 36, seed: int = SEED) -> dict[str, int]:
    """Module name -> bits for the 36-layer configuration: the per-layer draw of
    ``layer_bits`` applied to the modules of each linear (q/k/v share the fused q/k/v
    linear's draw, gate/up the gate/up linear's); the W8 lm_head."""
    out = {"lm_head": 8}
    for i, (qkv, o, gu, down) in enumerate(layer_bits(layers, seed)):
        p = f"model.layers.{i}."
        for m in ("q_proj", "k_proj", "v_proj"):
            out[p + "self_attn." + m] = qkv
        out[p + "self_attn.o_proj"] = o
        out[p + "mlp.gate_proj"] = gu
        out[p + "mlp.up_proj"] = gu
        out[p + "mlp.down_proj"] = down
    return out


class SyntheticCheckpoint:
    """Seeded stand-in for a quantized checkpoint, behind the loader interface the projection
    code takes (``bits(name)``, ``load(name, n, k) -> QuantMatrix``, the roles of
    src/model/checkpoint.rs:320-389).  Codes and scales of a module come from a sub-stream
    derived from its name, so every module differs and every load is reproducible.  With
    ``share_by_shape`` modules of one (bits, K, N) share codes (the benchmark's cheaper
    draw of a 36-layer model; every module is still uploaded separately)."""

    def __init__(self, bits: dict[str, int], seed: int = SEED, share_by_shape: bool = False):
        self._bits = dict(bits)
        self.seed = seed
        self.share_by_shape = share_by_shape
        self._cache = {}

    def bits(self, name: str) -> int:
        return self._bits[name]

    def stream_of(self, name: str, k: int, n: int) -> int:
        import zlib
        key = f"{self._bits[name]}:{k}:{n}" if self.share_by_shape else name
        return 100000 + zlib.crc32(key.encode()) % 1000000

    def codes(self, name: str, n: int, k: int):
        """(codes int8 [k][n], scales f32 [n]) of a module."""
        s = self.stream_of(name, k, n)
        hit = self._cache.get(s)
        if hit is None:
            bits = self._bits[name]
            hit = (weight_codes(bits, k, n, self.seed, s), weight_scales(n, self.seed, s))
            if self.share_by_shape:
                self._cache[s] = hit
        return hit

    def load(self, name: str, n: int, k: int):
        from .npu import QuantMatrix
        c, s = self.codes(name, n, k)
        return QuantMatrix(self._bits[name], k, n, c, s)
