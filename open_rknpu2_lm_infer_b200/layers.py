"""The quantized linears of a dense decoder layer and the quantized output head, loaded and
called the way the reference's dense model does it.

* ``DenseLayerLinears``: src/model/dense.rs:209-280 loads, per decoder layer, the q/k/v
  modules and the gate/up modules as two ``Projection``s (adjacent modules of one bit
  width fused into one matrix, src/model/projection.rs:142-189) and o_proj / down_proj as
  single linears.  At run time (src/model/dense.rs:425-530) the layer calls
  ``qkv.run(normalized)``, ``o.run(attended)``, then ``gate_up.run_swiglu(normalized ->
  middle)`` -- or, when gate and up are two matrices (different bit widths),
  ``gate_up.run`` into ``[rows][2f]`` followed by ``Cpu::swiglu`` -- and ``down.run(middle)``.
  Here the same calls run on device buffers: the fused MLP call (``qlinear_run_mlp_device``)
  when gate/up is one matrix, else the two gate/up parts into an f32 ``[rows][2f]`` buffer,
  ``qlinear_swiglu_device`` and the down call, with the reference's f32 middle either way.
* ``OutputHead``: the quantized vocabulary projection (src/model/output_head.rs:28-46,
  ``run`` :95-110): one linear ``lm_head`` [width] -> [vocab].

Everything between the linears (norms, RoPE, attention, residual adds) is not part of the
quantized-linear path and is not mirrored.
"""
from __future__ import annotations

import numpy as np

from .npu import Backend, Linear
from .projection import Projection, QuantLoader


class DenseLayerLinears:
    """The quantized linears of one dense decoder layer (src/model/dense.rs:209-280)."""

    def __init__(self, backend: Backend, qkv: Projection, gate_up: Projection, o: Linear,
                 down: Linear, hidden: int, q_width: int, kv_width: int, intermediate: int):
        self.backend = backend
        self.qkv, self.gate_up, self.o, self.down = qkv, gate_up, o, down
        self.hidden, self.q_width, self.kv_width, self.f = hidden, q_width, kv_width, intermediate
        self._bufs = {}

    @classmethod
    def load(cls, backend: Backend, loader: QuantLoader, prefix: str, hidden: int,
             q_heads: int, kv_heads: int, head_dim: int, intermediate: int
             ) -> "DenseLayerLinears":
        """Module names and shapes as src/model/dense.rs:213-227 builds them
        (``{prefix}self_attn.{q,k,v,o}_proj``, ``{prefix}mlp.{gate,up,down}_proj``)."""
        qw, kw = q_heads * head_dim, kv_heads * head_dim
        qkv = Projection.load(backend, loader, [(f"{prefix}self_attn.q_proj", qw),
                                                (f"{prefix}self_attn.k_proj", kw),
                                                (f"{prefix}self_attn.v_proj", kw)], hidden)
        gate_up = Projection.load(backend, loader, [(f"{prefix}mlp.gate_proj", intermediate),
                                                    (f"{prefix}mlp.up_proj", intermediate)],
                                  hidden)

        def single(name, n, k):
            return backend.load(loader.load(name, n, k), lambda: loader.load(name, n, k))

        o = single(f"{prefix}self_attn.o_proj", hidden, qw)
        down = single(f"{prefix}mlp.down_proj", hidden, intermediate)
        return cls(backend, qkv, gate_up, o, down, hidden, qw, kw, intermediate)

    @property
    def qkv_width(self) -> int:
        return self.q_width + 2 * self.kv_width

    def linears(self):
        """Every uploaded linear of the layer: (role, Linear, column offset)."""
        out = [("qkv", lin, off) for lin, off in self.qkv.parts]
        out += [("o", self.o, 0)]
        out += [("gate_up", lin, off) for lin, off in self.gate_up.parts]
        out += [("down", self.down, 0)]
        return out

    def close(self) -> None:
        self.qkv.close()
        self.gate_up.close()
        self.o.close()
        self.down.close()
        self._bufs = {}

    def _buf(self, key, shape, dtype, device):
        import torch
        b = self._bufs.get(key)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype or b.device != device:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[key] = b
        return b

    # -- the layer's calls on device buffers (fp16 / f32 torch tensors) ----------------
    def qkv_device(self, normalized, out, rows: int, stream=None) -> None:
        """``layer.qkv.run`` (src/model/dense.rs:435-441): out [rows][q + 2 kv]."""
        self.qkv.run_device(normalized, out, rows, stream=stream)

    def o_device(self, attended, out, rows: int, stream=None) -> None:
        """``layer.o.run`` (src/model/dense.rs:483-488): attended [rows][q] -> [rows][hidden]."""
        self.o.run_device(attended, out, rows, stream=stream)

    def mlp_device(self, normalized, out, rows: int, stream=None, middle=None) -> None:
        """The MLP (src/model/dense.rs:499-530): out [rows][hidden] = down(silu(g) * u) with the
        reference's f32 middle.  One gate/up matrix: ``qlinear_run_mlp_device``; two (gate and
        up of different bit widths): both parts into an f32 [rows][2f] buffer, the device
        SwiGLU into the middle (or `middle`, an f32 [rows][f] tensor the caller keeps), and
        the down call."""
        import torch
        if len(self.gate_up.parts) == 1 and middle is None:
            self.backend.run_mlp_device(self.gate_up.parts[0][0], self.down, normalized, out,
                                        rows, stream=stream)
            return
        dev = normalized.device
        if middle is None:
            middle = self._buf("middle", (rows, self.f), torch.float32, dev)
        if len(self.gate_up.parts) == 1:
            self.gate_up.parts[0][0].run_device(normalized, middle, rows, swiglu=True,
                                                stream=stream)
        else:
            gu = self._buf("gate_up", (rows, 2 * self.f), torch.float32, dev)
            self.gate_up.run_device(normalized, gu, rows, stream=stream)
            self.backend.swiglu_device(gu, middle, rows, 2 * self.f, stream=stream)
        self.down.run_device(middle, out, rows, stream=stream)


class OutputHead:
    """The quantized output projection (src/model/output_head.rs:28-46)."""

    def __init__(self, backend: Backend, linear: Linear, bits: int, vocab: int, width: int):
        self.backend, self.linear, self._bits = backend, linear, bits
        self.vocab, self.width = vocab, width

    @classmethod
    def quantized(cls, backend: Backend, loader: QuantLoader, vocab: int, width: int
                  ) -> "OutputHead":
        """``OutputHead::quantized``: the ``lm_head`` module, [width] -> [vocab]."""
        matrix = loader.load("lm_head", vocab, width)
        linear = backend.load(matrix, lambda: loader.load("lm_head", vocab, width))
        return cls(backend, linear, matrix.bits, vocab, width)

    def bits(self) -> int:
        return self._bits

    def prepare(self, rows: int) -> None:
        self.backend.prepare(rows)

    def run(self, input: np.ndarray, output: np.ndarray, rows: int) -> None:
        """src/model/output_head.rs:95-110 (host f32 buffers)."""
        if input.size != rows * self.width or output.size != rows * self.vocab:
            raise ValueError("lm_head shape mismatch")
        self.linear.run(input, output, rows)

    def run_device(self, x, out, rows: int, stream=None) -> None:
        self.linear.run_device(x, out, rows, stream=stream)

    def close(self) -> None:
        self.linear.close()
