"""Column-parallel (split-N) quantized linear over the ranks of a torch.distributed group.

Each rank holds output channels ``[r*N/g, (r+1)*N/g)`` of one QuantMatrix
(``qlinear_weights_create_shard``), runs the full activation rows through its shard, and the
per-rank fp16/f32 slabs are all-gathered over NCCL (NVLink) and assembled into ``[M][N]``
by ``qlinear_interleave_columns``.  Activations are replicated; the activation quantisation
runs on every rank and is deterministic, so every rank holds bit-identical codes and the
assembled output is bit-identical to a single-GPU run.  The reference is single-device;
this has no counterpart there.
"""
from __future__ import annotations

import numpy as np


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [lo, hi) of rank `rank` when n columns are split evenly over `world` ranks.
    Requires n % world == 0 (the all-gather moves equal slabs)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    if n % world:
        raise ValueError(f"N={n} is not divisible by {world} ranks")
    ns = n // world
    return rank * ns, (rank + 1) * ns


def assemble(gathered: np.ndarray) -> np.ndarray:
    """Host restatement of qlinear_interleave_columns: [g][M][N/g] -> [M][N]."""
    g, m, ns = gathered.shape
    return np.ascontiguousarray(np.transpose(gathered, (1, 0, 2)).reshape(m, g * ns))


class ShardedLinear:
    """One rank's shard of a column-parallel quantized linear."""

    def __init__(self, backend, matrix, group=None):
        import torch.distributed as dist
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n = matrix.n
        self.k = matrix.k
        lo, hi = shard_bounds(matrix.n, self.world, self.rank)
        self.ns = hi - lo
        self.linear = backend.load_shard(matrix, lo, hi)
        self._bufs = {}

    def _buf(self, key, shape, dtype, device):
        import torch
        b = self._bufs.get(key)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[key] = b
        return b

    def run_device(self, a, out, rows: int, stream=None) -> None:
        """a [rows][K] (fp16/f32, this rank's device); out [rows][N] fp16 or f32."""
        import torch
        import torch.distributed as dist
        local = self._buf("local", (rows, self.ns), out.dtype, out.device)
        self.linear.run_device(a, local, rows, stream=stream)
        if self.world == 1:
            out.copy_(local)
            return
        # slabs back to back, [g * rows][N/g]: the form every backend's all-gather accepts
        gathered = self._buf("gathered", (self.world * rows, self.ns), out.dtype, out.device)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        self.backend.interleave_columns(gathered, out, self.world, rows, self.ns,
                                        out.element_size(), stream=stream)
        del torch
