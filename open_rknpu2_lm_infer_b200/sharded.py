"""Column-parallel (split-N) quantized linear over the ranks of a torch.distributed group.

Each rank holds output channels ``[r*N/g, (r+1)*N/g)`` of one QuantMatrix
(``qlinear_weights_create_shard``) and runs the full activation rows through its shard.
Activations are replicated; the activation quantisation runs on every rank and is
deterministic, so every rank holds bit-identical codes and the output is bit-identical to a
single-GPU run.  Two ways to put the [M][N] output together on every rank:

* ``run_device``: the per-rank fp16/f32 slabs are all-gathered over NCCL (NVLink) and
  assembled into ``[M][N]`` by ``qlinear_interleave_columns``;
* ``run_exchange`` (``fused_exchange=True``): the kernels' epilogues store each rank's
  columns straight into every rank's ``[M][N]`` exchange buffer over NVLink while they
  compute (``qlinear_run_device_scatter``; the buffers are shared through CUDA IPC,
  ``qlinear_peer_buffer_*``), then a one-warp kernel raises this rank's flag in every rank's
  signal array and waits for all of them (``qlinear_peer_signal_wait``), so the output is
  complete on every rank.  No gather, no assembly pass, no collective per call.
  With ``multicast=True`` the exchange buffers are torch symmetric memory with an NVSwitch
  multicast (NVLS) mapping: the tensor-core GEMM stores each element once through the
  multicast address and the switch writes it into every rank's buffer
  (``qlinear_run_device_multicast``), so a rank sends its columns over NVLink once instead
  of once per peer.

``ShardedMLP`` splits a whole MLP block instead (gate/up columns and down rows together:
no gather of the middle, an exact all-reduce of int32 partial accumulators).

The reference is single-device; this has no counterpart there.
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


class _DeviceArray:
    """Zero-copy view of library-owned device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class ShardedLinear:
    """One rank's shard of a column-parallel quantized linear."""

    def __init__(self, backend, matrix, group=None, fused_exchange: bool = False,
                 max_rows: int = 0, out_dtype=None, multicast: bool = False):
        import torch.distributed as dist
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n = matrix.n
        self.k = matrix.k
        lo, hi = shard_bounds(matrix.n, self.world, self.rank)
        self.lo = lo
        self.ns = hi - lo
        self.linear = backend.load_shard(matrix, lo, hi)
        self._bufs = {}
        self.multicast = multicast
        self._xbufs = {}  # output dtype -> exchange buffer record (own, peers, view, type, mc)
        self._keep = []   # symmetric-memory tensors and handles of the multicast exchange
        self._default_dtype = None
        self._sig = None    # signal arrays in rank order (this rank's own at self.rank)
        self._epoch = 0
        if fused_exchange:
            self.add_exchange(max_rows, out_dtype)

    def add_exchange(self, max_rows: int, out_dtype=None) -> None:
        """Collective (every rank, same order): this rank allocates a [max_rows][N] exchange
        buffer of out_dtype (fp16 default, or f32), shares its CUDA IPC handle and maps the
        peers' buffers."""
        import torch
        import torch.distributed as dist
        from . import _lib as L
        if max_rows < 1:
            raise ValueError("fused exchange needs max_rows >= 1")
        dtype = out_dtype or torch.float16
        if dtype not in (torch.float16, torch.float32):
            raise TypeError(dtype)
        if dtype in self._xbufs:
            raise ValueError(f"exchange buffer for {dtype} exists")
        elem, typestr = (2, "<f2") if dtype == torch.float16 else (4, "<f4")
        if self.multicast:
            self._add_multicast_exchange(max_rows, dtype)
            return
        ptr, handle = self.backend.peer_buffer_create(max_rows * self.n * elem)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        peers = [self.backend.peer_buffer_open(h) for r, h in enumerate(handles) if r != self.rank]
        dev = torch.device("cuda", self.backend.device)
        view = torch.as_tensor(_DeviceArray(ptr, (max_rows, self.n), typestr), device=dev)
        self._xbufs[dtype] = {"own": ptr, "peers": peers, "view": view, "mc": 0,
                              "type": L.F16 if dtype == torch.float16 else L.F32}
        if self._default_dtype is None:
            self._default_dtype = dtype
        if self._sig is None:
            sptr, shandle = self.backend.peer_buffer_create(8 * self.world)
            shandles = [None] * self.world
            dist.all_gather_object(shandles, shandle, group=self.group)
            self._sig = [sptr if r == self.rank else self.backend.peer_buffer_open(h)
                         for r, h in enumerate(shandles)]

    def _add_multicast_exchange(self, max_rows: int, dtype) -> None:
        """Collective: the [max_rows][N] exchange buffer and the signal array in torch
        symmetric memory (every rank's copy mapped here, plus the NVSwitch multicast
        address of the buffers)."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from . import _lib as L
        group = self.group or dist.group.WORLD
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            symm_mem.enable_symm_mem_for_group(group.group_name)
        dev = torch.device("cuda", self.backend.device)
        buf = symm_mem.empty((max_rows, self.n), dtype=dtype, device=dev)
        hdl = symm_mem.rendezvous(buf, group.group_name)
        mc = int(hdl.multicast_ptr)
        if not mc:
            raise RuntimeError("multicast exchange: no NVSwitch multicast mapping on this node")
        # the handle's addresses are those of the symmetric allocation holding the tensor;
        # the tensor sits `off` bytes into it on every rank (and in the multicast mapping)
        off = buf.data_ptr() - int(hdl.buffer_ptrs[self.rank])
        if off < 0 or off != int(getattr(hdl, "offset", off)):
            raise RuntimeError("multicast exchange: unexpected symmetric-memory layout")
        ptrs = [int(p) + off for p in hdl.buffer_ptrs]
        mc += off
        self._keep += [buf, hdl]
        self._xbufs[dtype] = {"own": ptrs[self.rank],
                              "peers": [p for r, p in enumerate(ptrs) if r != self.rank],
                              "view": buf, "mc": mc,
                              "type": L.F16 if dtype == torch.float16 else L.F32}
        if self._default_dtype is None:
            self._default_dtype = dtype
        if self._sig is None:
            sig = symm_mem.empty((self.world,), dtype=torch.int64, device=dev)
            sig.zero_()
            hs = symm_mem.rendezvous(sig, group.group_name)
            self._keep += [sig, hs]
            soff = sig.data_ptr() - int(hs.buffer_ptrs[self.rank])
            self._sig = [int(p) + soff for p in hs.buffer_ptrs]
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)  # every rank's flags are zero before any signal

    @property
    def output(self):
        return self._xbufs[self._default_dtype]["view"] if self._xbufs else None

    def run_exchange(self, a, rows: int, stream=None, out_dtype=None):
        """Fused split-N: this rank's columns go straight into every rank's exchange buffer of
        out_dtype; returns the [rows][N] output (this rank's buffer), complete for the work
        queued on `stream` after the call.  Every rank makes the same calls in the same order
        (the signal epochs must match).  The caller keeps every rank from reading the previous
        output while a new call writes it."""
        key = out_dtype or self._default_dtype
        if key not in self._xbufs:
            raise RuntimeError("no exchange buffer for this output type (add_exchange)")
        x = self._xbufs[key]
        view = x["view"]
        if not 1 <= rows <= view.shape[0]:
            raise ValueError("rows out of range for the exchange buffer")
        if x["mc"]:
            self.linear.run_device_multicast(a, [x["own"]] + x["peers"], x["mc"], x["type"],
                                             self.n, self.lo, rows, stream=stream)
        else:
            self.linear.run_device_scatter(a, [x["own"]] + x["peers"], x["type"], self.n,
                                           self.lo, rows, stream=stream)
        self._epoch += 1
        self.backend.peer_signal_wait(self._sig, self.rank, self._epoch, stream=stream)
        return view[:rows]

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers, then frees its own."""
        import torch
        import torch.distributed as dist
        if self._xbufs and self.multicast:
            torch.cuda.synchronize(self.backend.device)  # no exchange kernel in flight
            dist.barrier(group=self.group)  # no rank still reads or writes a peer's buffer
            self._xbufs = {}
            self._sig = None
            self._keep = []
        elif self._xbufs:
            torch.cuda.synchronize(self.backend.device)  # no exchange kernel in flight
            for x in self._xbufs.values():
                for p in x["peers"]:
                    self.backend.peer_buffer_free(p, True)
            for r, p in enumerate(self._sig):
                if r != self.rank:
                    self.backend.peer_buffer_free(p, True)
            dist.barrier(group=self.group)  # every peer unmapped this rank's buffers
            for x in self._xbufs.values():
                self.backend.peer_buffer_free(x["own"], False)
            self.backend.peer_buffer_free(self._sig[self.rank], False)
            self._xbufs = {}
            self._sig = None
        self.linear.close()

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


def mlp_shard_matrices(gate_up, down, world: int, rank: int):
    """Rank `rank`'s pieces of an MLP block split over `world` ranks: the gate/up matrix
    (gate columns [0, h), up [h, 2h), src/model/checkpoint.rs:392-423) keeps the gate and up
    columns [lo, hi) of the middle width h -- so SwiGLU stays local -- and the down matrix
    (K = h) keeps its rows [lo, hi), a K slice.  Returns two QuantMatrix objects."""
    from .npu import QuantMatrix
    h = gate_up.n // 2
    if gate_up.n % 2 or down.k != h:
        raise ValueError("gate/up must have 2h columns and down h rows")
    lo, hi = shard_bounds(h, world, rank)
    gu = np.asarray(gate_up.codes).reshape(gate_up.k, gate_up.n)
    gsc = np.asarray(gate_up.scales).reshape(-1)
    codes = np.ascontiguousarray(np.concatenate([gu[:, lo:hi], gu[:, h + lo:h + hi]], axis=1))
    scales = np.ascontiguousarray(np.concatenate([gsc[lo:hi], gsc[h + lo:h + hi]]))
    dn = np.asarray(down.codes).reshape(down.k, down.n)
    return (QuantMatrix(gate_up.bits, gate_up.k, 2 * (hi - lo), codes, scales),
            QuantMatrix(down.bits, hi - lo, down.n, np.ascontiguousarray(dn[lo:hi]),
                        np.asarray(down.scales)))


class ShardedMLP:
    """One rank's share of an MLP block (gate/up + SwiGLU -> down, src/model/dense.rs:499-530)
    split over the ranks of a torch.distributed group without gathering the middle: the
    gate/up columns and the down rows are split together (``mlp_shard_matrices``), so each
    rank forms its slice of the middle locally; the down projection is then a K split whose
    whole-row activation scale comes from an all-reduce MAX of the slices' row maxima (M
    floats) and whose int32 partial accumulators are summed exactly by an all-reduce SUM
    (M x hidden int32) before one dequant.  The output on every rank is bit-identical to
    ``qlinear_run_mlp_device`` on one GPU (the same f32 middle, codes and accumulators)."""

    def __init__(self, backend, gate_up, down, group=None):
        import torch.distributed as dist
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        gu, dn = mlp_shard_matrices(gate_up, down, self.world, self.rank)
        self.hs, self.hidden = gu.n // 2, dn.n
        self.gate_up = backend.load(gu)
        self.down = backend.load(dn)
        self._bufs = {}

    def _buf(self, key, shape, dtype, device):
        import torch
        b = self._bufs.get(key)
        if b is None or tuple(b.shape) != tuple(shape) or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[key] = b
        return b

    def run_device(self, a, out, rows: int, stream=None) -> None:
        """a [rows][hidden] (fp16/f32, replicated); out [rows][hidden] fp16 or f32.  `stream`
        must be the current torch stream's handle (or None for it): the collectives are
        ordered after the kernels through it."""
        import torch
        import torch.distributed as dist
        current = torch.cuda.current_stream(a.device).cuda_stream
        if stream is None:
            stream = current
        if stream != current:
            # the all-reduces below run on torch's current stream: another stream would let
            # them start before the kernels that produce their inputs have finished
            raise ValueError("ShardedMLP.run_device: `stream` must be torch's current stream")
        dev = a.device
        mid = self._buf("mid", (rows, self.hs), torch.float32, dev)
        amax = self._buf("amax", (rows,), torch.float32, dev)
        acc = self._buf("acc", (rows, self.hidden), torch.int32, dev)
        self.gate_up.run_device(a, mid, rows, swiglu=True, stream=stream)
        self.backend.row_amax_device(mid, rows, self.hs, amax, stream=stream)
        if self.world > 1:
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        self.down.run_device_amax(mid, amax, acc, rows, stream=stream)
        if self.world > 1:
            dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        self.down.dequant_device(acc, amax, out, rows, stream=stream)

    def close(self) -> None:
        self.gate_up.close()
        self.down.close()
        self._bufs = {}
