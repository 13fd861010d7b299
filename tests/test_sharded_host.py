"""Split-N host logic on CPU with gloo ranks (no GPU): partitioning, the all-gather slab
order and the assembly reproduce the single-device output exactly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from open_rknpu2_lm_infer_b200 import workloads as W
from open_rknpu2_lm_infer_b200.sharded import assemble, shard_bounds


def test_shard_bounds():
    assert shard_bounds(28672, 8, 0) == (0, 3584)
    assert shard_bounds(28672, 8, 7) == (25088, 28672)
    with pytest.raises(ValueError):
        shard_bounds(100, 3, 0)
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    k, n, rows = 64, 96, 5
    w = W.weight_codes(4, k, n, stream=3)
    sw = W.weight_scales(n, stream=3)
    x = W.activations(rows, k, stream=3).astype(np.float32)
    lo, hi = shard_bounds(n, world, rank)
    local = O.linear(np.ascontiguousarray(w[:, lo:hi]), sw[lo:hi], x)  # this rank's slab
    gathered = torch.empty((world * rows, hi - lo), dtype=torch.float32)  # slabs back to back
    dist.all_gather_into_tensor(gathered, torch.from_numpy(local))
    full = assemble(gathered.numpy().reshape(world, rows, hi - lo))
    np.save(os.path.join(result_dir, f"rank{rank}.npy"), full)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_n_gather_assembly_matches_single_device(tmp_path, world):
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    k, n, rows = 64, 96, 5
    want = O.linear(W.weight_codes(4, k, n, stream=3), W.weight_scales(n, stream=3),
                    W.activations(rows, k, stream=3).astype(np.float32))
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"rank{r}.npy"), want)


def _mlp_rank_main(rank, world, port, result_dir):
    """One rank of the split-K MLP restated on the CPU: the same steps ShardedMLP.run_device
    takes (local gate/up slice + SwiGLU, all-reduce MAX of the row maxima, the slice quantised
    with the whole-row scale, int32 partial accumulators all-reduced with SUM, one dequant),
    with the oracle's arithmetic in place of the kernels."""
    from open_rknpu2_lm_infer_b200 import QuantMatrix
    from open_rknpu2_lm_infer_b200.sharded import mlp_shard_matrices
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    hidden, h, rows = 64, 48, 5
    gate_up = QuantMatrix(4, hidden, 2 * h, W.weight_codes(4, hidden, 2 * h, stream=7),
                          W.weight_scales(2 * h, stream=7))
    down = QuantMatrix(8, h, hidden, W.weight_codes(8, h, hidden, stream=8),
                       W.weight_scales(hidden, stream=8))
    gu, dn = mlp_shard_matrices(gate_up, down, world, rank)
    x = W.activations(rows, hidden, stream=9).astype(np.float32)
    mid = O.swiglu(O.linear(gu.codes, gu.scales, x))  # this rank's middle slice, f32
    amax = torch.from_numpy(np.abs(mid).max(axis=1).astype(np.float32))
    dist.all_reduce(amax, op=dist.ReduceOp.MAX)
    a = amax.numpy()
    scale = np.where(a == 0, np.float32(1), np.maximum(a / np.float32(127), O.F32_MIN))
    inv = (np.float32(1) / scale.astype(np.float32)).astype(np.float32)
    codes = np.clip(O.round_away((mid * inv[:, None]).astype(np.float32)), -127, 127)
    acc = torch.from_numpy(O.int_gemm(codes.astype(np.int8), dn.codes))
    dist.all_reduce(acc, op=dist.ReduceOp.SUM)
    y = O.dequant(acc.numpy(), scale.astype(np.float32), dn.scales)
    np.save(os.path.join(result_dir, f"mlp{rank}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_split_k_mlp_matches_single_device(tmp_path, world):
    """gate/up columns and down rows split together: every rank's output equals the unsplit
    block (f32 middle, src/model/dense.rs:499-530) bit for bit."""
    port = _free_port()
    mp.start_processes(_mlp_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    hidden, h, rows = 64, 48, 5
    x = W.activations(rows, hidden, stream=9).astype(np.float32)
    mid = O.swiglu(O.linear(W.weight_codes(4, hidden, 2 * h, stream=7),
                            W.weight_scales(2 * h, stream=7), x))
    want = O.linear(W.weight_codes(8, h, hidden, stream=8), W.weight_scales(hidden, stream=8), mid)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"mlp{r}.npy"), want)


def test_mlp_shard_matrices_partition():
    from open_rknpu2_lm_infer_b200 import QuantMatrix
    from open_rknpu2_lm_infer_b200.sharded import mlp_shard_matrices
    k, h, hidden = 8, 12, 10
    gu_codes = np.arange(k * 2 * h, dtype=np.int64).reshape(k, 2 * h) % 16 - 8
    gate_up = QuantMatrix(4, k, 2 * h, gu_codes.astype(np.int8),
                          np.arange(2 * h, dtype=np.float32) + 1)
    dn_codes = (np.arange(h * hidden) % 255 - 127).astype(np.int8).reshape(h, hidden)
    down = QuantMatrix(8, h, hidden, dn_codes, np.ones(hidden, np.float32))
    gu, dn = mlp_shard_matrices(gate_up, down, 3, 1)
    np.testing.assert_array_equal(gu.codes[:, :4], gu_codes[:, 4:8])       # gate columns
    np.testing.assert_array_equal(gu.codes[:, 4:], gu_codes[:, 16:20])     # their up columns
    np.testing.assert_array_equal(gu.scales, [5, 6, 7, 8, 17, 18, 19, 20])
    np.testing.assert_array_equal(dn.codes, dn_codes[4:8])                 # the K slice
    assert (gu.n, dn.k, dn.n) == (8, 4, hidden)
    with pytest.raises(ValueError):
        mlp_shard_matrices(gate_up, down, 5, 0)  # 12 middle columns over 5 ranks
