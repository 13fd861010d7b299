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
