"""Split-N on 2+ GPUs: the output assembled after an NCCL all-gather, and the output the
kernels' epilogues store straight into every rank's exchange buffer (fused exchange over
NVLink peer memory), both equal the single-GPU output bitwise; and the split-K MLP block
(ShardedMLP: NCCL all-reduces of row maxima and int32 accumulators) equals the single-GPU
block bitwise.  Runs as torchrun child
processes; skipped when fewer than 2 GPUs are visible."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import os, sys, datetime
sys.path.insert(0, os.environ["QL_ROOT"])
import numpy as np, torch, torch.distributed as dist
from open_rknpu2_lm_infer_b200 import Backend, QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W
from open_rknpu2_lm_infer_b200.sharded import ShardedLinear
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
b = Backend(device=rank)
for bits, k, n, rows in [(4, 2560, 4096, 300), (8, 4096, 2048, 3), (4, 8192, 28672 // 4, 64)]:
    qm = QuantMatrix(bits, k, n, W.weight_codes(bits, k, n, stream=n), W.weight_scales(n, stream=n))
    x = torch.from_numpy(W.activations(rows, k, stream=rows)).cuda()
    sh = ShardedLinear(b, qm)
    out = torch.empty((rows, n), dtype=torch.float16, device="cuda")
    sh.run_device(x, out, rows)
    full = b.load(qm)
    want = torch.empty((rows, n), dtype=torch.float16, device="cuda")
    full.run_device(x, want, rows)
    torch.cuda.synchronize()
    assert torch.equal(out, want), (rank, bits, k, n, rows)
    # fused exchange: the epilogues store every rank's columns into every rank's buffer
    for dtype in (torch.float16, torch.float32):
        fx = ShardedLinear(b, qm, fused_exchange=True, max_rows=rows, out_dtype=dtype)
        want_t = want if dtype == torch.float16 else torch.empty((rows, n), dtype=dtype, device="cuda")
        if dtype != torch.float16:
            full.run_device(x, want_t, rows)
        for _ in range(2):
            got = fx.run_exchange(x, rows)
            torch.cuda.synchronize()
            assert torch.equal(got, want_t), (rank, "fused", dtype, bits, k, n, rows)
        fx.close()
    # the exchange through NVSwitch multicast (torch symmetric memory, multimem stores)
    try:
        mx = ShardedLinear(b, qm, fused_exchange=True, max_rows=rows, multicast=True)
    except RuntimeError as e:
        print(f"rank {rank} multicast unavailable: {e}")
        mx = None
    if mx is not None:
        for _ in range(2):
            got = mx.run_exchange(x, rows)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (rank, "multicast", bits, k, n, rows)
        mx.close()
        print(f"rank {rank} multicast ok {bits} {k} {n} {rows}")
    sh.linear.close(); full.close()
# split-K MLP: gate/up columns and down rows split together, all-reduces of the row maxima
# and the int32 partial accumulators; equal to the single-GPU block bit for bit
from open_rknpu2_lm_infer_b200.sharded import ShardedMLP
hidden, h = 2560, 9728
gate_up = QuantMatrix(4, hidden, 2 * h, W.weight_codes(4, hidden, 2 * h, stream=90),
                      W.weight_scales(2 * h, stream=90))
down = QuantMatrix(8, h, hidden, W.weight_codes(8, h, hidden, stream=91),
                   W.weight_scales(hidden, stream=91))
gu_full, dn_full = b.load(gate_up), b.load(down)
mlp = ShardedMLP(b, gate_up, down)
for rows in (1, 300):
    x = torch.from_numpy(W.activations(rows, hidden, stream=92)).cuda()
    want = torch.empty((rows, hidden), dtype=torch.float16, device="cuda")
    b.run_mlp_device(gu_full, dn_full, x, want, rows)
    for _ in range(2):
        got = torch.empty((rows, hidden), dtype=torch.float16, device="cuda")
        mlp.run_device(x, got, rows)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (rank, "split-K MLP", rows)
mlp.close(); gu_full.close(); dn_full.close()
b.check()
dist.barrier()
dist.destroy_process_group()
print(f"rank {rank} ok")
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_equals_single_gpu(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD)
    env = dict(os.environ, QL_ROOT=ROOT, NCCL_NVLS_ENABLE="0")
    n = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", "29531", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
