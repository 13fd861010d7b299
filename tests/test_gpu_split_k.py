"""Row-parallel (split-K) MLP on one GPU with the ranks emulated (a rank's weights loaded
as their own objects, the collectives replaced by a max and an int32 sum on the device):
the C-ABI steps a rank takes -- gate/up slice with SwiGLU, qlinear_row_amax_device,
qlinear_run_device_amax into int32 partial accumulators, qlinear_dequant_device -- give the
single-GPU MLP block (qlinear_run_mlp_device, src/model/dense.rs:499-530) bit for bit, at the
decode (GEMV) and prefill (GEMM) row counts, with K slices that are not multiples of 128."""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W
from open_rknpu2_lm_infer_b200.sharded import mlp_shard_matrices

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,b1,b2,rows", [
    (2, 4, 8, 1), (2, 4, 8, 300), (4, 8, 4, 5), (8, 4, 8, 64), (8, 4, 4, 1),
])
def test_split_k_mlp_equals_single_gpu(backend, world, b1, b2, rows):
    hidden, h = 2560, 9728  # h / 8 = 1216: K slices padded to 1280
    gate_up = QuantMatrix(b1, hidden, 2 * h, W.weight_codes(b1, hidden, 2 * h, stream=80),
                          W.weight_scales(2 * h, stream=80))
    down = QuantMatrix(b2, h, hidden, W.weight_codes(b2, h, hidden, stream=81),
                       W.weight_scales(hidden, stream=81))
    a = torch.from_numpy(W.activations(rows, hidden, stream=82)).cuda()
    gu_full, dn_full = backend.load(gate_up), backend.load(down)
    for dtype in (torch.float16, torch.float32):
        want = torch.zeros((rows, hidden), dtype=dtype, device="cuda")
        backend.run_mlp_device(gu_full, dn_full, a, want, rows)
        mids, amaxes, parts = [], [], []
        for r in range(world):
            gu, dn = mlp_shard_matrices(gate_up, down, world, r)
            lgu, ldn = backend.load(gu), backend.load(dn)
            hs = gu.n // 2
            mid = torch.zeros((rows, hs), dtype=torch.float32, device="cuda")
            lgu.run_device(a, mid, rows, swiglu=True)
            amax = torch.zeros((rows,), dtype=torch.float32, device="cuda")
            backend.row_amax_device(mid, rows, hs, amax)
            mids.append((mid, ldn))
            amaxes.append(amax)
            lgu.close()
        gmax = torch.stack(amaxes).amax(dim=0)  # the all-reduce MAX
        # the row maxima are those of the whole middle row
        full_mid = torch.cat([m for m, _ in mids], dim=1).cpu().numpy()
        np.testing.assert_array_equal(gmax.cpu().numpy(), np.abs(full_mid).max(axis=1))
        for mid, ldn in mids:
            acc = torch.zeros((rows, hidden), dtype=torch.int32, device="cuda")
            ldn.run_device_amax(mid, gmax, acc, rows)
            parts.append(acc)
        acc = torch.stack(parts).sum(dim=0, dtype=torch.int32)  # the all-reduce SUM (exact)
        got = torch.zeros((rows, hidden), dtype=dtype, device="cuda")
        mids[0][1].dequant_device(acc, gmax, got, rows)
        backend.check()
        assert torch.equal(got, want), (world, b1, b2, rows, dtype)
        for _, ldn in mids:
            ldn.close()
    gu_full.close()
    dn_full.close()
