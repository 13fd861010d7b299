"""Chains of decode calls on one stream, with the GEMV's early launch of its dependent.

Every decode GEMV lets the next GEMV / GEMM call on its stream launch while it still runs;
the next call streams its own weights and waits (griddepcontrol.wait) before it reads its
activations or stores.  These tests run chains whose calls depend on each other through
memory -- read after write (a call's output is the next call's input), write after read and
write after write on one buffer -- back to back on one stream, and compare every result
with the same calls run one at a time with a device synchronisation between them, bit for
bit, and with the oracle.
"""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import QuantMatrix
from open_rknpu2_lm_infer_b200 import workloads as W

pytestmark = pytest.mark.gpu


def load(backend, bits, k, n, seed):
    w = W.weight_codes(bits, k, n, stream=seed)
    s = W.weight_scales(n, stream=seed)
    return backend.load(QuantMatrix(bits, k, n, w, s)), w, s


def test_chain_read_after_write(backend, coracle):
    """x -> A (W8 2560->9728) -> B (W4 9728->2560) -> C (W8 2560->2560) -> D (W4 2560->2x1024
    SwiGLU), f32 between the calls, M=1 and M=3; repeated 20 times back to back."""
    a, wa, sa = load(backend, 8, 2560, 9728, 200)
    b, wb, sb = load(backend, 4, 9728, 2560, 201)
    c, wc, sc = load(backend, 8, 2560, 2560, 202)
    d, wd, sd = load(backend, 4, 2560, 2048, 203)
    for rows in (1, 3):
        xh = W.activations(rows, 2560, stream=204 + rows)
        x = torch.from_numpy(xh).cuda()
        ya = torch.empty((rows, 9728), dtype=torch.float32, device="cuda")
        yb = torch.empty((rows, 2560), dtype=torch.float32, device="cuda")
        yc = torch.empty((rows, 2560), dtype=torch.float32, device="cuda")
        yd = torch.empty((rows, 1024), dtype=torch.float32, device="cuda")

        def chain(sync):
            for lin, src, dst, glu in ((a, x, ya, False), (b, ya, yb, False),
                                       (c, yb, yc, False), (d, yc, yd, True)):
                lin.run_device(src, dst, rows, swiglu=glu)
                if sync:
                    torch.cuda.synchronize()
            return [t.clone() for t in (ya, yb, yc, yd)]

        want = chain(sync=True)
        backend.check()
        for _ in range(20):
            got = chain(sync=False)
        torch.cuda.synchronize()
        backend.check()
        for g, w_ in zip(got, want):
            np.testing.assert_array_equal(g.cpu().numpy().view(np.uint32),
                                          w_.cpu().numpy().view(np.uint32))
        # the first link against the oracle, bit-exact (f32 output)
        np.testing.assert_array_equal(want[0].cpu().numpy(), coracle.linear(wa, sa, xh))
        # the second against the oracle on the GPU's own f32 input, bit-exact
        np.testing.assert_array_equal(want[1].cpu().numpy(),
                                      coracle.linear(wb, sb, want[0].cpu().numpy()))
    for lin in (a, b, c, d):
        lin.close()


def test_chain_reuses_buffers(backend, coracle):
    """One output buffer written by consecutive calls and read between them (write after
    read, write after write), independent calls on rotated weights, and a prefill GEMM call
    in the chain."""
    lins = [load(backend, bits, 2560, 4096, 210 + i) for i, bits in enumerate((8, 4, 8, 4))]
    back, wk, sk = load(backend, 8, 4096, 2560, 220)
    rows = 2
    xh = W.activations(rows, 2560, stream=221)
    x = torch.from_numpy(xh).cuda()
    x64 = torch.from_numpy(W.activations(64, 2560, stream=222)).cuda()
    y = torch.empty((rows, 4096), dtype=torch.float16, device="cuda")
    z = torch.empty((4, rows, 2560), dtype=torch.float16, device="cuda")
    g = torch.empty((64, 4096), dtype=torch.float16, device="cuda")

    def chain(sync):
        for i, (lin, _, _) in enumerate(lins):
            lin.run_device(x, y, rows)          # overwrites y (read by the previous call)
            back.run_device(y, z[i], rows)      # reads y
            if i == 1:
                lin.run_device(x64, g, 64)      # a GEMM call in the chain
            if sync:
                torch.cuda.synchronize()
        return z.clone(), g.clone()

    want_z, want_g = chain(sync=True)
    for _ in range(20):
        got_z, got_g = chain(sync=False)
    torch.cuda.synchronize()
    backend.check()
    np.testing.assert_array_equal(got_z.cpu().numpy().view(np.uint16),
                                  want_z.cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(got_g.cpu().numpy().view(np.uint16),
                                  want_g.cpu().numpy().view(np.uint16))
    for i, (lin, w, s) in enumerate(lins):
        yi = coracle.linear(w, s, xh).astype(np.float16)
        want = coracle.linear(wk, sk, yi).astype(np.float16)
        np.testing.assert_array_equal(want_z[i].cpu().numpy().view(np.uint16),
                                      want.view(np.uint16))
        lin.close()
    back.close()
