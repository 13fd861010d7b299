"""The quantized linears of dense decoder layers (src/model/dense.rs:209-280, :425-530) and
the quantized output head (src/model/output_head.rs:28-46) on the CUDA library, against the
oracle (src/npu.rs:1097-1121).

Layers at the Qwen3-4B shapes of the 36-layer configuration (hidden 2560, q/k/v 2560 ->
4096 + 1024 + 1024, o 4096 -> 2560, gate/up 2560 -> 2 x 9728, down 9728 -> 2560): two
layers of the seeded W4/W8 draw and one with mixed bit widths inside both projections (q W4
with k/v W8; gate W4 with up W8), decode (M=1) and prefill (M=512).  Every linear is
checked on its own input: fp16 outputs bit-exact against f16(oracle); the MLP's f32 middle
within 1e-3 relative of the oracle's SwiGLU (exp differs in the last bits) and its down
projection bit-exact against the oracle run on that middle.  The W8 lm_head 2560 -> 151936
at M=1 and M=512, bit-exact.
"""
import numpy as np
import pytest
import torch

from open_rknpu2_lm_infer_b200 import workloads as W
from open_rknpu2_lm_infer_b200.layers import DenseLayerLinears, OutputHead

pytestmark = pytest.mark.gpu

Q = W.QWEN3_4B
DIMS = dict(hidden=Q["hidden"], q_heads=Q["q_heads"], kv_heads=Q["kv_heads"],
            head_dim=Q["head_dim"], intermediate=Q["intermediate"])


def f16_bits(a):
    return np.asarray(a, np.float16).view(np.uint16)


def fused_codes(ck, prefix, names, k):
    parts = [ck.codes(prefix + n, w, k) for n, w in names]
    return np.concatenate([c for c, _ in parts], axis=1), np.concatenate([s for _, s in parts])


def layer_cases():
    bits = W.cfg3_module_bits()
    mixed = "model.layers.99."
    bits.update({mixed + "self_attn.q_proj": 4, mixed + "self_attn.k_proj": 8,
                 mixed + "self_attn.v_proj": 8, mixed + "self_attn.o_proj": 8,
                 mixed + "mlp.gate_proj": 4, mixed + "mlp.up_proj": 8,
                 mixed + "mlp.down_proj": 4})
    return bits, ["model.layers.0.", "model.layers.1.", mixed]


@pytest.mark.parametrize("rows", [1, 512])
def test_layer_linears_match_oracle(backend, coracle, rows):
    bits, prefixes = layer_cases()
    ck = W.SyntheticCheckpoint(bits)
    h, qw, kw, f = Q["hidden"], Q["q_heads"] * Q["head_dim"], Q["kv_heads"] * Q["head_dim"], \
        Q["intermediate"]
    x = W.activations(rows, h, stream=300)
    xa = W.activations(rows, qw, stream=301)
    xd, xad = torch.from_numpy(x).cuda(), torch.from_numpy(xa).cuda()
    groups = set()
    for p in prefixes:
        layer = DenseLayerLinears.load(backend, ck, p, **DIMS)
        groups.add((len(layer.qkv.parts), len(layer.gate_up.parts)))
        qkv = torch.zeros((rows, layer.qkv_width), dtype=torch.float16, device="cuda")
        o = torch.zeros((rows, h), dtype=torch.float16, device="cuda")
        mid = torch.zeros((rows, f), dtype=torch.float32, device="cuda")
        down = torch.zeros((rows, h), dtype=torch.float32, device="cuda")
        fused = torch.zeros((rows, h), dtype=torch.float32, device="cuda")
        layer.qkv_device(xd, qkv, rows)
        layer.o_device(xad, o, rows)
        layer.mlp_device(xd, down, rows, middle=mid)
        layer.mlp_device(xd, fused, rows)
        backend.check()
        # q/k/v: the modules side by side, whatever the grouping
        wq, sq = fused_codes(ck, p, [("self_attn.q_proj", qw), ("self_attn.k_proj", kw),
                                     ("self_attn.v_proj", kw)], h)
        np.testing.assert_array_equal(f16_bits(qkv.cpu().numpy()),
                                      f16_bits(coracle.linear(wq, sq, x)), err_msg=p + "qkv")
        wo, so = ck.codes(p + "self_attn.o_proj", h, qw)
        np.testing.assert_array_equal(f16_bits(o.cpu().numpy()),
                                      f16_bits(coracle.linear(wo, so, xa)), err_msg=p + "o")
        wg, sg = fused_codes(ck, p, [("mlp.gate_proj", f), ("mlp.up_proj", f)], h)
        want_mid = coracle.swiglu(coracle.linear(wg, sg, x))
        got_mid = mid.cpu().numpy()
        rel = np.abs(got_mid - want_mid) / np.maximum(np.abs(want_mid), 1.0)
        assert rel.max() <= 1e-3, (p, rel.max())
        wdn, sdn = ck.codes(p + "mlp.down_proj", h, f)
        want_down = coracle.linear(wdn, sdn, got_mid)
        np.testing.assert_array_equal(down.cpu().numpy(), want_down, err_msg=p + "down")
        # the fused MLP call gives the same bits as the explicit middle
        np.testing.assert_array_equal(fused.cpu().numpy().view(np.uint32),
                                      down.cpu().numpy().view(np.uint32), err_msg=p + "mlp")
        layer.close()
    assert (2, 2) in groups and (1, 1) in groups  # both run paths were exercised


def test_output_head_lm_head(backend, coracle):
    vocab, width = Q["vocab"], Q["hidden"]
    ck = W.SyntheticCheckpoint({"lm_head": 8})
    head = OutputHead.quantized(backend, ck, vocab, width)
    assert head.bits() == 8
    w, s = ck.codes("lm_head", vocab, width)
    for rows in (1, 512):
        x = W.activations(rows, width, stream=310 + rows)
        out = torch.zeros((rows, vocab), dtype=torch.float16, device="cuda")
        head.prepare(rows)
        head.run_device(torch.from_numpy(x).cuda(), out, rows)
        backend.check()
        np.testing.assert_array_equal(f16_bits(out.cpu().numpy()),
                                      f16_bits(coracle.linear(w, s, x)), err_msg=f"rows={rows}")
    # the reference's host call, f32 in and out
    x = W.activations(3, width, stream=320).astype(np.float32)
    out = np.zeros((3, vocab), np.float32)
    head.run(x, out, 3)
    np.testing.assert_array_equal(out, coracle.linear(w, s, x))
    head.close()
