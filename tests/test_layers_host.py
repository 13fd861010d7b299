"""DenseLayerLinears / OutputHead loading on the CPU (src/model/dense.rs:209-280,
src/model/output_head.rs:28-46): module names, grouping of the q/k/v and gate/up modules by
bit width, shapes, and the seeded checkpoint stand-in.  The linears are the numpy oracle
behind the fake backend of test_projection_host; tests/test_gpu_layers.py runs the layer
on the CUDA library."""
import numpy as np

from open_rknpu2_lm_infer_b200 import workloads as W
from open_rknpu2_lm_infer_b200.layers import DenseLayerLinears, OutputHead
from test_projection_host import FakeBackend

DIMS = dict(hidden=64, q_heads=4, kv_heads=2, head_dim=8, intermediate=48)


def bits_for(prefix, q, k, v, o, gate, up, down):
    return {prefix + "self_attn.q_proj": q, prefix + "self_attn.k_proj": k,
            prefix + "self_attn.v_proj": v, prefix + "self_attn.o_proj": o,
            prefix + "mlp.gate_proj": gate, prefix + "mlp.up_proj": up,
            prefix + "mlp.down_proj": down}


def test_uniform_bits_group_into_one_matrix_each():
    p = "model.layers.0."
    ck = W.SyntheticCheckpoint(bits_for(p, 4, 4, 4, 8, 4, 4, 8))
    be = FakeBackend()
    layer = DenseLayerLinears.load(be, ck, p, **DIMS)
    assert [off for _, off in layer.qkv.parts] == [0]
    assert layer.qkv.width == 32 + 2 * 16 == layer.qkv_width
    assert [off for _, off in layer.gate_up.parts] == [0] and layer.gate_up.width == 96
    shapes = [(m.bits, m.k, m.n) for m, _ in be.loaded]
    assert shapes == [(4, 64, 64), (4, 64, 96), (8, 32, 64), (8, 48, 64)]
    # the fused q/k/v matrix is the three modules side by side (checkpoint.rs:392-423)
    fused = np.asarray(be.loaded[0][0].codes).reshape(64, 64)
    for name, lo, hi in (("q_proj", 0, 32), ("k_proj", 32, 48), ("v_proj", 48, 64)):
        c, _ = ck.codes(p + "self_attn." + name, hi - lo, 64)
        np.testing.assert_array_equal(fused[:, lo:hi], c)


def test_mixed_bits_split_projections():
    p = "model.layers.3."
    ck = W.SyntheticCheckpoint(bits_for(p, 4, 8, 8, 4, 4, 8, 4))
    be = FakeBackend()
    layer = DenseLayerLinears.load(be, ck, p, **DIMS)
    assert [off for _, off in layer.qkv.parts] == [0, 32]       # [q] W4, [k v] W8
    assert [off for _, off in layer.gate_up.parts] == [0, 48]   # [gate] W4, [up] W8
    roles = [r for r, _, _ in layer.linears()]
    assert roles == ["qkv", "qkv", "o", "gate_up", "gate_up", "down"]


def test_output_head_loads_lm_head():
    ck = W.SyntheticCheckpoint({"lm_head": 8})
    be = FakeBackend()
    head = OutputHead.quantized(be, ck, vocab=300, width=64)
    assert head.bits() == 8 and (be.loaded[0][0].k, be.loaded[0][0].n) == (64, 300)
    x = W.activations(2, 64).astype(np.float32)
    out = np.zeros((2, 300), np.float32)
    head.run(x, out, 2)
    c, s = ck.codes("lm_head", 300, 64)
    from oracle import oracle as O
    np.testing.assert_array_equal(out, O.linear(c, s, x))


def test_cfg3_draw_and_loader_streams():
    bits = W.cfg3_module_bits()
    assert len(bits) == 36 * 7 + 1 and bits["lm_head"] == 8
    n_w4 = sum(v == 4 for k, v in bits.items() if k != "lm_head")
    assert 0.55 < n_w4 / (36 * 7) < 0.85  # the ~70% W4 draw
    ck = W.SyntheticCheckpoint(bits)
    a = ck.stream_of("model.layers.0.self_attn.q_proj", 2560, 4096)
    b = ck.stream_of("model.layers.1.self_attn.q_proj", 2560, 4096)
    assert a != b
    shared = W.SyntheticCheckpoint(bits, share_by_shape=True)
    same = [n for n in bits if n.endswith("down_proj") and bits[n] == 8][:2]
    assert shared.stream_of(same[0], 9728, 2560) == shared.stream_of(same[1], 9728, 2560)
