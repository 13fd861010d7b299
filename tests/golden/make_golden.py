"""Generate the golden fixtures in tests/golden/ (run once, in a checkout that has the
reference tree; the fixtures are committed and the tests never read the reference).

    python tests/golden/make_golden.py [--reference PATH_TO_open_rknpu2_lm_infer]

Where the expected values come from:

* Activation codes and scales: the reference's own numpy restatement of its A8
  quantiser, ``quantize`` in scripts/qwen35/audit_batch_attention_trace.py:17-23
  (reciprocal multiply, ties away from zero via copysign(floor(|v|+0.5), v), clamp to
  +-127), imported from the reference tree and applied row by row, as the reference's
  oracle does (src/npu.rs:1099-1110).  That function computes floor(|v| + 0.5) in f32,
  which differs from f32::round only at |v| = 0.5 - 2**-25; the script counts such
  elements in every fixture and requires the count to be zero, so the fixture agrees
  with both statements.  It has no zero-row branch, so no fixture row is all zero.
* Integer accumulators and outputs: exact int64 numpy matmul of those codes with the
  weight codes, then (f32(acc) * s_a) * s_w as two f32 products (src/npu.rs:1111-1117).
  This path shares no code with oracle/.
* Edge cases the reference's quantiser defines but its tests never reach (zero row,
  NaN, +-inf, values below FLT_MIN*127, exact .5 ties): expected codes written out by
  hand in this script from the Rust semantics (f32::max ignores NaN, f32::round ties
  away, `NaN as i32` is 0); see ``edge_cases``.

Data of the reference's two board tests (src/npu.rs:1161-1224 and
src/npu/narrow_projection.rs:3-68) comes from their deterministic generators, restated
in open_rknpu2_lm_infer_b200/workloads.py.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from open_rknpu2_lm_infer_b200 import workloads as W  # noqa: E402


def load_reference_quantize(ref_root: str):
    path = os.path.join(ref_root, "scripts", "qwen35", "audit_batch_attention_trace.py")
    spec = importlib.util.spec_from_file_location("ref_audit_trace", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.quantize


def per_row(quantize, x: np.ndarray):
    """Apply the reference's whole-array quantiser to each row; count the elements on
    which floor(|v|+0.5) and f32::round disagree."""
    x = np.asarray(x, dtype=np.float32)
    codes = np.empty(x.shape, np.int8)
    scales = np.empty(x.shape[0], np.float32)
    disagreements = 0
    for r in range(x.shape[0]):
        c, s = quantize(x[r])
        codes[r] = c.astype(np.int8)
        scales[r] = np.float32(s)
        scaled = (x[r] * (np.float32(1) / np.float32(s))).astype(np.float32)
        a = np.abs(scaled)
        disagreements += int(np.count_nonzero(a == np.float32(0.5) - np.float32(2.0 ** -25)))
    return codes, scales, disagreements


def linear_from_codes(codes, sa, w_kn, sw):
    acc = codes.astype(np.int64) @ w_kn.astype(np.int64)
    assert np.all(np.abs(acc) < 2 ** 31)
    acc = acc.astype(np.int32)
    t = (acc.astype(np.float32) * sa[:, None]).astype(np.float32)
    y = (t * sw[None, :]).astype(np.float32)
    return acc, y


def edge_cases():
    """Rows that exercise the quantiser's special cases, with expected results written
    from the Rust definitions (src/npu.rs:1099-1110)."""
    f = np.float32
    k = 8
    rows, exp_codes, exp_scales = [], [], []

    # 1. all-zero row: scale 1.0, codes 0.
    rows.append(np.zeros(k, f)); exp_scales.append(f(1.0)); exp_codes.append([0] * k)

    # 2. exact ties: amax 127 -> scale 1.0 -> inv 1.0; 2.5 -> 3, -2.5 -> -3, 0.5 -> 1,
    #    -0.5 -> -1, 126.5 -> 127 (ties away from zero).
    r = np.array([127, 2.5, -2.5, 0.5, -0.5, 126.5, 1.5, -127], f)
    rows.append(r); exp_scales.append(f(1.0)); exp_codes.append([127, 3, -3, 1, -1, 127, 2, -127])

    # 3. the value just below one half: 0.49999997 -> 0 under f32::round.
    v = f(0.5) - f(2.0 ** -25)
    r = np.array([127, v, -v, 0, 0, 0, 0, 0], f)
    rows.append(r); exp_scales.append(f(1.0)); exp_codes.append([127, 0, 0, 0, 0, 0, 0, 0])

    # 4. NaN is ignored by the max and quantises to 0 (`NaN as i32` = 0).
    r = np.array([np.nan, 127, -63.5, 0, 1, 2, 3, np.nan], f)
    rows.append(r); exp_scales.append(f(1.0)); exp_codes.append([0, 127, -64, 0, 1, 2, 3, 0])

    # 5. +inf: amax = inf, scale = inf, inv = 0; finite * 0 = 0, inf * 0 = NaN -> 0.
    r = np.array([np.inf, 1, -1, 5, 0, 0, 0, -3], f)
    rows.append(r); exp_scales.append(f(np.inf)); exp_codes.append([0] * k)

    # 6. tiny magnitudes: amax/127 < FLT_MIN -> scale = FLT_MIN.
    tiny = f(np.finfo(np.float32).tiny)
    r = np.array([tiny * f(2), -tiny * f(2), tiny, 0, 0, 0, 0, 0], f)
    s = tiny
    inv = f(1) / s
    exp = []
    for val in r:
        sc = f(val * inv)
        t = np.trunc(sc)
        q = t + np.sign(sc) if abs(sc - t) >= 0.5 else t
        exp.append(int(np.clip(q, -127, 127)))
    rows.append(r); exp_scales.append(s); exp_codes.append(exp)

    # 7. a generic row: amax 1.0 -> scale 1/127 (RN), inv = 1/scale (RN).
    r = np.array([1.0, -1.0, 0.25, -0.75, 0.5, 0.1, -0.3, 0.9], f)
    s = f(f(1.0) / f(127))
    inv = f(f(1) / s)
    exp = []
    for val in r:
        sc = f(val * inv)
        t = np.trunc(sc)
        q = t + np.sign(sc) if abs(sc - t) >= 0.5 else t
        exp.append(int(np.clip(q, -127, 127)))
    rows.append(r); exp_scales.append(s); exp_codes.append(exp)

    return (np.stack(rows).astype(np.float32), np.array(exp_codes, np.int8),
            np.array(exp_scales, np.float32))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QLINEAR_REFERENCE_TREE"),
                    help="root of the reference tree (or set QLINEAR_REFERENCE_TREE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference tree with --reference or QLINEAR_REFERENCE_TREE")
    quantize = load_reference_quantize(args.reference)
    out = {}
    total_disagree = 0

    # Board test quantized_linear_padding_and_swiglu (src/npu.rs:1161-1224).
    x = W.kat_input(256, 256)
    codes, sa, d = per_row(quantize, x)
    total_disagree += d
    out["kat_codes"], out["kat_scales"] = codes, sa
    for bits in (4, 8):
        w, sw = W.kat_matrix(bits)
        acc, y = linear_from_codes(codes, sa, w, sw)
        out[f"kat_w{bits}_acc"], out[f"kat_w{bits}_y"] = acc, y

    # Board test narrow_w8_gdn_gates_match_integer_oracle (src/npu/narrow_projection.rs).
    for n in (32, 64):
        w, sw, xn = W.narrow_kat(n)
        c, s, d = per_row(quantize, xn)
        total_disagree += d
        acc, y = linear_from_codes(c, s, w, sw)
        out[f"narrow_n{n}_codes"], out[f"narrow_n{n}_scales"] = c, s
        out[f"narrow_n{n}_y"] = y

    # Seeded activations with the benchmark distribution (fp16, 1% outlier channels).
    for name, rows, k, stream in (("seed_k2560", 16, 2560, 7), ("seed_k9728", 4, 9728, 8),
                                  ("seed_k8192", 2, 8192, 9), ("seed_k100", 5, 100, 10)):
        xh = W.activations(rows, k, stream=stream)
        c, s, d = per_row(quantize, xh.astype(np.float32))
        total_disagree += d
        out[f"{name}_x"], out[f"{name}_codes"], out[f"{name}_scales"] = xh, c, s
    # A seeded linear with an odd shape (K, N not multiples of the GPU tiles).
    xh = W.activations(3, 100, stream=11)
    w = W.weight_codes(4, 100, 72, stream=11)
    sw = W.weight_scales(72, stream=11)
    c, s, d = per_row(quantize, xh.astype(np.float32))
    total_disagree += d
    acc, y = linear_from_codes(c, s, w, sw)
    out.update(odd_x=xh, odd_w=w, odd_sw=sw, odd_acc=acc, odd_y=y)

    ex, ec, es = edge_cases()
    out.update(edge_x=ex, edge_codes=ec, edge_scales=es)

    assert total_disagree == 0, f"{total_disagree} elements at 0.5-2^-25; choose other inputs"
    out["floor_round_disagreements"] = np.array(total_disagree)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
