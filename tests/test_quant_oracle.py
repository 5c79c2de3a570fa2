"""The int8 row quantizer's CPU restatement on hand-checked cases (no GPU).

The engine's optional int8 weight-only mode has no counterpart in the
reference (its README lists INT8/INT4 weight transfer as unsupported), so the
known answers here follow the engine's documented rule: scale = max|w| / 127,
q = round-half-even(w / scale) clamped to [-127, 127], zero rows -> 0.
"""

import numpy as np

from oracle import quant_i8


def bf16_bits(values):
    f = np.asarray(values, dtype=np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)  # exact for bf16-representable values


def test_known_rows():
    w = bf16_bits([[127.0, -63.5, 0.5, 1.5, 2.5, -127.0, 0.0, 64.0],
                   [0.0] * 8,
                   [-1.0, 0.25, 0.5, 0.0, 0.0, 0.0, 0.0, 0.0]])
    q, scale = quant_i8.quantize_rows_i8(w)
    assert scale.tolist() == [1.0, 0.0, np.float32(1.0) / np.float32(127.0)]
    # row 0: scale 1, ties to even (0.5 -> 0, 1.5 -> 2, 2.5 -> 2, -63.5 -> -64)
    assert q[0].tolist() == [127, -64, 0, 2, 2, -127, 0, 64]
    assert q[1].tolist() == [0] * 8
    s = np.float32(1.0) / np.float32(127.0)
    expect = np.clip(np.rint(np.float32([-1.0, 0.25, 0.5]) / s), -127, 127).astype(int).tolist()
    assert q[2, :3].tolist() == expect == [-127, 32, 64]


def test_random_rows_bound_and_reconstruct():
    rng = np.random.default_rng(5)
    w = bf16_bits((rng.standard_normal((64, 512)) * 0.02).astype(np.float32))
    q, scale = quant_i8.quantize_rows_i8(w)
    f = quant_i8.bf16_to_f32(w).astype(np.float64)
    assert np.abs(q).max() == 127 and q.dtype == np.int8
    # every row reaches +-127 at its maximum; reconstruction error <= half a step
    assert (np.abs(q).max(axis=1) == 127).all()
    err = np.abs(quant_i8.dequantized(q, scale) - f)
    # (half a step, plus the fp32 rounding of the scale and of w / scale)
    assert (err <= scale.astype(np.float64)[:, None] * (0.5 + 1e-4)).all()
