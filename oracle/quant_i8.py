"""CPU restatement of the engine's int8 row quantizer (TEST INFRASTRUCTURE).

Only tests import this module, as the checker of ``cb_quantize_rows_i8``; the
product path never calls it. The reference has no quantized mode (its
README.md:156 lists INT8/INT4 weight transfer as unsupported), so there is no
reference algorithm to follow: this restates the engine's own documented
rule, in numpy fp32 arithmetic that reproduces the kernel's bits:

    s_r = fp32(max_k |w_rk|) / 127           (IEEE fp32 division)
    q_rk = clamp(rint(fp32(w_rk) / s_r), -127, 127)   (round half to even)
    an all-zero row: s_r = 0, q_r = 0

and the dequantized projection the int8 GEMVs approximate,
``x . (q * s)^T`` in float64.
"""

import numpy as np


def bf16_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 values."""

    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantize_rows_i8(w_bits):
    """w_bits: uint16 [rows, K] bf16 patterns -> (int8 [rows, K], float32 [rows])."""

    w = bf16_to_f32(w_bits)
    mx = np.abs(w).max(axis=1).astype(np.float32)
    scale = (mx / np.float32(127.0)).astype(np.float32)
    q = np.zeros(w.shape, dtype=np.int8)
    live = scale > 0
    if live.any():
        ratio = (w[live] / scale[live, None]).astype(np.float32)
        q[live] = np.clip(np.rint(ratio), -127, 127).astype(np.int8)
    return q, scale


def dequantized(q, scale):
    """float64 weights q * s of quantized rows."""

    return q.astype(np.float64) * scale.astype(np.float64)[:, None]
