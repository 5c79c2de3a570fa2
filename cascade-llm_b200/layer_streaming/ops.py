"""Torch operators ``torch.ops.cascade.*`` over the C ABI of libcascade_b200.

Each operator validates its tensors and launches one hand-written sm_100a
kernel on the current CUDA stream (no host synchronisation, so every
operator can be captured into a CUDA graph). Operators only have a CUDA
implementation: called with CPU tensors they raise, there is no fallback.
Reference op each one replaces is cited in ``include/cascade_b200.h``.
"""

import torch

from . import _native as nat

BF16 = torch.bfloat16
_LIB = torch.library.Library("cascade", "DEF")

_SCHEMAS = {
    "embedding": "embedding(Tensor ids, Tensor table, Tensor(a!) out) -> ()",
    "rmsnorm": "rmsnorm(Tensor x, Tensor weight, float eps, Tensor(a!) out) -> ()",
    "qkv_rope": (
        "qkv_rope(Tensor x, Tensor? norm_w, float eps, Tensor? wq, Tensor? wk, Tensor? wv, "
        "Tensor inv_freq, Tensor position, int token, Tensor(a!)? q_out, Tensor(b!)? k_cache, "
        "Tensor(c!)? v_cache, int q_heads=32, int kv_heads=8) -> ()"
    ),
    "proj_residual": "proj_residual(Tensor x, Tensor w, Tensor residual, Tensor(a!) out) -> ()",
    "proj_partial": "proj_partial(Tensor x, Tensor w, Tensor(a!) out) -> ()",
    "residual_add_f32": "residual_add_f32(Tensor x, Tensor sum, Tensor(a!) out) -> ()",
    "gate_up_swiglu": (
        "gate_up_swiglu(Tensor x, Tensor? norm_w, float eps, Tensor w_gate, Tensor w_up, "
        "Tensor(a!) out) -> ()"
    ),
    "gate_silu": "gate_silu(Tensor x, Tensor? norm_w, float eps, Tensor w_gate, Tensor(a!) out) -> ()",
    "up_mul": "up_mul(Tensor x, Tensor? norm_w, float eps, Tensor w_up, Tensor(a!) gate_act) -> ()",
    "lm_head_topk": (
        "lm_head_topk(Tensor x, Tensor? norm_w, float eps, Tensor w, int row_offset, int k, "
        "Tensor(a!)? logits, Tensor(b!) out_values, Tensor(c!) out_indices, Tensor(d!) workspace, "
        "Tensor(e!) ticket) -> ()"
    ),
    "topk_merge": (
        "topk_merge(Tensor? a_values, Tensor? a_indices, Tensor b_values, Tensor b_indices, int k, "
        "Tensor(a!) out_values, Tensor(b!) out_indices) -> ()"
    ),
    "attention": (
        "attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor position, int splits, int chunk, "
        "Tensor(a!) out, Tensor(b!) workspace, Tensor(c!) tickets) -> ()"
    ),
    "attention_oproj": (
        "attention_oproj(Tensor q, Tensor k_cache, Tensor v_cache, Tensor position, int splits, Tensor wo, "
        "Tensor residual, Tensor(a!) attn_out, Tensor(b!) out, Tensor(c!) workspace, Tensor(d!) tickets) -> ()"
    ),
    "position_set": "position_set(Tensor(a!) position, Tensor? src, int value) -> ()",
    "gemm_bf16": "gemm_bf16(Tensor a, Tensor w, Tensor(a!) out) -> ()",
    "prefill_attention": (
        "prefill_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor position, Tensor(a!) out) -> ()"
    ),
    "gemm_residual": "gemm_residual(Tensor a, Tensor w, Tensor residual, Tensor(a!) out) -> ()",
    "gemm_swiglu": "gemm_swiglu(Tensor a, Tensor w_gate, Tensor w_up, Tensor(a!) out) -> ()",
    "gemm_partial": "gemm_partial(Tensor a, Tensor w, Tensor(a!) out) -> ()",
    "gemm_silu": "gemm_silu(Tensor a, Tensor w_gate, Tensor(a!) out) -> ()",
    "gemm_mul": "gemm_mul(Tensor a, Tensor w_up, Tensor(a!) gate_act) -> ()",
    "prefill_qkv_rope": (
        "prefill_qkv_rope(Tensor xn, Tensor? wq, Tensor? wk, Tensor? wv, Tensor inv_freq, Tensor position, "
        "Tensor(a!)? q_out, Tensor(b!)? k_cache, Tensor(c!)? v_cache, int q_heads=32, int kv_heads=8) -> ()"
    ),
    "position_advance": "position_advance(Tensor(a!) position, int count) -> ()",
    "quantize_rows_i8": "quantize_rows_i8(Tensor w, Tensor(a!) q, Tensor(b!) scale) -> ()",
    "dequantize_rows_i8": "dequantize_rows_i8(Tensor q, Tensor scale, Tensor(a!) out) -> ()",
    "qkv_rope_i8": (
        "qkv_rope_i8(Tensor x, Tensor? norm_w, float eps, Tensor wq, Tensor sq, Tensor wk, Tensor sk, "
        "Tensor wv, Tensor sv, Tensor inv_freq, Tensor position, int token, Tensor(a!) q_out, "
        "Tensor(b!) k_cache, Tensor(c!) v_cache) -> ()"
    ),
    "proj_residual_i8": "proj_residual_i8(Tensor x, Tensor w, Tensor scale, Tensor residual, Tensor(a!) out) -> ()",
    "gate_up_swiglu_i8": (
        "gate_up_swiglu_i8(Tensor x, Tensor? norm_w, float eps, Tensor w_gate, Tensor s_gate, Tensor w_up, "
        "Tensor s_up, Tensor(a!) out) -> ()"
    ),
    "lm_head_topk_i8": (
        "lm_head_topk_i8(Tensor x, Tensor? norm_w, float eps, Tensor w, Tensor scale, int k, "
        "Tensor(a!)? logits, Tensor(b!) out_values, Tensor(c!) out_indices, Tensor(d!) workspace, "
        "Tensor(e!) ticket) -> ()"
    ),
}


def _stream(t):
    return nat.stream_ptr(t.device)


def embedding(ids, table, out):
    m = ids.numel()
    nat.check(
        nat.lib().cb_embedding(
            nat.ptr(ids, torch.int64, "ids"), m, nat.ptr(table, BF16, "table"),
            table.shape[0], table.shape[1], nat.ptr(out, BF16, "out"), _stream(out),
        ),
        "cascade.embedding",
    )


def rmsnorm(x, weight, eps, out):
    hidden = x.shape[-1]
    nat.check(
        nat.lib().cb_rmsnorm(
            nat.ptr(x, BF16, "x"), nat.ptr(weight, BF16, "weight"), x.numel() // hidden, hidden,
            float(eps), nat.ptr(out, BF16, "out"), _stream(out),
        ),
        "cascade.rmsnorm",
    )


def qkv_rope(x, norm_w, eps, wq, wk, wv, inv_freq, position, token, q_out, k_cache, v_cache,
             q_heads=32, kv_heads=8):
    cache = k_cache if k_cache is not None else v_cache
    cache_len = cache.shape[-2] if cache is not None else 0
    nat.check(
        nat.lib().cb_qkv_rope(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(wq, BF16, "wq"), nat.ptr(wk, BF16, "wk"), nat.ptr(wv, BF16, "wv"),
            nat.ptr(inv_freq, torch.float32, "inv_freq"), nat.ptr(position, torch.int32, "position"),
            int(token), nat.ptr(q_out, BF16, "q_out"), nat.ptr(k_cache, BF16, "k_cache"),
            nat.ptr(v_cache, BF16, "v_cache"), cache_len, int(q_heads), int(kv_heads), _stream(x),
        ),
        "cascade.qkv_rope",
    )


def proj_residual(x, w, residual, out):
    nat.check(
        nat.lib().cb_proj_residual(
            nat.ptr(x, BF16, "x"), w.shape[1], nat.ptr(w, BF16, "w"), w.shape[0],
            nat.ptr(residual, BF16, "residual"), nat.ptr(out, BF16, "out"), _stream(x),
        ),
        "cascade.proj_residual",
    )


def proj_partial(x, w, out):
    nat.check(
        nat.lib().cb_proj_partial(
            nat.ptr(x, BF16, "x"), w.shape[1], nat.ptr(w, BF16, "w"), w.shape[0],
            nat.ptr(out, torch.float32, "out"), _stream(x),
        ),
        "cascade.proj_partial",
    )


def residual_add_f32(x, sum, out):
    nat.check(
        nat.lib().cb_residual_add_f32(
            nat.ptr(x, BF16, "x"), nat.ptr(sum, torch.float32, "sum"), x.numel(), nat.ptr(out, BF16, "out"),
            _stream(x),
        ),
        "cascade.residual_add_f32",
    )


def gate_up_swiglu(x, norm_w, eps, w_gate, w_up, out):
    nat.check(
        nat.lib().cb_gate_up_swiglu(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(w_gate, BF16, "w_gate"), nat.ptr(w_up, BF16, "w_up"), w_gate.shape[0],
            nat.ptr(out, BF16, "out"), _stream(x),
        ),
        "cascade.gate_up_swiglu",
    )


def gate_silu(x, norm_w, eps, w_gate, out):
    nat.check(
        nat.lib().cb_gate_silu(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(w_gate, BF16, "w_gate"), nat.ptr(out, BF16, "out"), _stream(x),
        ),
        "cascade.gate_silu",
    )


def up_mul(x, norm_w, eps, w_up, gate_act):
    nat.check(
        nat.lib().cb_up_mul(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(w_up, BF16, "w_up"), nat.ptr(gate_act, BF16, "gate_act"), _stream(x),
        ),
        "cascade.up_mul",
    )


def lm_head_workspace_bytes(k):
    return int(nat.lib().cb_lm_head_workspace_bytes(int(k)))


def lm_head_topk(x, norm_w, eps, w, row_offset, k, logits, out_values, out_indices, workspace, ticket):
    nat.check(
        nat.lib().cb_lm_head_topk(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(w, BF16, "w"), w.shape[0], int(row_offset), int(k),
            nat.ptr(logits, torch.float32, "logits"), nat.ptr(out_values, torch.float32, "out_values"),
            nat.ptr(out_indices, torch.int64, "out_indices"), nat.ptr(workspace, None, "workspace"),
            nat.ptr(ticket, torch.int32, "ticket"), _stream(x),
        ),
        "cascade.lm_head_topk",
    )


def topk_merge(a_values, a_indices, b_values, b_indices, k, out_values, out_indices):
    na = 0 if a_values is None else a_values.numel()
    nat.check(
        nat.lib().cb_topk_merge(
            nat.ptr(a_values, torch.float32, "a_values"), nat.ptr(a_indices, torch.int64, "a_indices"),
            na, nat.ptr(b_values, torch.float32, "b_values"),
            nat.ptr(b_indices, torch.int64, "b_indices"), b_values.numel(), int(k),
            nat.ptr(out_values, torch.float32, "out_values"),
            nat.ptr(out_indices, torch.int64, "out_indices"), _stream(b_values),
        ),
        "cascade.topk_merge",
    )


def attention_workspace_bytes(m, splits):
    return int(nat.lib().cb_attention_workspace_bytes(int(m), int(splits)))


def attention(q, k_cache, v_cache, position, splits, chunk, out, workspace, tickets):
    kv_heads = k_cache.shape[-3]
    m = q.numel() // (kv_heads * 512)
    if tickets.numel() < kv_heads * m:
        raise ValueError("attention needs one ticket per KV head and token")
    nat.check(
        nat.lib().cb_attention(
            nat.ptr(q, BF16, "q"), nat.ptr(k_cache, BF16, "k_cache"), nat.ptr(v_cache, BF16, "v_cache"),
            k_cache.shape[-2], nat.ptr(position, torch.int32, "position"), m, kv_heads, int(splits), int(chunk),
            nat.ptr(out, BF16, "out"), nat.ptr(workspace, None, "workspace"),
            nat.ptr(tickets, torch.int32, "tickets"), _stream(q),
        ),
        "cascade.attention",
    )


def attention_oproj_max_splits():
    return int(nat.lib().cb_attention_oproj_max_splits())


def attention_oproj(q, k_cache, v_cache, position, splits, wo, residual, attn_out, out, workspace, tickets):
    """One-token attention (8 KV heads) fused with o_proj + residual add."""

    if k_cache.shape[-3] != 8 or q.numel() != 4096 or wo.shape != (4096, 4096):
        raise ValueError("attention_oproj is the one-token, 8-KV-head layout")
    if tickets.numel() < 10:
        raise ValueError("attention_oproj needs 10 zeroed tickets")
    nat.check(
        nat.lib().cb_attention_oproj(
            nat.ptr(q, BF16, "q"), nat.ptr(k_cache, BF16, "k_cache"), nat.ptr(v_cache, BF16, "v_cache"),
            k_cache.shape[-2], nat.ptr(position, torch.int32, "position"), int(splits), nat.ptr(wo, BF16, "wo"),
            nat.ptr(residual, BF16, "residual"), nat.ptr(attn_out, BF16, "attn_out"), nat.ptr(out, BF16, "out"),
            nat.ptr(workspace, None, "workspace"), nat.ptr(tickets, torch.int32, "tickets"), _stream(q),
        ),
        "cascade.attention_oproj",
    )


def _rows(t):
    return t.numel() // t.shape[-1]


def prefill_attention(q, k_cache, v_cache, position, out):
    kv_heads = k_cache.shape[-3]
    m = q.numel() // (kv_heads * 512)
    nat.check(
        nat.lib().cb_prefill_attention(
            nat.ptr(q, BF16, "q"), nat.ptr(k_cache, BF16, "k_cache"), nat.ptr(v_cache, BF16, "v_cache"),
            k_cache.shape[-2], nat.ptr(position, torch.int32, "position"), m, kv_heads,
            nat.ptr(out, BF16, "out"), _stream(q),
        ),
        "cascade.prefill_attention",
    )


def gemm_bf16(a, w, out):
    nat.check(
        nat.lib().cb_gemm_bf16(
            nat.ptr(a, BF16, "a"), _rows(a), a.shape[-1], nat.ptr(w, BF16, "w"), w.shape[0],
            nat.ptr(out, BF16, "out"), _stream(a),
        ),
        "cascade.gemm_bf16",
    )


def gemm_residual(a, w, residual, out):
    nat.check(
        nat.lib().cb_gemm_residual(
            nat.ptr(a, BF16, "a"), _rows(a), a.shape[-1], nat.ptr(w, BF16, "w"), w.shape[0],
            nat.ptr(residual, BF16, "residual"), nat.ptr(out, BF16, "out"), _stream(a),
        ),
        "cascade.gemm_residual",
    )


def gemm_partial(a, w, out):
    nat.check(
        nat.lib().cb_gemm_partial(
            nat.ptr(a, BF16, "a"), _rows(a), a.shape[-1], nat.ptr(w, BF16, "w"), w.shape[0],
            nat.ptr(out, torch.float32, "out"), _stream(a),
        ),
        "cascade.gemm_partial",
    )


def gemm_silu(a, w_gate, out):
    nat.check(
        nat.lib().cb_gemm_silu(
            nat.ptr(a, BF16, "a"), _rows(a), nat.ptr(w_gate, BF16, "w_gate"), w_gate.shape[0],
            nat.ptr(out, BF16, "out"), _stream(a),
        ),
        "cascade.gemm_silu",
    )


def gemm_mul(a, w_up, gate_act):
    nat.check(
        nat.lib().cb_gemm_mul(
            nat.ptr(a, BF16, "a"), _rows(a), nat.ptr(w_up, BF16, "w_up"), w_up.shape[0],
            nat.ptr(gate_act, BF16, "gate_act"), _stream(a),
        ),
        "cascade.gemm_mul",
    )


def gemm_swiglu(a, w_gate, w_up, out):
    nat.check(
        nat.lib().cb_gemm_swiglu(
            nat.ptr(a, BF16, "a"), _rows(a), nat.ptr(w_gate, BF16, "w_gate"), nat.ptr(w_up, BF16, "w_up"),
            w_gate.shape[0], nat.ptr(out, BF16, "out"), _stream(a),
        ),
        "cascade.gemm_swiglu",
    )


def prefill_qkv_rope(xn, wq, wk, wv, inv_freq, position, q_out, k_cache, v_cache, q_heads=32, kv_heads=8):
    nat.check(
        nat.lib().cb_prefill_qkv_rope(
            nat.ptr(xn, BF16, "xn"), _rows(xn), nat.ptr(wq, BF16, "wq"), nat.ptr(wk, BF16, "wk"),
            nat.ptr(wv, BF16, "wv"), int(q_heads), int(kv_heads), nat.ptr(inv_freq, torch.float32, "inv_freq"),
            nat.ptr(position, torch.int32, "position"), nat.ptr(q_out, BF16, "q_out"),
            nat.ptr(k_cache, BF16, "k_cache"), nat.ptr(v_cache, BF16, "v_cache"),
            (k_cache if k_cache is not None else v_cache).shape[-2] if (k_cache is not None or v_cache is not None)
            else 0, _stream(xn),
        ),
        "cascade.prefill_qkv_rope",
    )


def position_set(position, src, value):
    nat.check(
        nat.lib().cb_position_set(
            nat.ptr(position, torch.int32, "position"), nat.ptr(src, torch.int64, "src"),
            int(value), _stream(position),
        ),
        "cascade.position_set",
    )


def position_advance(position, count):
    nat.check(
        nat.lib().cb_position_advance(
            nat.ptr(position, torch.int32, "position"), int(count), _stream(position)
        ),
        "cascade.position_advance",
    )


def fill_normal_(tensor, key, std=0.02, offset=0):
    nat.check(
        nat.lib().cb_fill_normal_bf16(
            nat.ptr(tensor, BF16, "tensor"), tensor.numel(), int(offset), int(key), float(std),
            _stream(tensor),
        ),
        "cascade.fill_normal_",
    )
    return tensor


def fill_(tensor, value):
    nat.check(
        nat.lib().cb_fill_bf16(nat.ptr(tensor, BF16, "tensor"), tensor.numel(), float(value), _stream(tensor)),
        "cascade.fill_",
    )
    return tensor


def memcpy_h2d_async(dst, src):
    """cudaMemcpyAsync of a host tensor into a device tensor (same bytes)."""

    nbytes = src.numel() * src.element_size()
    if dst.numel() * dst.element_size() < nbytes:
        raise ValueError("destination is smaller than the source")
    if src.device.type != "cpu" or dst.device.type != "cuda":
        raise ValueError("memcpy_h2d_async copies host -> device")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise ValueError("memcpy_h2d_async needs contiguous tensors")
    nat.check(
        nat.lib().cb_memcpy_h2d_async(dst.data_ptr(), src.data_ptr(), nbytes, _stream(dst)),
        "cascade.memcpy_h2d_async",
    )


# ------------------------------------------------ int8 weight-only decode
# Optional reduced-precision mode (outside the bf16 parity contract): each
# weight matrix is an int8 [N, K] tensor plus fp32 row scales [N].
I8 = torch.int8
F32 = torch.float32


def quantize_rows_i8(w, q, scale):
    nat.check(
        nat.lib().cb_quantize_rows_i8(
            nat.ptr(w, BF16, "w"), w.shape[0], w.shape[1], nat.ptr(q, I8, "q"), nat.ptr(scale, F32, "scale"),
            _stream(w),
        ),
        "cascade.quantize_rows_i8",
    )


def dequantize_rows_i8(q, scale, out):
    nat.check(
        nat.lib().cb_dequantize_rows_i8(
            nat.ptr(q, I8, "q"), nat.ptr(scale, F32, "scale"), q.shape[0], q.shape[1], nat.ptr(out, BF16, "out"),
            _stream(q),
        ),
        "cascade.dequantize_rows_i8",
    )


def qkv_rope_i8(x, norm_w, eps, wq, sq, wk, sk, wv, sv, inv_freq, position, token, q_out, k_cache, v_cache):
    nat.check(
        nat.lib().cb_qkv_rope_i8(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(wq, I8, "wq"), nat.ptr(sq, F32, "sq"), nat.ptr(wk, I8, "wk"), nat.ptr(sk, F32, "sk"),
            nat.ptr(wv, I8, "wv"), nat.ptr(sv, F32, "sv"), nat.ptr(inv_freq, F32, "inv_freq"),
            nat.ptr(position, torch.int32, "position"), int(token), nat.ptr(q_out, BF16, "q_out"),
            nat.ptr(k_cache, BF16, "k_cache"), nat.ptr(v_cache, BF16, "v_cache"), k_cache.shape[-2],
            wq.shape[0] // 128, wk.shape[0] // 128, _stream(x),
        ),
        "cascade.qkv_rope_i8",
    )


def proj_residual_i8(x, w, scale, residual, out):
    nat.check(
        nat.lib().cb_proj_residual_i8(
            nat.ptr(x, BF16, "x"), w.shape[1], nat.ptr(w, I8, "w"), nat.ptr(scale, F32, "scale"), w.shape[0],
            nat.ptr(residual, BF16, "residual"), nat.ptr(out, BF16, "out"), _stream(x),
        ),
        "cascade.proj_residual_i8",
    )


def gate_up_swiglu_i8(x, norm_w, eps, w_gate, s_gate, w_up, s_up, out):
    nat.check(
        nat.lib().cb_gate_up_swiglu_i8(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps),
            nat.ptr(w_gate, I8, "w_gate"), nat.ptr(s_gate, F32, "s_gate"), nat.ptr(w_up, I8, "w_up"),
            nat.ptr(s_up, F32, "s_up"), w_gate.shape[0], nat.ptr(out, BF16, "out"), _stream(x),
        ),
        "cascade.gate_up_swiglu_i8",
    )


def lm_head_topk_i8(x, norm_w, eps, w, scale, k, logits, out_values, out_indices, workspace, ticket):
    nat.check(
        nat.lib().cb_lm_head_topk_i8(
            nat.ptr(x, BF16, "x"), nat.ptr(norm_w, BF16, "norm_w"), float(eps), nat.ptr(w, I8, "w"),
            nat.ptr(scale, F32, "scale"), w.shape[0], 0, int(k), nat.ptr(logits, F32, "logits"),
            nat.ptr(out_values, F32, "out_values"), nat.ptr(out_indices, torch.int64, "out_indices"),
            nat.ptr(workspace, None, "workspace"), nat.ptr(ticket, torch.int32, "ticket"), _stream(x),
        ),
        "cascade.lm_head_topk_i8",
    )


for _name, _schema in _SCHEMAS.items():
    _LIB.define(_schema)
    _LIB.impl(_name, globals()[_name], "CUDA")
