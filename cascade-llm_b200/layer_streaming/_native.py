"""Binding of libcascade_b200.so (the sm_100a kernels) for the Python host code.

The library exposes a plain C ABI (``include/cascade_b200.h``); this module
loads it with ctypes, checks tensors (device, dtype, contiguity, alignment)
and passes raw pointers plus the current CUDA stream. There is no fallback:
if the library or a GPU is missing, :func:`lib` raises.
"""

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get(
    "CASCADE_B200_LIB",
    os.path.join(os.path.dirname(_HERE), "lib", "libcascade_b200.so"),
)

_LOCK = threading.Lock()
_LIB = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

_SIGNATURES = {
    "cb_version": (_I, []),
    "cb_last_error": (ctypes.c_char_p, []),
    "cb_set_pdl": (_I, [_I]),
    "cb_sm_count": (_I, []),
    "cb_prepare": (_I, []),
    "cb_set_error_word": (_I, [_P]),
    "cb_set_trace": (_I, [_P]),
    "cb_set_l2_stage": (_I, [_I, _I, _I, _I, _I]),
    "cb_set_l2_stage_target": (_I, [_P, _P, _I, _I]),
    "cb_stream_key": (ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_char_p]),
    "cb_fill_normal_bf16": (_I, [_P, _I64, _I64, ctypes.c_uint64, ctypes.c_double, _P]),
    "cb_fill_bf16": (_I, [_P, _I64, _F, _P]),
    "cb_position_set": (_I, [_P, _P, ctypes.c_int32, _P]),
    "cb_position_advance": (_I, [_P, ctypes.c_int32, _P]),
    "cb_embedding": (_I, [_P, _I, _P, _I64, _I, _P, _P]),
    "cb_rmsnorm": (_I, [_P, _P, _I, _I, _F, _P, _P]),
    "cb_qkv_rope": (_I, [_P, _P, _F, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I64, _I, _I, _P]),
    "cb_proj_residual": (_I, [_P, _I, _P, _I, _P, _P, _P]),
    "cb_proj_partial": (_I, [_P, _I, _P, _I, _P, _P]),
    "cb_residual_add_f32": (_I, [_P, _P, _I, _P, _P]),
    "cb_gate_up_swiglu": (_I, [_P, _P, _F, _P, _P, _I, _P, _P]),
    "cb_gate_silu": (_I, [_P, _P, _F, _P, _P, _P]),
    "cb_up_mul": (_I, [_P, _P, _F, _P, _P, _P]),
    "cb_lm_head_workspace_bytes": (_I64, [_I]),
    "cb_lm_head_topk": (_I, [_P, _P, _F, _P, _I64, _I64, _I, _P, _P, _P, _P, _P, _P]),
    "cb_quantize_rows_i8": (_I, [_P, _I64, _I, _P, _P, _P]),
    "cb_dequantize_rows_i8": (_I, [_P, _P, _I64, _I, _P, _P]),
    "cb_qkv_rope_i8": (_I, [_P, _P, _F, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I64, _I, _I, _P]),
    "cb_proj_residual_i8": (_I, [_P, _I, _P, _P, _I, _P, _P, _P]),
    "cb_gate_up_swiglu_i8": (_I, [_P, _P, _F, _P, _P, _P, _P, _I, _P, _P]),
    "cb_lm_head_topk_i8": (_I, [_P, _P, _F, _P, _P, _I64, _I64, _I, _P, _P, _P, _P, _P, _P]),
    "cb_topk_merge": (_I, [_P, _P, _I, _P, _P, _I, _I, _P, _P, _P]),
    "cb_gemm_bf16": (_I, [_P, _I, _I, _P, _I, _P, _P]),
    "cb_gemm_residual": (_I, [_P, _I, _I, _P, _I, _P, _P, _P]),
    "cb_gemm_partial": (_I, [_P, _I, _I, _P, _I, _P, _P]),
    "cb_gemm_silu": (_I, [_P, _I, _P, _I, _P, _P]),
    "cb_gemm_mul": (_I, [_P, _I, _P, _I, _P, _P]),
    "cb_gemm_swiglu": (_I, [_P, _I, _P, _P, _I, _P, _P]),
    "cb_prefill_qkv_rope": (_I, [_P, _I, _P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _I64, _P]),
    "cb_prefill_attention": (_I, [_P, _P, _P, _I64, _P, _I, _I, _P, _P]),
    "cb_set_prefill_attention_tc": (_I, [_I]),
    "cb_host_copy": (_I, [_P, _P, _I64, _I]),
    "cb_read_file_ranges": (_I, [ctypes.c_char_p, _I, ctypes.POINTER(_I64), _PP, ctypes.POINTER(_I64), _I]),
    "cb_exchange_bytes": (_I64, []),
    "cb_exchange_alloc": (_I, [_PP]),
    "cb_exchange_free": (_I, [_P]),
    "cb_ipc_handle": (_I, [_P, _P]),
    "cb_ipc_open": (_I, [_P, _PP]),
    "cb_ipc_close": (_I, [_P]),
    "cb_set_exchange_wait_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "cb_proj_allreduce_residual": (_I, [_P, _I, _P, _I, _P, _P, _PP, _I, _I, _I, _I, _P, _P]),
    "cb_lm_head_topk_allgather": (
        _I, [_P, _P, _F, _P, _I64, _I64, _I, _P, _P, _P, _P, _PP, _I, _I, _I, _I, _P, _P]
    ),
    "cb_attention_workspace_bytes": (_I64, [_I, _I]),
    "cb_set_attention_cluster": (_I, [_I]),
    "cb_set_attention_min_chunk": (_I, [_I]),
    "cb_set_gemm_workspace": (_I, [_P, ctypes.c_int64, _P, _I]),
    "cb_gemm_split_k": (_I, [_I, _I, _I, _I]),
    "cb_attention": (_I, [_P, _P, _P, _I64, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "cb_attention_noalloc": (_I, [_P, _P, _P, _I64, _P, _I, _I, _I, _P, _P]),
    "cb_attention_oproj_max_splits": (_I, []),
    "cb_attention_oproj": (_I, [_P, _P, _P, _I64, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "cb_memcpy_h2d_async": (_I, [_P, _P, _I64, _P]),
    "cb_host_gather_rows": (_I, [_P, _P, _I64, _I64, _P, _I64]),
    "cb_ring_create": (_I, [_I, _PP, _I64, _P, _PP, _I64, _I, _PP]),
    "cb_ring_destroy": (_I, [_P]),
    "cb_ring_begin": (_I, [_P, _I, _PP, ctypes.POINTER(_I64), _P, _P, _I]),
    "cb_ring_acquire": (_I, [_P, _I, _PP]),
    "cb_ring_release": (_I, [_P, _I]),
    "cb_ring_end": (_I, [_P, _I, ctypes.POINTER(ctypes.c_double)]),
    "cb_ring_abort": (_I, [_P]),
}


def exported_symbols():
    """Names every header declaration maps to (used by the ABI tests)."""

    return sorted(_SIGNATURES)


def load_library(path=LIB_PATH):
    """dlopen the library and bind every entry point (no GPU needed)."""

    if not os.path.exists(path):
        raise RuntimeError(
            "libcascade_b200.so not found at {} - build it with "
            "`make -C cascade-llm_b200/csrc` (or __graft_entry__.build())".format(path)
        )
    handle = ctypes.CDLL(path)
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            _LIB = load_library()
    return _LIB


def check(code, what):
    if code != 0:
        message = lib().cb_last_error().decode(errors="replace")
        raise RuntimeError("{} failed (status {}): {}".format(what, code, message))


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def ptr(tensor, dtype=None, name="tensor"):
    """Device pointer of a contiguous CUDA tensor (None -> NULL)."""

    if tensor is None:
        return None
    if tensor.device.type != "cuda":
        raise RuntimeError("{} must be a CUDA tensor (got {})".format(name, tensor.device))
    if dtype is not None and tensor.dtype != dtype:
        raise TypeError("{} must be {} (got {})".format(name, dtype, tensor.dtype))
    if not tensor.is_contiguous():
        raise ValueError("{} must be contiguous".format(name))
    return tensor.data_ptr()


def stream_key(seed, name):
    return int(lib().cb_stream_key(int(seed) & (2**64 - 1), name.encode()))
