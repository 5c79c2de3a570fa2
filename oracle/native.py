"""ctypes access to the oracle's C restatements (test infrastructure only).

``oracle/seeded_init.c`` restates the engine's seeded weight initialiser and
``oracle/topk_merge.c`` the exact top-k of ``layer_streaming/vocab.py:11-32``.
The library is built by ``make -C oracle`` (``__graft_entry__.build()`` does
it); :func:`lib` builds it on first use when a C compiler is present.
"""

import ctypes
import os
import subprocess
import threading

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_LOCK = threading.Lock()
_LIB = None


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(_LIB_PATH):
                build()
            handle = ctypes.CDLL(_LIB_PATH)
            handle.oracle_fnv1a64.restype = ctypes.c_uint64
            handle.oracle_fnv1a64.argtypes = [ctypes.c_char_p]
            handle.oracle_stream_key.restype = ctypes.c_uint64
            handle.oracle_stream_key.argtypes = [ctypes.c_uint64, ctypes.c_char_p]
            handle.oracle_fill_normal_bf16.restype = None
            handle.oracle_fill_normal_bf16.argtypes = [
                ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                ctypes.c_uint64, ctypes.c_double,
            ]
            handle.oracle_uniform_ids.restype = None
            handle.oracle_uniform_ids.argtypes = [
                ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
            ]
            handle.oracle_topk.restype = None
            handle.oracle_topk.argtypes = [
                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                ctypes.c_void_p, ctypes.c_void_p,
            ]
            _LIB = handle
    return _LIB


def stream_key(seed, name):
    return int(lib().oracle_stream_key(int(seed) & (2**64 - 1), name.encode()))


def fill_normal_bf16(out, key, std=0.02, offset=0):
    """Fill a contiguous CPU bf16 tensor with elements [offset, offset+n)."""

    if out.device.type != "cpu" or out.dtype != torch.bfloat16:
        raise TypeError("oracle fill needs a CPU bf16 tensor")
    if not out.is_contiguous():
        raise ValueError("oracle fill needs a contiguous tensor")
    n = out.numel()
    handle = lib()
    base = out.data_ptr()
    workers = max(1, min(os.cpu_count() or 1, n // (1 << 20)))
    if workers == 1:
        handle.oracle_fill_normal_bf16(base, n, int(offset), int(key), float(std))
        return out
    step = (n + workers - 1) // workers
    step += step & 1

    def run(start):
        count = min(step, n - start)
        handle.oracle_fill_normal_bf16(
            base + 2 * start, count, int(offset) + start, int(key), float(std)
        )

    threads = [
        threading.Thread(target=run, args=(start,))
        for start in range(0, n, step)
    ]
    for thread in threads:
        thread.start()
    for thread in threads:
        thread.join()
    return out


def uniform_ids(count, key, bound):
    out = np.empty(int(count), dtype=np.int64)
    lib().oracle_uniform_ids(out.ctypes.data, out.size, int(key), int(bound))
    return torch.from_numpy(out)


def topk(values, k, indices=None):
    """Exact top-k, ties broken by smaller index (values: 1-D fp32)."""

    v = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
    idx = None
    if indices is not None:
        idx = np.ascontiguousarray(np.asarray(indices, dtype=np.int64).reshape(-1))
    k = int(min(k, v.size))
    out_v = np.empty(k, dtype=np.float32)
    out_i = np.empty(k, dtype=np.int64)
    lib().oracle_topk(
        v.ctypes.data, None if idx is None else idx.ctypes.data, v.size, k,
        out_v.ctypes.data, out_i.ctypes.data,
    )
    return out_v, out_i
