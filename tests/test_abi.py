"""The C-ABI library: it loads without a GPU and exports exactly what
include/cascade_b200.h declares; the Python binding covers every entry."""

import ctypes
import os
import re

import pytest

from conftest import REPO
from layer_streaming import _native

HEADER = os.path.join(REPO, "include", "cascade_b200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cb_[a-z0-9_]+)\s*\(", text)))


def test_header_declarations_are_all_bound():
    assert declared() == _native.exported_symbols()


def test_library_loads_and_exports_every_symbol():
    handle = _native.load_library()
    for name in declared():
        assert hasattr(handle, name), name
    assert handle.cb_version() == 100
    assert isinstance(handle.cb_last_error(), bytes)  # "" until a call fails on this thread


def test_stream_key_matches_oracle():
    from oracle import native

    handle = _native.load_library()
    for seed, name in [(0, "lm_head.weight"), (7, "model.layers.3.mlp.up_proj.weight"), (2**63, "")]:
        assert handle.cb_stream_key(seed, name.encode()) == native.stream_key(seed, name)


def test_invalid_arguments_fail_before_any_launch():
    handle = _native.load_library()
    # null pointers are rejected on the host: nothing reaches the GPU
    assert handle.cb_qkv_rope(None, None, 1e-5, None, None, None, None, None, 0, None, None, None, 0, 32, 8, None) != 0
    assert b"x must be" in handle.cb_last_error()
    assert handle.cb_attention(None, None, None, 0, None, 1, 8, 1, 64, None, None, None, None) != 0
    assert handle.cb_topk_merge(None, None, 0, None, None, 0, 10, None, None, None) != 0
    assert handle.cb_lm_head_topk(None, None, 0.0, None, 0, 0, 10, None, None, None, None, None, None) != 0


def test_ops_refuse_cpu_tensors():
    import torch
    from layer_streaming import ops  # noqa: F401 (registers torch.ops.cascade)

    x = torch.zeros(4096, dtype=torch.bfloat16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.cascade.rmsnorm(x, x, 1e-5, x)
