"""The allocation-free attention entry point (cb_attention_noalloc).

It serves callers that cannot allocate device memory themselves, such as a
host framework that owns the whole GPU memory budget, or a latency-critical
loop where cudaMalloc would synchronise the device. Its scratch is a fixed
static device array inside the library, so the test drives it through the
C ABI exactly like such a caller would (raw pointers, no workspace) and
compares every output with the workspace-taking cb_attention on the same
inputs, over consecutive calls that reuse the shared scratch. This file is
collected last so that a run stopping at the first failure has already run
every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


def _rand(shape, seed, device):
    gen = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(shape, generator=gen, device=device).to(BF16)


def _reference(lib, q, kc, vc, pos, tokens, splits, chunk, stream):
    out = torch.empty((tokens, 4096), dtype=BF16, device=q.device)
    workspace = torch.empty(lib.cb_attention_workspace_bytes(tokens, splits), dtype=torch.uint8, device=q.device)
    tickets = torch.zeros(8 * tokens, dtype=torch.int32, device=q.device)
    rc = lib.cb_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[1], pos.data_ptr(), tokens,
                          8, splits, chunk, out.data_ptr(), workspace.data_ptr(), tickets.data_ptr(), stream)
    assert rc == 0, lib.cb_last_error()
    return out


def test_noalloc_attention_matches_workspace_entry_point(cuda):
    from layer_streaming import _native

    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    length = 2048
    kc = _rand((8, length + 64, 128), 1, cuda)
    vc = _rand((8, length + 64, 128), 2, cuda)
    calls = [  # (tokens, first position, splits, chunk)
        (1, length - 1, 32, 64),     # one decode token at a 2K context
        (4, length - 4, 3, 704),     # a short causal chunk, other shape
        (1, length - 1, 32, 64),     # the first call again, after the scratch changed
    ]
    for index, (tokens, start, splits, chunk) in enumerate(calls):
        q = _rand((tokens, 4096), 10 + index, cuda)
        pos = torch.tensor([start], dtype=torch.int32, device=cuda)
        out = torch.full((tokens, 4096), float("nan"), dtype=BF16, device=cuda)
        rc = lib.cb_attention_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[1], pos.data_ptr(),
                                      tokens, splits, chunk, out.data_ptr(), stream)
        assert rc == 0, lib.cb_last_error()
        ref = _reference(lib, q, kc, vc, pos, tokens, splits, chunk, stream)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
        assert torch.equal(out, ref)  # same kernel and split order: identical bits


def test_noalloc_attention_rejects_requests_beyond_its_scratch(cuda):
    from layer_streaming import _native

    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    dummy = torch.zeros(16, dtype=BF16, device=cuda)
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    p = dummy.data_ptr()
    assert lib.cb_attention_noalloc(p, p, p, 1, pos.data_ptr(), 257, 1, 64, p, stream) != 0
    assert b"fixed scratch" in lib.cb_last_error()
    assert lib.cb_attention_noalloc(p, p, p, 1, pos.data_ptr(), 1, 300, 64, p, stream) != 0
    assert b"fixed scratch" in lib.cb_last_error()
    torch.cuda.synchronize()
