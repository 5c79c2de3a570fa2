"""Kernel-level parity on the GPU: every cascade kernel against the oracle's
restatement of the reference op (torch ops on the same device, same inputs).

Tolerances: projections are bf16 outputs of fp32 dot products whose
summation order differs from cuBLAS, so an output may sit one bf16 ulp away
(|d| <= 2^-8 |x|): rtol 1e-2 / atol 1e-2 with the mismatch fraction bounded.
Selection (top-k, merge) and data movement (embedding, cache writes, seeded
init) are bit-exact.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import llama_oracle as lo
from oracle import native

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def ops(cuda):
    from layer_streaming import ops as cascade_ops
    from layer_streaming import _native

    _native.check(_native.lib().cb_prepare(), "cb_prepare")
    return cascade_ops


def randn(shape, seed, std=1.0, device="cuda:0"):
    gen = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=gen, device=device) * std).to(BF16)


def assert_bf16_close(got, ref, frac=0.02, rtol=1e-2, atol=1e-2):
    got, ref = got.float(), ref.float()
    torch.testing.assert_close(got, ref, rtol=rtol, atol=atol)
    differ = (got != ref).float().mean().item()
    assert differ <= frac, "{:.4f} of outputs differ (> {})".format(differ, frac)


def test_fill_normal_matches_cpu_oracle(ops, cuda):
    key = native.stream_key(0, "model.layers.0.mlp.gate_proj.weight")
    n, offset = 8_000_003, 12345
    gpu = torch.empty(n, dtype=BF16, device=cuda)
    ops.fill_normal_(gpu, key, std=0.02, offset=offset)
    cpu = torch.empty(n, dtype=BF16)
    native.fill_normal_bf16(cpu, key, std=0.02, offset=offset)
    mismatches = int((gpu.cpu().view(torch.int16) != cpu.view(torch.int16)).sum())
    assert mismatches == 0


def test_embedding_gather_and_bad_id_reporting(ops, cuda):
    from layer_streaming import _native

    table = randn((1000, 4096), 1)
    ids = torch.tensor([3, 999, 0, 3, 512], device=cuda)
    out = torch.empty((5, 4096), dtype=BF16, device=cuda)
    ops.embedding(ids, table, out)
    assert torch.equal(out, table[ids])
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _native.lib().cb_set_error_word(err.data_ptr())
    try:
        ops.embedding(torch.tensor([1000], device=cuda), table, out[:1])
        torch.cuda.synchronize()
        assert int(err.item()) == 301  # reported, row 0 used, no fault
        assert torch.equal(out[0], table[0])
    finally:
        _native.lib().cb_set_error_word(None)


def test_rmsnorm(ops, cuda):
    x = randn((3, 4096), 2)
    w = (randn((4096,), 3, std=0.1).float() + 1).to(BF16)
    out = torch.empty_like(x)
    ops.rmsnorm(x, w, 1e-5, out)
    assert_bf16_close(out, lo.rms_norm(x, w), frac=0.01)


def _qkv_reference(x, norm_w, wq, wk, wv, position):
    normed = lo.rms_norm(x.view(1, 1, -1), norm_w)
    q = F.linear(normed, wq).view(1, 1, 32, 128).transpose(1, 2)
    k = F.linear(normed, wk).view(1, 1, 8, 128).transpose(1, 2)
    v = F.linear(normed, wv).view(1, 1, 8, 128).transpose(1, 2)
    cos, sin = lo.rope_cos_sin(torch.tensor([[position]], device=x.device), lo.llama3_inv_freq(device=x.device))
    q, k = lo.apply_rope(q, k, cos, sin)
    return q.reshape(4096), k.reshape(8, 128), v.reshape(8, 128)


@pytest.mark.parametrize("position", [0, 37, 5000])
def test_qkv_rope_matches_reference(ops, cuda, position):
    x = randn((4096,), 10 + position)
    norm_w = (randn((4096,), 11, std=0.1).float() + 1).to(BF16)
    wq, wk, wv = randn((4096, 4096), 12, 0.02), randn((1024, 4096), 13, 0.02), randn((1024, 4096), 14, 0.02)
    inv = lo.llama3_inv_freq(device=cuda)
    length = position + 3
    kc = torch.full((8, length, 128), 7.0, dtype=BF16, device=cuda)
    vc = torch.full((8, length, 128), 7.0, dtype=BF16, device=cuda)
    pos = torch.tensor([position], dtype=torch.int32, device=cuda)
    q = torch.empty(4096, dtype=BF16, device=cuda)
    ops.qkv_rope(x, norm_w, 1e-5, wq, wk, wv, inv, pos, 0, q, kc, vc)
    rq, rk, rv = _qkv_reference(x, norm_w, wq, wk, wv, position)
    assert_bf16_close(q, rq)
    assert_bf16_close(kc[:, position], rk)
    assert_bf16_close(vc[:, position], rv)
    untouched = torch.cat([kc[:, :position], kc[:, position + 1:], vc[:, :position], vc[:, position + 1:]], dim=1)
    assert bool((untouched == 7.0).all())
    # matrix granularity: q, k and v as separate units give the same bits
    q2 = torch.empty_like(q)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    ops.qkv_rope(x, norm_w, 1e-5, wq, None, None, inv, pos, 0, q2, None, None)
    ops.qkv_rope(x, norm_w, 1e-5, None, wk, None, inv, pos, 0, None, kc2, None)
    ops.qkv_rope(x, norm_w, 1e-5, None, None, wv, inv, pos, 0, None, None, vc2)
    assert torch.equal(q2, q)
    assert torch.equal(kc2[:, position], kc[:, position])
    assert torch.equal(vc2[:, position], vc[:, position])


@pytest.mark.parametrize("k_dim", [4096, 14336])
def test_proj_residual(ops, cuda, k_dim):
    x = randn((k_dim,), 20)
    w = randn((4096, k_dim), 21, 0.02)
    res = randn((4096,), 22)
    out = torch.empty_like(res)
    ops.proj_residual(x, w, res, out)
    assert_bf16_close(out, res + F.linear(x.view(1, -1), w).view(-1))
    # in place (out aliases the residual), as the executor uses it
    res2 = res.clone()
    ops.proj_residual(x, w, res2, res2)
    assert torch.equal(res2, out)


def test_gate_up_swiglu_and_split_units(ops, cuda):
    x = randn((4096,), 30)
    norm_w = (randn((4096,), 31, std=0.1).float() + 1).to(BF16)
    wg, wu = randn((14336, 4096), 32, 0.02), randn((14336, 4096), 33, 0.02)
    out = torch.empty(14336, dtype=BF16, device=cuda)
    ops.gate_up_swiglu(x, norm_w, 1e-5, wg, wu, out)
    normed = lo.rms_norm(x.view(1, -1), norm_w)
    ref = (F.silu(F.linear(normed, wg)) * F.linear(normed, wu)).view(-1)
    assert_bf16_close(out, ref, frac=0.03)
    split = torch.empty_like(out)
    ops.gate_silu(x, norm_w, 1e-5, wg, split)
    assert_bf16_close(split, F.silu(F.linear(normed, wg)).view(-1))
    ops.up_mul(x, norm_w, 1e-5, wu, split)
    assert torch.equal(split, out)


def _topk_oracle(values, k):
    v, i = native.topk(values.detach().float().cpu().numpy(), k)
    return torch.from_numpy(v), torch.from_numpy(i)


@pytest.mark.parametrize("rows,offset,k", [(128256, 0, 10), (16384, 114688 - 16384, 10), (13568, 114688, 64), (2, 5, 1)])
def test_lm_head_topk(ops, cuda, rows, offset, k):
    x = randn((4096,), 40)
    norm_w = torch.ones(4096, dtype=BF16, device=cuda)
    w = randn((rows, 4096), 41, 0.02)
    logits = torch.empty(rows, dtype=torch.float32, device=cuda)
    values = torch.empty(k, dtype=torch.float32, device=cuda)
    indices = torch.empty(k, dtype=torch.int64, device=cuda)
    ws = torch.full((ops.lm_head_workspace_bytes(k),), 0xAB, dtype=torch.uint8, device=cuda)  # scratch
    ticket = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):  # the ticket is left zero for the next launch
        ops.lm_head_topk(x, norm_w, 1e-5, w, offset, k, logits, values, indices, ws, ticket)
        ref_logits = F.linear(lo.rms_norm(x.view(1, -1), norm_w), w).float().view(-1)
        assert_bf16_close(logits, ref_logits, frac=0.02, rtol=1e-2, atol=2e-2)
        # the selection is exact on the kernel's own logits
        ov, oi = _topk_oracle(logits, k)
        assert torch.equal(values.cpu(), ov)
        assert torch.equal(indices.cpu(), oi + offset)
    # without the logits output: same top-k
    v2, i2 = torch.empty_like(values), torch.empty_like(indices)
    ops.lm_head_topk(x, norm_w, 1e-5, w, offset, k, None, v2, i2, ws, ticket)
    assert torch.equal(v2, values) and torch.equal(i2, indices)
    assert int(ticket.item()) == 0


@pytest.mark.parametrize("patterns,k", [(1, 10), (1, 64), (3, 10), (7, 64)])
def test_lm_head_topk_massive_ties(ops, cuda, patterns, k):
    """A head whose rows repeat `patterns` distinct rows: every logit takes
    one of `patterns` values, so every CTA's candidate list ties with every
    other's and the selection rests on the row-id rule alone (smaller id
    first). Covers the merge that loads all candidates into registers (k=10)
    and the threshold-filter merge (k=64) under the ties that bf16 logits
    produce."""

    rows = 128256
    x = randn((4096,), 42)
    norm_w = torch.ones(4096, dtype=BF16, device=cuda)
    base = randn((patterns, 4096), 43, 0.02)
    w = base.repeat((rows + patterns - 1) // patterns, 1)[:rows].contiguous()
    logits = torch.empty(rows, dtype=torch.float32, device=cuda)
    values = torch.empty(k, dtype=torch.float32, device=cuda)
    indices = torch.empty(k, dtype=torch.int64, device=cuda)
    ws = torch.full((ops.lm_head_workspace_bytes(k),), 0xAB, dtype=torch.uint8, device=cuda)
    ticket = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):
        ops.lm_head_topk(x, norm_w, 1e-5, w, 0, k, logits, values, indices, ws, ticket)
        # identical rows give identical logits
        assert torch.equal(logits.view(-1, 1)[:patterns * (rows // patterns)].view(-1, patterns),
                           logits[:patterns].expand(rows // patterns, patterns))
        ov, oi = _topk_oracle(logits, k)
        assert torch.equal(values.cpu(), ov)
        assert torch.equal(indices.cpu(), oi)
    best = int(torch.argmax(logits[:patterns]).item()) if patterns > 1 else 0
    if int((logits[:patterns] == logits[best]).sum()) == 1:
        # one pattern holds the maximum: the k smallest ids of that pattern
        assert indices.cpu().tolist() == [best + patterns * i for i in range(k)]
    assert int(ticket.item()) == 0


def test_topk_merge_with_ties(ops, cuda):
    gen = torch.Generator().manual_seed(5)
    a_v = torch.randint(0, 20, (37,), generator=gen).float()
    b_v = torch.randint(0, 20, (300,), generator=gen).float()
    a_i = torch.randperm(5000, generator=gen)[:37]
    b_i = torch.randperm(5000, generator=gen)[:300] + 5000
    for k in (1, 10, 64):
        out_v = torch.empty(k, dtype=torch.float32, device=cuda)
        out_i = torch.empty(k, dtype=torch.int64, device=cuda)
        ops.topk_merge(a_v.to(cuda), a_i.to(cuda), b_v.to(cuda), b_i.to(cuda), k, out_v, out_i)
        ov, oi = native.topk(torch.cat([a_v, b_v]).numpy(), k, indices=torch.cat([a_i, b_i]).numpy())
        assert out_v.cpu().tolist() == ov.tolist()
        assert out_i.cpu().tolist() == oi.tolist()


def test_merge_topk_api_matches_reference_case(cuda):
    from layer_streaming.vocab import merge_topk

    logits = torch.tensor([[[-2.0, 7.0, 1.0, 3.0, 9.0, -1.0, 8.0, 4.0]]], device=cuda)
    values = indices = None
    for start in (0, 3, 6):
        part = logits[..., start:start + 3]
        lv, li = torch.topk(part, k=min(3, part.shape[-1]), dim=-1)
        values, indices = merge_topk(values, indices, lv, li + start, top_k=3)
    ev, ei = torch.topk(logits, k=3, dim=-1)
    assert torch.equal(values, ev) and torch.equal(indices, ei)


def _cache_with_rope(length, capacity, seed, device):
    """Config 1: K/V ~N(0,1) with RoPE applied at positions 0..L-1."""

    k = randn((1, 8, length, 128), seed)
    v = randn((1, 8, length, 128), seed + 1)
    cos, sin = lo.rope_cos_sin(torch.arange(length, device=device).unsqueeze(0), lo.llama3_inv_freq(device=device))
    _, k = lo.apply_rope(k, k, cos, sin)
    kc = torch.zeros((8, capacity, 128), dtype=BF16, device=device)
    vc = torch.zeros((8, capacity, 128), dtype=BF16, device=device)
    kc[:, :length] = k[0]
    vc[:, :length] = v[0]
    return kc, vc, k, v


def _attention_fp32(q, k, v, mask=None):
    """Upcast reference: fp32 scores, softmax and PV (q [1,32,M,128])."""

    k = k.float().repeat_interleave(4, dim=1)
    v = v.float().repeat_interleave(4, dim=1)
    s = q.float() @ k.transpose(-1, -2) / (128 ** 0.5)
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    return torch.softmax(s, dim=-1) @ v


@pytest.mark.parametrize("length", [1, 37, 2048, 8192, 32768])
def test_decode_attention_config1(ops, cuda, length):
    capacity = length + 64
    kc, vc, k, v = _cache_with_rope(length, capacity, 50, cuda)
    q = randn((1, 32, 1, 128), 52)
    pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda)
    sdpa = lo.attention(q, k, v, causal=False).view(4096)
    exact = _attention_fp32(q, k, v).transpose(1, 2).reshape(4096)
    from layer_streaming.llama31 import attention_split

    configs = {
        attention_split(1, length, torch.cuda.get_device_properties(0).multi_processor_count),
        (1, -(-length // 64) * 64),                 # one CTA per KV head
        (4, -(-length // 64) * 64),                 # three of four splits empty
    }
    for splits, chunk in sorted(configs):
        out = torch.empty(4096, dtype=BF16, device=cuda)
        ws = torch.full((ops.attention_workspace_bytes(1, splits),), 0xAB, dtype=torch.uint8, device=cuda)
        tickets = torch.zeros(8, dtype=torch.int32, device=cuda)
        for _ in range(2):  # tickets are reset for the next launch
            ops.attention(q.view(4096), kc, vc, pos, splits, chunk, out, ws, tickets)
            torch.testing.assert_close(out.float(), sdpa.float(), rtol=2e-2, atol=2e-2)
            # at least as close to the fp32 result as torch's bf16 SDPA is
            assert (out.float() - exact).abs().max() <= (sdpa.float() - exact).abs().max() + 4e-3
        assert int(tickets.abs().sum()) == 0


@pytest.mark.parametrize("start,tokens", [(0, 6), (100, 5), (0, 64)])
def test_causal_multi_token_attention(ops, cuda, start, tokens):
    length = start + tokens
    kc, vc, k, v = _cache_with_rope(length, length + 8, 60, cuda)
    q = randn((1, 32, tokens, 128), 62)
    pos = torch.tensor([start], dtype=torch.int32, device=cuda)
    qi = torch.arange(start, start + tokens, device=cuda).view(-1, 1)
    mask = torch.arange(length, device=cuda).view(1, -1) <= qi
    exact = _attention_fp32(q, k, v, mask).transpose(1, 2).reshape(tokens, 4096)
    if start == 0:
        ref = lo.attention(q, k, v, causal=True).view(tokens, 4096).float()
    else:
        ref = F.scaled_dot_product_attention(
            q, k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1), attn_mask=mask
        ).transpose(1, 2).reshape(tokens, 4096).float()
    out = torch.empty((tokens, 4096), dtype=BF16, device=cuda)
    splits, chunk = 2, max(64, -(-length // 128) * 64)
    ws = torch.full((ops.attention_workspace_bytes(tokens, splits),), 0xAB, dtype=torch.uint8, device=cuda)
    tickets = torch.zeros(8 * tokens, dtype=torch.int32, device=cuda)
    ops.attention(q.transpose(1, 2).contiguous().view(tokens, 4096), kc, vc, pos, splits, chunk, out, ws, tickets)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    assert (out.float() - exact).abs().max() <= (ref - exact).abs().max() + 4e-3


def test_position_counter(ops, cuda):
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.position_set(pos, None, 41)
    ops.position_advance(pos, 1)
    assert int(pos.item()) == 42
    ops.position_set(pos, torch.tensor([7], device=cuda), 0)
    ops.position_advance(pos, 6)
    assert int(pos.item()) == 13


def test_attention_scratch_reuse_across_shapes(ops, cuda):
    """One workspace and one ticket array serve a 6-token prefill and then
    one-token decode steps (the executor's pattern): the partials are pure
    scratch and the tickets come back zero after every launch."""

    length = 9
    kc, vc, k, v = _cache_with_rope(length, 64, 70, cuda)
    ws = torch.full((ops.attention_workspace_bytes(6, 3),), 0x7F, dtype=torch.uint8, device=cuda)
    tickets = torch.zeros(48, dtype=torch.int32, device=cuda)
    for start, tokens, splits in ((0, 6, 3), (6, 1, 1), (7, 1, 2), (8, 1, 1)):
        q = randn((1, 32, tokens, 128), 71 + start)
        pos = torch.tensor([start], dtype=torch.int32, device=cuda)
        out = torch.empty((tokens, 4096), dtype=BF16, device=cuda)
        ops.attention(q.transpose(1, 2).contiguous().view(tokens, 4096), kc, vc, pos, splits, 64, out, ws, tickets)
        qi = torch.arange(start, start + tokens, device=cuda).view(-1, 1)
        mask = torch.arange(start + tokens, device=cuda).view(1, -1) <= qi
        exact = _attention_fp32(q, k[:, :, :start + tokens], v[:, :, :start + tokens], mask)
        torch.testing.assert_close(out.float(), exact.transpose(1, 2).reshape(tokens, 4096), rtol=2e-2, atol=2e-2)
        assert int(tickets.abs().sum()) == 0


def test_attention_with_too_few_splits_reports_code_204(ops, cuda):
    """The step position lives on the device, so the host cannot check that
    splits x chunk covers it: the kernel records code 204 instead of leaving
    the tail out silently, and a covering launch afterwards is clean."""

    from layer_streaming import _native

    length = 300
    kc, vc, k, v = _cache_with_rope(length, length + 64, 60, cuda)
    q = randn((1, 32, 1, 128), 61).view(4096)
    pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib = _native.lib()
    lib.cb_set_error_word(err.data_ptr())
    try:
        out = torch.empty(4096, dtype=BF16, device=cuda)
        splits, chunk = 2, 128  # covers 256 of the 300 visible positions
        ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
        tickets = torch.zeros(8, dtype=torch.int32, device=cuda)
        ops.attention(q, kc, vc, pos, splits, chunk, out, ws, tickets)
        torch.cuda.synchronize()
        assert int(err.item()) == 204
        assert int(tickets.abs().sum()) == 0
        err.zero_()
        splits, chunk = 3, 128
        ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
        ops.attention(q, kc, vc, pos, splits, chunk, out, ws, tickets)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        sdpa = lo.attention(q.view(1, 32, 1, 128), k, v, causal=False).view(4096)
        torch.testing.assert_close(out.float(), sdpa.float(), rtol=2e-2, atol=2e-2)
    finally:
        lib.cb_set_error_word(None)


@pytest.mark.parametrize("length", [1, 37, 300, 2048, 5000, 8192])
def test_adaptive_split_chunks(ops, cuda, length):
    """chunk = 0: the kernel sizes the splits from the device position, so one
    launch configuration serves every length (SDPA tolerance, tickets zero)."""

    kc, vc, k, v = _cache_with_rope(length, length + 64, 70, cuda)
    q = randn((1, 32, 1, 128), 71)
    pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda)
    sdpa = lo.attention(q, k, v, causal=False).view(4096)
    for splits in (1, 16, 37):
        out = torch.empty(4096, dtype=BF16, device=cuda)
        ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
        tickets = torch.zeros(8, dtype=torch.int32, device=cuda)
        ops.attention(q.view(4096), kc, vc, pos, splits, 0, out, ws, tickets)
        torch.testing.assert_close(out.float(), sdpa.float(), rtol=2e-2, atol=2e-2)
        assert int(tickets.abs().sum()) == 0


@pytest.mark.parametrize("length", [1, 37, 300, 2048, 8192])
def test_fused_attention_oproj_equals_separate_kernels(ops, cuda, length):
    """cb_attention_oproj == cb_attention (chunk 0) + cb_proj_residual, bit
    for bit, on two launches in a row (the counters return to zero)."""

    from layer_streaming import _native

    kc, vc, k, v = _cache_with_rope(length, length + 64, 80, cuda)
    q = randn((1, 32, 1, 128), 81).view(4096)
    wo = randn((4096, 4096), 82, 0.02)
    x = randn((4096,), 83)
    pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib = _native.lib()
    lib.cb_set_error_word(err.data_ptr())
    try:
        for splits in sorted({1, 8, 16, ops.attention_oproj_max_splits()}):
            ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
            tickets = torch.zeros(16, dtype=torch.int32, device=cuda)
            attn_ref = torch.empty(4096, dtype=BF16, device=cuda)
            ops.attention(q, kc, vc, pos, splits, 0, attn_ref, ws, tickets)
            want = torch.empty(4096, dtype=BF16, device=cuda)
            ops.proj_residual(attn_ref, wo, x, want)
            for _ in range(2):
                attn = torch.empty(4096, dtype=BF16, device=cuda)
                out = x.clone()
                ops.attention_oproj(q, kc, vc, pos, splits, wo, out, attn, out, ws, tickets)
                torch.cuda.synchronize()
                assert torch.equal(attn, attn_ref), splits
                assert torch.equal(out, want), splits
                assert int(tickets.abs().sum()) == 0
            assert int(err.item()) == 0
    finally:
        lib.cb_set_error_word(None)


@pytest.mark.parametrize("length", [1, 37, 300, 2048])
def test_cluster_merge_equals_global_merge(ops, cuda, length):
    """One-token launches with splits <= 16 merge inside a thread-block
    cluster (distributed shared memory); the outputs are bit-identical to the
    global-memory merge and within SDPA tolerance."""

    from layer_streaming import _native

    lib = _native.lib()
    kc, vc, k, v = _cache_with_rope(length, length + 64, 90, cuda)
    q = randn((1, 32, 1, 128), 91).view(4096)
    pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda)
    sdpa = lo.attention(q.view(1, 32, 1, 128), k, v, causal=False).view(4096)
    previous = lib.cb_set_attention_cluster(1)
    try:
        for splits in (1, 4, 16):
            outs = []
            for cluster in (0, 1):
                lib.cb_set_attention_cluster(cluster)
                out = torch.empty(4096, dtype=BF16, device=cuda)
                ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
                tickets = torch.zeros(8, dtype=torch.int32, device=cuda)
                ops.attention(q, kc, vc, pos, splits, 0, out, ws, tickets)
                torch.cuda.synchronize()
                assert int(tickets.abs().sum()) == 0
                outs.append(out)
            assert torch.equal(outs[0], outs[1]), splits
            torch.testing.assert_close(outs[1].float(), sdpa.float(), rtol=2e-2, atol=2e-2)
    finally:
        lib.cb_set_attention_cluster(previous)
