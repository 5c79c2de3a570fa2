"""Prefill GEMMs on the tcgen05 tensor cores against torch and the decode path.

The GEMM accumulates in fp32 in a different order than cuBLAS, so a bf16
output may sit one ulp away; each case is held to rtol/atol 1e-2 of the torch
op with the mismatch fraction bounded, and to be at least as close to the
fp64 result as torch's own bf16 output (plus one bf16 ulp of slack). The fused
epilogues (residual, SwiGLU, RoPE + KV-cache write) are checked against the
decode GEMV kernels, which share their rounding points.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import llama_oracle as lo

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def ops(cuda):
    from layer_streaming import _native
    from layer_streaming import ops as cascade_ops

    _native.check(_native.lib().cb_prepare(), "cb_prepare")
    return cascade_ops


def randn(shape, seed, std=1.0, device="cuda:0"):
    gen = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=gen, device=device) * std).to(BF16)


def close_to_torch(got, a, w, extra=None):
    ref = F.linear(a, w)
    exact = a.double() @ w.double().T
    if extra is not None:
        ref = (extra.float() + ref.float()).to(BF16)
        exact = extra.double() + exact
    torch.testing.assert_close(got.float(), ref.float(), rtol=1e-2, atol=1e-2)
    assert (got.float() != ref.float()).float().mean().item() <= 0.05
    ulp = exact.abs().max().item() * 2.0 ** -8
    assert (got.double() - exact).abs().max().item() <= (ref.double() - exact).abs().max().item() + ulp


@pytest.mark.parametrize("m,k,n", [(128, 4096, 4096), (6, 4096, 6144), (200, 4096, 256), (512, 14336, 4096),
                                   (64, 512, 4096), (300, 1792, 128)])
def test_gemm_bf16_matches_torch(ops, cuda, m, k, n):
    a = randn((m, k), 1000 + m, 1.0)
    w = randn((n, k), 1001 + n, 0.02)
    out = torch.full((m, n), 7.0, dtype=BF16, device=cuda)
    ops.gemm_bf16(a, w, out)
    torch.cuda.synchronize()
    close_to_torch(out, a, w)


@pytest.mark.parametrize("m,k", [(64, 4096), (512, 14336), (77, 2048)])
def test_gemm_residual_matches_torch(ops, cuda, m, k):
    a = randn((m, k), 1100 + m, 1.0)
    w = randn((4096, k), 1101, 0.02)
    res = randn((m, 4096), 1102, 1.0)
    out = torch.empty_like(res)
    ops.gemm_residual(a, w, res, out)
    close_to_torch(out, a, w, extra=res)
    # in place, as the prefill path uses it
    res2 = res.clone()
    ops.gemm_residual(a, w, res2, res2)
    assert torch.equal(res2, out)


@pytest.mark.parametrize("m,k", [(64, 512), (300, 14336)])
def test_gemm_partial_is_the_unrounded_sum(ops, cuda, m, k):
    a = randn((m, k), 1150 + m, 1.0)
    w = randn((4096, k), 1151, 0.02)
    part = torch.empty((m, 4096), dtype=torch.float32, device=cuda)
    ops.gemm_partial(a, w, part)
    exact = a.double() @ w.double().T
    bound = 1e-6 * k ** 0.5 * (a.double().abs() @ w.double().abs().T) + 1e-6
    assert bool(((part.double() - exact).abs() <= 8 * bound).all())
    # rounded, it is the plain GEMM's output
    out = torch.empty((m, 4096), dtype=BF16, device=cuda)
    ops.gemm_bf16(a, w, out)
    assert torch.equal(part.to(BF16), out)


@pytest.mark.parametrize("m,rows", [(128, 14336), (33, 1792)])
def test_gemm_swiglu_matches_decode_kernel(ops, cuda, m, rows):
    a = randn((m, 4096), 1200 + m, 1.0)
    wg, wu = randn((rows, 4096), 1201, 0.02), randn((rows, 4096), 1202, 0.02)
    out = torch.empty((m, rows), dtype=BF16, device=cuda)
    ops.gemm_swiglu(a, wg, wu, out)
    ref = (F.silu(F.linear(a, wg)) * F.linear(a, wu)).float()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    # the decode kernel on each row (no norm): same rounding points; silu(bf16(g)) * bf16(u)
    # compounds a one-ulp difference of either factor, so two ulps (2e-2) apart at most
    per_row = torch.empty_like(out)
    for i in range(m):
        ops.gate_up_swiglu(a[i], None, 1e-5, wg, wu, per_row[i])
    torch.testing.assert_close(out.float(), per_row.float(), rtol=2e-2, atol=2e-2)
    assert (out != per_row).float().mean().item() <= 0.05


def test_split_swiglu_and_single_matrix_qkv_equal_the_fused_gemms(ops, cuda):
    """The `matrix` granularity's separate units give the fused kernels' bits."""

    m = 70
    a = randn((m, 4096), 1250, 1.0)
    wg, wu = randn((14336, 4096), 1251, 0.02), randn((14336, 4096), 1252, 0.02)
    fused = torch.empty((m, 14336), dtype=BF16, device=cuda)
    ops.gemm_swiglu(a, wg, wu, fused)
    split = torch.empty_like(fused)
    ops.gemm_silu(a, wg, split)
    ops.gemm_mul(a, wu, split)
    assert torch.equal(split, fused)
    wq, wk, wv = randn((4096, 4096), 1253, 0.02), randn((1024, 4096), 1254, 0.02), randn((1024, 4096), 1255, 0.02)
    inv = lo.llama3_inv_freq(device=cuda)
    pos = torch.tensor([11], dtype=torch.int32, device=cuda)
    q = torch.empty((m, 4096), dtype=BF16, device=cuda)
    kc = torch.zeros((8, 100, 128), dtype=BF16, device=cuda)
    vc = torch.zeros_like(kc)
    ops.prefill_qkv_rope(a, wq, wk, wv, inv, pos, q, kc, vc)
    q2, kc2, vc2 = torch.empty_like(q), torch.zeros_like(kc), torch.zeros_like(vc)
    ops.prefill_qkv_rope(a, wq, None, None, inv, pos, q2, None, None)
    ops.prefill_qkv_rope(a, None, wk, None, inv, pos, None, kc2, None)
    ops.prefill_qkv_rope(a, None, None, wv, inv, pos, None, None, vc2)
    assert torch.equal(q2, q) and torch.equal(kc2, kc) and torch.equal(vc2, vc)


@pytest.mark.parametrize("start,m,q_heads,kv_heads", [(0, 6, 32, 8), (100, 128, 32, 8), (7, 200, 8, 2),
                                                     (5, 1100, 32, 8)])
def test_prefill_qkv_rope_matches_decode_kernel(ops, cuda, start, m, q_heads, kv_heads):
    xn = randn((m, 4096), 1300 + m, 1.0)
    wq = randn((q_heads * 128, 4096), 1301, 0.02)
    wk = randn((kv_heads * 128, 4096), 1302, 0.02)
    wv = randn((kv_heads * 128, 4096), 1303, 0.02)
    inv = lo.llama3_inv_freq(device=cuda)
    cap = start + m + 5
    pos = torch.tensor([start], dtype=torch.int32, device=cuda)
    q = torch.empty((m, q_heads * 128), dtype=BF16, device=cuda)
    kc = torch.full((kv_heads, cap, 128), 7.0, dtype=BF16, device=cuda)
    vc = torch.full_like(kc, 7.0)
    ops.prefill_qkv_rope(xn, wq, wk, wv, inv, pos, q, kc, vc, q_heads, kv_heads)
    # the decode kernel, token by token (no norm: xn is already normalised)
    q2 = torch.empty_like(q)
    kc2 = torch.full_like(kc, 7.0)
    vc2 = torch.full_like(kc, 7.0)
    for i in range(m):
        ops.qkv_rope(xn[i], None, 1e-5, wq, wk, wv, inv, pos, i, q2[i], kc2, vc2, q_heads, kv_heads)
    torch.cuda.synchronize()
    # RoPE subtracts two rounded products: a one-ulp difference of the projection
    # (|q| ~ 2-4, ulp 1/64) can survive the cancellation, so the absolute bound is
    # the projection's ulp rather than the output's
    for got, ref in ((q, q2), (kc, kc2), (vc, vc2)):
        torch.testing.assert_close(got.float(), ref.float(), rtol=1e-2, atol=2e-2)
        assert (got != ref).float().mean().item() <= 0.05
    # nothing outside the step's positions was written
    outside = torch.cat([kc[:, :start], kc[:, start + m:], vc[:, :start], vc[:, start + m:]], dim=1)
    assert bool((outside == 7.0).all())


def _causal_reference(q, k, v, start):
    """fp32 causal GQA attention: q [1, H, M, 128], k/v [1, KV, L, 128]; query
    t sits at position start + t."""

    groups = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(groups, dim=1)
    vf = v.float().repeat_interleave(groups, dim=1)
    m, length = q.shape[2], k.shape[2]
    s = q.float() @ kf.transpose(-1, -2) / (128 ** 0.5)
    qi = torch.arange(start, start + m, device=q.device).view(-1, 1)
    mask = torch.arange(length, device=q.device).view(1, -1) <= qi
    s = s.masked_fill(~mask, float("-inf"))
    return torch.softmax(s, dim=-1) @ vf


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("start,m,kv_heads", [(0, 6, 8), (0, 64, 8), (100, 5, 8), (37, 200, 2), (1000, 130, 1),
                                              (0, 512, 8), (5, 33, 8), (4000, 512, 8), (130, 1, 4)])
def test_prefill_attention_matches_causal_reference(ops, cuda, start, m, kv_heads, tc):
    """Both prefill attention kernels (tcgen05 with S and O in TMEM, and the
    mma.sync one) against causal SDPA and the fp32 result; cache rows past
    the chunk hold NaN (never written), which must not reach the output."""

    from layer_streaming import _native

    previous = _native.lib().cb_set_prefill_attention_tc(tc)
    try:
        _prefill_attention_case(ops, cuda, start, m, kv_heads)
    finally:
        _native.lib().cb_set_prefill_attention_tc(previous)


@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
def test_prefill_attention_maximum_jumps_in_a_later_tile(ops, cuda, tc):
    """One key in a later 128-position tile aligned with one query row: that
    row's running maximum jumps (O rescaled for it alone), its neighbours'
    does not."""

    from layer_streaming import _native

    previous = _native.lib().cb_set_prefill_attention_tc(tc)
    try:
        _prefill_attention_case(ops, cuda, 300, 40, 8, spike=True)
    finally:
        _native.lib().cb_set_prefill_attention_tc(previous)


def _prefill_attention_case(ops, cuda, start, m, kv_heads, spike=False):
    length = start + m
    cap = length + 37
    k = randn((1, kv_heads, length, 128), 1400 + m)
    v = randn((1, kv_heads, length, 128), 1401 + m)
    q = randn((1, 4 * kv_heads, m, 128), 1402 + m)
    if spike:  # key 200 (tile 1) of KV head 0 = 3 x the query of token 5, head 1
        k[0, 0, 200] = (3 * q[0, 1, 5].float()).to(BF16)
    kc = torch.full((kv_heads, cap, 128), float("nan"), dtype=BF16, device=cuda)  # past the end: never read
    vc = torch.full_like(kc, float("nan"))
    kc[:, :length] = k[0]
    vc[:, :length] = v[0]
    pos = torch.tensor([start], dtype=torch.int32, device=cuda)
    out = torch.empty((m, 4 * kv_heads * 128), dtype=BF16, device=cuda)
    ops.prefill_attention(q[0].transpose(0, 1).contiguous().view(m, -1), kc, vc, pos, out)
    exact = _causal_reference(q, k, v, start)[0].transpose(0, 1).reshape(m, -1)
    sdpa = F.scaled_dot_product_attention(
        q, k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1),
        attn_mask=(torch.arange(length, device=cuda).view(1, -1)
                   <= torch.arange(start, length, device=cuda).view(-1, 1)))[0].transpose(0, 1).reshape(m, -1)
    assert bool(torch.isfinite(out.float()).all())
    torch.testing.assert_close(out.float(), sdpa.float(), rtol=2e-2, atol=2e-2)
    # P is rounded to bf16 before PV (as the reference's bf16 SDPA does): within
    # the bf16 SDPA's own distance from the fp32 result, plus a bf16 ulp
    assert (out.float() - exact).abs().max() <= (sdpa.float() - exact).abs().max() + 1e-2
    # and the split-KV decode kernel on the same step agrees
    ws = torch.empty(ops.attention_workspace_bytes(m, 1), dtype=torch.uint8, device=cuda)
    tickets = torch.zeros(kv_heads * m, dtype=torch.int32, device=cuda)
    ref = torch.empty_like(out)
    ops.attention(q[0].transpose(0, 1).contiguous().view(m, -1), kc, vc, pos, 1, -(-length // 64) * 64, ref, ws,
                  tickets)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.fixture
def split_k(ops, cuda):
    """Registers a split-K workspace for the test (and unregisters it)."""

    from layer_streaming import _native

    lib = _native.lib()
    ws = torch.empty(48 << 18, dtype=torch.float32, device=cuda)  # 48 MB
    tickets = torch.zeros(1024, dtype=torch.int32, device=cuda)
    _native.check(lib.cb_set_gemm_workspace(ws.data_ptr(), 48 << 20, tickets.data_ptr(), 1024), "workspace")
    try:
        yield lib, tickets
    finally:
        lib.cb_set_gemm_workspace(None, 0, None, 0)


def _unsplit(lib, fn):
    lib.cb_set_gemm_workspace(None, 0, None, 0)
    fn()


@pytest.mark.parametrize("m", [1, 6, 16, 64])
def test_split_k_gemms_match_unsplit_and_torch(ops, cuda, split_k, m):
    """Short chunks split each tile's K range over several CTAs; the last CTA
    sums the fp32 slices in slice order and runs the same epilogue. The
    outputs stay within one bf16 ulp of the unsplit kernel (a different fp32
    summation order) and meet the torch criteria; the tickets return to 0."""

    from layer_streaming import _native

    lib, tickets = split_k
    a = randn((m, 4096), 1500 + m, 1.0)
    wo = randn((4096, 4096), 1501, 0.02)
    wd = randn((4096, 14336), 1502, 0.02)
    h = randn((m, 14336), 1503, 1.0)
    res = randn((m, 4096), 1504, 1.0)
    wg, wu = randn((14336, 4096), 1505, 0.02), randn((14336, 4096), 1506, 0.02)
    wq, wk, wv = randn((4096, 4096), 1507, 0.02), randn((1024, 4096), 1508, 0.02), randn((1024, 4096), 1509, 0.02)
    inv = lo.llama3_inv_freq(device=cuda)
    pos = torch.tensor([3], dtype=torch.int32, device=cuda)
    assert lib.cb_gemm_split_k(m, 14336, 4096, 0) == 9  # down: 32 tiles x 9 K slices
    same_split = lib.cb_gemm_split_k(m, 4096, 14336, 1) == lib.cb_gemm_split_k(m, 4096, 14336, 0)
    # the slice count depends on K alone; K = 4096 is not split (measured slower)
    assert lib.cb_gemm_split_k(m, 4096, 4096, 0) == lib.cb_gemm_split_k(m, 4096, 6144, 0) == 1
    assert lib.cb_gemm_split_k(65, 14336, 4096, 0) == 1  # longer chunks are not split

    def run_all():
        out = {}
        out["o"] = torch.empty((m, 4096), dtype=BF16, device=cuda)
        ops.gemm_residual(a, wo, res, out["o"])
        out["down"] = torch.empty((m, 4096), dtype=BF16, device=cuda)
        ops.gemm_residual(h, wd, res, out["down"])
        out["bf16"] = torch.empty((m, 4096), dtype=BF16, device=cuda)
        ops.gemm_bf16(a, wo, out["bf16"])
        out["partial"] = torch.empty((m, 4096), dtype=torch.float32, device=cuda)
        ops.gemm_partial(h, wd, out["partial"])
        out["swiglu"] = torch.empty((m, 14336), dtype=BF16, device=cuda)
        ops.gemm_swiglu(a, wg, wu, out["swiglu"])
        out["silu_mul"] = torch.empty((m, 14336), dtype=BF16, device=cuda)
        ops.gemm_silu(a, wg, out["silu_mul"])
        ops.gemm_mul(a, wu, out["silu_mul"])
        out["q"] = torch.empty((m, 4096), dtype=BF16, device=cuda)
        out["kc"] = torch.full((8, m + 8, 128), 7.0, dtype=BF16, device=cuda)
        out["vc"] = torch.full_like(out["kc"], 7.0)
        ops.prefill_qkv_rope(a, wq, wk, wv, inv, pos, out["q"], out["kc"], out["vc"])
        torch.cuda.synchronize()
        return out

    split = run_all()
    assert int(tickets.abs().sum()) == 0
    _unsplit(lib, lambda: None)
    plain = run_all()

    def proj_ulp(proj):
        # one bf16 ulp of the largest projection value: the residual epilogue
        # rounds the projection before the add, so when residual and
        # projection cancel, a one-ulp flip of the projection is what the
        # (small) output differs by
        return 2.0 ** (torch.floor(torch.log2(proj.abs().max().float())).item() - 7)

    # allowed difference from the unsplit kernel: one ulp of the projection
    # (residual modes), two ulps of the output where two rounded values are
    # combined (SwiGLU: silu(bf16 g) * bf16 u; RoPE: a difference of rounded
    # products), one ulp of a plain store
    ulp = {"o": proj_ulp(F.linear(a, wo)) + proj_ulp(plain["o"]),
           "down": proj_ulp(F.linear(h, wd)) + proj_ulp(plain["down"]),
           "bf16": proj_ulp(plain["bf16"]), "vc": proj_ulp(plain["vc"][:, 3:3 + m]),
           "swiglu": 2 * proj_ulp(plain["swiglu"]), "silu_mul": 2 * proj_ulp(plain["silu_mul"]),
           "q": 2 * proj_ulp(plain["q"]), "kc": 2 * proj_ulp(plain["kc"][:, 3:3 + m])}
    for name in plain:
        if name == "partial":
            exact = h.double() @ wd.double().T
            bound = 1e-6 * 14336 ** 0.5 * (h.double().abs() @ wd.double().abs().T) + 1e-6
            assert bool(((split[name].double() - exact).abs() <= 8 * bound).all())
            continue
        got, ref = split[name].float(), plain[name].float()
        assert (got - ref).abs().max().item() <= ulp[name], name
        assert (got != ref).float().mean().item() <= 0.05, name
    close_to_torch(split["bf16"], a, wo)
    for name, proj in (("o", F.linear(a, wo)), ("down", F.linear(h, wd))):
        ref = (res.float() + proj.float()).to(BF16).float()
        assert (split[name].float() - ref).abs().max().item() <= ulp[name], name
        assert (split[name].float() != ref).float().mean().item() <= 0.05, name
    # the `matrix` granularity's gate / up GEMMs give the fused kernel's bits
    # when both split K the same way (else: one fp32 summation order apart)
    if same_split:
        assert torch.equal(split["swiglu"], split["silu_mul"])
    else:
        assert (split["swiglu"].float() - split["silu_mul"].float()).abs().max().item() <= ulp["swiglu"]
    outside = torch.cat([split["kc"][:, :3], split["kc"][:, 3 + m:]], dim=1)
    assert bool((outside == 7.0).all())
