"""Int8 weight-only decode projections (the engine's optional low-precision
weight transfer mode) on the GPU.

The reference has no quantized mode, so these kernels are held to their own
documented arithmetic: the quantizer bit-exactly to its CPU restatement
(oracle/quant_i8.py), each int8 projection to the reference op computed with
the dequantized weights (q * scale) in fp32 - a one-bf16-ulp summation-order
difference allowed, as for the bf16 kernels - and the whole int8 model to the
bf16 engine within a bound on the quantization noise (not the bf16 parity
contract).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import llama_oracle as lo
from oracle import quant_i8

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


def quantize(ops, w):
    q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    s = torch.empty(w.shape[0], dtype=torch.float32, device=w.device)
    ops.quantize_rows_i8(w, q, s)
    return q, s


def lin8(x, q, s):
    """bf16(x . (q * s)^T) in fp32, as F.linear would return it."""

    return ((x.float() @ q.float().T) * s).to(BF16)


def ulp(t):
    """One bf16 ulp of the largest |t|."""

    return 2.0 ** (torch.floor(torch.log2(t.float().abs().max())).item() - 7)


def close(got, ref, tol, frac=0.05):
    got, ref = got.float(), ref.float()
    assert (got - ref).abs().max().item() <= tol
    assert (got != ref).float().mean().item() <= frac


def test_quantizer_matches_cpu_restatement(ops, cuda):
    w = randn((300, 4096), 50, 0.02)
    w[7] = 0  # an all-zero row: scale 0, q 0
    w[11, :8] = torch.tensor([127, -63.5, 0.5, 1.5, 2.5, -127, 0, 64], dtype=BF16)  # exact ties at scale 1
    w[11, 8:] = 0
    q, s = quantize(ops, w)
    rq, rs = quant_i8.quantize_rows_i8(w.cpu().view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert q[11, :8].tolist() == [127, -64, 0, 2, 2, -127, 0, 64]


@pytest.mark.parametrize("k_dim", [4096, 14336])
def test_proj_residual_i8(ops, cuda, k_dim):
    x = randn((k_dim,), 51)
    w = randn((4096, k_dim), 52, 0.02)
    res = randn((4096,), 53)
    q, s = quantize(ops, w)
    out = torch.empty_like(res)
    ops.proj_residual_i8(x, q, s, res, out)
    proj = lin8(x.view(1, -1), q, s).view(-1)
    ref = (res.float() + proj.float()).to(BF16)
    # one ulp of the projection (rounded before the residual add) plus one of the output
    close(out, ref, ulp(proj) + ulp(ref))
    res2 = res.clone()
    ops.proj_residual_i8(x, q, s, res2, res2)  # in place
    assert torch.equal(res2, out)


def test_gate_up_swiglu_i8(ops, cuda):
    x = randn((4096,), 54)
    norm_w = (randn((4096,), 55, std=0.1).float() + 1).to(BF16)
    wg, wu = randn((14336, 4096), 56, 0.02), randn((14336, 4096), 57, 0.02)
    (qg, sg), (qu, su) = quantize(ops, wg), quantize(ops, wu)
    out = torch.empty(14336, dtype=BF16, device=cuda)
    ops.gate_up_swiglu_i8(x, norm_w, 1e-5, qg, sg, qu, su, out)
    normed = lo.rms_norm(x.view(1, -1), norm_w)
    g, u = lin8(normed, qg, sg).view(-1), lin8(normed, qu, su).view(-1)
    ref = (F.silu(g.float()).to(BF16).float() * u.float()).to(BF16)
    close(out, ref, 2 * ulp(ref) + 2e-2 * ulp(g))


@pytest.mark.parametrize("position", [0, 700])
def test_qkv_rope_i8(ops, cuda, position):
    x = randn((4096,), 60 + position)
    norm_w = (randn((4096,), 61, std=0.1).float() + 1).to(BF16)
    wq, wk, wv = randn((4096, 4096), 62, 0.02), randn((1024, 4096), 63, 0.02), randn((1024, 4096), 64, 0.02)
    (qq, sq), (qk, sk), (qv, sv) = quantize(ops, wq), quantize(ops, wk), quantize(ops, wv)
    inv = lo.llama3_inv_freq(device=cuda)
    kc = torch.full((8, position + 3, 128), 7.0, dtype=BF16, device=cuda)
    vc = torch.full_like(kc, 7.0)
    pos = torch.tensor([position], dtype=torch.int32, device=cuda)
    q = torch.empty(4096, dtype=BF16, device=cuda)
    ops.qkv_rope_i8(x, norm_w, 1e-5, qq, sq, qk, sk, qv, sv, inv, pos, 0, q, kc, vc)
    normed = lo.rms_norm(x.view(1, 1, -1), norm_w)
    rq = lin8(normed.view(1, -1), qq, sq).view(1, 1, 32, 128).transpose(1, 2)
    rk = lin8(normed.view(1, -1), qk, sk).view(1, 1, 8, 128).transpose(1, 2)
    rv = lin8(normed.view(1, -1), qv, sv).view(8, 128)
    cos, sin = lo.rope_cos_sin(torch.tensor([[position]], device=cuda), inv)
    rq, rk = lo.apply_rope(rq, rk, cos, sin)
    # RoPE subtracts rounded products: a one-ulp projection difference can
    # survive the cancellation, so the bound is two ulps of the projection
    close(q, rq.reshape(4096), 2 * ulp(rq))
    close(kc[:, position], rk.reshape(8, 128), 2 * ulp(rk))
    close(vc[:, position], rv, ulp(rv))
    untouched = torch.cat([kc[:, :position], kc[:, position + 1:], vc[:, :position], vc[:, position + 1:]], dim=1)
    assert bool((untouched == 7.0).all())


def test_lm_head_topk_i8(ops, cuda):
    x = randn((4096,), 70)
    norm_w = torch.ones(4096, dtype=BF16, device=cuda)
    w = randn((128256, 4096), 71, 0.02)
    q, s = quantize(ops, w)
    del w
    k = 10
    values = torch.empty(k, device=cuda)
    indices = torch.empty(k, dtype=torch.int64, device=cuda)
    logits = torch.empty(128256, device=cuda)
    ws = torch.empty(ops.lm_head_workspace_bytes(k), dtype=torch.uint8, device=cuda)
    ticket = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.lm_head_topk_i8(x, norm_w, 1e-5, q, s, k, logits, values, indices, ws, ticket)
    normed = lo.rms_norm(x.view(1, -1), norm_w)
    ref_logits = lin8(normed, q, s).float().view(-1)
    close(logits, ref_logits, ulp(ref_logits))
    # the kernel's own logits select its top-k exactly (ties: smaller index)
    top_v, _ = torch.topk(logits, k)
    assert torch.equal(values, top_v)
    assert torch.equal(logits[indices], values)
    assert int(ticket.item()) == 0


def test_int8_engine_tracks_the_bf16_engine(cuda, hbm_engine, meta):
    """Config 0 (seeded weights, 6-token prompt) through the int8 executor:
    the one-token steps read int8 weights (about half the bytes) and follow
    the bf16 engine within the quantization noise; prefill stays bf16."""

    import layer_streaming as ls

    from conftest import Config

    _, _, resident, runtime = hbm_engine
    ids = torch.tensor(meta["prompt_ids"], dtype=torch.int64, device=cuda).view(1, -1)

    def run(fmt, forced=None, steps=4):
        """Prefill, then `steps` one-token steps fed `forced` ids (or the run's own picks)."""

        executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=10, decode_weights=fmt)
        out = []
        with torch.inference_mode():
            state = executor.finish(runtime.run(executor, executor.begin(ids)))
            token = state.topk_indices[..., 0].reshape(1, 1)
            for step in range(steps):
                if forced is not None:
                    token = forced[step].view(1, 1)
                fed = token.clone()
                state = executor.finish(runtime.run(executor, executor.begin(fed)))
                out.append((fed, state.logits.view(-1).clone(), state.topk_indices.view(-1).clone()))
                token = state.topk_indices[..., 0].reshape(1, 1)
        executor.check_errors()
        return out

    bf16 = run("bf16")
    int8 = run("int8", forced=[fed for fed, _, _ in bf16])  # teacher-forced with the bf16 engine's ids
    for (_, lb, ib), (_, l8, i8) in zip(bf16, int8):
        cos = F.cosine_similarity(lb.double(), l8.double(), dim=0).item()
        overlap = len(set(ib.tolist()) & set(i8.tolist()))
        print("int8 vs bf16: logits cosine {:.5f}, top-10 overlap {}/10, top-1 {} / {}".format(
            cos, overlap, int(i8[0]), int(ib[0])))
        assert cos > 0.98


def test_streamed_int8_transfer(cuda, arena, hbm_engine, meta):
    """The reference's streamed mode with int8 units (transfer='int8'): about
    half the H2D bytes per token; its one-token steps give the bits of the
    HBM-resident int8 executor (same quantized weights, same kernels), and a
    multi-token prompt (prefill GEMMs on dequantized units) tracks the bf16
    engine within the quantization noise."""

    import layer_streaming as ls

    from conftest import Config, make_store

    plan = ls.build_llama31_8b_plan("matrix_group")
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    streamed = ls.DoubleBufferRuntime(plan, store, resident, cuda, weights="streamed", transfer="int8", profile=True)
    _, _, hbm_resident, hbm_runtime = hbm_engine

    def run(executor, runtime, prompt, steps, forced=None):
        """Per step (top-k, logits, the residual stream after the last layer)."""

        out = []
        with torch.inference_mode():
            ids = prompt
            for step in range(steps):
                state = executor.finish(runtime.run(executor, executor.begin(ids)))
                out.append((state.topk_indices.clone(), state.logits.clone(), executor._x[0].clone()))
                ids = state.topk_indices[..., 0].reshape(1, 1) if forced is None else forced[step].view(1, 1)
        executor.check_errors()
        return out

    # every step one token: both paths run the int8 GEMVs on identical int8
    # layer weights, so the residual stream after the 32 layers is the same
    # bits (the HBM int8 executor also quantizes its resident LM head, the
    # streamed transfer only the layer units, so the logits differ)
    first = torch.tensor([[meta["prompt_ids"][0]]], dtype=torch.int64, device=cuda)
    forced = torch.tensor(meta["prompt_ids"][1:5], dtype=torch.int64, device=cuda)
    got = run(ls.Llama31DecodeExecutor(Config(), resident, top_k=10), streamed, first, 4, forced)
    ref = run(ls.Llama31DecodeExecutor(Config(), hbm_resident, top_k=10, decode_weights="int8"), hbm_runtime,
              first, 4, forced)
    for (_, _, h1), (_, _, h2) in zip(got, ref):
        assert torch.equal(h1, h2)
    moved = streamed.last_profile["h2d_bytes"]
    assert abs(moved - streamed.int8_arena.nbytes) == 0
    assert 0.49 < moved / plan.stream_bytes_per_token < 0.51
    # a 6-token prompt: prefill on dequantized units, then int8 one-token steps
    ids = torch.tensor(meta["prompt_ids"], dtype=torch.int64, device=cuda).view(1, -1)
    got = run(ls.Llama31DecodeExecutor(Config(), resident, top_k=10), streamed, ids, 3)
    ref = run(ls.Llama31DecodeExecutor(Config(), hbm_resident, top_k=10), hbm_runtime, ids, 3)
    cos = F.cosine_similarity(got[0][1].view(-1).double(), ref[0][1].view(-1).double(), dim=0).item()
    print("streamed int8 prefill vs bf16: logits cosine {:.5f}".format(cos))
    assert cos > 0.98
