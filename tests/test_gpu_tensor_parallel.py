"""Tensor-parallel decode on the GPU.

Kernel level (one GPU): a rank's shard kernels give exactly the bits of the
matching slice of the full computation (query / KV heads, FFN rows), the
partial projections match an fp32 reference for every shard width, and the
fused exchange kernels over a world of one are bit-identical to the
single-GPU kernels.

Model level: the tensor-parallel decoder over a world of one reproduces the
reference's golden run through both exchange paths, and
over two GPUs (when the box has them, via torchrun of tests/tp_worker.py) it
meets the same top-k criteria against the golden run through both exchange
paths (teacher-forced), decodes the golden greedy ids up to the first golden
near-tie, and every rank holds the same bits.
"""

import ctypes
import json
import os
import subprocess
import sys
import time

import pytest
import torch
import torch.nn.functional as F

import parity
from conftest import REPO, golden_path
from oracle.seeded import prompt_ids

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


@pytest.mark.parametrize("k_dim", [512, 1024, 1792, 2048, 3584, 4096, 7168, 14336])
def test_partial_projection_every_shard_width(ops, cuda, k_dim):
    x = randn((k_dim,), 100 + k_dim)
    w = randn((4096, k_dim), 101, 0.02)
    res = randn((4096,), 102)
    partial = torch.empty(4096, dtype=torch.float32, device=cuda)
    ops.proj_partial(x, w, partial)
    exact = (w.double() @ x.double()).float()
    # fp32 accumulation of k_dim products of bf16 values: a few ulps of the sum of |terms|
    bound = 1e-6 * k_dim ** 0.5 * (w.double().abs() @ x.double().abs()).float() + 1e-6
    assert bool(((partial - exact).abs() <= bound * 8).all())
    # partial + separate residual add == the fused residual projection, bit for bit
    fused = torch.empty_like(res)
    ops.proj_residual(x, w, res, fused)
    split = torch.empty_like(res)
    ops.residual_add_f32(res, partial, split)
    assert torch.equal(fused, split)


def test_shard_kernels_equal_full_slices(ops, cuda):
    """qkv_rope over 8 query / 2 KV heads, gate_up over 3584 rows and
    attention over 2 KV heads (a rank of four) equal the full kernels' slices."""

    world, rank = 4, 1
    qh, kvh, ffn = 32 // world, 8 // world, 14336 // world
    x = randn((4096,), 110)
    norm_w = (randn((4096,), 111, std=0.1).float() + 1).to(BF16)
    wq, wk, wv = randn((4096, 4096), 112, 0.02), randn((1024, 4096), 113, 0.02), randn((1024, 4096), 114, 0.02)
    inv = torch.linspace(1e-4, 1.0, 64, device=cuda)
    length, position = 300, 299
    pos = torch.tensor([position], dtype=torch.int32, device=cuda)
    kc = randn((8, length, 128), 115)
    vc = randn((8, length, 128), 116)
    q = torch.empty(4096, dtype=BF16, device=cuda)
    ops.qkv_rope(x, norm_w, 1e-5, wq, wk, wv, inv, pos, 0, q, kc, vc)
    q_rows = slice(rank * qh * 128, (rank + 1) * qh * 128)
    kv_rows = slice(rank * kvh * 128, (rank + 1) * kvh * 128)
    heads = slice(rank * kvh, (rank + 1) * kvh)
    kc_s = kc[heads].clone()
    vc_s = vc[heads].clone()
    kc_s[:, position] = 0
    vc_s[:, position] = 0
    q_s = torch.empty(qh * 128, dtype=BF16, device=cuda)
    ops.qkv_rope(x, norm_w, 1e-5, wq[q_rows].contiguous(), wk[kv_rows].contiguous(), wv[kv_rows].contiguous(),
                 inv, pos, 0, q_s, kc_s, vc_s, qh, kvh)
    assert torch.equal(q_s, q[q_rows])
    assert torch.equal(kc_s, kc[heads]) and torch.equal(vc_s, vc[heads])

    # attention of this rank's heads, same split
    splits, chunk = 3, 128
    out = torch.empty(4096, dtype=BF16, device=cuda)
    ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=cuda)
    tickets = torch.zeros(8, dtype=torch.int32, device=cuda)
    ops.attention(q, kc, vc, pos, splits, chunk, out, ws, tickets)
    out_s = torch.empty(qh * 128, dtype=BF16, device=cuda)
    ops.attention(q_s, kc_s, vc_s, pos, splits, chunk, out_s, ws, tickets)
    assert torch.equal(out_s, out[q_rows])
    assert int(tickets.abs().sum()) == 0

    wg, wu = randn((14336, 4096), 117, 0.02), randn((14336, 4096), 118, 0.02)
    full = torch.empty(14336, dtype=BF16, device=cuda)
    ops.gate_up_swiglu(x, norm_w, 1e-5, wg, wu, full)
    rows = slice(rank * ffn, (rank + 1) * ffn)
    part = torch.empty(ffn, dtype=BF16, device=cuda)
    ops.gate_up_swiglu(x, norm_w, 1e-5, wg[rows].contiguous(), wu[rows].contiguous(), part)
    assert torch.equal(part, full[rows])


def _exchange(lib, native):
    own = ctypes.c_void_p()
    native.check(lib.cb_exchange_alloc(ctypes.byref(own)), "cb_exchange_alloc")
    return own, (ctypes.c_void_p * 1)(own.value)


def test_exchange_kernels_world_of_one_equal_local_kernels(ops, cuda):
    from layer_streaming import _native

    lib = _native.lib()
    own, pointers = _exchange(lib, _native)
    stream = _native.stream_ptr(cuda)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for k_dim in (4096, 14336):
            x = randn((k_dim,), 120 + k_dim)
            w = randn((4096, k_dim), 121, 0.02)
            res = randn((4096,), 122)
            want = torch.empty_like(res)
            ops.proj_residual(x, w, res, want)
            for step in range(3):
                for slot in (0, 1, 2, 63):
                    out = res.clone()
                    _native.check(lib.cb_proj_allreduce_residual(
                        x.data_ptr(), k_dim, w.data_ptr(), 4096, out.data_ptr(), out.data_ptr(), pointers, 0, 1,
                        slot, 66, epoch.data_ptr(), stream), "cb_proj_allreduce_residual")
                    assert torch.equal(out, want), (k_dim, step, slot)
                ops.position_advance(epoch, 1)
        # LM head: local top-k gathered over a world of one
        h = randn((4096,), 130)
        norm = (randn((4096,), 131, std=0.1).float() + 1).to(BF16)
        head = randn((16032, 4096), 132, 0.02)
        ws = torch.empty(ops.lm_head_workspace_bytes(10), dtype=torch.uint8, device=cuda)
        ticket = torch.zeros(1, dtype=torch.int32, device=cuda)
        v1 = torch.empty(10, dtype=torch.float32, device=cuda)
        i1 = torch.empty(10, dtype=torch.int64, device=cuda)
        ops.lm_head_topk(h, norm, 1e-5, head, 5000, 10, None, v1, i1, ws, ticket)
        v2, i2 = torch.empty_like(v1), torch.empty_like(i1)
        _native.check(lib.cb_lm_head_topk_allgather(
            h.data_ptr(), norm.data_ptr(), 1e-5, head.data_ptr(), 16032, 5000, 10, v2.data_ptr(), i2.data_ptr(),
            ws.data_ptr(), ticket.data_ptr(), pointers, 0, 1, 64, 66, epoch.data_ptr(), stream),
            "cb_lm_head_topk_allgather")
        assert torch.equal(v1, v2) and torch.equal(i1, i2)
        torch.cuda.synchronize()
    finally:
        lib.cb_exchange_free(own)


def test_exchange_arguments_are_validated(cuda):
    from layer_streaming import _native

    lib = _native.lib()
    null = (ctypes.c_void_p * 2)(None, None)
    assert lib.cb_proj_allreduce_residual(None, 4096, None, 4096, None, None, null, 0, 2, 0, 66, None, None) != 0
    x = torch.zeros(4096, dtype=BF16, device=cuda)
    w = torch.zeros((2, 4096), dtype=BF16, device=cuda)
    out = torch.zeros(2, dtype=BF16, device=cuda)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    own, pointers = _exchange(lib, _native)
    try:
        for rank, world, slot, slots in ((1, 1, 0, 66), (0, 9, 0, 66), (0, 1, 66, 66), (0, 1, 0, 65)):
            rc = lib.cb_proj_allreduce_residual(x.data_ptr(), 4096, w.data_ptr(), 2, out.data_ptr(), out.data_ptr(),
                                                pointers, rank, world, slot, slots, epoch.data_ptr(), None)
            assert rc != 0, (rank, world, slot, slots)
    finally:
        lib.cb_exchange_free(own)


def test_exchange_wait_runs_out_and_reports(ops, cuda):
    """Failure detection of the fused exchanges on one GPU, without a fault:
    a world of two whose second "peer" is a local exchange buffer that no
    kernel writes. With a 1 ms limit the projection gives up, records code
    120 (the LM head's gather 121) and returns; the same buffers then serve a
    normal launch, bit-identical to the local kernel."""

    from layer_streaming import _native

    lib = _native.lib()
    own, single = _exchange(lib, _native)
    ghost, _ = _exchange(lib, _native)
    pair = (ctypes.c_void_p * 2)(own.value, ghost.value)
    stream = _native.stream_ptr(cuda)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    x = randn((4096,), 140)
    w = randn((4096, 4096), 141, 0.02)
    res = randn((4096,), 142)
    h = randn((4096,), 143)
    head = randn((16384, 4096), 144, 0.02)
    ws = torch.empty(ops.lm_head_workspace_bytes(10), dtype=torch.uint8, device=cuda)
    ticket = torch.zeros(1, dtype=torch.int32, device=cuda)
    values = torch.empty(10, dtype=torch.float32, device=cuda)
    indices = torch.empty(10, dtype=torch.int64, device=cuda)
    lib.cb_set_error_word(err.data_ptr())
    previous = lib.cb_set_exchange_wait_ns(1_000_000)
    try:
        assert previous == 2_000_000_000
        out = res.clone()
        torch.cuda.synchronize()
        started = time.perf_counter()
        _native.check(lib.cb_proj_allreduce_residual(
            x.data_ptr(), 4096, w.data_ptr(), 4096, out.data_ptr(), out.data_ptr(), pair, 0, 2, 0, 66,
            epoch.data_ptr(), stream), "cb_proj_allreduce_residual")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - started
        assert int(err.item()) == 120
        assert elapsed < 1.0, elapsed  # one limit per waiting thread, not per awaited word
        err.zero_()
        _native.check(lib.cb_lm_head_topk_allgather(
            h.data_ptr(), None, 1e-5, head.data_ptr(), 16384, 0, 10, values.data_ptr(), indices.data_ptr(),
            ws.data_ptr(), ticket.data_ptr(), pair, 0, 2, 1, 66, epoch.data_ptr(), stream),
            "cb_lm_head_topk_allgather")
        torch.cuda.synchronize()
        assert int(err.item()) == 121
        assert int(ticket.item()) == 0
    finally:
        lib.cb_set_exchange_wait_ns(0)
    try:
        # the next step on the same buffers (world of one) is clean and exact
        err.zero_()
        ops.position_advance(epoch, 1)
        want = torch.empty_like(res)
        ops.proj_residual(x, w, res, want)
        out = res.clone()
        _native.check(lib.cb_proj_allreduce_residual(
            x.data_ptr(), 4096, w.data_ptr(), 4096, out.data_ptr(), out.data_ptr(), single, 0, 1, 0, 66,
            epoch.data_ptr(), stream), "cb_proj_allreduce_residual")
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        assert int(err.item()) == 0
    finally:
        lib.cb_set_error_word(None)
        lib.cb_exchange_free(own)
        lib.cb_exchange_free(ghost)


class Config:
    hidden_size = 4096
    intermediate_size = 14336
    num_hidden_layers = 32
    num_attention_heads = 32
    num_key_value_heads = 8
    vocab_size = 128256
    rms_norm_eps = 1e-5
    rope_parameters = {
        "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192, "rope_theta": 500000.0,
    }


def _greedy(decoder, ids, steps):
    out = []
    with torch.inference_mode():
        for _ in range(steps):
            state = decoder(ids)
            out.append((state.topk_values.reshape(-1).cpu(), state.topk_indices.reshape(-1).cpu()))
            ids = state.topk_indices[..., 0].reshape(1, 1)
    decoder.check_errors()
    return out


def test_world_of_one_decoder_reproduces_golden_run(cuda):
    from layer_streaming.tensor_parallel import TensorParallelDecoder, TensorParallelWeights

    meta = json.load(open(golden_path("config0.json")))
    weights = TensorParallelWeights.seeded(1, 0, cuda, seed=meta["weight_seed"])
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    runs = {}
    for exchange in ("peer", "nccl"):
        decoder = TensorParallelDecoder(Config(), weights, top_k=meta["top_k"], exchange=exchange)
        runs[exchange] = _greedy(decoder, ids, 1 + meta["decode_steps"])
        decoder.close()
    for (v1, i1), (v2, i2) in zip(runs["peer"], runs["nccl"]):
        assert torch.equal(v1, v2) and torch.equal(i1, i2)
    gpu_topk = parity.reference_gpu_topk(weights.tensors, meta, cuda)
    for step, ((values, indices), record) in enumerate(zip(runs["peer"], meta["steps"])):
        failure = parity.topk_values_failure(values, record, gpu_topk[step])
        assert failure is None, "step {}: {}".format(step, failure)
        failure, tie = parity.greedy_failure(step, int(indices[0]), record, meta)
        assert failure is None, "step {}: {}".format(step, failure)
        if tie:
            break  # free-running greedy decoding parts from the reference's after a near-tie


def test_world_of_one_streamed_shards_equal_resident(cuda):
    """Row e3 on one GPU: the decoder streaming its layer shards from a pinned
    shard arena through two device slots (the reference's H2D mode, per
    rank) gives the resident decoder's bits; the profile reports the H2D
    rate of the rank's stream."""

    from layer_streaming.tensor_parallel import TensorParallelDecoder, TensorParallelWeights

    meta = json.load(open(golden_path("config0.json")))
    resident = TensorParallelWeights.seeded(1, 0, cuda, seed=meta["weight_seed"])
    streamed = TensorParallelWeights.seeded(1, 0, cuda, seed=meta["weight_seed"], stream_layers=True)
    assert streamed.streamed and streamed.arena.storage.is_pinned()
    assert streamed.arena.nbytes >= 32 * 436_207_616
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    runs = []
    for weights in (resident, streamed):
        decoder = TensorParallelDecoder(Config(), weights, top_k=meta["top_k"], profile=True)
        runs.append(_greedy(decoder, ids, 3))
        if weights is streamed:
            prof = decoder.last_stream
            gbps = prof["h2d_bytes"] / 1e9 / (prof["h2d_event_sum_ms"] / 1000.0)
            print("streamed shard: {} bytes per step, {:.1f} GB/s H2D, pass {:.1f} ms".format(
                prof["h2d_bytes"], gbps, prof["gpu_pipeline_ms"]))
            assert prof["h2d_bytes"] == 2 * sum(unit[3] for unit in streamed.arena.units)
        decoder.close()
    for (v1, i1), (v2, i2) in zip(*runs):
        assert torch.equal(v1, v2) and torch.equal(i1, i2)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs on the box")
def test_two_gpu_decoder_reproduces_golden_run():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(REPO, "tests", "tp_worker.py")]
    proc = subprocess.run(["timeout", "-k", "30", "900"] + cmd, env=env, capture_output=True, text=True)
    print(proc.stdout[-4000:])
    print(proc.stderr[-4000:])
    assert proc.returncode == 0
    assert "TP-PARITY-OK" in proc.stdout
