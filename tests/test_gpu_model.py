"""Model-level parity on the GPU.

Seeded random-init Llama-3.1-8B, the 6-token seeded prompt, prefill + 8
greedy decode steps, top-k 10, driven exactly like tools/run_llama31.py
(plan -> store -> ResidentDeviceArena -> DoubleBufferRuntime [->
VocabStreamingRuntime] -> executor.begin/run/finish). Checked against
  * the golden run of the reference's own code (tests/golden/config0.*),
  * the oracle's restatement running with torch ops on the same GPU and the
    same device weights (the reference's PyTorch GPU path),
with the north-star criteria: top-k values within rtol 2e-2 / atol 2e-2 and
ids identical wherever the neighbouring gaps exceed that tolerance, greedy
ids identical over the 8 decode steps. Full logits: after 32 random-init
layers the reference's own GPU and CPU runs differ by up to ~0.3 (mean
~0.05), so the engine is held to that noise floor (cosine, max-abs, RMSE)
rather than to a per-element 2e-2 that the reference fails against itself;
the per-element tolerance is checked per layer (kernel tests, smoke).
"""

import pytest
import torch
from safetensors.torch import load_file

import parity
from conftest import Config, engine_weights, golden_path, make_store
from oracle import llama_oracle as lo
from oracle.seeded import prompt_ids

pytestmark = pytest.mark.gpu

RTOL = ATOL = 2e-2


@pytest.fixture(scope="module")
def golden():
    return load_file(golden_path("config0.safetensors"))


def generate(executor, runtime, ids, steps):
    """The tools/run_llama31.py loop; returns per-step (values, indices, logits)."""

    out = []
    with torch.inference_mode():
        for _ in range(steps):
            state = executor.begin(ids)
            state = runtime.run(executor, state)
            state = executor.finish(state)
            out.append((
                state.topk_values.reshape(-1).cpu(),
                state.topk_indices.reshape(-1).cpu(),
                None if state.logits is None else state.logits.reshape(-1).cpu(),
            ))
            ids = state.topk_indices[..., 0]
    executor.check_errors()
    return out


@pytest.fixture(scope="module")
def reference_gpu_topk(cuda, hbm_engine, meta):
    """Top-k values of the reference's PyTorch ops on this GPU (the oracle's
    restatement on the same device weights), fed the golden run's inputs."""

    return parity.reference_gpu_topk(engine_weights(hbm_engine), meta, cuda)


def check_against_golden(results, meta, gpu_topk, free_running=False):
    """Top-k values within rtol/atol 2e-2 of the reference's PyTorch path on
    this GPU, and of the reference's CPU run (golden) up to the distance
    between the reference's own GPU and CPU values; ranks identical where the
    logit gaps around them exceed the tolerance; greedy ids identical."""

    for step, ((values, indices, _), record) in enumerate(zip(results, meta["steps"])):
        if free_running and step > 0 and int(results[step - 1][1][0]) != meta["greedy_ids"][step - 1]:
            return  # the previous pick broke a near-tie the other way: the inputs differ from here
        ref_v = torch.tensor(record["topk_values"])
        failure = parity.topk_values_failure(values, record, gpu_topk[step])
        assert failure is None, "step {}: {}".format(step, failure)
        for j in range(len(ref_v)):
            tol = ATOL + RTOL * abs(float(ref_v[j]))
            before = float(ref_v[j - 1] - ref_v[j]) if j else float("inf")
            after = float(ref_v[j] - ref_v[j + 1]) if j + 1 < len(ref_v) else record["k_k1_gap"]
            if before > tol and after > tol:
                assert int(indices[j]) == record["topk_indices"][j], (step, j)
        if step < 8:  # teacher-forced: every step is compared
            failure, tie = parity.greedy_failure(step, int(indices[0]), record, meta)
            assert failure is None, "step {}: {}".format(step, failure)
            if tie:
                print("step {}: near-tie broken as {} (the reference's CPU run picked {}, its GPU path {})".format(
                    step, int(indices[0]), meta["greedy_ids"][step], int(gpu_topk.indices[step][0])))


def logit_stats(a, b):
    d = (a - b).abs()
    cos = float(torch.nn.functional.cosine_similarity(a.view(1, -1), b.view(1, -1)))
    return {"max": float(d.max()), "mean": float(d.mean()), "rmse": float(d.pow(2).mean().sqrt()), "cos": cos}


def test_config0_parity_with_reference(cuda, hbm_engine, meta, golden, reference_gpu_topk):
    """Engine (HBM weights, graph replay) vs the reference's run (golden, CPU)
    and vs the reference's PyTorch ops on this GPU (oracle), both fed the
    reference's token path. Full logits use the reference's own comparison
    metrics (benchmarks/compare_real_logits.py: max-abs, RMSE, cosine, top-10):
    the engine must sit within the reference's GPU-vs-CPU noise floor."""

    import layer_streaming as ls

    plan, store, resident, runtime = hbm_engine
    oracle = lo.OracleDecoder(engine_weights(hbm_engine), top_k=meta["top_k"])
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"], return_full_logits=True)
    results = []
    with torch.inference_mode():
        for step, record in enumerate(meta["steps"]):
            ids = torch.tensor([record["input_ids"]], device=cuda)
            state = executor.finish(runtime.run(executor, executor.begin(ids)))
            engine = state.logits.reshape(-1).float().cpu()
            results.append((state.topk_values.reshape(-1).cpu(), state.topk_indices.reshape(-1).cpu(), engine))
            reference_gpu = oracle.step(ids)["logits"][0, -1].float().cpu()
            reference_cpu = golden["step{}.logits".format(step)].float()
            e_c = logit_stats(engine, reference_cpu)
            g_c = logit_stats(reference_gpu, reference_cpu)
            e_g = logit_stats(engine, reference_gpu)
            print("step {}: engine-vs-refCPU {} | refGPU-vs-refCPU {} | engine-vs-refGPU {}".format(
                step, {k: round(v, 5) for k, v in e_c.items()}, {k: round(v, 5) for k, v in g_c.items()},
                {k: round(v, 5) for k, v in e_g.items()}))
            # the reference's own GPU-vs-CPU disagreement is the noise floor
            for stats in (e_c, e_g):
                assert 1.0 - stats["cos"] <= 1.5 * (1.0 - g_c["cos"]) + 1e-4
                assert stats["max"] <= 1.5 * g_c["max"] + 0.05
                assert stats["rmse"] <= 1.5 * g_c["rmse"]
            top_engine = set(torch.topk(engine, 10).indices.tolist())
            assert len(top_engine & set(record["topk_indices"])) >= 8
    executor.check_errors()
    check_against_golden(results, meta, reference_gpu_topk)


def test_config0_greedy_generation(cuda, hbm_engine, meta, reference_gpu_topk):
    """The tools/run_llama31.py loop on the engine's own greedy path."""

    import layer_streaming as ls

    plan, store, resident, runtime = hbm_engine
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"])
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    results = generate(executor, runtime, ids, 1 + meta["decode_steps"])
    engine_ids = [int(indices[0]) for _, indices, _ in results]
    print("greedy ids, engine:    {}".format(engine_ids))
    print("greedy ids, reference: {}".format(meta["greedy_ids"][:len(engine_ids)]))
    for step, ((values, _, _), record) in enumerate(zip(results, meta["steps"])):
        print("step {}: top-1/top-2 gap engine {:.4f}, reference {:.4f} (tolerance {:.4f})".format(
            step, float(values[0] - values[1]), record["topk_values"][0] - record["topk_values"][1],
            parity.tolerance(record["topk_values"][0])))
    check_against_golden(results, meta, reference_gpu_topk, free_running=True)


def test_eager_and_graph_replay_are_identical(cuda, hbm_engine, meta):
    import layer_streaming as ls

    plan, store, resident, runtime = hbm_engine
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    runs = []
    for graphs in (True, False):
        executor = ls.Llama31DecodeExecutor(
            Config(), resident, top_k=meta["top_k"], return_full_logits=True, use_graphs=graphs
        )
        runs.append(generate(executor, runtime, ids, 5))
    for (v1, i1, l1), (v2, i2, l2) in zip(*runs):
        assert torch.equal(v1, v2) and torch.equal(i1, i2) and torch.equal(l1, l2)


def test_l2_staging_is_only_a_cache_hint(cuda, hbm_engine, meta):
    """The attention launches prefetch part of the layer's gate+up weights into
    L2 (on by default); with every kind of staging switched off, or with the
    QKV and o_proj launches staging too, the decode steps give the same bits."""

    import layer_streaming as ls
    from layer_streaming import _native

    lib = _native.lib()
    _, _, resident, runtime = hbm_engine
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    settings = {
        "default": [],
        "off": [(1, 0, 0, 0, 0)],
        "all kinds": [(0, 3, 4, 4, 0), (2, 1, 4, 8, 0), (1, 3, 10, 12, 1)],
    }
    runs = {}
    try:
        for name, knobs in settings.items():
            lib.cb_set_l2_stage(1, 3, 10, 4, 0)  # the default
            for knob in knobs:
                _native.check(lib.cb_set_l2_stage(*knob), "cb_set_l2_stage")
            executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"], return_full_logits=True)
            runs[name] = generate(executor, runtime, ids, 4)
    finally:
        lib.cb_set_l2_stage(0, 0, 0, 0, 0)
        lib.cb_set_l2_stage(1, 3, 10, 4, 0)
        lib.cb_set_l2_stage(2, 0, 0, 0, 0)
    for name in ("off", "all kinds"):
        for (v1, i1, l1), (v2, i2, l2) in zip(runs["default"], runs[name]):
            assert torch.equal(v1, v2) and torch.equal(i1, i2) and torch.equal(l1, l2), name


def test_resident_head_returns_last_token_logits(cuda, hbm_engine, meta):
    """Like the reference's resident head (llama31.py:330-339), ``finish``
    fills ``state.logits`` without being asked: the last token's fp32 row,
    whose top-k is the returned top-k."""

    import layer_streaming as ls

    _, _, resident, runtime = hbm_engine
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"])
    with torch.inference_mode():
        state = executor.finish(runtime.run(executor, executor.begin(ids)))
    assert state.logits is not None and tuple(state.logits.shape) == (1, 1, 128256)
    assert state.logits.dtype == torch.float32
    values, _ = torch.topk(state.logits[:, -1, :], meta["top_k"], dim=-1)
    assert torch.equal(values.reshape(-1), state.topk_values.reshape(-1))
    # (torch.topk orders equal logits arbitrarily: check the ids by lookup)
    row = state.logits[0, -1]
    assert torch.equal(row[state.topk_indices.reshape(-1)], state.topk_values.reshape(-1))


def test_streamed_runtime_and_vocab_match(cuda, arena, hbm_engine, meta, reference_gpu_topk):
    """The reference's own mode: H2D two-slot streaming + streamed vocab."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group", stream_vocab=True)
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda, profile=True)
    vocab = ls.VocabStreamingRuntime(plan, store, runtime, profile=True)
    executor = ls.Llama31DecodeExecutor(Config(), resident, vocab_runtime=vocab, top_k=meta["top_k"],
                                        return_full_logits=True)
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    streamed = generate(executor, runtime, ids, 3)
    check_against_golden(streamed, meta, reference_gpu_topk)
    assert runtime.last_profile["h2d_bytes"] == plan.stream_bytes_per_token
    assert vocab.last_profile["chunk_count"] == 8

    # same bits as the hbm-resident engine (same kernels; only the LM-head
    # kernel runs per chunk, and chunking does not change any logit)
    _, _, hbm_resident, hbm_runtime = hbm_engine
    hbm = ls.Llama31DecodeExecutor(Config(), hbm_resident, top_k=meta["top_k"], return_full_logits=True)
    resident_run = generate(hbm, hbm_runtime, ids, 3)
    for (v1, i1, l1), (v2, i2, l2) in zip(streamed, resident_run):
        assert torch.equal(v1, v2) and torch.equal(i1, i2) and torch.equal(l1, l2)


@pytest.mark.parametrize("granularity", ["matrix", "layer"])
def test_other_granularities_give_same_tokens(cuda, arena, hbm_engine, meta, granularity):
    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan(granularity)
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda, weights="streamed")
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"], return_full_logits=True)
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    got = generate(executor, runtime, ids, 2)
    _, _, hbm_resident, hbm_runtime = hbm_engine
    ref = generate(ls.Llama31DecodeExecutor(Config(), hbm_resident, top_k=meta["top_k"], return_full_logits=True),
                   hbm_runtime, ids, 2)
    for (v1, i1, l1), (v2, i2, l2) in zip(got, ref):
        assert torch.equal(i1, i2) and torch.equal(l1, l2)


def test_slot_reuse_waits_for_compute(cuda, arena, meta):
    """Race check of the two-slot protocol: delay every unit's compute; the
    copy stream must still wait for the slot to be released (same results)."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group", stream_vocab=True)
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda)
    vocab = ls.VocabStreamingRuntime(plan, store, runtime)
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    plain = ls.Llama31DecodeExecutor(Config(), resident, vocab_runtime=vocab, top_k=meta["top_k"])
    base = generate(plain, runtime, ids, 2)

    class Slow:
        def __init__(self, inner):
            self.inner = inner

        def __call__(self, unit, weights, state):
            torch.cuda._sleep(2_000_000)  # ~1 ms of GPU time before the unit's kernels
            return self.inner(unit, weights, state)

    slow_exec = ls.Llama31DecodeExecutor(Config(), resident, vocab_runtime=vocab, top_k=meta["top_k"])
    slow = []
    with torch.inference_mode():
        state_ids = ids
        for _ in range(2):
            state = slow_exec.begin(state_ids)
            state = runtime.run(Slow(slow_exec), state)
            state = slow_exec.finish(state)
            slow.append((state.topk_values.reshape(-1).cpu(), state.topk_indices.reshape(-1).cpu()))
            state_ids = state.topk_indices[..., 0]
    for (v1, i1, _), (v2, i2) in zip(base, slow):
        assert torch.equal(v1, v2) and torch.equal(i1, i2)


def test_pinned_staging_store_end_to_end(cuda, arena, hbm_engine, meta):
    """The reference's pinned_staging mode on the GPU: a PAGEABLE host arena
    plus two pinned staging buffers (and two pinned LM-head chunk buffers);
    the slot ring's native stager copies every unit into a staging buffer
    before its DMA. Same bits as the HBM-resident engine; the profile reports
    the staging copies and the H2D rate next to the full-pinned mode's."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group", stream_vocab=True)

    def pageable(elements, dtype=None, device=None, pin_memory=False):
        return torch.empty(elements, dtype=dtype, device=device, pin_memory=pin_memory)

    store = ls.create_weight_store(plan, "pinned_staging", tensor_factory=pageable)
    assert not store.arena.is_pinned() and all(s.is_pinned() for s in store.staging_slots)
    store.arena.copy_(arena.arena)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda, profile=True)
    vocab = ls.VocabStreamingRuntime(plan, store, runtime, profile=True)
    assert vocab.extra_pinned_cpu_bytes == 256 * 4096 * 2 + 2 * plan.vocab.chunk_elements * 2
    executor = ls.Llama31DecodeExecutor(Config(), resident, vocab_runtime=vocab, top_k=meta["top_k"],
                                        return_full_logits=True)
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    staged = generate(executor, runtime, ids, 3)
    profile = runtime.last_profile
    print("pinned_staging: {:.1f} GB/s H2D, {} staging copies ({:.1f} ms, max {:.1f}), source wait {:.1f} ms, "
          "pipeline {:.1f} ms; LM head {:.1f} GB/s".format(
              profile["h2d_effective_gbps"], profile["staging_copy_count"], profile["staging_event_sum_ms"],
              profile["staging_event_max_ms"], profile["source_wait_ms"], profile["gpu_pipeline_ms"],
              vocab.last_profile["h2d_effective_gbps"]))
    assert profile["staging_copy_count"] == len(plan.units)
    assert profile["h2d_bytes"] == plan.stream_bytes_per_token

    _, _, hbm_resident, hbm_runtime = hbm_engine
    hbm = ls.Llama31DecodeExecutor(Config(), hbm_resident, top_k=meta["top_k"], return_full_logits=True)
    resident_run = generate(hbm, hbm_runtime, ids, 3)
    for (v1, i1, l1), (v2, i2, l2) in zip(staged, resident_run):
        assert torch.equal(v1, v2) and torch.equal(i1, i2) and torch.equal(l1, l2)
    store.close()


def test_streamed_pass_recovers_after_a_failing_unit(cuda, arena, meta):
    """A compute callback that raises mid-pass: the slot ring drops the
    queued copies, waits for the started ones and serves the next pass."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group")
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda)
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"])
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(cuda)
    want = generate(executor, runtime, ids, 1)

    class Boom(Exception):
        pass

    def failing(unit, weights, state):
        if unit.layer_index == 3:
            raise Boom()
        return state

    with pytest.raises(Boom):
        runtime.run(failing, None)
    again = ls.Llama31DecodeExecutor(Config(), resident, top_k=meta["top_k"])
    got = generate(again, runtime, ids, 1)
    assert torch.equal(want[0][0], got[0][0]) and torch.equal(want[0][1], got[0][1])
