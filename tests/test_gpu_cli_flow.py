"""The drop-in path of ``tools/run_llama31.py`` on a real checkpoint (GPU).

The reference's CLI (``tools/run_llama31.py:53-155``) loads a local
checkpoint with ``AutoConfig`` / ``AutoTokenizer`` and
``store.load_checkpoint``, builds plan -> store -> ``ResidentDeviceArena`` ->
``DoubleBufferRuntime`` [-> ``VocabStreamingRuntime``] ->
``Llama31DecodeExecutor``, generates ``--max-new-tokens`` greedy tokens and
reports ``runtime.stats.as_dict()``, ``store.pinned_cpu_bytes``,
``vocab_runtime.extra_pinned_cpu_bytes`` and ``plan.host_arena_bytes`` /
``stream_bytes_per_token``. :func:`cli_flow` makes exactly those calls, in
that order, against this package, on the seeded checkpoint that
``write_seeded_checkpoint`` writes (Llama-3.1-8B geometry, byte-level
tokenizer stand-in). Every vocab mode x weight mode must generate the same
ids as the HBM-resident engine fed the same prompt.
"""

import os
import time

import pytest
import torch

from conftest import Config

pytestmark = pytest.mark.gpu

PROMPT = "The meaning of life is"
NEW_TOKENS = 8


@pytest.fixture(scope="module")
def checkpoint(cuda, tmp_path_factory):
    from layer_streaming.checkpoint import write_seeded_checkpoint

    out = tmp_path_factory.mktemp("llama31-seed0")
    started = time.perf_counter()
    write_seeded_checkpoint(out, seed=0, device=cuda)
    print("seeded checkpoint written in {:.1f} s".format(time.perf_counter() - started))
    return out


def cli_flow(checkpoint, device, vocab_mode, weight_store="full_pinned", granularity="matrix_group"):
    """tools/run_llama31.py:53-155, call for call, returning its report and ids."""

    from transformers import AutoConfig, AutoTokenizer

    from layer_streaming import (
        DoubleBufferRuntime,
        Llama31DecodeExecutor,
        ResidentDeviceArena,
        VocabStreamingRuntime,
        build_llama31_8b_plan,
        create_weight_store,
    )

    config = AutoConfig.from_pretrained(checkpoint, local_files_only=True)
    tokenizer = AutoTokenizer.from_pretrained(checkpoint, local_files_only=True)
    plan = build_llama31_8b_plan(granularity, tie_word_embeddings=bool(config.tie_word_embeddings),
                                 stream_vocab=(vocab_mode == "streamed"))
    store = create_weight_store(plan, weight_store)
    started = time.perf_counter()
    store.load_checkpoint(checkpoint)
    load_seconds = time.perf_counter() - started
    torch.cuda.set_device(device)
    resident = ResidentDeviceArena(plan, store, device)
    runtime = DoubleBufferRuntime(plan, store, resident, device)
    vocab_runtime = VocabStreamingRuntime(plan, store, runtime) if plan.vocab is not None else None
    executor = Llama31DecodeExecutor(config, resident, vocab_runtime=vocab_runtime, top_k=10)
    input_ids = tokenizer(PROMPT, return_tensors="pt", add_special_tokens=True).input_ids.to(device)
    generated, latencies = [], []
    with torch.inference_mode():
        state = executor.finish(runtime.run(executor, executor.begin(input_ids)))
        token = state.topk_indices[..., 0]
        generated.append(token)
        for _ in range(NEW_TOKENS - 1):
            began = time.perf_counter()
            state = executor.finish(runtime.run(executor, executor.begin(token)))
            token = state.topk_indices[..., 0]
            torch.cuda.synchronize(device)
            latencies.append((time.perf_counter() - began) * 1000.0)
            generated.append(token)
    ids = torch.cat(generated, dim=-1).cpu()
    report = {
        "generated_text": tokenizer.decode(ids[0], skip_special_tokens=True),
        "checkpoint_load_seconds": load_seconds,
        "decode_token_latencies_ms": latencies,
        "runtime": runtime.stats.as_dict(),
        "cpu_pinned_bytes": store.pinned_cpu_bytes,
        "vocab_extra_pinned_cpu_bytes": vocab_runtime.extra_pinned_cpu_bytes if vocab_runtime else 0,
        "plan": {"host_arena_bytes": plan.host_arena_bytes, "stream_bytes_per_token": plan.stream_bytes_per_token},
    }
    store.close()
    return report, ids[0].tolist(), input_ids


@pytest.mark.parametrize("weights", ["streamed", "hbm"])
@pytest.mark.parametrize("vocab_mode", ["resident", "streamed"])
def test_cli_flow_on_seeded_checkpoint(cuda, checkpoint, hbm_engine, vocab_mode, weights, monkeypatch):
    import layer_streaming as ls

    monkeypatch.setenv("CASCADE_B200_WEIGHTS", weights)
    report, ids, prompt = cli_flow(checkpoint, cuda, vocab_mode)
    print("{} vocab, {} weights: ids {} | load {:.1f} s | decode ms/token {}".format(
        vocab_mode, weights, ids, report["checkpoint_load_seconds"],
        [round(x, 2) for x in report["decode_token_latencies_ms"]]))
    for key in ("transfer_units", "slot_bytes", "two_slot_bytes", "device_slot_count", "device_slots_bytes",
                "resident_bytes", "weight_gpu_bytes"):
        assert key in report["runtime"]
    assert report["plan"]["host_arena_bytes"] == 16060522496
    assert report["cpu_pinned_bytes"] == report["plan"]["host_arena_bytes"]
    assert (report["vocab_extra_pinned_cpu_bytes"] > 0) == (vocab_mode == "streamed")

    # the same prompt through the seeded HBM engine (fill_seeded bits = checkpoint bits)
    _, _, resident, runtime = hbm_engine
    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=10)
    want, token = [], prompt
    with torch.inference_mode():
        for _ in range(NEW_TOKENS):
            state = executor.finish(runtime.run(executor, executor.begin(token)))
            token = state.topk_indices[..., 0]
            want.append(int(token.reshape(-1)[0]))
    assert ids == want
