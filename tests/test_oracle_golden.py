"""Pins the oracle to the reference: every restatement in oracle/ reproduces
the vectors that tests/golden/make_golden.py recorded from the reference's
own layer_streaming code (CPU, bit-exact where the same torch CPU ops run)."""

import json
import os

import numpy as np
import pytest
import torch
from safetensors.torch import load_file

from conftest import golden_path
from oracle import llama_oracle as lo
from oracle import native
from oracle.seeded import fill_model, prompt_ids, seeded


@pytest.fixture(scope="module")
def ops_golden():
    return load_file(golden_path("ops.safetensors"))


def test_rms_norm_matches_reference(ops_golden):
    x = seeded((3, 4096), "golden.rms.x")
    w = seeded((4096,), "golden.rms.w", std=0.1, mean=1.0)
    assert torch.equal(lo.rms_norm(x, w), ops_golden["rms.out"])


def test_rope_tables_match_reference(ops_golden):
    positions = ops_golden["rope.positions"]
    cos, sin = lo.rope_cos_sin(positions, lo.llama3_inv_freq())
    assert torch.equal(cos[0], ops_golden["rope.cos"])
    assert torch.equal(sin[0], ops_golden["rope.sin"])


def _attention_chain(calls):
    """Re-run the reference's attention calls (RoPE, cache append, SDPA)."""

    inv = lo.llama3_inv_freq()
    cache = None
    outs = {}
    for length, start in calls:
        tag = "attn.L{}at{}".format(length, start)
        q = seeded((1, length, 4096), tag + ".q").view(1, length, 32, 128).transpose(1, 2)
        k = seeded((1, length, 1024), tag + ".k").view(1, length, 8, 128).transpose(1, 2)
        v = seeded((1, length, 1024), tag + ".v").view(1, length, 8, 128).transpose(1, 2)
        cos, sin = lo.rope_cos_sin(torch.arange(start, start + length).unsqueeze(0), inv)
        q, k = lo.apply_rope(q, k, cos, sin)
        had_past = cache is not None
        if had_past:
            k = torch.cat((cache[0], k), dim=-2)
            v = torch.cat((cache[1], v), dim=-2)
        cache = (k, v)
        outs[tag] = (lo.attention(q, k, v, causal=not had_past and length > 1), cache)
    return outs


@pytest.mark.parametrize("calls", [[(6, 0)], [(36, 0), (1, 36)], [(64, 0), (1, 64), (1, 65)]])
def test_attention_matches_reference(ops_golden, calls):
    for tag, (out, cache) in _attention_chain(calls).items():
        assert torch.equal(out, ops_golden[tag + ".out"]), tag
        if tag + ".cache_k" in ops_golden:
            assert torch.equal(cache[0].contiguous(), ops_golden[tag + ".cache_k"])
            assert torch.equal(cache[1].contiguous(), ops_golden[tag + ".cache_v"])


def test_merge_topk_restatements_match_reference():
    for case in json.load(open(golden_path("merge_topk.json"))):
        logits = torch.tensor([[case["logits"]]])
        values = indices = None
        for start in range(0, logits.shape[-1], case["chunk"]):
            part = logits[..., start:start + case["chunk"]]
            lv, li = torch.topk(part, k=min(case["k"], part.shape[-1]), dim=-1)
            values, indices = lo.merge_topk(values, indices, lv, li + start, case["k"])
        assert values.reshape(-1).tolist() == case["values"]
        # the C oracle: same values; indices equal wherever values are distinct
        cv, ci = native.topk(np.array(case["logits"], dtype=np.float32), case["k"])
        assert cv.tolist() == case["values"]
        for value in set(case["values"]):
            got = sorted(i for i, v in zip(ci.tolist(), cv.tolist()) if v == value)
            ref = sorted(i for i, v in zip(case["indices"], case["values"]) if v == value)
            if case["values"].count(value) == sum(1 for x in case["logits"] if x == value):
                assert got == ref  # every tied copy is inside the top-k: same set


def test_c_topk_breaks_ties_by_index():
    values, indices = native.topk([1.0, 3.0, 3.0, 2.0, 3.0, 0.5, 3.0, 2.0], 5)
    assert values.tolist() == [3.0, 3.0, 3.0, 3.0, 2.0]
    assert indices.tolist() == [1, 2, 4, 6, 3]


def test_generator_is_offset_consistent():
    key = native.stream_key(0, "some.tensor")
    full = torch.empty(4099, dtype=torch.bfloat16)
    native.fill_normal_bf16(full, key)
    part = torch.empty(1000, dtype=torch.bfloat16)
    native.fill_normal_bf16(part, key, offset=1001)
    assert torch.equal(part, full[1001:2001])
    big = torch.empty(3_000_001, dtype=torch.bfloat16)
    native.fill_normal_bf16(big, key)  # threaded path
    assert torch.equal(big[:4099], full)
    assert abs(float(big.float().std()) - 0.02) < 2e-4


def _enough_memory(gib):
    try:
        pages = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    except (ValueError, OSError):
        return True
    return pages >= gib * (1 << 30)


@pytest.mark.slow
def test_config0_oracle_reproduces_reference_run():
    """BASELINE config 0 end to end on the CPU: seeded 8B weights, 6-token
    prompt, prefill + 8 greedy steps; top-k and logits equal the reference's."""

    if not _enough_memory(20):
        pytest.skip("needs ~20 GiB of free host memory")
    meta = json.load(open(golden_path("config0.json")))
    golden = load_file(golden_path("config0.safetensors"))
    from layer_streaming.plan import build_llama31_8b_plan

    plan = build_llama31_8b_plan("matrix_group")
    weights = {k: torch.empty(s.shape, dtype=torch.bfloat16) for k, s in plan.tensors.items()}
    fill_model(sorted(weights), weights.__getitem__, seed=meta["weight_seed"])
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1)
    assert ids.reshape(-1).tolist() == meta["prompt_ids"]
    decoder = lo.OracleDecoder(weights, top_k=meta["top_k"])
    with torch.inference_mode():
        for step, record in enumerate(meta["steps"]):
            result = decoder.step(ids)
            assert result["values"].reshape(-1).tolist() == record["topk_values"]
            assert torch.equal(result["logits"][0, -1].to(torch.bfloat16), golden["step{}.logits".format(step)])
            assert int(result["indices"].reshape(-1)[0]) == meta["greedy_ids"][step]
            ids = result["indices"][..., 0]
