"""Layout contract: the reference's own plan tests (tests/test_plan.py:11-95)
plus SHA-256 pins of every plan the reference builds (tests/golden/plan_layouts.json)."""

import hashlib
import json

import pytest

from conftest import golden_path
from layer_streaming.plan import MIB, Granularity, build_llama31_8b_plan


def sha(obj):
    return hashlib.sha256(json.dumps(obj, sort_keys=True).encode()).hexdigest()


def test_matrix_is_default_and_uses_largest_projection():
    plan = build_llama31_8b_plan()
    assert plan.granularity == Granularity.MATRIX
    assert len(plan.units) == 32 * 7
    assert plan.slot_bytes == 112 * MIB
    assert plan.two_slot_bytes == 224 * MIB
    assert plan.stream_bytes_per_token == 32 * 416 * MIB


def test_layer_plan_allocates_two_whole_layer_slots():
    plan = build_llama31_8b_plan("layer")
    assert len(plan.units) == 32
    assert plan.slot_bytes == 416 * MIB
    assert plan.two_slot_bytes == 832 * MIB


def test_matrix_group_uses_four_whole_matrix_groups_per_layer():
    plan = build_llama31_8b_plan("matrix_group")
    assert plan.granularity == Granularity.MATRIX_GROUP
    assert len(plan.units) == 32 * 4
    assert [u.operation for u in plan.units[:4]] == ["qkv", "o_proj", "gate_up", "down_proj"]
    assert plan.slot_bytes == 224 * MIB
    assert plan.two_slot_bytes == 448 * MIB


def test_separate_embedding_and_head_are_resident():
    plan = build_llama31_8b_plan("matrix")
    keys = {p.tensor.key for p in plan.resident}
    assert "model.embed_tokens.weight" in keys and "lm_head.weight" in keys
    assert plan.resident_bytes == int(2004.5078125 * MIB)
    assert plan.aliases == {}


def test_tied_head_alias_does_not_duplicate_gpu_memory():
    untied = build_llama31_8b_plan("matrix", tie_word_embeddings=False)
    tied = build_llama31_8b_plan("matrix", tie_word_embeddings=True)
    assert tied.aliases["lm_head.weight"] == "model.embed_tokens.weight"
    assert untied.resident_bytes - tied.resident_bytes == 1002 * MIB


def test_matrix_plan_saves_608_mib_of_device_slots():
    layer = build_llama31_8b_plan("layer")
    matrix = build_llama31_8b_plan("matrix")
    assert layer.two_slot_bytes - matrix.two_slot_bytes == 608 * MIB
    assert 1.0 - matrix.two_slot_bytes / layer.two_slot_bytes == pytest.approx(0.7307692307692308)


def test_streamed_vocab_is_cpu_only_and_uses_128_mib_chunks():
    plan = build_llama31_8b_plan("matrix", stream_vocab=True)
    resident = {p.tensor.key for p in plan.resident}
    host_only = {p.tensor.key for p in plan.host_only}
    assert "model.embed_tokens.weight" not in resident and "lm_head.weight" not in resident
    assert host_only == {"model.embed_tokens.weight", "lm_head.weight"}
    assert plan.resident_bytes == 532480
    assert plan.vocab.chunk_bytes == 128 * MIB
    assert plan.vocab.chunk_rows == 16384
    assert plan.vocab.chunk_count == 8
    assert plan.slot_bytes == 128 * MIB
    assert plan.two_slot_bytes == 256 * MIB
    assert plan.host_arena_bytes == 16060522496
    assert plan.vocab.chunk_range(7) == (114688, 128256)


@pytest.mark.parametrize("gran", ["matrix", "matrix_group", "layer"])
@pytest.mark.parametrize("stream", [False, True])
@pytest.mark.parametrize("tied", [False, True])
def test_layout_is_byte_identical_to_reference(gran, stream, tied):
    golden = json.load(open(golden_path("plan_layouts.json")))
    name = "{}|stream={}|tied={}".format(gran, int(stream), int(tied))
    plan = build_llama31_8b_plan(gran, tie_word_embeddings=tied, stream_vocab=stream)
    offsets = {k: plan.tensor_host_offset(k) for k in sorted(plan.tensors)}
    assert sha(plan.as_dict()) == golden[name]["as_dict_sha256"]
    assert sha(offsets) == golden[name]["offsets_sha256"]
    assert plan.host_arena_bytes == golden[name]["host_arena_bytes"]


def test_unknown_tensor_raises():
    with pytest.raises(KeyError):
        build_llama31_8b_plan().tensor_host_offset("model.layers.99.bogus")
    with pytest.raises(ValueError):
        build_llama31_8b_plan(stream_vocab=True, vocab_chunk_bytes=100)


@pytest.mark.parametrize("kv_heads", [8, 4, 2, 1])
def test_attention_split_policy(kv_heads):
    """The split-KV layout covers every position with chunks of whole 64-position
    sub-chunks and targets about two CTAs per SM (148 SMs), within the kernel's
    grid limits and the allocation-free entry point's one-token capacity."""

    from layer_streaming.llama31 import attention_split

    sms = 148
    for tokens in (1, 2, 6):
        for length in (1, 63, 64, 65, 2048, 2049, 4096, 8192, 32768, 131072):
            splits, chunk = attention_split(tokens, length, sms, kv_heads=kv_heads)
            assert chunk >= 64 and chunk % 64 == 0
            assert splits * chunk >= length and (splits - 1) * chunk < length  # no empty split
            assert 1 <= splits <= 65535
            ctas = splits * kv_heads * tokens
            assert ctas <= max(2 * sms, kv_heads * tokens) or chunk == 64
            if tokens == 1 and kv_heads == 8:
                assert splits <= 252  # cb_attention_noalloc holds 252 one-token splits
