"""Checkpoint writer / loader and the native host I/O (CPU, except the last test).

* ``cb_host_copy`` and ``cb_read_file_ranges`` move bytes exactly, across
  task boundaries and thread counts;
* ``write_safetensors`` files read back with the ``safetensors`` library, and
  ``load_safetensors_into`` fills preallocated tensors (BF16 direct, F32
  converted);
* the tokenizer stand-in and ``config.json`` load with ``AutoTokenizer`` /
  ``AutoConfig`` as the reference's CLI loads them (``tools/run_llama31.py``);
* on a GPU: a seeded checkpoint written by ``write_seeded_checkpoint`` loads
  back bit-identical to ``fill_seeded``'s arena.
"""

import ctypes
import json

import numpy as np
import pytest
import torch

from layer_streaming import _native
from layer_streaming import checkpoint as ck


def test_host_copy_exact_for_any_thread_count():
    lib = _native.load_library()
    rng = np.random.default_rng(1)
    src = rng.integers(0, 256, size=(20 << 20) + 12345, dtype=np.uint8)
    for threads in (1, 3, 0):
        dst = np.zeros_like(src)
        assert lib.cb_host_copy(dst.ctypes.data, src.ctypes.data, src.size, threads) == 0
        assert np.array_equal(dst, src)
    assert lib.cb_host_copy(None, None, 5, 1) != 0


def test_read_file_ranges_exact(tmp_path):
    lib = _native.load_library()
    rng = np.random.default_rng(2)
    data = rng.integers(0, 256, size=3_000_001, dtype=np.uint8)
    path = tmp_path / "blob.bin"
    data.tofile(path)
    ranges = [(0, 17), (100, 1_000_000), (2_999_000, 1001), (5, 0)]
    outs = [np.zeros(size, dtype=np.uint8) for _, size in ranges]
    n = len(ranges)
    rc = lib.cb_read_file_ranges(
        str(path).encode(), n, (ctypes.c_int64 * n)(*[o for o, _ in ranges]),
        (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs]), (ctypes.c_int64 * n)(*[s for _, s in ranges]), 4)
    assert rc == 0
    for (offset, size), out in zip(ranges, outs):
        assert np.array_equal(out, data[offset:offset + size])
    # past the end of the file: an error, not a hang or a partial success
    short = np.zeros(10, dtype=np.uint8)
    rc = lib.cb_read_file_ranges(str(path).encode(), 1, (ctypes.c_int64 * 1)(2_999_995),
                                 (ctypes.c_void_p * 1)(short.ctypes.data), (ctypes.c_int64 * 1)(10), 1)
    assert rc != 0
    assert lib.cb_read_file_ranges(str(tmp_path / "missing").encode(), 1, (ctypes.c_int64 * 1)(0),
                                   (ctypes.c_void_p * 1)(short.ctypes.data), (ctypes.c_int64 * 1)(1), 1) != 0


def test_safetensors_writer_and_parallel_reader(tmp_path):
    from safetensors import safe_open

    gen = torch.Generator().manual_seed(3)
    a = torch.randn((33, 17), generator=gen).to(torch.bfloat16)
    b = torch.randn(5, generator=gen)
    path = tmp_path / "x.safetensors"
    ck.write_safetensors(path, [("a.weight", a.shape, torch.bfloat16, lambda: a),
                                ("b.weight", b.shape, torch.float32, lambda: b)])
    with safe_open(str(path), framework="pt") as source:
        assert torch.equal(source.get_tensor("a.weight"), a)
        assert torch.equal(source.get_tensor("b.weight"), b)
    targets = {"a.weight": torch.zeros((33, 17), dtype=torch.bfloat16),
               "b.weight": torch.zeros(5, dtype=torch.bfloat16)}
    loaded = ck.load_safetensors_into({"a.weight": path, "b.weight": path}, targets, threads=2)
    assert loaded == {"a.weight", "b.weight"}
    assert torch.equal(targets["a.weight"], a)
    assert torch.equal(targets["b.weight"], b.to(torch.bfloat16))
    with pytest.raises(ValueError):
        ck.load_safetensors_into({"a.weight": path}, {"a.weight": torch.zeros((17, 33), dtype=torch.bfloat16)})


def test_tokenizer_and_config_load_like_the_reference_cli(tmp_path):
    from transformers import AutoConfig, AutoTokenizer

    ck.write_tokenizer(tmp_path)
    (tmp_path / "config.json").write_text(json.dumps(ck.llama31_8b_config_dict()))
    config = AutoConfig.from_pretrained(tmp_path, local_files_only=True)
    for name, value in (("hidden_size", 4096), ("intermediate_size", 14336), ("num_hidden_layers", 32),
                        ("num_attention_heads", 32), ("num_key_value_heads", 8), ("vocab_size", 128256)):
        assert getattr(config, name) == value
    assert not config.tie_word_embeddings
    tokenizer = AutoTokenizer.from_pretrained(tmp_path, local_files_only=True)
    text = "The meaning of life is"
    ids = tokenizer(text, return_tensors="pt", add_special_tokens=True).input_ids
    assert ids[0, 0].item() == ck.BOS_ID and ids.shape[1] == 1 + len(text.encode())
    assert int(ids.max()) < ck.VOCAB
    assert tokenizer.decode(ids[0], skip_special_tokens=True) == text
    assert tokenizer.decode([115650, 98334]) != ""  # any model output id decodes
    # the engine's executor accepts the config (the reference CLI passes it through)
    from layer_streaming.llama31 import llama3_inv_freq

    assert llama3_inv_freq(config).shape == (64,)


@pytest.mark.gpu
def test_seeded_checkpoint_round_trip(cuda, tmp_path):
    """A small plan written by the seeded writer loads back bit-identical to
    fill_seeded (the 8B plan is the same code over larger shapes)."""

    from layer_streaming.plan import TensorSpec, build_llama31_8b_plan

    full = build_llama31_8b_plan("matrix_group")
    # keep the norms and two matrices of the real plan's keys, at reduced size
    keep = ["model.norm.weight", "model.layers.0.input_layernorm.weight",
            "model.layers.0.self_attn.k_proj.weight", "model.layers.0.mlp.down_proj.weight"]
    assert all(k in full.tensors for k in keep)
    writer_plan = type("P", (), {})()
    writer_plan.tensors = {k: TensorSpec(k, (4096,) if "norm" in k else (256, 4096 if "k_proj" in k else 1024))
                           for k in keep}
    ck.write_seeded_checkpoint(tmp_path, seed=7, shard_bytes=1 << 20, device=cuda, plan=writer_plan)
    index = json.loads((tmp_path / "model.safetensors.index.json").read_text())
    assert set(index["weight_map"]) == set(keep)
    targets = {k: torch.empty(s.shape, dtype=torch.bfloat16) for k, s in writer_plan.tensors.items()}
    files = {k: tmp_path / name for k, name in index["weight_map"].items()}
    assert ck.load_safetensors_into(files, targets) == set(keep)
    from layer_streaming import ops

    for key, tensor in targets.items():
        want = torch.empty(tensor.shape, dtype=torch.bfloat16, device=cuda)
        if "norm" in key:
            want.fill_(1.0)
        else:
            ops.fill_normal_(want, _native.stream_key(7, key), std=0.02)
        assert torch.equal(tensor, want.cpu()), key
