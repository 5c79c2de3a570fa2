#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/Cascade-LLM [--skip-model]

It imports the reference's own ``layer_streaming`` package (never this
repository's engine) and records what it computes:

* ``plan_layouts.json``  - ``build_llama31_8b_plan`` for every granularity /
  vocab mode / tie combination: SHA-256 of ``as_dict()`` and of every
  ``tensor_host_offset``, plus the headline numbers (layer_streaming/plan.py).
* ``merge_topk.json``    - ``merge_topk`` on chunked random vectors
  (layer_streaming/vocab.py:11-32).
* ``ops.safetensors``    - ``_rms_norm`` (llama31.py:21-25), the executor's
  RoPE cos/sin (llama31.py:206-212) and ``_attention_output`` for a causal
  6-, 36- and 64-token prefill followed by 1-token decode steps
  (llama31.py:182-234), on seeded inputs.
* ``config0.safetensors`` / ``config0.json``: the full
  Llama-3.1-8B geometry with seeded random-init weights (the oracle's
  generator, oracle/seeded_init.c), a 6-token seeded prompt, prefill plus
  8 greedy decode steps through ``Llama31DecodeExecutor`` on the CPU
  (resident vocabulary), driven unit by unit over the matrix_group plan the
  way ``DoubleBufferRuntime.run`` does (runtime.py:185-230).

The weights themselves are not stored: tests regenerate them from the seed.
"""

import argparse
import hashlib
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

WEIGHT_SEED = 0
PROMPT_SEED = 1
PROMPT_LEN = 6
DECODE_STEPS = 8
TOP_K = 10


def sha(obj):
    return hashlib.sha256(json.dumps(obj, sort_keys=True).encode()).hexdigest()


def llama_config():
    from transformers import LlamaConfig

    return LlamaConfig(
        hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=8, vocab_size=128256,
        rms_norm_eps=1e-5, max_position_embeddings=131072, rope_theta=500000.0,
        rope_scaling={
            "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
            "high_freq_factor": 4.0, "original_max_position_embeddings": 8192,
        },
        tie_word_embeddings=False,
    )


class CpuResident(dict):
    """Dict-like stand-in for ResidentDeviceArena on the CPU."""

    device = torch.device("cpu")


def seeded(shape, name, std=1.0, mean=0.0):
    from oracle.seeded import seeded as oracle_seeded

    return oracle_seeded(shape, name, std=std, mean=mean, seed=WEIGHT_SEED)


def make_plans(ls):
    out = {}
    for gran in ("matrix", "matrix_group", "layer"):
        for stream in (False, True):
            for tied in (False, True):
                plan = ls.build_llama31_8b_plan(gran, tie_word_embeddings=tied, stream_vocab=stream)
                offsets = {k: plan.tensor_host_offset(k) for k in sorted(plan.tensors)}
                name = "{}|stream={}|tied={}".format(gran, int(stream), int(tied))
                out[name] = {
                    "as_dict_sha256": sha(plan.as_dict()),
                    "offsets_sha256": sha(offsets),
                    "units": len(plan.units),
                    "slot_bytes": plan.slot_bytes,
                    "two_slot_bytes": plan.two_slot_bytes,
                    "stream_bytes_per_token": plan.stream_bytes_per_token,
                    "resident_bytes": plan.resident_bytes,
                    "host_arena_bytes": plan.host_arena_bytes,
                    "first_unit": plan.as_dict()["units"][0],
                    "last_unit": plan.as_dict()["units"][-1],
                    "resident_head": plan.as_dict()["resident"][:3],
                    "host_only": plan.as_dict()["host_only"],
                    "vocab": plan.as_dict()["vocab"],
                }
    return out


def make_merge_cases(ls):
    cases = []
    logits = [-2.0, 7.0, 1.0, 3.0, 9.0, -1.0, 8.0, 4.0]
    cases.append({"logits": logits, "chunk": 3, "k": 3})
    gen = torch.Generator().manual_seed(7)
    for n, chunk, k in ((1000, 128, 10), (4099, 1000, 10), (300, 300, 1), (64, 7, 20)):
        values = torch.randn(n, generator=gen).to(torch.bfloat16).float()
        cases.append({"logits": values.tolist(), "chunk": chunk, "k": k})
    for case in cases:
        row = torch.tensor([[case["logits"]]])
        vals = idx = None
        for start in range(0, row.shape[-1], case["chunk"]):
            part = row[..., start:start + case["chunk"]]
            lv, li = torch.topk(part, k=min(case["k"], part.shape[-1]), dim=-1)
            vals, idx = ls.merge_topk(vals, idx, lv, li + start, case["k"])
        case["values"] = vals.reshape(-1).tolist()
        case["indices"] = idx.reshape(-1).tolist()
    return cases


def make_ops(ls, config):
    from layer_streaming.llama31 import DecodeState, Llama31DecodeExecutor, _rms_norm

    tensors = {}
    x = seeded((3, 4096), "golden.rms.x")
    w = seeded((4096,), "golden.rms.w", std=0.1, mean=1.0)
    tensors["rms.out"] = _rms_norm(x, w, 1e-5)

    executor = Llama31DecodeExecutor(config, CpuResident())
    positions = torch.tensor([[0, 1, 2, 5, 100, 2047, 8191, 8192, 32767, 131071]])
    cos, sin = executor.rotary(torch.empty(1, dtype=torch.bfloat16), positions)
    tensors["rope.positions"], tensors["rope.cos"], tensors["rope.sin"] = positions, cos[0], sin[0]

    def attention_call(length, position_start, keep_cache=False):
        state = DecodeState(
            hidden_states=torch.empty(1, length, 4096, dtype=torch.bfloat16),
            position_ids=torch.arange(position_start, position_start + length).unsqueeze(0),
        )
        tag = "attn.L{}at{}".format(length, position_start)
        q = seeded((1, length, 4096), tag + ".q")
        k = seeded((1, length, 1024), tag + ".k")
        v = seeded((1, length, 1024), tag + ".v")
        state.layer_values = {"q": q, "k": k, "v": v}
        out = executor._attention_output(0, state)
        tensors[tag + ".out"] = out
        if keep_cache:
            key, value = executor.kv_cache.entries[0]
            tensors[tag + ".cache_k"] = key.contiguous()
            tensors[tag + ".cache_v"] = value.contiguous()

    # inputs are seeded (regenerated by the tests); only outputs are stored
    attention_call(6, 0, keep_cache=True)   # causal prefill on an empty cache
    executor.kv_cache.clear()
    attention_call(36, 0)                   # prefill 36 positions, then one decode step
    attention_call(1, 36, keep_cache=True)
    executor.kv_cache.clear()
    attention_call(64, 0)                   # prefill 64, then two decode steps
    attention_call(1, 64)
    attention_call(1, 65, keep_cache=True)
    return tensors


def weight_fingerprint(tensor_of):
    """SHA-256 of a few slices of the seeded weights (checks regeneration)."""

    slices = {
        "model.embed_tokens.weight": lambda t: t[:4],
        "model.layers.0.self_attn.q_proj.weight": lambda t: t.reshape(-1)[:65536],
        "model.layers.31.mlp.down_proj.weight": lambda t: t.reshape(-1)[-65536:],
        "lm_head.weight": lambda t: t[-1:],
    }
    return {
        key: hashlib.sha256(cut(tensor_of(key)).contiguous().view(torch.int16).numpy().tobytes()).hexdigest()
        for key, cut in slices.items()
    }


def fill_seeded_weights(plan, tensor_of):
    """Seeded random init of every non-alias tensor: N(0, 0.02), norms = 1."""

    from oracle.seeded import fill_model

    fill_model([k for k, s in plan.tensors.items() if s.alias_of is None], tensor_of, seed=WEIGHT_SEED)


def make_config0(ls, config):
    from layer_streaming.llama31 import Llama31DecodeExecutor, _rms_norm

    plan = ls.build_llama31_8b_plan("matrix_group", stream_vocab=False)

    def unpinned(elements, **kwargs):
        kwargs.pop("pin_memory", None)
        return torch.empty(elements, **kwargs)

    store = ls.FullPinnedWeightStore(plan, tensor_factory=unpinned)
    started = time.time()
    fill_seeded_weights(plan, store.tensor)
    print("weights filled in {:.1f}s".format(time.time() - started), flush=True)
    resident = CpuResident({p.tensor.key: store.tensor(p.tensor.key) for p in plan.resident})
    executor = Llama31DecodeExecutor(config, resident, top_k=TOP_K)
    from oracle.seeded import prompt_ids

    prompt = prompt_ids(PROMPT_LEN, seed=PROMPT_SEED)
    ids = prompt.view(1, -1)
    tensors, steps = {}, []
    with torch.inference_mode():
        for step in range(1 + DECODE_STEPS):
            started = time.time()
            state = executor.begin(ids)
            for unit in plan.units:
                source = store.unit_source(unit)
                views = {
                    piece.tensor.key: source[
                        piece.unit_offset_elements:piece.unit_offset_elements + piece.tensor.numel
                    ].view(piece.tensor.shape)
                    for piece in unit.pieces
                }
                state = executor(unit, views, state)
            hidden = state.hidden_states
            state = executor.finish(state)
            last = state.logits[0, -1]
            tensors["step{}.logits".format(step)] = last.to(torch.bfloat16)
            tensors["step{}.hidden".format(step)] = hidden[0, -1].contiguous()
            # the streamed-vocabulary head (vocab.py:239-261) on the same hidden state
            normed = _rms_norm(hidden, resident["model.norm.weight"], 1e-5)[:, -1:, :]
            sv = si = None
            head = resident["lm_head.weight"]
            for start in range(0, 128256, 16384):
                part = torch.nn.functional.linear(normed, head[start:start + 16384]).float()
                lv, li = torch.topk(part, k=TOP_K, dim=-1)
                sv, si = ls.merge_topk(sv, si, lv, li + start, TOP_K)
            sorted_logits = torch.sort(last, descending=True).values
            steps.append({
                "input_ids": ids.reshape(-1).tolist(),
                "topk_values": state.topk_values.reshape(-1).tolist(),
                "topk_indices": state.topk_indices.reshape(-1).tolist(),
                "streamed_topk_values": sv.reshape(-1).tolist(),
                "streamed_topk_indices": si.reshape(-1).tolist(),
                "top1_top2_gap": float(sorted_logits[0] - sorted_logits[1]),
                "k_k1_gap": float(sorted_logits[TOP_K - 1] - sorted_logits[TOP_K]),
                "seconds": time.time() - started,
            })
            print("step", step, steps[-1]["topk_indices"][:3], "{:.2f}s".format(steps[-1]["seconds"]), flush=True)
            ids = state.topk_indices[..., 0]
    meta = {
        "weight_seed": WEIGHT_SEED,
        "prompt_seed": PROMPT_SEED,
        "prompt_ids": prompt.tolist(),
        "top_k": TOP_K,
        "decode_steps": DECODE_STEPS,
        "greedy_ids": [s["topk_indices"][0] for s in steps],
        "steps": steps,
        "weight_fingerprint": weight_fingerprint(store.tensor),
        "torch": torch.__version__,
        "threads": torch.get_num_threads(),
        "plan": "matrix_group, resident vocabulary",
    }
    return tensors, meta


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    parser.add_argument("--skip-model", action="store_true")
    args = parser.parse_args()
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.abspath(args.reference))
    import layer_streaming as ls
    from safetensors.torch import save_file

    if not os.path.abspath(ls.__file__).startswith(os.path.abspath(args.reference)):
        raise SystemExit("imported the wrong layer_streaming: " + ls.__file__)
    config = llama_config()
    with open(os.path.join(HERE, "plan_layouts.json"), "w") as out:
        json.dump(make_plans(ls), out, indent=1, sort_keys=True)
    with open(os.path.join(HERE, "merge_topk.json"), "w") as out:
        json.dump(make_merge_cases(ls), out)
    save_file(make_ops(ls, config), os.path.join(HERE, "ops.safetensors"))
    if not args.skip_model:
        tensors, meta = make_config0(ls, config)
        save_file(tensors, os.path.join(HERE, "config0.safetensors"))
        with open(os.path.join(HERE, "config0.json"), "w") as out:
            json.dump(meta, out, indent=1)


if __name__ == "__main__":
    main()
