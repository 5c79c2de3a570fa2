"""Seeded inputs and weights shared by the golden generator and the tests
(TEST INFRASTRUCTURE ONLY).

``seeded(shape, name)`` is element-for-element the engine's
``cb_fill_normal_bf16`` stream ``stream_key(seed, name)``; ``fill_model`` writes
the random-init Llama-3.1-8B of the benchmark configurations (matrices
N(0, 0.02), norm weights 1) into any mapping of bf16 CPU tensors.
"""

import torch

from . import native

WEIGHT_SEED = 0
PROMPT_SEED = 1


def seeded(shape, name, std=1.0, mean=0.0, seed=WEIGHT_SEED):
    n = 1
    for s in shape:
        n *= int(s)
    out = torch.empty(n, dtype=torch.bfloat16)
    native.fill_normal_bf16(out, native.stream_key(seed, name), std=std)
    out = out.view(*shape)
    if mean:
        out = (out.float() + mean).to(torch.bfloat16)
    return out


def is_norm(key):
    return key.endswith("layernorm.weight") or key == "model.norm.weight"


def fill_model(keys, tensor_of, seed=WEIGHT_SEED, std=0.02):
    for key in keys:
        target = tensor_of(key)
        if is_norm(key):
            target.fill_(1.0)
        else:
            native.fill_normal_bf16(target.view(-1), native.stream_key(seed, key), std=std)


def prompt_ids(length=6, seed=PROMPT_SEED, vocab=128256):
    return native.uniform_ids(length, native.stream_key(seed, "prompt"), vocab)
