"""Shared test set-up: import paths, the `gpu` marker and common fixtures.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host
logic, ABI loading); `-m gpu` runs the CUDA parity tests on a B200.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "cascade-llm_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for path in (REPO, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: regenerates the full 8B seeded model on the CPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA GPU (run the gpu tests on a B200)")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def golden_path(name):
    return os.path.join(GOLDEN, name)


class Config:
    """Llama-3.1-8B config fields the executor reads (AutoConfig stand-in)."""

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


@pytest.fixture(scope="session")
def meta():
    import json

    with open(golden_path("config0.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def arena(cuda, meta):
    """One pinned, seeded host arena shared by every model test (its layout
    is the same for every plan granularity)."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group")
    store = ls.create_weight_store(plan, "full_pinned")
    store.fill_seeded(seed=meta["weight_seed"], device=cuda)
    return store


def make_store(arena, plan, mode="full_pinned"):
    """A store of `plan` over the shared arena, through the stores'
    tensor_factory seam (the arena request returns the shared tensor)."""

    import torch

    import layer_streaming as ls

    assert plan.host_arena_elements == arena.plan.host_arena_elements

    def factory(elements, dtype=None, device=None, pin_memory=False):
        if elements == plan.host_arena_elements:
            return arena.arena
        return torch.empty(elements, dtype=dtype, device=device, pin_memory=pin_memory)

    return ls.create_weight_store(plan, mode, tensor_factory=factory)


@pytest.fixture(scope="session")
def hbm_engine(cuda, arena):
    """matrix_group plan with every unit resident in HBM (the bench's mode)."""

    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group")
    store = make_store(arena, plan)
    resident = ls.ResidentDeviceArena(plan, store, cuda)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, cuda, weights="hbm")
    return plan, store, resident, runtime


def engine_weights(hbm_engine):
    """{reference tensor name: device view} of the resident engine (the
    oracle runs the reference's torch ops over the same device weights)."""

    plan, _, resident, runtime = hbm_engine
    weights = dict(resident.views)
    for index in range(len(plan.units)):
        weights.update(runtime.unit_views(index))
    return weights
