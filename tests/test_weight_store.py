"""Host arena: the reference's store tests (tests/test_weight_store.py:67-108)
with its GPU-less seams (tensor_factory, fake events), plus checkpoint loading
and host-side failure detection (missing tensors, shape mismatches)."""

import json

import pytest
import torch

from layer_streaming.plan import ModelPlan, ResidentPlacement, TensorSpec, TransferUnit, UnitPiece
from layer_streaming.weight_store import (
    FullPinnedWeightStore,
    PinnedStagingWeightStore,
    WeightStoreMode,
    create_weight_store,
)


def tiny_plan():
    streamed = TensorSpec("stream.weight", (2, 2))
    resident = TensorSpec("resident.weight", (2,), resident=True)
    unit = TransferUnit("unit", 0, "q_proj", (UnitPiece(streamed, 0),), 4, 0)
    return ModelPlan(
        model_id="tiny",
        granularity="matrix",
        tensors={streamed.key: streamed, resident.key: resident},
        units=(unit,),
        resident=(ResidentPlacement(resident, 4, 0),),
        aliases={},
        host_arena_elements=6,
        resident_arena_elements=2,
        slot_elements=4,
    )


class RecordingFactory:
    def __init__(self):
        self.pin_flags = []

    def __call__(self, elements, **kwargs):
        self.pin_flags.append(bool(kwargs.pop("pin_memory")))
        return torch.empty(elements, **kwargs)


class FakeEvent:
    def __init__(self):
        self.synchronized = False

    def synchronize(self):
        self.synchronized = True


def test_full_pinned_requests_one_pinned_arena():
    factory = RecordingFactory()
    store = FullPinnedWeightStore(tiny_plan(), tensor_factory=factory)
    assert factory.pin_flags == [True]
    assert store.pinned_cpu_bytes == 12
    assert store.mode == WeightStoreMode.FULL_PINNED
    store.close()


def test_staging_has_pageable_store_and_two_pinned_slots():
    factory = RecordingFactory()
    plan = tiny_plan()
    store = PinnedStagingWeightStore(plan, tensor_factory=factory)
    assert factory.pin_flags == [False, True, True]
    assert store.pinned_cpu_bytes == plan.two_slot_bytes
    store.close()


def test_staging_copies_unit_and_waits_before_reuse():
    plan = tiny_plan()
    store = PinnedStagingWeightStore(plan, tensor_factory=RecordingFactory())
    store.arena[:4] = torch.tensor([1.0, 2.0, 3.0, 4.0], dtype=torch.bfloat16)
    event = FakeEvent()
    staged = store.prepare_unit(plan.units[0], 0, reuse_event=event).result()
    assert event.synchronized
    assert staged.float().tolist() == [1.0, 2.0, 3.0, 4.0]
    assert store.profile_stats()["staging_copy_count"] == 1
    store.close()


def test_full_pinned_prepare_returns_arena_view():
    plan = tiny_plan()
    store = create_weight_store(plan, "full_pinned", tensor_factory=RecordingFactory())
    store.arena[:4] = torch.tensor([5.0, 6.0, 7.0, 8.0], dtype=torch.bfloat16)
    view = store.prepare_unit(plan.units[0], 0).result()
    assert view.data_ptr() == store.arena.data_ptr()
    assert store.tensor("stream.weight").shape == (2, 2)


def _unpinned(elements, **kwargs):
    kwargs.pop("pin_memory", None)
    return torch.empty(elements, **kwargs)


def test_load_checkpoint_single_file_and_index(tmp_path):
    from safetensors.torch import save_file

    plan = tiny_plan()
    tensors = {"stream.weight": torch.arange(4.0).view(2, 2), "resident.weight": torch.tensor([9.0, 10.0])}
    save_file(tensors, str(tmp_path / "model.safetensors"))
    store = FullPinnedWeightStore(plan, tensor_factory=_unpinned).load_checkpoint(tmp_path)
    assert store.loaded
    assert store.arena.float().tolist() == [0.0, 1.0, 2.0, 3.0, 9.0, 10.0]

    sharded = tmp_path / "sharded"
    sharded.mkdir()
    save_file({"stream.weight": tensors["stream.weight"]}, str(sharded / "a.safetensors"))
    save_file({"resident.weight": tensors["resident.weight"]}, str(sharded / "b.safetensors"))
    (sharded / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {"stream.weight": "a.safetensors", "resident.weight": "b.safetensors"}})
    )
    store = FullPinnedWeightStore(plan, tensor_factory=_unpinned).load_checkpoint(sharded)
    assert store.arena.float().tolist() == [0.0, 1.0, 2.0, 3.0, 9.0, 10.0]


def test_load_checkpoint_rejects_missing_and_misshapen(tmp_path):
    from safetensors.torch import save_file

    plan = tiny_plan()
    save_file({"stream.weight": torch.zeros(2, 2)}, str(tmp_path / "model.safetensors"))
    with pytest.raises(KeyError):
        FullPinnedWeightStore(plan, tensor_factory=_unpinned).load_checkpoint(tmp_path)
    bad = tmp_path / "bad"
    bad.mkdir()
    save_file({"stream.weight": torch.zeros(4), "resident.weight": torch.zeros(2)}, str(bad / "model.safetensors"))
    with pytest.raises(ValueError):
        FullPinnedWeightStore(plan, tensor_factory=_unpinned).load_checkpoint(bad)
    with pytest.raises(FileNotFoundError):
        FullPinnedWeightStore(plan, tensor_factory=_unpinned).load_checkpoint(tmp_path / "nowhere")


def test_unallocated_store_raises():
    store = FullPinnedWeightStore(tiny_plan(), allocate=False)
    with pytest.raises(RuntimeError):
        store.tensor("stream.weight")


def test_native_row_gather_and_out_of_range_ids():
    """cb_host_gather_rows: the streamed-vocabulary embedding's host gather."""

    from layer_streaming import _native

    lib = _native.load_library()
    table = torch.arange(40, dtype=torch.float32).view(10, 4).to(torch.bfloat16)
    ids = torch.tensor([3, 0, 9, 3], dtype=torch.int64)
    out = torch.zeros(4, 4, dtype=torch.bfloat16)
    assert lib.cb_host_gather_rows(out.data_ptr(), table.data_ptr(), 10, 8, ids.data_ptr(), 4) == 0
    assert torch.equal(out, table[ids])
    bad = torch.tensor([2, 10], dtype=torch.int64)
    out.zero_()
    assert lib.cb_host_gather_rows(out.data_ptr(), table.data_ptr(), 10, 8, bad.data_ptr(), 2) != 0
    assert b"outside" in lib.cb_last_error()
    assert int(out.abs().sum()) == 0  # rejected before any copy


def test_staging_worker_reports_copy_failures():
    plan = tiny_plan()
    store = PinnedStagingWeightStore(plan, tensor_factory=RecordingFactory())

    class BrokenEvent:
        def synchronize(self):
            raise RuntimeError("the DMA failed")

    with pytest.raises(RuntimeError, match="DMA failed"):
        store.prepare_unit(plan.units[0], 1, reuse_event=BrokenEvent()).result()
    # the worker survives and serves the next request
    assert store.prepare_unit(plan.units[0], 0).result().numel() == 4
    store.close()
