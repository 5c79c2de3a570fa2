"""Packed CPU weight arenas: full-pinned and pinned-staging modes.

Same API as the reference (``layer_streaming/weight_store.py:15-318``): one
BF16 host arena laid out by :mod:`plan`; ``full_pinned`` page-locks all of it
so every transfer unit can be DMA'd straight from the arena, while
``pinned_staging`` keeps a pageable arena plus ``slot_count`` pinned staging
slots filled by worker threads. ``tensor_factory`` is the allocation seam the
reference's tests use to run without a GPU.

Additions: :meth:`BaseWeightStore.fill_seeded` writes the seeded random-init
weights of the benchmark configurations (generated on the GPU by
``cb_fill_normal_bf16``, norms = 1); :meth:`load_checkpoint` parses each
safetensors header once and reads the tensor bytes straight into the arena
with parallel ``pread`` on native threads; the staging store's pageable ->
pinned copies run on native threads (``cb_host_copy``).
"""

import json
import os
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from enum import Enum
from pathlib import Path

import torch

from .plan import ModelPlan


class WeightStoreMode(str, Enum):
    FULL_PINNED = "full_pinned"
    PINNED_STAGING = "pinned_staging"


def _checkpoint_files(checkpoint):
    """{tensor key: file} for an indexed checkpoint, None for one file."""

    checkpoint = Path(checkpoint)
    index = checkpoint / "model.safetensors.index.json"
    if index.exists():
        weight_map = json.loads(index.read_text(encoding="utf-8")).get("weight_map")
        if not isinstance(weight_map, dict):
            raise ValueError("{} has no weight_map".format(index))
        return {key: checkpoint / name for key, name in weight_map.items()}
    if (checkpoint / "model.safetensors").exists():
        return None
    raise FileNotFoundError(
        "expected model.safetensors or model.safetensors.index.json in {}".format(checkpoint)
    )


def _native_copy_ok(target, source):
    """Both CPU, contiguous, same dtype and size, and the native library present."""

    if target.device.type != "cpu" or source.device.type != "cpu" or target.dtype != source.dtype:
        return False
    if not (target.is_contiguous() and source.is_contiguous()) or target.numel() != source.numel():
        return False
    from . import _native

    try:
        _native.lib()
    except (OSError, RuntimeError):
        return False
    return True


def is_norm(key):
    return key.endswith("layernorm.weight") or key == "model.norm.weight"


class BaseWeightStore:
    """Packed CPU arena shared by both memory modes."""

    def __init__(self, plan, pin_full_arena, allocate=True, tensor_factory=None):
        if not isinstance(plan, ModelPlan):
            raise TypeError("plan must be a ModelPlan")
        self.plan = plan
        self.pin_full_arena = bool(pin_full_arena)
        self.tensor_factory = tensor_factory or torch.empty
        self.arena = None
        self._loaded = False
        if allocate:
            self.allocate()

    @property
    def mode(self):
        raise NotImplementedError

    @property
    def pinned_cpu_bytes(self):
        raise NotImplementedError

    @property
    def allocated(self):
        return self.arena is not None

    @property
    def loaded(self):
        return self._loaded

    def allocate(self):
        if self.arena is None:
            self.arena = self.tensor_factory(
                self.plan.host_arena_elements,
                dtype=torch.bfloat16,
                device="cpu",
                pin_memory=self.pin_full_arena,
            )
        return self.arena

    def _view(self, key):
        spec = self.plan.tensors[key]
        if spec.alias_of is not None:
            return self._view(spec.alias_of)
        start = self.plan.tensor_host_offset(key)
        return self.arena[start:start + spec.numel].view(spec.shape)

    def tensor(self, key):
        if self.arena is None:
            raise RuntimeError("weight arena has not been allocated")
        return self._view(self.plan.aliases.get(key, key))

    def unit_source(self, unit, slot_index=None):
        if self.arena is None:
            raise RuntimeError("weight arena has not been allocated")
        start = unit.host_offset_elements
        return self.arena[start:start + unit.elements]

    def required_keys(self):
        return sorted(k for k, s in self.plan.tensors.items() if s.alias_of is None)

    def load_checkpoint(self, checkpoint, threads=0):
        """Copy a local safetensors checkpoint into the packed arena (as bf16).

        Each file's header is parsed once and every tensor's bytes are read
        straight into its arena view by parallel ``pread`` on native threads
        (``threads`` = 0: up to 16); non-BF16 tensors are converted.
        """

        from .checkpoint import load_safetensors_into

        if self.arena is None:
            self.allocate()
        required = set(self.required_keys())
        weight_map = _checkpoint_files(checkpoint)
        if weight_map is None:
            files = {key: Path(checkpoint) / "model.safetensors" for key in required}
        else:
            missing = required.difference(weight_map)
            if missing:
                raise KeyError(
                    "checkpoint index misses required tensors: {}".format(", ".join(sorted(missing)[:8]))
                )
            files = {key: weight_map[key] for key in required}
        targets = {key: self._view(key) for key in required}
        with torch.inference_mode():
            loaded = load_safetensors_into(files, targets, threads)
        missing = required.difference(loaded)
        if missing:
            raise KeyError("checkpoint misses required tensors: {}".format(", ".join(sorted(missing)[:8])))
        self._loaded = True
        return self

    def fill_seeded(self, seed=0, std=0.02, device="cuda:0", chunk_elements=1 << 27):
        """Seeded random-init weights: N(0, std) matrices, norm weights = 1.

        Element i of tensor ``key`` is element i of the counter-based stream
        ``cb_stream_key(seed, key)``; the values are generated on ``device``
        in chunks and copied into the arena, so any process (and the CPU
        oracle) regenerates the same bits.
        """

        from . import ops
        from ._native import stream_key

        if self.arena is None:
            self.allocate()
        device = torch.device(device)
        buffer = torch.empty(chunk_elements, dtype=torch.bfloat16, device=device)
        with torch.inference_mode():
            for key in self.required_keys():
                target = self._view(key).reshape(-1)
                if is_norm(key):
                    target.fill_(1.0)
                    continue
                k = stream_key(seed, key)
                for start in range(0, target.numel(), chunk_elements):
                    n = min(chunk_elements, target.numel() - start)
                    ops.fill_normal_(buffer[:n], k, std=std, offset=start)
                    target[start:start + n].copy_(buffer[:n])
        torch.cuda.synchronize(device)
        self._loaded = True
        return self

    def close(self):
        self.arena = None
        self._loaded = False

    def reset_profile(self):
        return None

    def profile_stats(self):
        return {}


class FullPinnedWeightStore(BaseWeightStore):
    """All checkpoint weights remain in page-locked CPU memory."""

    def __init__(self, plan, allocate=True, tensor_factory=None):
        super().__init__(plan, pin_full_arena=True, allocate=allocate, tensor_factory=tensor_factory)

    @property
    def mode(self):
        return WeightStoreMode.FULL_PINNED

    @property
    def pinned_cpu_bytes(self):
        return self.plan.host_arena_bytes

    def prepare_unit(self, unit, slot_index, reuse_event=None):
        future = Future()
        future.set_result(self.unit_source(unit))
        return future


class PinnedStagingWeightStore(BaseWeightStore):
    """Pageable full store plus reusable page-locked staging slots."""

    def __init__(self, plan, allocate=True, tensor_factory=None, worker_count=2, copy_threads=None):
        self.staging_slots = None
        self.worker_count = int(worker_count)
        # native threads per staging copy (the workers' copies run concurrently)
        self.copy_threads = int(copy_threads or max(1, min(8, (os.cpu_count() or 2) // max(1, self.worker_count))))
        self._executor = None
        self._profile_lock = threading.Lock()
        self._stage_ms = []
        super().__init__(plan, pin_full_arena=False, allocate=allocate, tensor_factory=tensor_factory)

    @property
    def mode(self):
        return WeightStoreMode.PINNED_STAGING

    @property
    def pinned_cpu_bytes(self):
        return self.plan.two_slot_bytes

    def allocate(self):
        arena = super().allocate()
        if self.staging_slots is None:
            self.staging_slots = [
                self.tensor_factory(
                    self.plan.slot_elements, dtype=torch.bfloat16, device="cpu", pin_memory=True
                )
                for _ in range(self.plan.slot_count)
            ]
        if self._executor is None:
            self._executor = ThreadPoolExecutor(
                max_workers=self.worker_count, thread_name_prefix="weight-stage"
            )
        return arena

    def _stage(self, unit, slot_index, reuse_event):
        started = time.perf_counter()
        if reuse_event is not None:
            # the DMA that last read this staging slot must have finished
            reuse_event.synchronize()
        target = self.staging_slots[slot_index][:unit.elements]
        source = self.unit_source(unit)
        if _native_copy_ok(target, source):
            # pageable -> pinned on native threads (one thread cannot reach the PCIe rate)
            from . import _native

            _native.check(
                _native.lib().cb_host_copy(target.data_ptr(), source.data_ptr(),
                                           source.numel() * source.element_size(), self.copy_threads),
                "cb_host_copy",
            )
        else:
            target.copy_(source)
        with self._profile_lock:
            self._stage_ms.append((time.perf_counter() - started) * 1000.0)
        return target

    def prepare_unit(self, unit, slot_index, reuse_event=None):
        if self.staging_slots is None or self._executor is None:
            raise RuntimeError("staging store has not been allocated")
        return self._executor.submit(self._stage, unit, slot_index, reuse_event)

    def close(self):
        if self._executor is not None:
            self._executor.shutdown(wait=True)
            self._executor = None
        self.staging_slots = None
        super().close()

    def reset_profile(self):
        with self._profile_lock:
            self._stage_ms = []

    def profile_stats(self):
        with self._profile_lock:
            durations = list(self._stage_ms)
        return {
            "staging_copy_count": len(durations),
            "staging_event_sum_ms": sum(durations),
            "staging_event_max_ms": max(durations) if durations else 0.0,
        }


def create_weight_store(plan, mode=WeightStoreMode.FULL_PINNED, allocate=True, tensor_factory=None):
    mode = WeightStoreMode(mode)
    if mode == WeightStoreMode.FULL_PINNED:
        return FullPinnedWeightStore(plan, allocate=allocate, tensor_factory=tensor_factory)
    return PinnedStagingWeightStore(plan, allocate=allocate, tensor_factory=tensor_factory)
