"""Host weight arenas of the two memory modes.

Public surface of the reference's ``layer_streaming/weight_store.py:15-318``
(class names, constructor signatures, ``mode``, ``pinned_cpu_bytes``,
``tensor``, ``unit_source``, ``prepare_unit``, ``load_checkpoint``, the
``tensor_factory`` allocation seam and the staging profile keys), organised
around what the streaming ring needs:

* :class:`HostArena` is the packed BF16 arena laid out by :mod:`plan`: it
  resolves tensor keys (aliases included) and transfer units to views and
  hands the ring each unit's host span;
* ``full_pinned`` page-locks the whole arena, so a unit's span is DMA'd
  straight from it;
* ``pinned_staging`` keeps the arena pageable and allocates one pinned
  staging buffer per device slot; the streamed runtime passes those buffers
  to the native slot ring (``csrc/slot_ring.cu``), whose stager thread copies
  each unit into them on native threads right before its DMA.
  :meth:`PinnedStagingWeightStore.prepare_unit` stages one unit on request
  (the reference's per-unit entry, kept for callers and tests).

Additions: :meth:`BaseWeightStore.fill_seeded` writes the seeded random-init
weights of the benchmark configurations (generated on the GPU by
``cb_fill_normal_bf16``, norms = 1); :meth:`BaseWeightStore.load_checkpoint`
reads safetensors bytes straight into the arena with parallel ``pread``.
"""

import json
import os
import queue
import threading
import time
from concurrent.futures import Future
from enum import Enum
from pathlib import Path

import torch

from .plan import ModelPlan


class WeightStoreMode(str, Enum):
    FULL_PINNED = "full_pinned"
    PINNED_STAGING = "pinned_staging"


def is_norm(key):
    return key.endswith("layernorm.weight") or key == "model.norm.weight"


def checkpoint_layout(checkpoint):
    """Where each tensor of a local safetensors checkpoint lives.

    ``{key: file}`` from ``model.safetensors.index.json``, or ``None`` when
    the checkpoint is the single file ``model.safetensors``.
    """

    root = Path(checkpoint)
    index = root / "model.safetensors.index.json"
    if index.is_file():
        mapping = json.loads(index.read_text(encoding="utf-8")).get("weight_map")
        if not isinstance(mapping, dict):
            raise ValueError("{}: no weight_map object".format(index))
        return {key: root / name for key, name in mapping.items()}
    if (root / "model.safetensors").is_file():
        return None
    raise FileNotFoundError("{} holds neither model.safetensors nor model.safetensors.index.json".format(root))


class HostArena:
    """The plan's packed BF16 arena (one 1-D host tensor) and its views."""

    def __init__(self, plan, storage):
        self.plan = plan
        self.storage = storage

    def view(self, key):
        """View of tensor ``key`` (an alias resolves to its target)."""

        plan = self.plan
        key = plan.aliases.get(key, key)
        spec = plan.tensors[key]
        while spec.alias_of is not None:
            spec = plan.tensors[spec.alias_of]
        begin = plan.tensor_host_offset(spec.key)
        return self.storage.narrow(0, begin, spec.numel).view(spec.shape)

    def unit(self, unit):
        """The contiguous 1-D span of transfer unit ``unit``."""

        return self.storage.narrow(0, unit.host_offset_elements, unit.elements)

    def span(self, unit):
        """(host address, bytes) of the unit's span, for the slot ring."""

        return self.storage.data_ptr() + 2 * unit.host_offset_elements, 2 * unit.elements

    def is_pinned(self):
        return self.storage.is_pinned()


class BaseWeightStore:
    """Packed CPU arena shared by both memory modes."""

    def __init__(self, plan, pin_full_arena, allocate=True, tensor_factory=None):
        if not isinstance(plan, ModelPlan):
            raise TypeError("plan must be a ModelPlan")
        self.plan = plan
        self.pin_full_arena = bool(pin_full_arena)
        self.tensor_factory = tensor_factory or torch.empty
        self._host = None
        self._loaded = False
        if allocate:
            self.allocate()

    # -- mode-specific facts
    @property
    def mode(self):
        raise NotImplementedError

    @property
    def pinned_cpu_bytes(self):
        raise NotImplementedError

    def staging_buffers(self):
        """Pinned staging buffers the slot ring copies through (None: the
        arena itself is pinned)."""

        return None

    # -- arena
    @property
    def arena(self):
        return None if self._host is None else self._host.storage

    @property
    def allocated(self):
        return self._host is not None

    @property
    def loaded(self):
        return self._loaded

    def _request(self, elements, pinned):
        return self.tensor_factory(elements, dtype=torch.bfloat16, device="cpu", pin_memory=pinned)

    def allocate(self):
        if self._host is None:
            self._host = HostArena(self.plan, self._request(self.plan.host_arena_elements, self.pin_full_arena))
        return self._host.storage

    def _arena(self):
        if self._host is None:
            raise RuntimeError("the weight arena is not allocated (allocate=False and no allocate() yet)")
        return self._host

    def tensor(self, key):
        return self._arena().view(key)

    def unit_source(self, unit, slot_index=None):
        return self._arena().unit(unit)

    def unit_spans(self, units):
        """Host spans of ``units`` in order (what the slot ring copies)."""

        host = self._arena()
        return [host.span(unit) for unit in units]

    def required_keys(self):
        return sorted(key for key, spec in self.plan.tensors.items() if spec.alias_of is None)

    # -- filling the arena
    def load_checkpoint(self, checkpoint, threads=0):
        """Copy a local safetensors checkpoint into the packed arena (as bf16).

        Each file's header is parsed once and every tensor's bytes are read
        straight into its arena view by parallel ``pread`` on native threads
        (``threads`` = 0: up to 16); non-BF16 tensors are converted.
        """

        from .checkpoint import load_safetensors_into

        self.allocate()
        wanted = self.required_keys()
        layout = checkpoint_layout(checkpoint)
        if layout is None:
            single = Path(checkpoint) / "model.safetensors"
            files = dict.fromkeys(wanted, single)
        else:
            absent = [key for key in wanted if key not in layout]
            if absent:
                raise KeyError("the checkpoint index lacks {} required tensor(s), e.g. {}".format(
                    len(absent), ", ".join(absent[:8])))
            files = {key: layout[key] for key in wanted}
        with torch.inference_mode():
            got = load_safetensors_into(files, {key: self.tensor(key) for key in wanted}, threads)
        absent = [key for key in wanted if key not in got]
        if absent:
            raise KeyError("the checkpoint lacks {} required tensor(s), e.g. {}".format(
                len(absent), ", ".join(absent[:8])))
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

        self.allocate()
        scratch = torch.empty(chunk_elements, dtype=torch.bfloat16, device=torch.device(device))
        with torch.inference_mode():
            for key in self.required_keys():
                flat = self.tensor(key).reshape(-1)
                if is_norm(key):
                    flat.fill_(1.0)
                    continue
                stream = stream_key(seed, key)
                for begin in range(0, flat.numel(), chunk_elements):
                    part = scratch[:min(chunk_elements, flat.numel() - begin)]
                    ops.fill_normal_(part, stream, std=std, offset=begin)
                    flat[begin:begin + part.numel()].copy_(part)
        torch.cuda.synchronize(device)
        self._loaded = True
        return self

    def close(self):
        self._host = None
        self._loaded = False

    def reset_profile(self):
        return None

    def profile_stats(self):
        return {}


class FullPinnedWeightStore(BaseWeightStore):
    """All checkpoint weights remain in page-locked CPU memory."""

    def __init__(self, plan, allocate=True, tensor_factory=None):
        super().__init__(plan, True, allocate=allocate, tensor_factory=tensor_factory)

    @property
    def mode(self):
        return WeightStoreMode.FULL_PINNED

    @property
    def pinned_cpu_bytes(self):
        return self.plan.host_arena_bytes

    def prepare_unit(self, unit, slot_index, reuse_event=None):
        """The unit's span of the pinned arena, as an already-resolved future."""

        done = Future()
        done.set_result(self.unit_source(unit))
        return done


class _StagingWorker:
    """One daemon thread that runs staging requests in submission order."""

    def __init__(self):
        self._requests = queue.SimpleQueue()
        self._thread = threading.Thread(target=self._loop, name="cascade-staging", daemon=True)
        self._thread.start()

    def _loop(self):
        while True:
            request = self._requests.get()
            if request is None:
                return
            future, job = request
            if future.set_running_or_notify_cancel():
                try:
                    future.set_result(job())
                except BaseException as error:  # handed to the waiting caller
                    future.set_exception(error)

    def submit(self, job):
        future = Future()
        self._requests.put((future, job))
        return future

    def stop(self):
        self._requests.put(None)
        self._thread.join()


class PinnedStagingWeightStore(BaseWeightStore):
    """Pageable full store plus reusable page-locked staging slots."""

    def __init__(self, plan, allocate=True, tensor_factory=None, worker_count=2, copy_threads=None):
        # worker_count is the reference's staging concurrency; here the slot
        # ring stages one unit at a time with a multi-threaded copy instead
        self.worker_count = int(worker_count)
        cores = os.cpu_count() or 2
        self.copy_threads = int(copy_threads or max(1, min(16, cores)))
        self.staging_slots = None
        self._worker = None
        self._stats_lock = threading.Lock()
        self._copy_ms = []
        super().__init__(plan, False, allocate=allocate, tensor_factory=tensor_factory)

    @property
    def mode(self):
        return WeightStoreMode.PINNED_STAGING

    @property
    def pinned_cpu_bytes(self):
        return self.plan.two_slot_bytes

    def allocate(self):
        storage = super().allocate()
        if self.staging_slots is None:
            self.staging_slots = [self._request(self.plan.slot_elements, True) for _ in range(self.plan.slot_count)]
        return storage

    def staging_buffers(self):
        if self.staging_slots is None:
            raise RuntimeError("the staging buffers are not allocated")
        return self.staging_slots

    def _copy_into_slot(self, unit, slot_index, reuse_event):
        began = time.perf_counter()
        if reuse_event is not None:
            reuse_event.synchronize()  # the DMA that last read this buffer has finished
        source = self.unit_source(unit)
        target = self.staging_slots[slot_index].narrow(0, 0, unit.elements)
        host_copy(target, source, self.copy_threads)
        with self._stats_lock:
            self._copy_ms.append((time.perf_counter() - began) * 1000.0)
        return target

    def prepare_unit(self, unit, slot_index, reuse_event=None):
        """Stage ``unit`` into staging buffer ``slot_index`` in the background
        (after ``reuse_event``, the DMA that last read the buffer); the
        future's result is the pinned staged span."""

        if self.staging_slots is None:
            raise RuntimeError("the staging buffers are not allocated")
        if self._worker is None:
            self._worker = _StagingWorker()
        return self._worker.submit(lambda: self._copy_into_slot(unit, slot_index, reuse_event))

    def close(self):
        if self._worker is not None:
            self._worker.stop()
            self._worker = None
        self.staging_slots = None
        super().close()

    def reset_profile(self):
        with self._stats_lock:
            self._copy_ms = []

    def profile_stats(self):
        with self._stats_lock:
            ms = list(self._copy_ms)
        return {
            "staging_copy_count": len(ms),
            "staging_event_sum_ms": float(sum(ms)),
            "staging_event_max_ms": float(max(ms, default=0.0)),
        }


def host_copy(target, source, threads=0):
    """``target.copy_(source)`` for host tensors, on native threads when both
    are contiguous bf16 of one size and the native library is present."""

    same = (
        target.device.type == source.device.type == "cpu"
        and target.dtype == source.dtype
        and target.numel() == source.numel()
        and target.is_contiguous()
        and source.is_contiguous()
    )
    if same:
        from . import _native

        try:
            lib = _native.lib()
        except (OSError, RuntimeError):
            lib = None
        if lib is not None:
            _native.check(
                lib.cb_host_copy(target.data_ptr(), source.data_ptr(), source.numel() * source.element_size(),
                                 int(threads)),
                "cb_host_copy",
            )
            return target
    return target.copy_(source)


def create_weight_store(plan, mode=WeightStoreMode.FULL_PINNED, allocate=True, tensor_factory=None):
    kinds = {
        WeightStoreMode.FULL_PINNED: FullPinnedWeightStore,
        WeightStoreMode.PINNED_STAGING: PinnedStagingWeightStore,
    }
    return kinds[WeightStoreMode(mode)](plan, allocate=allocate, tensor_factory=tensor_factory)
