"""Device residency and the two-slot copy/compute pipeline.

Mirrors ``layer_streaming/runtime.py:11-268`` of the reference:

* :class:`ResidentDeviceArena` copies the plan's resident tensors (norms, and
  the vocabulary when it is not streamed) to the GPU once;
* :class:`DoubleBufferRuntime` runs ``compute_unit(unit, views, state)`` for
  every transfer unit of a token. In the reference's **streamed** mode each
  unit is copied host->device (``cudaMemcpyAsync`` from the pinned arena) into
  slot ``i % 2`` on a copy stream; the compute stream waits for that copy and
  the copy stream waits until compute has released the slot two units later.

Added: the **hbm** weight mode (``weights="hbm"``, or the environment variable
``CASCADE_B200_WEIGHTS=hbm`` so that an unchanged caller picks it up): B200
holds the whole 16 GB model, so every transfer unit is copied to HBM once at
construction and ``run`` only launches compute. When the executor provides
``run_units_resident`` (this package's executor does), the whole layer stack
of a one-token step is replayed as a single captured CUDA graph.
"""

import os
import time
from dataclasses import dataclass

import torch

from . import ops
from .plan import ModelPlan

WEIGHT_MODES = ("streamed", "hbm")


@dataclass
class RuntimeStats:
    transfer_units: int
    slot_bytes: int
    two_slot_bytes: int
    device_slot_count: int
    device_slots_bytes: int
    resident_bytes: int
    weight_gpu_bytes: int

    def as_dict(self):
        return {
            "transfer_units": self.transfer_units,
            "slot_bytes": self.slot_bytes,
            "two_slot_bytes": self.two_slot_bytes,
            "device_slot_count": self.device_slot_count,
            "device_slots_bytes": self.device_slots_bytes,
            "resident_bytes": self.resident_bytes,
            "weight_gpu_bytes": self.weight_gpu_bytes,
        }


def _require_cuda(device):
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("the B200 engine requires a CUDA device")
    return device


def _h2d(dst, src):
    """Host -> device copy on the current stream (pinned: asynchronous)."""

    ops.memcpy_h2d_async(dst, src.contiguous())


class ResidentDeviceArena:
    """GPU allocation for the plan's resident tensors and aliases."""

    def __init__(self, plan, store, device):
        if not isinstance(plan, ModelPlan):
            raise TypeError("plan must be a ModelPlan")
        self.plan = plan
        self.store = store
        self.device = _require_cuda(device)
        self.arena = torch.empty(plan.resident_arena_elements, dtype=torch.bfloat16, device=self.device)
        self.views = {}
        with torch.cuda.device(self.device):
            for placement in plan.resident:
                spec = placement.tensor
                start = placement.device_offset_elements
                view = self.arena[start:start + spec.numel].view(spec.shape)
                _h2d(view, store.tensor(spec.key))
                self.views[spec.key] = view
            for alias, target in plan.aliases.items():
                self.views[alias] = self.views[target]
            torch.cuda.current_stream(self.device).synchronize()

    @property
    def nbytes(self):
        return self.plan.resident_bytes

    def __getitem__(self, key):
        return self.views[key]

    def __contains__(self, key):
        return key in self.views


class DoubleBufferRuntime:
    """Two device slots with a copy stream and a compute stream.

    ``compute_unit`` is called as ``compute_unit(unit, weight_views, state)``
    and must enqueue all work on the current (compute) stream; weight views
    must not escape the call because their slot is reused two units later.

    ``weights`` selects ``"streamed"`` (the reference's behaviour, default)
    or ``"hbm"`` (all units resident in device memory); ``None`` reads
    ``CASCADE_B200_WEIGHTS``.
    """

    def __init__(self, plan, store, resident, device="cuda:0", slot_count=None, profile=False,
                 weights=None):
        self.device = _require_cuda(device)
        self.plan = plan
        self.store = store
        self.resident = resident
        self.weights = (weights or os.environ.get("CASCADE_B200_WEIGHTS", "streamed")).lower()
        if self.weights not in WEIGHT_MODES:
            raise ValueError("weights must be one of {}".format(WEIGHT_MODES))
        self.slot_count = plan.slot_count if slot_count is None else int(slot_count)
        if self.slot_count not in (1, 2):
            raise ValueError("slot_count must be 1 or 2")
        self.profile = bool(profile)
        self.last_profile = None
        # hbm mode needs slots only to stream a host-only vocabulary
        need_slots = self.weights == "streamed" or plan.vocab is not None
        self.device_slots = [
            torch.empty(plan.slot_elements, dtype=torch.bfloat16, device=self.device)
            for _ in range(self.slot_count if need_slots else 0)
        ]
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.compute_stream = torch.cuda.Stream(device=self.device)
        self.coordinator = torch.cuda.current_stream(self.device)
        self.unit_arena = None
        self._resident_views = None
        if self.weights == "hbm":
            self._load_units()

    # ------------------------------------------------------------ hbm mode
    def _load_units(self):
        total = sum(unit.elements for unit in self.plan.units)
        self.unit_arena = torch.empty(total, dtype=torch.bfloat16, device=self.device)
        self._unit_base = {}
        cursor = 0
        with torch.cuda.device(self.device):
            for unit in self.plan.units:
                dst = self.unit_arena[cursor:cursor + unit.elements]
                _h2d(dst, self.store.unit_source(unit))
                self._unit_base[unit.unit_id] = dst
                cursor += unit.elements
            torch.cuda.current_stream(self.device).synchronize()
        self._resident_views = [self._unit_views(u, self._unit_base[u.unit_id]) for u in self.plan.units]

    def unit_views(self, index):
        """Device views of unit ``index`` (hbm mode: stable addresses)."""

        return self._resident_views[index]

    @property
    def stats(self):
        slots = len(self.device_slots)
        resident_units = 0 if self.unit_arena is None else self.unit_arena.numel() * 2
        return RuntimeStats(
            transfer_units=len(self.plan.units),
            slot_bytes=self.plan.slot_bytes,
            two_slot_bytes=self.plan.two_slot_bytes,
            device_slot_count=slots,
            device_slots_bytes=slots * self.plan.slot_bytes,
            resident_bytes=self.plan.resident_bytes,
            weight_gpu_bytes=slots * self.plan.slot_bytes + self.plan.resident_bytes + resident_units,
        )

    @staticmethod
    def _unit_views(unit, base):
        return {
            piece.tensor.key: base[piece.unit_offset_elements:piece.unit_offset_elements + piece.tensor.numel].view(
                piece.tensor.shape
            )
            for piece in unit.pieces
        }

    def run(self, compute_unit, state):
        if not self.plan.units:
            return state
        if self.weights == "hbm":
            return self._run_resident(compute_unit, state)
        return self._run_streamed(compute_unit, state)

    def _run_resident(self, compute_unit, state):
        started = time.perf_counter()
        begin = end = None
        if self.profile:
            begin = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            begin.record(self.coordinator)
        fast = getattr(compute_unit, "run_units_resident", None)
        if fast is not None:
            state = fast(self, state)
        else:
            for index, unit in enumerate(self.plan.units):
                state = compute_unit(unit, self._resident_views[index], state)
        if self.profile:
            end.record(self.coordinator)
            end.synchronize()
            gpu_ms = begin.elapsed_time(end)
            self.last_profile = {
                "wall_ms": (time.perf_counter() - started) * 1000.0,
                "host_submit_ms": 0.0,
                "source_wait_ms": 0.0,
                "gpu_pipeline_ms": gpu_ms,
                "h2d_event_sum_ms": 0.0,
                "compute_event_sum_ms": gpu_ms,
                "h2d_bytes": 0,
                "h2d_effective_gbps": 0.0,
            }
        return state

    # ------------------------------------------------------------ streamed
    def _run_streamed(self, compute_unit, state):
        wall_started = time.perf_counter()
        units = self.plan.units
        n = len(units)
        profile = self.profile
        timing = dict(enable_timing=True)
        if profile:
            pipe_start, pipe_end = torch.cuda.Event(**timing), torch.cuda.Event(**timing)
            copy_ev = [(torch.cuda.Event(**timing), torch.cuda.Event(**timing)) for _ in units]
            comp_ev = [(torch.cuda.Event(**timing), torch.cuda.Event(**timing)) for _ in units]
            pipe_start.record(self.coordinator)
            self.copy_stream.wait_event(pipe_start)
            self.compute_stream.wait_event(pipe_start)
        else:
            # order both streams after work already queued by the caller
            self.copy_stream.wait_stream(self.coordinator)
            self.compute_stream.wait_stream(self.coordinator)
        ready = [torch.cuda.Event() for _ in units]
        free = [torch.cuda.Event() for _ in units]
        if hasattr(self.store, "reset_profile"):
            self.store.reset_profile()
        staged = {i: self.store.prepare_unit(units[i], i) for i in range(min(self.slot_count, n))}
        staging = getattr(self.store.mode, "value", "") == "pinned_staging"
        source_wait_ms = 0.0
        submit_started = time.perf_counter()
        for index, unit in enumerate(units):
            slot_index = index % self.slot_count
            slot = self.device_slots[slot_index]
            waited = time.perf_counter()
            source = staged.pop(index).result()
            source_wait_ms += (time.perf_counter() - waited) * 1000.0
            if index >= self.slot_count:
                self.copy_stream.wait_event(free[index - self.slot_count])
            with torch.cuda.stream(self.copy_stream):
                if profile:
                    copy_ev[index][0].record(self.copy_stream)
                ops.memcpy_h2d_async(slot[:unit.elements], source)
                if profile:
                    copy_ev[index][1].record(self.copy_stream)
                ready[index].record(self.copy_stream)
            ahead = index + self.slot_count
            if ahead < n:
                # a staging slot may be refilled once its DMA has finished
                staged[ahead] = self.store.prepare_unit(
                    units[ahead], slot_index, reuse_event=ready[index] if staging else None
                )
            self.compute_stream.wait_event(ready[index])
            with torch.cuda.stream(self.compute_stream):
                if profile:
                    comp_ev[index][0].record(self.compute_stream)
                state = compute_unit(unit, self._unit_views(unit, slot), state)
                if profile:
                    comp_ev[index][1].record(self.compute_stream)
                free[index].record(self.compute_stream)
        submit_ms = (time.perf_counter() - submit_started) * 1000.0
        self.coordinator.wait_event(free[-1])
        if profile:
            pipe_end.record(self.coordinator)
        self.coordinator.synchronize()
        if profile:
            h2d_ms = sum(a.elapsed_time(b) for a, b in copy_ev)
            compute_ms = sum(a.elapsed_time(b) for a, b in comp_ev)
            self.last_profile = {
                "wall_ms": (time.perf_counter() - wall_started) * 1000.0,
                "host_submit_ms": submit_ms,
                "source_wait_ms": source_wait_ms,
                "gpu_pipeline_ms": pipe_start.elapsed_time(pipe_end),
                "h2d_event_sum_ms": h2d_ms,
                "compute_event_sum_ms": compute_ms,
                "h2d_bytes": self.plan.stream_bytes_per_token,
                "h2d_effective_gbps": (self.plan.stream_bytes_per_token / 1e9) / (h2d_ms / 1000.0),
            }
            if hasattr(self.store, "profile_stats"):
                self.last_profile.update(self.store.profile_stats())
        return state


def HBMResidentRuntime(plan, store, resident, device="cuda:0", profile=False):
    """DoubleBufferRuntime with every transfer unit resident in HBM."""

    return DoubleBufferRuntime(plan, store, resident, device=device, profile=profile, weights="hbm")
