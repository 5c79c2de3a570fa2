"""Device residency and the two-slot copy/compute pipeline.

Public surface of the reference's ``layer_streaming/runtime.py:11-268``
(``RuntimeStats``, ``ResidentDeviceArena``, ``DoubleBufferRuntime`` with
``run(compute_unit, state)``, ``stats``, ``device_slots``, ``copy_stream``,
``compute_stream``, ``coordinator``, ``profile`` and the ``last_profile``
keys), over two weight modes:

* **streamed** (the reference's mode, default): every transfer unit of a
  step goes host -> device through the device slots. The pipeline itself is
  native (:class:`~layer_streaming.streaming.SlotRing` over
  ``csrc/slot_ring.cu``): unit i lands in slot ``i % slots`` on the copy
  stream, the compute stream waits for it, and unit ``i + slots`` is copied
  into the same slot once the compute stream has released unit i. With the
  pinned-staging store the ring's native stager copies each unit into a
  pinned staging buffer right before its DMA.
* **hbm** (added; ``weights="hbm"`` or ``CASCADE_B200_WEIGHTS=hbm`` so an
  unchanged caller picks it up): B200 holds the whole 16 GB model, so every
  unit is copied to HBM once at construction and ``run`` only launches
  compute; with this package's executor a one-token step is replayed as one
  captured CUDA graph.

The streamed mode can also move its units as int8 rows with fp32 scales
(``transfer="int8"`` or ``CASCADE_B200_TRANSFER=int8``: about half the PCIe
bytes, reduced precision; :mod:`layer_streaming.int8_transfer`).
"""

import os
import time
from dataclasses import dataclass

import torch

from . import ops
from .plan import ModelPlan
from .streaming import SlotRing

WEIGHT_MODES = ("streamed", "hbm")
TRANSFER_FORMATS = ("bf16", "int8")


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
        return dict(self.__dict__)


def _cuda_device(device):
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is unavailable")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("the B200 engine requires a CUDA device")
    return device


def _upload(pairs, device):
    """Copy (device view, host tensor) pairs, one async copy each, and wait."""

    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        for target, source in pairs:
            ops.memcpy_h2d_async(target, source.contiguous())
        stream.synchronize()


def _piece_views(unit, base):
    """{tensor key: view} of a unit laid out from the 1-D device tensor base."""

    views = {}
    for piece in unit.pieces:
        spec = piece.tensor
        views[spec.key] = base.narrow(0, piece.unit_offset_elements, spec.numel).view(spec.shape)
    return views


class ResidentDeviceArena:
    """GPU allocation for the plan's resident tensors and aliases."""

    def __init__(self, plan, store, device):
        if not isinstance(plan, ModelPlan):
            raise TypeError("plan must be a ModelPlan")
        self.plan = plan
        self.store = store
        self.device = _cuda_device(device)
        self.arena = torch.empty(plan.resident_arena_elements, dtype=torch.bfloat16, device=self.device)
        self.views = {}
        pairs = []
        for placement in plan.resident:
            spec = placement.tensor
            view = self.arena.narrow(0, placement.device_offset_elements, spec.numel).view(spec.shape)
            self.views[spec.key] = view
            pairs.append((view, store.tensor(spec.key)))
        _upload(pairs, self.device)
        self.views.update({alias: self.views[target] for alias, target in plan.aliases.items()})

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
    ``CASCADE_B200_WEIGHTS``. ``transfer`` (streamed mode) selects ``"bf16"``
    units (the reference's) or ``"int8"`` units (int8 rows + fp32 scales,
    handed to ``compute_unit`` as ``{key: (int8, scales)}``); ``None`` reads
    ``CASCADE_B200_TRANSFER``.
    """

    def __init__(self, plan, store, resident, device="cuda:0", slot_count=None, profile=False,
                 weights=None, transfer=None):
        self.device = _cuda_device(device)
        self.plan = plan
        self.store = store
        self.resident = resident
        self.weights = str(weights or os.environ.get("CASCADE_B200_WEIGHTS", "streamed")).lower()
        if self.weights not in WEIGHT_MODES:
            raise ValueError("weights must be one of {}".format(WEIGHT_MODES))
        self.transfer = str(transfer or os.environ.get("CASCADE_B200_TRANSFER", "bf16")).lower()
        if self.transfer not in TRANSFER_FORMATS:
            raise ValueError("transfer must be one of {}".format(TRANSFER_FORMATS))
        if self.transfer == "int8" and self.weights != "streamed":
            raise ValueError("transfer='int8' is the streamed mode's (HBM-resident int8: the executor's "
                             "decode_weights='int8')")
        self.slot_count = plan.slot_count if slot_count is None else int(slot_count)
        if self.slot_count not in (1, 2):
            raise ValueError("slot_count must be 1 or 2")
        self.profile = bool(profile)
        self.last_profile = None
        # the hbm mode keeps slots only for a streamed vocabulary
        slots = self.slot_count if (self.weights == "streamed" or plan.vocab is not None) else 0
        self.device_slots = [
            torch.empty(plan.slot_elements, dtype=torch.bfloat16, device=self.device) for _ in range(slots)
        ]
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.compute_stream = torch.cuda.Stream(device=self.device)
        self.coordinator = torch.cuda.current_stream(self.device)
        self.unit_arena = None
        self.int8_arena = None
        self._views = None
        self._ring = None
        if self.weights == "hbm":
            self._load_units()
        elif self.transfer == "int8":
            from .int8_transfer import Int8UnitArena

            self.int8_arena = Int8UnitArena(plan, store, self.device)
            self._views = [self.int8_arena.views(i, self.device_slots[i % slots]) for i in range(len(plan.units))]
            self._ring = SlotRing(self.device_slots, self.copy_stream)  # the int8 arena is pinned
        else:
            self._views = [_piece_views(unit, self.device_slots[i % slots]) for i, unit in enumerate(plan.units)]
            staging = store.staging_buffers() if hasattr(store, "staging_buffers") else None
            if staging is not None:
                staging = staging[:slots]
            self._ring = SlotRing(self.device_slots, self.copy_stream, staging=staging,
                                  copy_threads=getattr(store, "copy_threads", 0))

    # ------------------------------------------------------------ hbm mode
    def _load_units(self):
        units = self.plan.units
        self.unit_arena = torch.empty(sum(u.elements for u in units), dtype=torch.bfloat16, device=self.device)
        bases, pairs, cursor = [], [], 0
        for unit in units:
            base = self.unit_arena.narrow(0, cursor, unit.elements)
            bases.append(base)
            pairs.append((base, self.store.unit_source(unit)))
            cursor += unit.elements
        _upload(pairs, self.device)
        self._views = [_piece_views(unit, base) for unit, base in zip(units, bases)]

    def unit_views(self, index):
        """Device views of unit ``index`` (hbm mode: stable addresses)."""

        if self.weights != "hbm":
            raise RuntimeError("unit_views is the hbm mode's resident layout")
        return self._views[index]

    @property
    def stats(self):
        slots = len(self.device_slots)
        resident_units = 0 if self.unit_arena is None else 2 * self.unit_arena.numel()
        return RuntimeStats(
            transfer_units=len(self.plan.units),
            slot_bytes=self.plan.slot_bytes,
            two_slot_bytes=self.plan.two_slot_bytes,
            device_slot_count=slots,
            device_slots_bytes=slots * self.plan.slot_bytes,
            resident_bytes=self.plan.resident_bytes,
            weight_gpu_bytes=slots * self.plan.slot_bytes + self.plan.resident_bytes + resident_units,
        )

    def run(self, compute_unit, state):
        if not self.plan.units:
            return state
        if self.weights == "hbm":
            return self._run_resident(compute_unit, state)
        return self._run_streamed(compute_unit, state)

    def _run_resident(self, compute_unit, state):
        started = time.perf_counter()
        if self.profile:
            marks = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            marks[0].record(self.coordinator)
        replay = getattr(compute_unit, "run_units_resident", None)
        if replay is not None:
            state = replay(self, state)
        else:
            for unit, views in zip(self.plan.units, self._views):
                state = compute_unit(unit, views, state)
        if self.profile:
            marks[1].record(self.coordinator)
            marks[1].synchronize()
            gpu_ms = marks[0].elapsed_time(marks[1])
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
        units = self.plan.units
        views = self._views
        box = [state]

        def body(index, slot):
            box[0] = compute_unit(units[index], views[index], box[0])

        if hasattr(self.store, "reset_profile"):
            self.store.reset_profile()
        spans = self.int8_arena.spans() if self.int8_arena is not None else self.store.unit_spans(units)
        numbers = self._ring.run(spans, body, self.compute_stream, self.coordinator, profile=self.profile)
        if self.profile:
            profile = {key: numbers[key] for key in (
                "wall_ms", "host_submit_ms", "source_wait_ms", "gpu_pipeline_ms", "h2d_event_sum_ms",
                "compute_event_sum_ms")}
            moved = self.plan.stream_bytes_per_token
            if self.int8_arena is not None:
                moved += self.int8_arena.nbytes - 2 * sum(unit.elements for unit in units)
            profile["h2d_bytes"] = moved
            profile["h2d_effective_gbps"] = (moved / 1e9) / max(numbers["h2d_event_sum_ms"] / 1000.0, 1e-12)
            if self.store.mode == "pinned_staging" and self.int8_arena is None:
                for key in ("staging_copy_count", "staging_event_sum_ms", "staging_event_max_ms"):
                    profile[key] = numbers[key]
            self.last_profile = profile
        return box[0]


def HBMResidentRuntime(plan, store, resident, device="cuda:0", profile=False):
    """DoubleBufferRuntime with every transfer unit resident in HBM."""

    return DoubleBufferRuntime(plan, store, resident, device=device, profile=profile, weights="hbm")
