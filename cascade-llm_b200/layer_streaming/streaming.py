"""Host -> device streaming of weight spans through a ring of device slots.

:class:`SlotRing` drives the native ``cb_ring_*`` pipeline
(``csrc/slot_ring.cu``): the streamed weight mode of
:class:`~layer_streaming.runtime.DoubleBufferRuntime` (the reference's
``runtime.py:137-268``) and the streamed LM head of
:class:`~layer_streaming.vocab.VocabStreamingRuntime` (``vocab.py:207-266``)
both hand it a list of host spans and a per-span body; copies, stream
ordering, staging of pageable spans and the profile events all live in the
native ring, so the Python loop only enqueues each span's kernels.
"""

import ctypes
import time

import torch

from . import _native


def host_span(tensor):
    """(address, bytes) of a contiguous CPU tensor."""

    if tensor.device.type != "cpu":
        raise ValueError("a streamed span must live in host memory")
    if not tensor.is_contiguous():
        raise ValueError("a streamed span must be contiguous")
    return tensor.data_ptr(), tensor.numel() * tensor.element_size()


class SlotRing:
    """``slots`` (equal-sized device tensors) fed on ``copy_stream``.

    ``staging`` (None, or one pinned host tensor per slot) selects the
    pageable-source path: each span is first copied into a staging buffer by
    the ring's native stager (``copy_threads`` threads).
    """

    def __init__(self, slots, copy_stream, staging=None, copy_threads=0):
        if not slots:
            raise ValueError("a slot ring needs at least one device slot")
        self.slots = list(slots)
        self.slot_bytes = min(s.numel() * s.element_size() for s in self.slots)
        self.copy_stream = copy_stream
        self.staging = None if staging is None else list(staging)
        lib = _native.lib()
        dev = (ctypes.c_void_p * len(self.slots))(*[s.data_ptr() for s in self.slots])
        stage = None
        stage_bytes = 0
        if self.staging is not None:
            if len(self.staging) != len(self.slots):
                raise ValueError("one staging buffer per device slot")
            stage = (ctypes.c_void_p * len(self.staging))(*[s.data_ptr() for s in self.staging])
            stage_bytes = min(s.numel() * s.element_size() for s in self.staging)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.slots[0].device):
            _native.check(
                lib.cb_ring_create(len(self.slots), dev, self.slot_bytes, copy_stream.cuda_stream, stage,
                                   stage_bytes, int(copy_threads), ctypes.byref(handle)),
                "cb_ring_create",
            )
        self._handle = handle
        self._lib = lib

    def close(self):
        if self._handle is not None and self._handle.value:
            self._lib.cb_ring_destroy(self._handle)
        self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass

    def run(self, spans, body, compute_stream, coordinator, profile=False):
        """Stream ``spans`` ([(address, bytes)]) and call ``body(i, slot)``
        for each with ``compute_stream`` current, once span i is in ``slot``
        (a device tensor). Returns the pass statistics (host-side ms and,
        with ``profile``, the event timings)."""

        n = len(spans)
        if n == 0:
            return None
        lib = self._lib
        sources = (ctypes.c_void_p * n)(*[a for a, _ in spans])
        sizes = (ctypes.c_int64 * n)(*[b for _, b in spans])
        started = time.perf_counter()
        _native.check(
            lib.cb_ring_begin(self._handle, n, sources, sizes, compute_stream.cuda_stream, coordinator.cuda_stream,
                              1 if profile else 0),
            "cb_ring_begin",
        )
        ptr = ctypes.c_void_p()
        submit = time.perf_counter()
        try:
            with torch.cuda.stream(compute_stream):
                for i in range(n):
                    _native.check(lib.cb_ring_acquire(self._handle, i, ctypes.byref(ptr)), "cb_ring_acquire")
                    body(i, self.slots[i % len(self.slots)])
                    _native.check(lib.cb_ring_release(self._handle, i), "cb_ring_release")
        except BaseException:
            lib.cb_ring_abort(self._handle)
            raise
        submit_ms = (time.perf_counter() - submit) * 1000.0
        stats = (ctypes.c_double * 8)()
        _native.check(lib.cb_ring_end(self._handle, n - 1, stats), "cb_ring_end")
        return {
            "wall_ms": (time.perf_counter() - started) * 1000.0,
            "host_submit_ms": submit_ms,
            "gpu_pipeline_ms": stats[0],
            "h2d_event_sum_ms": stats[1],
            "compute_event_sum_ms": stats[2],
            "source_wait_ms": stats[3],
            "staging_copy_count": int(stats[4]),
            "staging_event_sum_ms": stats[5],
            "staging_event_max_ms": stats[6],
            "h2d_bytes": int(stats[7]),
        }
