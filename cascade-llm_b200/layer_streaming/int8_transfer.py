"""Int8 weight transfer for the streamed runtime (optional, reduced precision).

The reference streams every transfer unit in bf16 over PCIe and lists
INT8/INT4 weight transfer as unsupported (its README.md:156). Here each unit
can instead cross PCIe as int8 rows with one fp32 scale per row (w ~= q * s,
``cb_quantize_rows_i8``): about half the bytes per token. The packed layout of
a unit is, for each of its matrices in plan order, the int8 matrix and then
its fp32 scales, every block at a 256-byte offset, so a unit is one
contiguous span that the native slot ring copies into a device slot like a
bf16 unit.

:class:`Int8UnitArena` quantizes the store's units once, on the device, into
a pinned host arena; :meth:`Int8UnitArena.views` interprets a device slot
holding unit i as ``{key: (int8 [N, K], fp32 [N])}``. The executor runs a
one-token step on those views with the int8 GEMVs and dequantizes a unit to
bf16 (``cb_dequantize_rows_i8``) for the tensor-core prefill GEMMs.
"""

from dataclasses import dataclass
from typing import Tuple

import torch

from . import ops

_ALIGN = 256


def _align(n):
    return -(-n // _ALIGN) * _ALIGN


@dataclass(frozen=True)
class Int8Piece:
    key: str
    shape: Tuple[int, int]
    q_offset: int      # bytes from the unit's start
    scale_offset: int  # bytes from the unit's start


@dataclass(frozen=True)
class Int8Unit:
    pieces: Tuple[Int8Piece, ...]
    nbytes: int
    host_offset: int


def unit_layout(unit, host_offset=0):
    """The int8 layout of a bf16 transfer unit (every piece a 2-D matrix)."""

    pieces, cursor = [], 0
    for piece in unit.pieces:
        spec = piece.tensor
        if len(spec.shape) != 2:
            raise ValueError("int8 transfer packs matrices only ({} is {}-D)".format(spec.key, len(spec.shape)))
        rows, cols = spec.shape
        q_offset = cursor
        cursor = _align(cursor + rows * cols)
        scale_offset = cursor
        cursor = _align(cursor + rows * 4)
        pieces.append(Int8Piece(spec.key, (rows, cols), q_offset, scale_offset))
    return Int8Unit(tuple(pieces), cursor, host_offset)


class Int8UnitArena:
    """Pinned host copy of every transfer unit of ``plan`` as int8 rows + fp32 scales."""

    def __init__(self, plan, store, device):
        self.plan = plan
        self.device = torch.device(device)
        units, offset = [], 0
        for unit in plan.units:
            packed = unit_layout(unit, offset)
            units.append(packed)
            offset += packed.nbytes
        self.units = units
        self.host = torch.empty(offset, dtype=torch.uint8).pin_memory()
        self._quantize_from(store)

    @property
    def nbytes(self):
        return self.host.numel()

    @property
    def max_unit_bytes(self):
        return max(u.nbytes for u in self.units)

    def _quantize_from(self, store):
        """Each unit: bf16 host span -> device, quantize, packed int8 -> host."""

        plan = self.plan
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            biggest = max(unit.elements for unit in plan.units)
            dev_bf16 = torch.empty(biggest, dtype=torch.bfloat16, device=self.device)
            dev_packed = torch.empty(self.max_unit_bytes, dtype=torch.uint8, device=self.device)
            for unit, packed in zip(plan.units, self.units):
                ops.memcpy_h2d_async(dev_bf16.narrow(0, 0, unit.elements), store.unit_source(unit).contiguous())
                for piece, spec_piece in zip(packed.pieces, unit.pieces):
                    rows, cols = piece.shape
                    w = dev_bf16.narrow(0, spec_piece.unit_offset_elements, rows * cols).view(rows, cols)
                    q, scale = self._split(dev_packed, piece)
                    ops.quantize_rows_i8(w, q, scale)
                self.host.narrow(0, packed.host_offset, packed.nbytes).copy_(
                    dev_packed.narrow(0, 0, packed.nbytes), non_blocking=True)
                stream.synchronize()  # the device buffers are reused by the next unit

    @staticmethod
    def _split(buffer, piece):
        rows, cols = piece.shape
        q = buffer.narrow(0, piece.q_offset, rows * cols).view(torch.int8).view(rows, cols)
        scale = buffer.narrow(0, piece.scale_offset, rows * 4).view(torch.float32)
        return q, scale

    def spans(self):
        """(host address, bytes) of every unit, in plan order (what the ring copies)."""

        base = self.host.data_ptr()
        return [(base + u.host_offset, u.nbytes) for u in self.units]

    def views(self, index, slot):
        """{key: (int8 [N, K], fp32 [N])} of unit ``index`` held in device ``slot``."""

        raw = slot.view(torch.uint8)
        if raw.numel() < self.units[index].nbytes:
            raise ValueError("device slot is smaller than the int8 unit")
        return {piece.key: self._split(raw, piece) for piece in self.units[index].pieces}
