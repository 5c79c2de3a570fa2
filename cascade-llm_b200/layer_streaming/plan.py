"""Static BF16 packing plan for Llama-3.1-8B (the layout contract).

Same public types and byte-identical layout as the reference
(``layer_streaming/plan.py:15-457``): every offset, unit, slot and vocab
chunk size is part of the drop-in contract (checkpoints are packed into the
host arena by it, and the reference's tests pin its numbers), so the
algorithm is kept while the code is this engine's own:

* tensors are packed in checkpoint order: per layer q, k, v, o, gate, up,
  down, each piece 256-byte aligned inside its transfer unit and each unit
  256-byte aligned in the host arena (``plan.py:12, :206-243``);
* units per layer by granularity: 7 matrices, 4 matrix groups
  (qkv | o | gate_up | down) or 1 layer (``:343-379``);
* after the units: host-only vocab tensors (streamed vocabulary), then the
  resident tensors (embedding + head unless streamed, 65 norms), each
  aligned on the host and on the device (``:381-417``);
* vocab chunk = floor(chunk_bytes / row_bytes) rows (``:423-441``);
  slot = the largest unit or vocab chunk (``:442-444``).
"""

from dataclasses import dataclass
from enum import Enum
from math import prod
from typing import Mapping, Optional, Tuple

MIB = 1024 * 1024
BF16_BYTES = 2
ALIGNMENT_BYTES = 256
_ALIGN = ALIGNMENT_BYTES // BF16_BYTES

HIDDEN = 4096
INTERMEDIATE = 14336
KV_WIDTH = 1024
VOCAB = 128256
LAYERS = 32
MODEL_ID = "meta-llama/Llama-3.1-8B"


class Granularity(str, Enum):
    """Smallest independently transferred model unit."""

    MATRIX = "matrix"
    MATRIX_GROUP = "matrix_group"
    LAYER = "layer"


def _round_up(value, multiple):
    return -(-value // multiple) * multiple


@dataclass(frozen=True)
class TensorSpec:
    key: str
    shape: Tuple[int, ...]
    resident: bool = False
    alias_of: Optional[str] = None

    @property
    def numel(self):
        return prod(self.shape)

    @property
    def nbytes(self):
        return self.numel * BF16_BYTES


@dataclass(frozen=True)
class UnitPiece:
    tensor: TensorSpec
    unit_offset_elements: int


@dataclass(frozen=True)
class TransferUnit:
    unit_id: str
    layer_index: int
    operation: str
    pieces: Tuple[UnitPiece, ...]
    elements: int
    host_offset_elements: int

    @property
    def nbytes(self):
        return self.elements * BF16_BYTES


@dataclass(frozen=True)
class ResidentPlacement:
    tensor: TensorSpec
    host_offset_elements: int
    device_offset_elements: int


@dataclass(frozen=True)
class HostPlacement:
    """CPU-only tensor placement inside the shared packed host arena."""

    tensor: TensorSpec
    host_offset_elements: int


@dataclass(frozen=True)
class VocabPlan:
    """Row-contiguous CPU vocabulary layout shared by lookup and projection."""

    embedding_key: str
    lm_head_key: str
    vocab_size: int
    hidden_size: int
    chunk_rows: int
    chunk_elements: int
    chunk_bytes: int
    chunk_count: int

    def chunk_range(self, index):
        """(first_row, end_row) of vocab chunk ``index``."""

        start = index * self.chunk_rows
        return start, min(start + self.chunk_rows, self.vocab_size)


@dataclass(frozen=True)
class ModelPlan:
    model_id: str
    granularity: Granularity
    tensors: Mapping[str, TensorSpec]
    units: Tuple[TransferUnit, ...]
    resident: Tuple[ResidentPlacement, ...]
    aliases: Mapping[str, str]
    host_arena_elements: int
    resident_arena_elements: int
    slot_elements: int
    dtype_bytes: int = BF16_BYTES
    slot_count: int = 2
    host_only: Tuple[HostPlacement, ...] = ()
    vocab: Optional[VocabPlan] = None

    @property
    def slot_bytes(self):
        return self.slot_elements * self.dtype_bytes

    @property
    def two_slot_bytes(self):
        return self.slot_count * self.slot_bytes

    @property
    def stream_bytes_per_token(self):
        return sum(unit.nbytes for unit in self.units)

    @property
    def resident_bytes(self):
        return self.resident_arena_elements * self.dtype_bytes

    @property
    def host_arena_bytes(self):
        return self.host_arena_elements * self.dtype_bytes

    def tensor_host_offset(self, key):
        """Element offset of ``key`` in the packed host arena."""

        table = self.__dict__.get("_offsets")
        if table is None:
            table = {}
            for unit in self.units:
                for piece in unit.pieces:
                    table.setdefault(
                        piece.tensor.key, unit.host_offset_elements + piece.unit_offset_elements
                    )
            for placement in self.resident:
                table.setdefault(placement.tensor.key, placement.host_offset_elements)
            for placement in self.host_only:
                table.setdefault(placement.tensor.key, placement.host_offset_elements)
            object.__setattr__(self, "_offsets", table)
        if key in table:
            return table[key]
        if key in self.aliases:
            return self.tensor_host_offset(self.aliases[key])
        raise KeyError(key)

    def as_dict(self):
        """JSON-ready summary (same keys and order as the reference's report)."""

        vocab = self.vocab
        return {
            "model_id": self.model_id,
            "granularity": self.granularity.value,
            "dtype": "torch.bfloat16",
            "dtype_bytes": self.dtype_bytes,
            "transfer_unit_count": len(self.units),
            "stream_bytes_per_token": self.stream_bytes_per_token,
            "slot_count": self.slot_count,
            "slot_bytes": self.slot_bytes,
            "two_slot_bytes": self.two_slot_bytes,
            "resident_bytes": self.resident_bytes,
            "host_arena_bytes": self.host_arena_bytes,
            "aliases": dict(self.aliases),
            "vocab": None if vocab is None else {
                "embedding_key": vocab.embedding_key,
                "lm_head_key": vocab.lm_head_key,
                "vocab_size": vocab.vocab_size,
                "hidden_size": vocab.hidden_size,
                "chunk_rows": vocab.chunk_rows,
                "chunk_bytes": vocab.chunk_bytes,
                "chunk_count": vocab.chunk_count,
            },
            "units": [
                {
                    "unit_id": u.unit_id,
                    "layer_index": u.layer_index,
                    "operation": u.operation,
                    "bytes": u.nbytes,
                    "pieces": [
                        {
                            "key": pc.tensor.key,
                            "shape": list(pc.tensor.shape),
                            "unit_offset_bytes": pc.unit_offset_elements * self.dtype_bytes,
                        }
                        for pc in u.pieces
                    ],
                }
                for u in self.units
            ],
            "resident": [
                {
                    "key": rp.tensor.key,
                    "shape": list(rp.tensor.shape),
                    "bytes": rp.tensor.nbytes,
                    "device_offset_bytes": rp.device_offset_elements * self.dtype_bytes,
                }
                for rp in self.resident
            ],
            "host_only": [
                {
                    "key": hp.tensor.key,
                    "shape": list(hp.tensor.shape),
                    "bytes": hp.tensor.nbytes,
                    "host_offset_bytes": hp.host_offset_elements * self.dtype_bytes,
                }
                for hp in self.host_only
            ],
        }


_PROJECTIONS = (
    ("self_attn", "q_proj", (HIDDEN, HIDDEN)),
    ("self_attn", "k_proj", (KV_WIDTH, HIDDEN)),
    ("self_attn", "v_proj", (KV_WIDTH, HIDDEN)),
    ("self_attn", "o_proj", (HIDDEN, HIDDEN)),
    ("mlp", "gate_proj", (INTERMEDIATE, HIDDEN)),
    ("mlp", "up_proj", (INTERMEDIATE, HIDDEN)),
    ("mlp", "down_proj", (HIDDEN, INTERMEDIATE)),
)
# matrix_group units: (operation, first projection index, end index)
_GROUPS = (("qkv", 0, 3), ("o_proj", 3, 4), ("gate_up", 4, 6), ("down_proj", 6, 7))


def _pack_unit(unit_id, layer, operation, tensors, cursor):
    pieces, inner = [], 0
    for spec in tensors:
        inner = _round_up(inner, _ALIGN)
        pieces.append(UnitPiece(spec, inner))
        inner += spec.numel
    start = _round_up(cursor, _ALIGN)
    unit = TransferUnit(
        unit_id=unit_id,
        layer_index=layer,
        operation=operation,
        pieces=tuple(pieces),
        elements=_round_up(inner, _ALIGN),
        host_offset_elements=start,
    )
    return unit, start + unit.elements


def build_llama31_8b_plan(
    granularity=Granularity.MATRIX,
    tie_word_embeddings=False,
    stream_vocab=False,
    vocab_chunk_bytes=128 * MIB,
):
    """Packed BF16 plan for the official Llama-3.1-8B geometry.

    Same signature and defaults as the reference (``plan.py:246-251``).
    ``tie_word_embeddings`` aliases ``lm_head.weight`` to the embedding;
    ``stream_vocab`` keeps both vocab matrices host-only, streamed in chunks
    of ``vocab_chunk_bytes``.
    """

    granularity = Granularity(granularity)
    specs = {}

    def spec(key, shape, resident=False, alias_of=None):
        specs[key] = TensorSpec(key, tuple(shape), resident, alias_of)
        return specs[key]

    embed = spec("model.embed_tokens.weight", (VOCAB, HIDDEN), resident=not stream_vocab)
    spec(
        "lm_head.weight",
        (VOCAB, HIDDEN),
        resident=not stream_vocab,
        alias_of=embed.key if tie_word_embeddings else None,
    )
    layers, norms = [], []
    for layer in range(LAYERS):
        prefix = "model.layers.{}".format(layer)
        layers.append(tuple(
            spec("{}.{}.{}.weight".format(prefix, block, name), shape)
            for block, name, shape in _PROJECTIONS
        ))
        norms.append(spec(prefix + ".input_layernorm.weight", (HIDDEN,), resident=True))
        norms.append(spec(prefix + ".post_attention_layernorm.weight", (HIDDEN,), resident=True))
    norms.append(spec("model.norm.weight", (HIDDEN,), resident=True))

    units, cursor = [], 0
    for layer, mats in enumerate(layers):
        if granularity == Granularity.LAYER:
            groups = (("layer", mats),)
            ids = ("layer_{:02d}".format(layer),)
        elif granularity == Granularity.MATRIX:
            groups = tuple((name, (m,)) for (_, name, _), m in zip(_PROJECTIONS, mats))
            ids = tuple("layer_{:02d}.{}".format(layer, name) for name, _ in groups)
        else:
            groups = tuple((op, mats[a:b]) for op, a, b in _GROUPS)
            ids = tuple("layer_{:02d}.{}".format(layer, op) for op, _ in groups)
        for unit_id, (operation, members) in zip(ids, groups):
            unit, cursor = _pack_unit(unit_id, layer, operation, members, cursor)
            units.append(unit)

    vocab_specs = [embed] + ([] if tie_word_embeddings else [specs["lm_head.weight"]])
    host_only = []
    if stream_vocab:
        for item in vocab_specs:
            cursor = _round_up(cursor, _ALIGN)
            host_only.append(HostPlacement(item, cursor))
            cursor += item.numel
    resident, device_cursor = [], 0
    for item in ([] if stream_vocab else vocab_specs) + norms:
        cursor = _round_up(cursor, _ALIGN)
        device_cursor = _round_up(device_cursor, _ALIGN)
        resident.append(ResidentPlacement(item, cursor, device_cursor))
        cursor += item.numel
        device_cursor += item.numel

    vocab = None
    if stream_vocab:
        row_bytes = HIDDEN * BF16_BYTES
        if int(vocab_chunk_bytes) < row_bytes:
            raise ValueError("vocab chunk must hold at least one row")
        rows = int(vocab_chunk_bytes) // row_bytes
        vocab = VocabPlan(
            embedding_key=embed.key,
            lm_head_key="lm_head.weight",
            vocab_size=VOCAB,
            hidden_size=HIDDEN,
            chunk_rows=rows,
            chunk_elements=rows * HIDDEN,
            chunk_bytes=rows * HIDDEN * BF16_BYTES,
            chunk_count=-(-VOCAB // rows),
        )
    slot = max(unit.elements for unit in units)
    if vocab is not None:
        slot = max(slot, vocab.chunk_elements)
    return ModelPlan(
        model_id=MODEL_ID,
        granularity=granularity,
        tensors=specs,
        units=tuple(units),
        resident=tuple(resident),
        aliases={"lm_head.weight": embed.key} if tie_word_embeddings else {},
        host_arena_elements=_round_up(cursor, _ALIGN),
        resident_arena_elements=_round_up(device_cursor, _ALIGN),
        slot_elements=slot,
        host_only=tuple(host_only),
        vocab=vocab,
    )
