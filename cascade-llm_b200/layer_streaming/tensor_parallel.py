"""Tensor-parallel Llama-3.1-8B decode across the GPUs of one node.

The reference executes one request on one GPU (``llama31.py:82-352``); this
module splits the same decode step over N = 1, 2, 4 or 8 GPUs, one process
per GPU (``torchrun``), with the Megatron split of a Llama block:

* rank r holds query heads ``[32r/N, 32(r+1)/N)`` and KV heads
  ``[8r/N, 8(r+1)/N)`` (a query head keeps its GQA KV head on the same rank),
  rows ``[14336r/N, 14336(r+1)/N)`` of gate_proj / up_proj, the matching
  COLUMNS of o_proj and down_proj, and vocabulary rows
  ``[128256r/N, 128256(r+1)/N)`` of the LM head; the embedding table, the
  norms and the residual stream are replicated;
* attention, the QKV / gate-up projections and the LM head run on local
  shards with no communication (with ``stream_layers`` weights each rank
  streams only its own layer shards from a pinned host arena through two
  device slots every step, the reference's H2D mode split N ways); o_proj and down_proj produce fp32 partial
  sums that are all-reduced before the residual add (two exchanges per
  layer), and the LM head's per-rank top-k candidates are all-gathered and
  merged (one exchange per token).

Two exchange paths:

``"peer"`` (default): the exchanges are fused into the projection kernels
(``cb_proj_allreduce_residual``, ``cb_lm_head_topk_allgather``): each CTA
stores its partial rows straight into every rank's exchange buffer over
NVLink (CUDA IPC mappings) and waits only for the same CTA of its peers, so a
one-token step is the single-GPU kernel sequence with no extra launches; it
is captured into one CUDA graph per context-length bucket. Multi-token steps
(prefill) use NCCL all-reduces of ``[M, 4096]`` partials.

``"nccl"``: every exchange is a ``torch.distributed`` NCCL collective between
stand-alone kernels (the baseline the fused path is measured against);
steps run eagerly.

Every rank ends a step with the same top-k (same bits); the residual stream
stays bit-identical across ranks because partials are summed in a fixed rank
order.
"""

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native, ops
from .llama31 import DecodeState, StaticKVCache, _matrix_key, attention_split, llama3_inv_freq

HIDDEN = 4096
FFN = 14336
HEADS = 32
KV_HEADS = 8
HEAD_DIM = 128
LAYERS = 32
VOCAB = 128256
SLOTS = 2 * LAYERS + 2  # exchange slots per step (even): o and down per layer, the LM head
LM_SLOT = 2 * LAYERS
_TOPK_MAX = 64
WORLD_SIZES = (1, 2, 4, 8)

_ROW_SPLIT = {"q_proj": HEADS * HEAD_DIM, "k_proj": KV_HEADS * HEAD_DIM, "v_proj": KV_HEADS * HEAD_DIM,
              "gate_proj": FFN, "up_proj": FFN}
_COLUMN_SPLIT = {"o_proj": HEADS * HEAD_DIM, "down_proj": FFN}


def _check_world(world, rank):
    if world not in WORLD_SIZES:
        raise ValueError("tensor parallelism over {} GPUs: Llama-3.1-8B splits over 1, 2, 4 or 8".format(world))
    if not 0 <= rank < world:
        raise ValueError("rank {} outside world {}".format(rank, world))


def shard_spec(key, world, rank):
    """``(dim, start, stop)`` of rank ``rank``'s part of tensor ``key``, or
    ``None`` when the tensor is replicated (embedding, norms)."""

    _check_world(world, rank)
    if key == "lm_head.weight":
        per = VOCAB // world
        return 0, rank * per, (rank + 1) * per
    name = key.split(".")[-2] if key.endswith(".weight") else ""
    if name in _ROW_SPLIT:
        per = _ROW_SPLIT[name] // world
        return 0, rank * per, (rank + 1) * per
    if name in _COLUMN_SPLIT:
        per = _COLUMN_SPLIT[name] // world
        return 1, rank * per, (rank + 1) * per
    return None


def shard_tensor(tensor, key, world, rank):
    """This rank's part of ``tensor`` (a contiguous copy, or ``tensor``
    itself when replicated)."""

    spec = shard_spec(key, world, rank)
    if spec is None:
        return tensor
    dim, start, stop = spec
    return tensor.narrow(dim, start, stop - start).contiguous()


def model_keys(layers=LAYERS):
    keys = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
    for layer in range(layers):
        keys.append("model.layers.{}.input_layernorm.weight".format(layer))
        keys.append("model.layers.{}.post_attention_layernorm.weight".format(layer))
        keys.extend(_matrix_key(layer, name) for name in
                    ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"))
    return keys


def full_shape(key):
    if key in ("model.embed_tokens.weight", "lm_head.weight"):
        return (VOCAB, HIDDEN)
    if key.endswith("layernorm.weight") or key == "model.norm.weight":
        return (HIDDEN,)
    name = key.split(".")[-2]
    if name in ("q_proj", "o_proj"):
        return (HIDDEN, HIDDEN)
    if name in ("k_proj", "v_proj"):
        return (KV_HEADS * HEAD_DIM, HIDDEN)
    if name in ("gate_proj", "up_proj"):
        return (FFN, HIDDEN)
    if name == "down_proj":
        return (HIDDEN, FFN)
    raise KeyError(key)


# the transfer units of a rank's streamed layer shards, in stream order per
# layer: (unit, [(matrix, rows, columns) of this rank's shard ...]); a unit's
# pieces are consecutive rows of one contiguous block
def shard_units(world):
    q, kv, f = HEADS * HEAD_DIM // world, KV_HEADS * HEAD_DIM // world, FFN // world
    return (
        ("qkv", (("q_proj", q, HIDDEN), ("k_proj", kv, HIDDEN), ("v_proj", kv, HIDDEN))),
        ("o_proj", (("o_proj", HIDDEN, HIDDEN // world),)),
        ("gate_up", (("gate_proj", f, HIDDEN), ("up_proj", f, HIDDEN))),
        ("down_proj", (("down_proj", HIDDEN, f),)),
    )


class ShardArena:
    """A rank's layer shards packed for H2D streaming: the 4 units of every
    layer back to back (each unit 256-byte aligned) in ONE host arena
    (pinned by default), so the rank streams only its own shard - 1/N of the
    reference's per-token transfer (weight_store.py:184-206 streams the
    whole model) - through the same two-slot pipeline."""

    ALIGN = 128  # elements (256 bytes)

    def __init__(self, world, rank, layers=LAYERS, pin=True):
        _check_world(world, rank)
        self.world = world
        self.rank = rank
        self.layers = layers
        self.units = []  # (layer, unit name, element offset, elements, ((key, offset, rows, cols), ...))
        cursor = 0
        for layer in range(layers):
            for name, pieces in shard_units(world):
                placed, inner = [], 0
                for matrix, rows, cols in pieces:
                    placed.append((_matrix_key(layer, matrix), inner, rows, cols))
                    inner += rows * cols
                self.units.append((layer, name, cursor, inner, tuple(placed)))
                cursor += -(-inner // self.ALIGN) * self.ALIGN
        self.elements = cursor
        self.unit_elements = max(u[3] for u in self.units)
        self.storage = torch.empty(cursor, dtype=torch.bfloat16, pin_memory=pin)

    @property
    def nbytes(self):
        return 2 * self.elements

    def host_view(self, key):
        for _, _, offset, _, pieces in self.units:
            for k, inner, rows, cols in pieces:
                if k == key:
                    return self.storage.narrow(0, offset + inner, rows * cols).view(rows, cols)
        raise KeyError(key)

    def spans(self):
        base = self.storage.data_ptr()
        return [(base + 2 * offset, 2 * elements) for _, _, offset, elements, _ in self.units]

    def views(self, index, slot):
        """{key: device view} of unit ``index`` landed in ``slot``."""

        return {k: slot.narrow(0, inner, rows * cols).view(rows, cols)
                for k, inner, rows, cols in self.units[index][4]}


class TensorParallelWeights:
    """This rank's weight shards: resident in HBM (bf16), or with the layer
    matrices in a :class:`ShardArena` streamed every step (``arena``) and
    only the embedding, the norms and the LM-head shard resident."""

    def __init__(self, world, rank, device, tensors, arena=None):
        _check_world(world, rank)
        self.world = world
        self.rank = rank
        self.device = torch.device(device)
        self.tensors = tensors
        self.arena = arena

    def __getitem__(self, key):
        return self.tensors[key]

    def __contains__(self, key):
        return key in self.tensors

    @property
    def streamed(self):
        return self.arena is not None

    @property
    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in self.tensors.values())

    @staticmethod
    def _is_layer_matrix(key):
        return key.startswith("model.layers.") and not key.endswith("layernorm.weight")

    @classmethod
    def from_store(cls, store, world, rank, device, stream_layers=False):
        """Shards of a loaded weight store (host arena, ``store.tensor(key)``);
        ``stream_layers`` packs the layer matrices into a pinned
        :class:`ShardArena` instead of HBM."""

        device = torch.device(device)
        arena = ShardArena(world, rank) if stream_layers else None
        tensors = {}
        with torch.cuda.device(device):
            for key in model_keys():
                part = shard_tensor(store.tensor(key), key, world, rank)
                if arena is not None and cls._is_layer_matrix(key):
                    arena.host_view(key).copy_(part)
                else:
                    tensors[key] = part.to(device=device, non_blocking=False)
        return cls(world, rank, device, tensors, arena)

    @classmethod
    def seeded(cls, world, rank, device, seed=0, std=0.02, stream_layers=False):
        """The seeded random-init model of ``BaseWeightStore.fill_seeded``
        (element i of ``key`` = element i of stream ``cb_stream_key(seed,
        key)``; norms = 1), generated on the GPU and sharded: every rank's
        shards are slices of the same full tensors. ``stream_layers`` keeps
        the layer matrices in a pinned :class:`ShardArena` (streamed mode)."""

        from .weight_store import is_norm

        device = torch.device(device)
        arena = ShardArena(world, rank) if stream_layers else None
        tensors = {}
        with torch.cuda.device(device), torch.inference_mode():
            scratch = torch.empty(VOCAB * HIDDEN, dtype=torch.bfloat16, device=device)
            for key in model_keys():
                shape = full_shape(key)
                numel = 1
                for d in shape:
                    numel *= d
                full = scratch[:numel].view(shape)
                if is_norm(key):
                    full.fill_(1.0)
                else:
                    ops.fill_normal_(full, _native.stream_key(seed, key), std=std)
                if arena is not None and cls._is_layer_matrix(key):
                    arena.host_view(key).copy_(shard_tensor(full, key, world, rank))
                else:
                    tensors[key] = shard_tensor(full, key, world, rank).clone()
            del scratch
            torch.cuda.synchronize(device)
        return cls(world, rank, device, tensors, arena)


@dataclass
class _Group:
    """World/rank of the decoder's process group (world 1 without one)."""

    group: object
    world: int
    rank: int

    @classmethod
    def of(cls, group):
        if dist.is_available() and dist.is_initialized():
            return cls(group, dist.get_world_size(group), dist.get_rank(group))
        return cls(None, 1, 0)

    def all_reduce(self, tensor):
        if self.world > 1:
            dist.all_reduce(tensor, group=self.group)

    def all_gather(self, tensor):
        if self.world == 1:
            return tensor.unsqueeze(0)
        out = torch.empty((self.world,) + tuple(tensor.shape), dtype=tensor.dtype, device=tensor.device)
        dist.all_gather_into_tensor(out, tensor.contiguous(), group=self.group)
        return out

    def barrier(self):
        if self.world == 1:
            return
        if dist.get_backend(self.group) == "nccl":
            # a one-element all-reduce on this rank's device, then a host wait
            token = torch.zeros(1, device=torch.cuda.current_device())
            dist.all_reduce(token, group=self.group)
            token.item()
        else:
            dist.barrier(group=self.group)


class ExchangeBuffers:
    """This rank's exchange buffer and the peers' buffers mapped into this
    process (CUDA IPC), as the host pointer array the exchange kernels take."""

    def __init__(self, group, device):
        lib = _native.lib()
        self.group = group
        self.device = torch.device(device)
        self.own = ctypes.c_void_p()
        self._opened = []
        with torch.cuda.device(self.device):
            _native.check(lib.cb_exchange_alloc(ctypes.byref(self.own)), "cb_exchange_alloc")
            pointers = [None] * group.world
            pointers[group.rank] = self.own.value
            if group.world > 1:
                handle = (ctypes.c_uint8 * 64)()
                _native.check(lib.cb_ipc_handle(self.own, handle), "cb_ipc_handle")
                mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
                handles = group.all_gather(mine).cpu()
                for q in range(group.world):
                    if q == group.rank:
                        continue
                    raw = (ctypes.c_uint8 * 64)(*handles[q].tolist())
                    peer = ctypes.c_void_p()
                    _native.check(lib.cb_ipc_open(raw, ctypes.byref(peer)), "cb_ipc_open")
                    self._opened.append(peer.value)
                    pointers[q] = peer.value
            self.pointers = (ctypes.c_void_p * group.world)(*pointers)
        # no rank may push into a buffer before its owner has zeroed it
        torch.cuda.synchronize(self.device)
        group.barrier()

    def close(self):
        lib = _native.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for peer in self._opened:
                lib.cb_ipc_close(ctypes.c_void_p(peer))
            self._opened = []
            if self.own.value:
                lib.cb_exchange_free(self.own)
                self.own = ctypes.c_void_p()


class TensorParallelDecoder:
    """One request decoded by all ranks of ``group`` (the default group when
    ``torch.distributed`` is initialised, else a world of one).

    ``decoder(input_ids)`` runs one step (prefill of the prompt, then one
    token per call) and returns a :class:`DecodeState` whose
    ``topk_values`` / ``topk_indices`` ``[1, 1, k]`` (device tensors) are the
    same on every rank. Full logits are not produced.
    """

    def __init__(self, config, weights, group=None, top_k=10, max_length=None, use_graphs=True,
                 exchange="peer", profile=False):
        for name, value in (("hidden_size", HIDDEN), ("intermediate_size", FFN),
                            ("num_hidden_layers", LAYERS), ("num_attention_heads", HEADS),
                            ("num_key_value_heads", KV_HEADS), ("vocab_size", VOCAB)):
            if getattr(config, name, None) != value:
                raise ValueError("config {}={} is not Llama-3.1-8B value {}".format(
                    name, getattr(config, name, None), value))
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.group = _Group.of(group)
        if (self.group.world, self.group.rank) != (weights.world, weights.rank):
            raise ValueError("weights are rank {} of {}, the process group is rank {} of {}".format(
                weights.rank, weights.world, self.group.rank, self.group.world))
        self.top_k = int(top_k)
        if not 1 <= self.top_k <= _TOPK_MAX:
            raise ValueError("top_k must be in [1, {}]".format(_TOPK_MAX))
        self.config = config
        self.weights = weights
        self.exchange = exchange
        self.device = weights.device
        if self.device.type != "cuda":
            raise RuntimeError("tensor-parallel decode needs CUDA devices (there is no CPU path)")
        world = self.group.world
        self.q_heads = HEADS // world
        self.kv_heads = KV_HEADS // world
        self.ffn = FFN // world
        self.vocab_rows = VOCAB // world
        self.eps = float(getattr(config, "rms_norm_eps", 1e-5))
        # a streamed step waits on the host for its copies: it runs eagerly
        self.use_graphs = bool(use_graphs) and exchange == "peer" and not weights.streamed
        self.profile = bool(profile)
        self.last_stream = None
        lib = _native.lib()
        with torch.cuda.device(self.device):
            _native.check(lib.cb_prepare(), "cb_prepare")
            self.kv_cache = StaticKVCache(LAYERS, capacity=max_length, kv_heads=self.kv_heads)
            self.kv_cache.bind(self.device)
            self.inv_freq = llama3_inv_freq(config).to(self.device)
            self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
            _native.check(lib.cb_set_error_word(self.error_word.data_ptr()), "cb_set_error_word")
            self.lm_workspace = torch.empty(ops.lm_head_workspace_bytes(self.top_k), dtype=torch.uint8,
                                            device=self.device)
            self.lm_ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.values = torch.empty((1, 1, self.top_k), dtype=torch.float32, device=self.device)
            self.indices = torch.empty((1, 1, self.top_k), dtype=torch.int64, device=self.device)
            self._ids_dev = torch.zeros(1, dtype=torch.int64, device=self.device)  # one-token step input
        self.exchange_buffers = ExchangeBuffers(self.group, self.device) if exchange == "peer" else None
        self._ring = None
        if weights.streamed:
            # two device slots of the largest unit, fed from this rank's pinned shard arena
            from .streaming import SlotRing

            self.slots = [torch.empty(weights.arena.unit_elements, dtype=torch.bfloat16, device=self.device)
                          for _ in range(2)]
            self.copy_stream = torch.cuda.Stream(device=self.device)
            self.compute_stream = torch.cuda.Stream(device=self.device)
            self._ring = SlotRing(self.slots, self.copy_stream)
        self.sm_count = int(lib.cb_sm_count())
        self._graphs = {}
        self._rows = 0
        self._attn_ws = None
        self._attn_ws_bytes = 0
        self._tokens = 0
        self._buffers(1)

    # ---------------------------------------------------------------- buffers
    def _buffers(self, rows):
        if rows <= self._rows:
            return
        rows = max(rows, 2 * self._rows)
        dev = self.device
        local = self.q_heads * HEAD_DIM
        self._x = torch.empty((rows, HIDDEN), dtype=torch.bfloat16, device=dev)
        self._xn = torch.empty((rows, HIDDEN), dtype=torch.bfloat16, device=dev)  # normalised rows (prefill)
        self._q = torch.empty((rows, local), dtype=torch.bfloat16, device=dev)
        self._attn = torch.empty((rows, local), dtype=torch.bfloat16, device=dev)
        self._mlp = torch.empty((rows, self.ffn), dtype=torch.bfloat16, device=dev)
        self._partial = torch.empty((rows, HIDDEN), dtype=torch.float32, device=dev)
        self._tickets = torch.zeros(self.kv_heads * rows, dtype=torch.int32, device=dev)
        self._rows = rows
        self._graphs.clear()

    def _attention_workspace(self, tokens, splits):
        need = ops.attention_workspace_bytes(tokens, splits)
        if need > self._attn_ws_bytes:
            self._attn_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._attn_ws_bytes = need
            self._graphs.clear()
        return self._attn_ws

    def attention_config(self, tokens, length):
        return attention_split(tokens, length, self.sm_count, kv_heads=self.kv_heads)

    def check_errors(self):
        code = int(self.error_word.item())
        if code:
            self.error_word.zero_()
            raise RuntimeError("a cascade kernel reported device error code {}".format(code))

    def close(self):
        self._graphs.clear()
        if self._ring is not None:
            self._ring.close()
            self._ring = None
        if self.exchange_buffers is not None:
            self.exchange_buffers.close()
            self.exchange_buffers = None

    # ---------------------------------------------------------------- a step
    def _w(self, layer, name):
        return self.weights[_matrix_key(layer, name)]

    def _exchange_args(self, slot):
        buf = self.exchange_buffers
        return (buf.pointers, self.group.rank, self.group.world, slot, SLOTS, self.epoch.data_ptr())

    def _proj(self, layer, which, source, weight, tokens, fused):
        """x += all-reduce(source . W_shard^T) for o_proj / down_proj."""

        if fused:
            lib = _native.lib()
            stream = _native.stream_ptr(self.device)
            _native.check(
                lib.cb_proj_allreduce_residual(
                    source[0].data_ptr(), weight.shape[1], weight.data_ptr(), weight.shape[0],
                    self._x[0].data_ptr(), self._x[0].data_ptr(),
                    *self._exchange_args(2 * layer + which), stream),
                "cb_proj_allreduce_residual",
            )
            return
        if tokens > 1:
            ops.gemm_partial(source[:tokens], weight, self._partial[:tokens])
        else:
            ops.proj_partial(source[0], weight, self._partial[0])
        self.group.all_reduce(self._partial[:tokens])
        ops.residual_add_f32(self._x[:tokens], self._partial[:tokens], self._x[:tokens])

    def _unit(self, layer, unit, mats, tokens, splits, chunk, fused):
        """One transfer unit of a layer (``qkv``, ``o_proj``, ``gate_up`` or
        ``down_proj``) with its weight matrices ``mats`` (resident shards, or
        views of a device slot in the streamed mode)."""

        w = self.weights
        cache = self.kv_cache
        pos = cache.position
        kc, vc = cache.key(layer), cache.value(layer)
        m = lambda name: mats[_matrix_key(layer, name)]
        if unit == "qkv":
            norm_in = w["model.layers.{}.input_layernorm.weight".format(layer)]
            if tokens > 1:  # prefill: tcgen05 GEMM over the step's tokens
                ops.rmsnorm(self._x[:tokens], norm_in, self.eps, self._xn[:tokens])
                ops.prefill_qkv_rope(self._xn[:tokens], m("q_proj"), m("k_proj"), m("v_proj"), self.inv_freq, pos,
                                     self._q[:tokens], kc, vc, self.q_heads, self.kv_heads)
            else:
                ops.qkv_rope(self._x[0], norm_in, self.eps, m("q_proj"), m("k_proj"), m("v_proj"), self.inv_freq,
                             pos, 0, self._q[0], kc, vc, self.q_heads, self.kv_heads)
        elif unit == "o_proj":
            if tokens > 1:
                ops.prefill_attention(self._q[:tokens], kc, vc, pos, self._attn[:tokens])
            else:
                ws = self._attention_workspace(tokens, splits)
                ops.attention(self._q[:tokens], kc, vc, pos, splits, chunk, self._attn[:tokens], ws, self._tickets)
            self._proj(layer, 0, self._attn, m("o_proj"), tokens, fused)
        elif unit == "gate_up":
            norm_post = w["model.layers.{}.post_attention_layernorm.weight".format(layer)]
            if tokens > 1:
                ops.rmsnorm(self._x[:tokens], norm_post, self.eps, self._xn[:tokens])
                ops.gemm_swiglu(self._xn[:tokens], m("gate_proj"), m("up_proj"), self._mlp[:tokens])
            else:
                ops.gate_up_swiglu(self._x[0], norm_post, self.eps, m("gate_proj"), m("up_proj"), self._mlp[0])
        else:
            self._proj(layer, 1, self._mlp, m("down_proj"), tokens, fused)

    def _layer(self, layer, tokens, splits, chunk, fused):
        for unit, _ in shard_units(self.group.world):
            self._unit(layer, unit, self.weights, tokens, splits, chunk, fused)

    def _head(self, tokens):
        last = self._x[tokens - 1]
        w = self.weights
        k = self.top_k
        offset = self.group.rank * self.vocab_rows
        if self.exchange == "peer":
            lib = _native.lib()
            _native.check(
                lib.cb_lm_head_topk_allgather(
                    last.data_ptr(), w["model.norm.weight"].data_ptr(), self.eps, w["lm_head.weight"].data_ptr(),
                    self.vocab_rows, offset, k, self.values.data_ptr(), self.indices.data_ptr(),
                    self.lm_workspace.data_ptr(), self.lm_ticket.data_ptr(), *self._exchange_args(LM_SLOT),
                    _native.stream_ptr(self.device)),
                "cb_lm_head_topk_allgather",
            )
        else:
            values = torch.empty(k, dtype=torch.float32, device=self.device)
            indices = torch.empty(k, dtype=torch.int64, device=self.device)
            ops.lm_head_topk(last, w["model.norm.weight"], self.eps, w["lm_head.weight"], offset, k, None,
                             values, indices, self.lm_workspace, self.lm_ticket)
            all_values = self.group.all_gather(values).reshape(-1)
            all_indices = self.group.all_gather(indices).reshape(-1)
            ops.topk_merge(None, None, all_values, all_indices, k, self.values.view(-1), self.indices.view(-1))

    def _step(self, tokens, splits, chunk):
        fused = self.exchange == "peer" and tokens == 1
        if self.weights.streamed:
            arena = self.weights.arena

            def body(index, slot):
                layer, unit = arena.units[index][0], arena.units[index][1]
                self._unit(layer, unit, arena.views(index, slot), tokens, splits, chunk, fused)

            self.last_stream = self._ring.run(arena.spans(), body, self.compute_stream,
                                              torch.cuda.current_stream(self.device), profile=self.profile)
        else:
            for layer in range(LAYERS):
                self._layer(layer, tokens, splits, chunk, fused)
        self._head(tokens)
        ops.position_advance(self.kv_cache.position, tokens)
        ops.position_advance(self.epoch, 1)

    def __call__(self, input_ids, position_ids=None):
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("one unpadded request per decoder")
        tokens = int(input_ids.shape[1])
        if tokens < 1:
            raise ValueError("input_ids is empty")
        past = self.kv_cache.length
        if position_ids is not None and int(position_ids.reshape(-1)[0]) != past:
            raise ValueError("position_ids must continue the cached sequence")
        with torch.cuda.device(self.device):
            self.kv_cache.reserve(past + tokens)
            self._buffers(tokens)
            if tokens == 1 and self.use_graphs:
                # the id goes into a persistent device slot (asynchronous from
                # pinned memory); the step's graph starts with its embedding
                self._ids_dev.copy_(input_ids.reshape(-1), non_blocking=True)
                self._replay()
            else:
                ids = input_ids.reshape(-1).to(device=self.device, dtype=torch.int64)
                ops.embedding(ids, self.weights["model.embed_tokens.weight"], self._x[:tokens])
                splits, chunk = self.attention_config(tokens, past + tokens)
                self._step(tokens, splits, chunk)
        self.kv_cache.length += tokens
        self._tokens = tokens
        return DecodeState(
            hidden_states=self._x[:tokens].view(1, tokens, HIDDEN),
            position_ids=torch.arange(past, past + tokens, dtype=torch.long).unsqueeze(0),
            topk_values=self.values,
            topk_indices=self.indices,
        )

    def _replay(self):
        length = self.kv_cache.length + 1
        bucket = min(max(64, 1 << (length - 1).bit_length()), self.kv_cache.capacity)
        splits, chunk = self.attention_config(1, bucket)
        key = (bucket, self.kv_cache.generation, self._rows)
        graph = self._graphs.get(key)
        if graph is None:
            self._attention_workspace(1, splits)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ops.embedding(self._ids_dev, self.weights["model.embed_tokens.weight"], self._x[:1])
                self._step(1, splits, chunk)
            # every rank captured the same graph; start replaying together
            torch.cuda.synchronize(self.device)
            self.group.barrier()
            self._graphs[key] = graph
        graph.replay()
