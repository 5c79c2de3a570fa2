"""Llama-3.1-8B decode executor on the sm_100a kernels.

Drop-in for ``layer_streaming/llama31.py`` of the reference: the same class
names, constructor signature, ``begin / __call__(unit, weights, state) /
finish`` protocol and :class:`DecodeState` fields. Every tensor op of the
reference is replaced by one fused kernel per transfer unit:

==============  =====================================================  ============================
unit            reference ops (llama31.py)                             kernel (torch.ops.cascade)
==============  =====================================================  ============================
qkv / q,k,v     RMSNorm :173-179, 3x F.linear :241-245, RoPE :206-212,  qkv_rope (prefill:
                KV-cache cat :44-50                                    rmsnorm + prefill_qkv_rope)
o_proj          repeat_kv + SDPA :182-234, F.linear + residual :246-250 attention, proj_residual
                                                                       (prefill: prefill_attention,
                                                                       gemm_residual)
gate_up / g,u   RMSNorm :255-263, F.linear, silu :264-271              gate_up_swiglu (gate_silu,
                                                                       up_mul for ``matrix``;
                                                                       prefill: gemm_swiglu)
down_proj       gate*up, F.linear + residual :272-280                 proj_residual (prefill:
                                                                       gemm_residual)
finish          RMSNorm :325-329, LM head + topk :330-348              lm_head_topk (+ vocab path)
==============  =====================================================  ============================

Multi-token steps (the prompt) run the fused units as tcgen05 tensor-core
GEMMs over all the step's tokens; the ``matrix`` granularity's separate q/k/v
and gate/up units keep the per-token GEMVs.

The KV cache is pre-allocated (:class:`StaticKVCache`, ``[layers, 2, 8,
capacity, 128]``) and the request position is a device counter, so a
one-token step has no host synchronisation and no allocation: with the
weights resident in HBM (``DoubleBufferRuntime(weights="hbm")``) the whole
layer stack of a decode step is captured once per context-length bucket and
replayed as one CUDA graph.
"""

import math
import os
from dataclasses import dataclass, field

import torch

from . import _native, ops

LLAMA31_8B_MODEL_ID = "meta-llama/Llama-3.1-8B"
MATRIX_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
_UNIT_OPS = {
    "layer": ("qkv", "o_proj", "gate_up", "down_proj"),
    "qkv": ("qkv",),
    "gate_up": ("gate_up",),
}
_TOPK_MAX = 64
# prefill chunks of at most this many tokens split the GEMMs' K range (one
# 128-row tile leaves most SMs idle); workspace and per-tile tickets
_SPLIT_K_MAX_TOKENS = 64
_SPLIT_K_BYTES = 16 << 20
_SPLIT_K_TICKETS = 1024
_DEFAULT_CAPACITY = 8192


def _matrix_key(layer, name):
    block = "self_attn" if name in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
    return "model.layers.{}.{}.{}.weight".format(layer, block, name)


def llama3_inv_freq(config):
    """Inverse RoPE frequencies (fp32 [64]) for the config's rope parameters.

    The llama3 frequency scaling of transformers'
    ``_compute_llama3_parameters`` (modeling_rope_utils.py:550-626), which
    the reference reaches through ``LlamaRotaryEmbedding`` (llama31.py:125),
    evaluated once with the same fp32 operations.
    """

    params = dict(getattr(config, "rope_parameters", None) or {})
    scaling = getattr(config, "rope_scaling", None) or {}
    params = {**scaling, **params}
    theta = float(params.get("rope_theta", getattr(config, "rope_theta", 500000.0)))
    dim = config.hidden_size // config.num_attention_heads
    exponents = torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float)
    inv_freq = 1.0 / (theta ** (exponents / dim))
    rope_type = params.get("rope_type", params.get("type", "default"))
    if rope_type == "default":
        return inv_freq
    if rope_type != "llama3":
        raise ValueError("unsupported rope_type {!r} (llama3 or default)".format(rope_type))
    factor = params["factor"]
    low = params["low_freq_factor"]
    high = params["high_freq_factor"]
    old_len = params["original_max_position_embeddings"]
    wavelen = 2 * math.pi / inv_freq
    scaled = torch.where(wavelen > old_len / low, inv_freq / factor, inv_freq)
    smooth = (old_len / wavelen - low) / (high - low)
    smoothed = (1 - smooth) * scaled / factor + smooth * scaled
    medium = ~(wavelen < old_len / high) * ~(wavelen > old_len / low)
    return torch.where(medium, smoothed, scaled)


FUSED_ATTENTION_MAX_LENGTH = 8192  # CASCADE_B200_FUSED_ATTENTION=1: one-token steps up to this context
FUSED_ATTENTION_SPLITS = 18        # run attention + o_proj as one kernel (144 attention CTAs, 152 for W_o)


def attention_split(tokens, length, sm_count, kv_heads=8):
    """(splits, chunk) for the split-KV attention kernel: about two CTAs per
    SM over (splits x KV heads x tokens), chunks a multiple of 64 positions."""

    target = max(1, (2 * sm_count) // (kv_heads * tokens))
    per_split = -(-length // target)
    chunk = max(64, -(-per_split // 64) * 64)
    return -(-length // chunk), chunk


class StaticKVCache:
    """Pre-allocated single-request KV cache ``[layers, 2, 8, capacity, 128]``.

    Replaces ``SimpleKVCache`` (llama31.py:34-54), which re-allocates and
    copies the whole cache with ``torch.cat`` on every token. Keys are stored
    after RoPE, like the reference. ``position`` is the device int32 counter
    of the next position; ``length`` is its host mirror. The storage is
    allocated when an executor binds the cache to its device.
    """

    def __init__(self, layer_count=32, capacity=None, kv_heads=8, head_dim=128):
        self.layer_count = int(layer_count)
        self.capacity = int(capacity or os.environ.get("CASCADE_B200_MAX_LENGTH", _DEFAULT_CAPACITY))
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.storage = None
        self.position = None
        self.length = 0
        self.generation = 0  # bumped when storage moves (invalidates graphs)

    def bind(self, device):
        if self.storage is None:
            self._allocate(torch.device(device), self.capacity)
        return self

    def _allocate(self, device, capacity):
        storage = torch.empty(
            (self.layer_count, 2, self.kv_heads, capacity, self.head_dim), dtype=torch.bfloat16, device=device
        )
        if self.storage is not None and self.length:
            storage[:, :, :, :self.length].copy_(self.storage[:, :, :, :self.length])
        self.storage = storage
        if self.position is None:
            self.position = torch.zeros(1, dtype=torch.int32, device=device)
        self.capacity = capacity
        self.generation += 1

    def reserve(self, length):
        """Grow (copying the valid prefix) so that ``length`` positions fit."""

        if length > self.capacity:
            self._allocate(self.storage.device, max(length, 2 * self.capacity))

    def key(self, layer):
        return self.storage[layer, 0]

    def value(self, layer):
        return self.storage[layer, 1]

    def sequence_length(self):
        return self.length

    @property
    def entries(self):
        """Per-layer ``(key, value)`` views ``[1, 8, length, 128]`` (None if empty)."""

        if self.storage is None or self.length == 0:
            return [None] * self.layer_count
        return [
            (self.storage[i, 0, :, :self.length].unsqueeze(0), self.storage[i, 1, :, :self.length].unsqueeze(0))
            for i in range(self.layer_count)
        ]

    def clear(self):
        self.length = 0
        if self.position is not None:
            ops.position_set(self.position, None, 0)


SimpleKVCache = StaticKVCache


@dataclass
class DecodeState:
    hidden_states: torch.Tensor
    position_ids: torch.Tensor
    layer_values: dict = field(default_factory=dict)
    logits: object = None
    topk_values: object = None
    topk_indices: object = None


class Llama31DecodeExecutor:
    """Stateful callbacks consumed by :class:`DoubleBufferRuntime`.

    One unpadded request: a multi-token prefill, then one-token decode steps
    (``allow_chunked_prefill=True`` additionally accepts multi-token steps
    after the prefill, which the reference refuses). ``max_length`` sizes the
    KV cache (grown on demand). ``use_graphs`` enables CUDA-graph replay of
    one-token steps when the runtime keeps the weights in HBM.
    """

    def __init__(self, config, resident, kv_cache=None, vocab_runtime=None, top_k=10,
                 return_full_logits=False, max_length=None, allow_chunked_prefill=False,
                 use_graphs=True, decode_weights=None):
        expected = {
            "hidden_size": 4096,
            "intermediate_size": 14336,
            "num_hidden_layers": 32,
            "num_attention_heads": 32,
            "num_key_value_heads": 8,
            "vocab_size": 128256,
        }
        for name, value in expected.items():
            if getattr(config, name, None) != value:
                raise ValueError(
                    "config {}={} is not Llama-3.1-8B value {}".format(name, getattr(config, name, None), value)
                )
        self.config = config
        self.resident = resident
        self.vocab_runtime = vocab_runtime
        self.top_k = int(top_k)
        self.return_full_logits = bool(return_full_logits)
        if self.top_k < 1:
            raise ValueError("top_k must be positive")
        if self.top_k > _TOPK_MAX:
            raise ValueError("the fused LM-head kernel supports top_k <= {}".format(_TOPK_MAX))
        self.device = torch.device(resident.device)
        if self.device.type != "cuda":
            raise RuntimeError("the B200 executor needs a CUDA device (there is no CPU path)")
        self.eps = float(getattr(config, "rms_norm_eps", 1e-5))
        self.allow_chunked_prefill = bool(allow_chunked_prefill)
        self.use_graphs = bool(use_graphs) and os.environ.get("CASCADE_B200_GRAPHS", "1") != "0"
        lib = _native.lib()
        with torch.cuda.device(self.device):
            _native.check(lib.cb_prepare(), "cb_prepare")
            self.kv_cache = kv_cache if kv_cache is not None else StaticKVCache(config.num_hidden_layers)
            if not isinstance(self.kv_cache, StaticKVCache):
                raise TypeError("kv_cache must be a StaticKVCache (SimpleKVCache)")
            if max_length is not None:
                self.kv_cache.capacity = max(self.kv_cache.capacity, int(max_length))
            self.kv_cache.bind(self.device)
            self.inv_freq = llama3_inv_freq(config).to(self.device)
            self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
            _native.check(lib.cb_set_error_word(self.error_word.data_ptr()), "cb_set_error_word")
            self.lm_workspace = torch.empty(
                ops.lm_head_workspace_bytes(self.top_k), dtype=torch.uint8, device=self.device
            )
            self.lm_ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._ids_dev = torch.zeros(1, dtype=torch.int64, device=self.device)  # one-token step input
        self._embed_pending = False
        self.sm_count = int(lib.cb_sm_count())
        self.fuse_attention = os.environ.get("CASCADE_B200_FUSED_ATTENTION", "0") == "1"
        self._fused_max_splits = int(lib.cb_attention_oproj_max_splits())
        self._graphs = {}
        # layer -> (gate, up) device views of the HBM-resident runtime `_stage_owner`; `_stage_active`
        # is set only while run_units_resident issues a one-token step
        self._stage_slabs, self._stage_owner, self._stage_active = {}, None, False
        self._split_k_ws = self._split_k_tickets = None
        # optional int8 weight-only one-token steps (HBM-resident runtimes):
        # key -> (int8 [N, K], fp32 scales [N]) quantized from `_i8_owner`'s views
        self.decode_weights = decode_weights or os.environ.get("CASCADE_B200_DECODE_WEIGHTS", "bf16")
        if self.decode_weights not in ("bf16", "int8"):
            raise ValueError("decode_weights must be 'bf16' or 'int8'")
        self._i8, self._i8_owner, self._i8_active, self._i8_step = {}, None, False, False
        self._deq = None  # bf16 scratch of a unit that arrived as int8 (prefill)
        self._rows = 0
        self._buffers(1)
        self._attn_ws = None
        self._attn_ws_bytes = 0
        self._tokens = 0

    # ---------------------------------------------------------------- buffers
    def _buffers(self, rows):
        """Activation rows: residual stream x, q, attention output, mlp."""

        if rows <= self._rows:
            return
        rows = max(rows, 2 * self._rows)
        dev = self.device
        self._x = torch.empty((rows, 4096), dtype=torch.bfloat16, device=dev)
        self._xn = torch.empty((rows, 4096), dtype=torch.bfloat16, device=dev)  # normalised rows (prefill)
        self._q = torch.empty((rows, 4096), dtype=torch.bfloat16, device=dev)
        self._attn = torch.empty((rows, 4096), dtype=torch.bfloat16, device=dev)
        self._mlp = torch.empty((rows, 14336), dtype=torch.bfloat16, device=dev)
        # per (token, KV head) tickets, then the fused kernel's two counters (kept zero by the kernels)
        self._tickets = torch.zeros(8 * rows + 8, dtype=torch.int32, device=dev)
        self._rows = rows
        self._graphs.clear()

    def attention_config(self, tokens, length):
        """(splits, chunk, fused) of the decode attention for `length` keys:
        chunk 0 lets the kernel size the splits from the device position, so
        one captured launch serves every length up to `length`; fused runs
        attention and o_proj as one kernel (one-token steps)."""

        if tokens == 1 and self.fuse_attention and length <= FUSED_ATTENTION_MAX_LENGTH:
            return min(FUSED_ATTENTION_SPLITS, self._fused_max_splits), 0, True
        splits, _ = attention_split(tokens, length, self.sm_count)
        return splits, 0, False

    def _attention_workspace(self, tokens, splits):
        need = ops.attention_workspace_bytes(tokens, splits)
        if need > self._attn_ws_bytes:
            self._attn_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._attn_ws_bytes = need
            self._graphs.clear()
        return self._attn_ws

    def check_errors(self):
        """Raise if a kernel reported a timed-out wait or a bad index."""

        code = int(self.error_word.item())
        if code:
            self.error_word.zero_()
            raise RuntimeError("a cascade kernel reported device error code {}".format(code))

    # ---------------------------------------------------------------- protocol
    def begin(self, input_ids, position_ids=None):
        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("first runtime supports one unpadded request")
        past = self.kv_cache.sequence_length()
        tokens = int(input_ids.shape[1])
        if tokens < 1:
            raise ValueError("input_ids is empty")
        if past and tokens != 1 and not self.allow_chunked_prefill:
            raise ValueError("after prefill, only one-token decode calls are supported")
        self._i8_step = False  # set by run_units_resident for an int8 one-token step
        with torch.cuda.device(self.device):
            if position_ids is not None:
                start = int(position_ids.reshape(-1)[0])
                if start != past:
                    raise ValueError("position_ids must continue the cached sequence ({} != {})".format(start, past))
            self.kv_cache.reserve(past + tokens)
            self._buffers(tokens)
            ids = input_ids.reshape(-1)
            if tokens == 1 and self.vocab_runtime is None:
                # one-token step: the id goes into a persistent device slot
                # (asynchronous from pinned memory) and the embedding runs
                # with the first unit, inside the step's graph when replayed
                self._ids_dev.copy_(ids, non_blocking=True)
                self._embed_pending = True
            else:
                if ids.device != self.device or ids.dtype != torch.int64 or not ids.is_contiguous():
                    ids = ids.to(device=self.device, dtype=torch.int64).contiguous()
                self._embed_pending = False
                if self.vocab_runtime is None:
                    ops.embedding(ids, self.resident["model.embed_tokens.weight"], self._x[:tokens])
                else:
                    self._x[:tokens].copy_(self.vocab_runtime.embedding(ids.view(1, -1)).view(tokens, -1))
        self._tokens = tokens
        return DecodeState(
            hidden_states=self._x[:tokens].view(1, tokens, 4096),
            position_ids=torch.arange(past, past + tokens, dtype=torch.long).unsqueeze(0),
        )

    def _unit(self, layer, operation, weights, splits=None, chunk=None, fused=None):
        if 1 < self._tokens <= _SPLIT_K_MAX_TOKENS:
            # the registration lives only for this unit's launches: the
            # workspace belongs to this executor
            self._register_split_k()
            try:
                return self._unit_ops(layer, operation, weights, splits, chunk, fused)
            finally:
                _native.lib().cb_set_gemm_workspace(None, 0, None, 0)
        return self._unit_ops(layer, operation, weights, splits, chunk, fused)

    def _unit_ops(self, layer, operation, weights, splits=None, chunk=None, fused=None):
        tokens = self._tokens
        if tokens == 1 and self._i8_active:
            if splits is None:
                splits, chunk, fused = self.attention_config(1, self.kv_cache.length + 1)
            return self._unit_i8(layer, operation, splits, chunk)
        cache = self.kv_cache
        eps = self.eps
        pos = cache.position
        res = self.resident
        norm_in = res["model.layers.{}.input_layernorm.weight".format(layer)]
        norm_post = res["model.layers.{}.post_attention_layernorm.weight".format(layer)]
        w = lambda name: weights[_matrix_key(layer, name)]
        kc, vc = cache.key(layer), cache.value(layer)
        # multi-token steps (prefill) run the fused units as tcgen05 GEMMs
        gemm = tokens > 1
        if not gemm and self._stage_active:
            self._stage_target(layer, operation)
        if operation in ("qkv", "q_proj", "k_proj", "v_proj") and gemm:
            wq = w("q_proj") if operation in ("qkv", "q_proj") else None
            wk = w("k_proj") if operation in ("qkv", "k_proj") else None
            wv = w("v_proj") if operation in ("qkv", "v_proj") else None
            ops.rmsnorm(self._x[:tokens], norm_in, eps, self._xn[:tokens])
            ops.prefill_qkv_rope(self._xn[:tokens], wq, wk, wv, self.inv_freq, pos,
                                 self._q[:tokens] if wq is not None else None,
                                 kc if wk is not None else None, vc if wv is not None else None)
        elif operation in ("qkv", "q_proj", "k_proj", "v_proj"):
            wq = w("q_proj") if operation in ("qkv", "q_proj") else None
            wk = w("k_proj") if operation in ("qkv", "k_proj") else None
            wv = w("v_proj") if operation in ("qkv", "v_proj") else None
            for m in range(tokens):
                ops.qkv_rope(
                    self._x[m], norm_in, eps, wq, wk, wv, self.inv_freq, pos, m,
                    self._q[m] if wq is not None else None,
                    kc if wk is not None else None, vc if wv is not None else None,
                )
        elif operation == "o_proj":
            wo = w("o_proj")
            if gemm:  # prefill: causal flash attention on the tensor cores
                ops.prefill_attention(self._q[:tokens], kc, vc, pos, self._attn[:tokens])
                ops.gemm_residual(self._attn[:tokens], wo, self._x[:tokens], self._x[:tokens])
                return
            if splits is None:
                splits, chunk, fused = self.attention_config(tokens, cache.length + tokens)
            ws = self._attention_workspace(tokens, splits)
            if fused:
                ops.attention_oproj(self._q[0], kc, vc, pos, splits, wo, self._x[0], self._attn[0], self._x[0], ws,
                                    self._tickets)
            else:
                ops.attention(self._q[:tokens], kc, vc, pos, splits, chunk, self._attn[:tokens], ws, self._tickets)
                ops.proj_residual(self._attn[0], wo, self._x[0], self._x[0])
        elif operation == "gate_up":
            wg, wu = w("gate_proj"), w("up_proj")
            if gemm:
                ops.rmsnorm(self._x[:tokens], norm_post, eps, self._xn[:tokens])
                ops.gemm_swiglu(self._xn[:tokens], wg, wu, self._mlp[:tokens])
            else:
                ops.gate_up_swiglu(self._x[0], norm_post, eps, wg, wu, self._mlp[0])
        elif operation in ("gate_proj", "up_proj") and gemm:
            ops.rmsnorm(self._x[:tokens], norm_post, eps, self._xn[:tokens])
            if operation == "gate_proj":
                ops.gemm_silu(self._xn[:tokens], w("gate_proj"), self._mlp[:tokens])
            else:
                ops.gemm_mul(self._xn[:tokens], w("up_proj"), self._mlp[:tokens])
        elif operation == "gate_proj":
            for m in range(tokens):
                ops.gate_silu(self._x[m], norm_post, eps, w("gate_proj"), self._mlp[m])
        elif operation == "up_proj":
            for m in range(tokens):
                ops.up_mul(self._x[m], norm_post, eps, w("up_proj"), self._mlp[m])
        elif operation == "down_proj":
            wd = w("down_proj")
            if gemm:
                ops.gemm_residual(self._mlp[:tokens], wd, self._x[:tokens], self._x[:tokens])
            else:
                ops.proj_residual(self._mlp[0], wd, self._x[0], self._x[0])
        else:
            raise ValueError("unknown Llama operation {}".format(operation))

    def _collect_int8(self, runtime):
        """Quantize every decode weight matrix of `runtime` (and the resident
        LM head) to int8 rows with fp32 scales, once, on the device."""

        q8 = {}
        with torch.cuda.device(self.device):
            for index in range(len(runtime.plan.units)):
                for key, t in runtime.unit_views(index).items():
                    if t.dim() == 2 and key not in q8:
                        q = torch.empty(t.shape, dtype=torch.int8, device=self.device)
                        scale = torch.empty(t.shape[0], dtype=torch.float32, device=self.device)
                        ops.quantize_rows_i8(t, q, scale)
                        q8[key] = (q, scale)
            if self.vocab_runtime is None:
                head = self.resident["lm_head.weight"]
                q = torch.empty(head.shape, dtype=torch.int8, device=self.device)
                scale = torch.empty(head.shape[0], dtype=torch.float32, device=self.device)
                ops.quantize_rows_i8(head, q, scale)
                q8["lm_head.weight"] = (q, scale)
        self._i8, self._i8_owner = q8, id(runtime)

    def _unit_i8(self, layer, operation, splits, chunk, weights8=None):
        """One-token unit with int8 weights (the bf16 kernels' fused epilogues);
        weights8: {key: (int8, scales)} (default: the HBM-resident quantized copy)."""

        cache, eps, pos, res = self.kv_cache, self.eps, self.kv_cache.position, self.resident
        table = self._i8 if weights8 is None else weights8
        q8 = lambda name: table[_matrix_key(layer, name)]
        kc, vc = cache.key(layer), cache.value(layer)
        if operation == "qkv":
            (wq, sq), (wk, sk), (wv, sv) = q8("q_proj"), q8("k_proj"), q8("v_proj")
            ops.qkv_rope_i8(self._x[0], res["model.layers.{}.input_layernorm.weight".format(layer)], eps, wq, sq,
                            wk, sk, wv, sv, self.inv_freq, pos, 0, self._q[0], kc, vc)
        elif operation == "o_proj":
            ws = self._attention_workspace(1, splits)
            ops.attention(self._q[:1], kc, vc, pos, splits, chunk, self._attn[:1], ws, self._tickets)
            wo, so = q8("o_proj")
            ops.proj_residual_i8(self._attn[0], wo, so, self._x[0], self._x[0])
        elif operation == "gate_up":
            (wg, sg), (wu, su) = q8("gate_proj"), q8("up_proj")
            ops.gate_up_swiglu_i8(self._x[0], res["model.layers.{}.post_attention_layernorm.weight".format(layer)],
                                  eps, wg, sg, wu, su, self._mlp[0])
        elif operation == "down_proj":
            wd, sd = q8("down_proj")
            ops.proj_residual_i8(self._mlp[0], wd, sd, self._x[0], self._x[0])
        else:
            raise ValueError("int8 decode weights need the matrix_group or layer granularity (got {})".format(
                operation))

    def _register_split_k(self):
        """Short chunks (a few-token prompt): let the prefill GEMMs split K over
        the SMs (``cb_set_gemm_workspace``) through this executor's fp32
        workspace and zeroed per-tile tickets, allocated on first use."""

        if self._split_k_ws is None:
            self._split_k_ws = torch.empty(_SPLIT_K_BYTES // 4, dtype=torch.float32, device=self.device)
            self._split_k_tickets = torch.zeros(_SPLIT_K_TICKETS, dtype=torch.int32, device=self.device)
        _native.check(
            _native.lib().cb_set_gemm_workspace(self._split_k_ws.data_ptr(), _SPLIT_K_BYTES,
                                                self._split_k_tickets.data_ptr(), _SPLIT_K_TICKETS),
            "cb_set_gemm_workspace",
        )

    def _stage_target(self, layer, operation):
        """One-token steps with HBM-resident weights: the QKV, attention and
        o_proj launches of a layer may pre-stage that layer's gate+up weights
        into L2 (``cb_set_l2_stage``); the target is set before the layer's
        QKV and cleared before its gate+up."""

        if operation == "qkv":
            slabs = self._stage_slabs.get(layer)
            if slabs is not None:
                wg, wu = slabs
                _native.check(
                    _native.lib().cb_set_l2_stage_target(wg.data_ptr(), wu.data_ptr(), wg.shape[0], wg.shape[1]),
                    "cb_set_l2_stage_target",
                )
        elif operation in ("gate_up", "gate_proj"):
            _native.lib().cb_set_l2_stage_target(None, None, 0, 0)

    def _collect_stage_slabs(self, runtime):
        slabs = {}
        for index, unit in enumerate(runtime.plan.units):
            views = runtime.unit_views(index)
            gate = _matrix_key(unit.layer_index, "gate_proj")
            up = _matrix_key(unit.layer_index, "up_proj")
            if gate in views and up in views:
                slabs[unit.layer_index] = (views[gate], views[up])
        self._stage_slabs, self._stage_owner = slabs, id(runtime)

    def _after_last_unit(self):
        # the step's K/V are cached: advance the device position counter
        ops.position_advance(self.kv_cache.position, self._tokens)
        self.kv_cache.length += self._tokens

    def _embed_one(self):
        ops.embedding(self._ids_dev, self.resident["model.embed_tokens.weight"], self._x[:1])

    def _dequantized(self, weights8):
        """bf16 views of a unit that arrived as int8 rows (prefill GEMMs)."""

        need = sum(q.numel() for q, _ in weights8.values())
        if self._deq is None or self._deq.numel() < need:
            self._deq = torch.empty(need, dtype=torch.bfloat16, device=self.device)
        views, cursor = {}, 0
        for key, (q, scale) in weights8.items():
            out = self._deq.narrow(0, cursor, q.numel()).view(q.shape)
            ops.dequantize_rows_i8(q, scale, out)
            views[key] = out
            cursor += q.numel()
        return views

    def __call__(self, unit, weights, state):
        if self._embed_pending:
            self._embed_one()
            self._embed_pending = False
        int8 = bool(weights) and isinstance(next(iter(weights.values())), tuple)  # streamed int8 transfer
        if int8 and self._tokens > 1:
            weights, int8 = self._dequantized(weights), False
        for operation in _UNIT_OPS.get(unit.operation, (unit.operation,)):
            if int8:
                splits, chunk, _ = self.attention_config(1, self.kv_cache.length + 1)
                self._unit_i8(unit.layer_index, operation, splits, chunk, weights)
                continue
            self._unit(unit.layer_index, operation, weights)
        if unit.layer_index == self.config.num_hidden_layers - 1 and unit.operation in ("layer", "down_proj"):
            self._after_last_unit()
        return state

    def run_units_resident(self, runtime, state):
        """All units of a step with HBM-resident weights (graph replay for M=1)."""

        units = runtime.plan.units
        if self._tokens == 1 and self._stage_owner != id(runtime):
            self._collect_stage_slabs(runtime)
        i8 = self._tokens == 1 and self.decode_weights == "int8"
        if i8 and self._i8_owner != id(runtime):
            self._collect_int8(runtime)
        self._i8_step = i8
        if not self.use_graphs or self._tokens != 1:
            self._stage_active = self._tokens == 1 and not i8
            self._i8_active = i8
            try:
                for index, unit in enumerate(units):
                    state = self(unit, runtime.unit_views(index), state)
            finally:
                self._stage_active = self._i8_active = False
                _native.lib().cb_set_l2_stage_target(None, None, 0, 0)
            return state
        length = self.kv_cache.length + 1
        bucket = max(64, 1 << (length - 1).bit_length())
        bucket = min(bucket, self.kv_cache.capacity)
        splits, chunk, fused = self.attention_config(1, bucket)
        embed = self._embed_pending  # the graph starts with the embedding of the step's id
        key = (id(runtime), bucket, self.kv_cache.generation, self._rows, embed, fused)
        graph = self._graphs.get(key)
        if graph is None:
            self._attention_workspace(1, splits)
            graph = torch.cuda.CUDAGraph()
            saved = self.kv_cache.length
            with torch.cuda.graph(graph):
                if embed:
                    self._embed_one()
                self._stage_active = not i8
                self._i8_active = i8
                try:
                    for index, unit in enumerate(units):
                        for operation in _UNIT_OPS.get(unit.operation, (unit.operation,)):
                            self._unit(unit.layer_index, operation, runtime.unit_views(index), splits, chunk, fused)
                finally:
                    self._stage_active = self._i8_active = False
                    _native.lib().cb_set_l2_stage_target(None, None, 0, 0)
                ops.position_advance(self.kv_cache.position, 1)
            self.kv_cache.length = saved
            self._graphs[key] = graph
        graph.replay()
        self._embed_pending = False
        self.kv_cache.length += 1
        return state

    def finish(self, state):
        tokens = self._tokens
        last = self._x[tokens - 1]
        k = min(self.top_k, self.config.vocab_size)
        with torch.cuda.device(self.device):
            if self.vocab_runtime is None:
                values = torch.empty((1, 1, k), dtype=torch.float32, device=self.device)
                indices = torch.empty((1, 1, k), dtype=torch.int64, device=self.device)
                # the last token's logits, always (the reference's resident head
                # returns every position's [1, M, vocab]; a decode step has M = 1)
                logits = torch.empty((1, 1, self.config.vocab_size), dtype=torch.float32, device=self.device)
                if self._i8_step:
                    head, scale = self._i8["lm_head.weight"]
                    ops.lm_head_topk_i8(last, self.resident["model.norm.weight"], self.eps, head, scale, k,
                                        logits.view(-1), values.view(-1), indices.view(-1), self.lm_workspace,
                                        self.lm_ticket)
                else:
                    ops.lm_head_topk(
                        last, self.resident["model.norm.weight"], self.eps, self.resident["lm_head.weight"], 0, k,
                        logits.view(-1), values.view(-1), indices.view(-1),
                        self.lm_workspace, self.lm_ticket,
                    )
            else:
                normed = torch.empty((1, 1, 4096), dtype=torch.bfloat16, device=self.device)
                ops.rmsnorm(last, self.resident["model.norm.weight"], self.eps, normed.view(-1))
                result = self.vocab_runtime.lm_head_topk(normed, top_k=k, return_full_logits=self.return_full_logits)
                values, indices, logits = result["values"], result["indices"], result["logits"]
        state.topk_values = values
        state.topk_indices = indices
        state.logits = logits
        return state
