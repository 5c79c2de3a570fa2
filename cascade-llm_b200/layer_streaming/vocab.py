"""Row lookup and the chunked (vocabulary-streamed) LM head.

Public surface of the reference's ``layer_streaming/vocab.py:11-300``:

* :func:`merge_topk` - exact top-k of the union of two candidate sets
  (``vocab.py:11-32``), computed by the ``cascade.topk_merge`` kernel;
* :class:`VocabStreamingRuntime` - shares the transformer runtime's device
  slots and streams. ``embedding`` gathers the requested rows of the host
  table into pinned staging rows on the host (``cb_host_gather_rows``) and
  copies them to the GPU (``vocab.py:100-131``); ``lm_head_topk`` streams the
  LM head's ``chunk_rows`` slices (7 x 16,384 + 13,568 rows) through the
  native slot ring (``csrc/slot_ring.cu``, staged through two pinned chunk
  buffers for the pinned-staging store) and runs ONE fused kernel per slice
  (logits + per-CTA top-k + in-kernel merge, ``cascade.lm_head_topk``), then
  one k-way merge of all slices' candidates (``vocab.py:207-266``).

Ties: the reference's ``torch.topk`` leaves the order of equal logits
unspecified; these kernels rank larger values first, then smaller indices.
"""

import torch

from . import _native, ops
from .streaming import SlotRing, host_span
from .weight_store import WeightStoreMode


def merge_topk(current_values, current_indices, candidate_values, candidate_indices, top_k):
    """Merge two candidate sets exactly (CUDA tensors, one row)."""

    if candidate_values.device.type != "cuda":
        raise RuntimeError("merge_topk runs on the GPU (cascade.topk_merge); got CPU tensors")
    if candidate_values.numel() != candidate_values.shape[-1]:
        raise ValueError("merge_topk supports a single row (batch 1)")
    lead = tuple(candidate_values.shape[:-1])
    flat = lambda v, i: (v.reshape(-1).float().contiguous(), i.reshape(-1).to(torch.int64).contiguous())
    b_v, b_i = flat(candidate_values, candidate_indices)
    a_v = a_i = None
    if current_values is not None:
        a_v, a_i = flat(current_values, current_indices)
    keep = min(int(top_k), b_v.numel() + (0 if a_v is None else a_v.numel()))
    values = torch.empty(lead + (keep,), dtype=torch.float32, device=b_v.device)
    indices = torch.empty(lead + (keep,), dtype=torch.int64, device=b_v.device)
    ops.topk_merge(a_v, a_i, b_v, b_i, keep, values.view(-1), indices.view(-1))
    return values, indices


class VocabStreamingRuntime:
    """Share transformer slots for embedding lookup and LM-head chunks."""

    def __init__(self, plan, store, transformer_runtime, embedding_staging_rows=256, profile=False):
        vocab = plan.vocab
        if vocab is None:
            raise ValueError("this plan keeps the vocabulary resident (stream_vocab=False)")
        slots = transformer_runtime.device_slots
        if len(slots) != 2:
            raise ValueError("the streamed vocabulary needs the runtime's two device slots (got {})".format(len(slots)))
        if slots[0].numel() < vocab.chunk_elements:
            raise ValueError("a device slot ({} elements) cannot hold a vocab chunk ({})".format(
                slots[0].numel(), vocab.chunk_elements))
        if int(embedding_staging_rows) < 1:
            raise ValueError("embedding_staging_rows must be at least 1")
        self.plan = plan
        self.vocab = vocab
        self.store = store
        self.transformer_runtime = transformer_runtime
        self.device = transformer_runtime.device
        self.device_slots = slots
        self.copy_stream = transformer_runtime.copy_stream
        self.compute_stream = transformer_runtime.compute_stream
        self.coordinator = transformer_runtime.coordinator
        self.profile = bool(profile)
        self.last_profile = None
        self.last_embedding_bytes = 0
        self.embedding_staging_rows = int(embedding_staging_rows)
        pinned_rows = lambda n: torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
        self.embedding_staging = pinned_rows(self.embedding_staging_rows * vocab.hidden_size).view(
            self.embedding_staging_rows, vocab.hidden_size)
        # the pinned-staging store keeps the head pageable: two pinned chunk buffers
        staged = store.mode == WeightStoreMode.PINNED_STAGING
        self.head_staging_slots = [pinned_rows(vocab.chunk_elements) for _ in range(2)] if staged else None
        self._ring = SlotRing(slots, self.copy_stream, staging=self.head_staging_slots,
                              copy_threads=getattr(store, "copy_threads", 0))
        self._scratch = {}

    @property
    def gpu_slot_bytes(self):
        return sum(slot.numel() * slot.element_size() for slot in self.device_slots)

    @property
    def extra_pinned_cpu_bytes(self):
        buffers = [self.embedding_staging] + list(self.head_staging_slots or [])
        return sum(b.numel() * b.element_size() for b in buffers)

    def embedding(self, input_ids):
        """Gather only the requested host rows and copy them to the GPU."""

        shape = tuple(input_ids.shape)
        ids = input_ids.detach().reshape(-1).to(device="cpu", dtype=torch.int64).contiguous()
        hidden = self.vocab.hidden_size
        table = self.store.tensor(self.vocab.embedding_key)
        out = torch.empty((ids.numel(), hidden), dtype=torch.bfloat16, device=self.device)
        lib = _native.lib()
        for begin in range(0, ids.numel(), self.embedding_staging_rows):
            part = ids[begin:begin + self.embedding_staging_rows]
            rows = self.embedding_staging[:part.numel()]
            rc = lib.cb_host_gather_rows(rows.data_ptr(), table.data_ptr(), table.shape[0], 2 * hidden,
                                         part.data_ptr(), part.numel())
            if rc != 0:
                raise IndexError("token id out of vocabulary range: {}".format(lib.cb_last_error().decode()))
            with torch.cuda.stream(self.copy_stream):
                ops.memcpy_h2d_async(out[begin:begin + part.numel()], rows)
            self.copy_stream.synchronize()  # the staging rows are refilled next
        self.last_embedding_bytes = 2 * hidden * ids.numel()
        return out.view(shape + (hidden,))

    def _workspace(self, top_k):
        """Per-top_k device scratch: candidates of every chunk, the fused
        kernel's workspace and its zeroed ticket."""

        scratch = self._scratch.get(top_k)
        if scratch is None:
            need = self.vocab.chunk_count * top_k
            scratch = (
                torch.empty(need, dtype=torch.float32, device=self.device),
                torch.empty(need, dtype=torch.int64, device=self.device),
                torch.empty(ops.lm_head_workspace_bytes(top_k), dtype=torch.uint8, device=self.device),
                torch.zeros(1, dtype=torch.int32, device=self.device),
            )
            self._scratch[top_k] = scratch
        return scratch

    def lm_head_topk(self, hidden_states, top_k=10, return_full_logits=False):
        """Stream the head in row chunks and keep an exact global top-k.

        ``hidden_states``: the final-normalised last token ``[1, 1, hidden]``
        (bf16, on the GPU). Returns ``{"values", "indices", "logits"}`` like
        the reference; ``logits`` is fp32 ``[1, 1, vocab]`` when requested.
        """

        vocab = self.vocab
        if hidden_states.shape[-1] != vocab.hidden_size:
            raise ValueError("hidden state width does not match vocabulary")
        if top_k < 1 or top_k > vocab.vocab_size:
            raise ValueError("top_k is outside vocabulary range")
        if top_k > 64:
            raise ValueError("the fused LM-head kernel supports top_k <= 64")
        if hidden_states.numel() != vocab.hidden_size or not hidden_states.is_contiguous():
            raise ValueError("lm_head_topk expects one contiguous token row")
        hidden = hidden_states.reshape(-1)
        cand_v, cand_i, workspace, ticket = self._workspace(top_k)
        logits = None
        if return_full_logits:
            logits = torch.empty(tuple(hidden_states.shape[:-1]) + (vocab.vocab_size,), dtype=torch.float32,
                                 device=self.device)
        head = self.store.tensor(vocab.lm_head_key)
        ranges = [vocab.chunk_range(c) for c in range(vocab.chunk_count)]
        spans = [host_span(head[a:b].reshape(-1)) for a, b in ranges]
        if self.head_staging_slots is None and not head.is_pinned():
            raise RuntimeError("the full-pinned store's LM head is not in pinned memory")
        kept = [0]

        def body(c, slot):
            a, b = ranges[c]
            k = min(top_k, b - a)
            weight = slot[:(b - a) * vocab.hidden_size].view(b - a, vocab.hidden_size)
            ops.lm_head_topk(hidden, None, 0.0, weight, a, k, None if logits is None else logits.view(-1)[a:b],
                             cand_v[kept[0]:kept[0] + k], cand_i[kept[0]:kept[0] + k], workspace, ticket)
            kept[0] += k
            if c == len(ranges) - 1:  # the merge of all chunks closes the last span
                keep = min(top_k, kept[0])
                out_v = torch.empty(tuple(hidden_states.shape[:-1]) + (keep,), dtype=torch.float32,
                                    device=self.device)
                out_i = torch.empty(tuple(hidden_states.shape[:-1]) + (keep,), dtype=torch.int64, device=self.device)
                ops.topk_merge(None, None, cand_v[:kept[0]], cand_i[:kept[0]], keep, out_v.view(-1), out_i.view(-1))
                result.update(values=out_v, indices=out_i)

        result = {"values": None, "indices": None, "logits": logits}
        numbers = self._ring.run(spans, body, self.compute_stream, self.coordinator, profile=self.profile)
        if self.profile:
            moved = numbers["h2d_bytes"]
            self.last_profile = {
                "wall_ms": numbers["wall_ms"],
                "pipeline_ms": numbers["gpu_pipeline_ms"],
                "h2d_event_sum_ms": numbers["h2d_event_sum_ms"],
                "compute_event_sum_ms": numbers["compute_event_sum_ms"],
                "h2d_bytes": moved,
                "h2d_effective_gbps": (moved / 1e9) / max(numbers["h2d_event_sum_ms"] / 1000.0, 1e-12),
                "chunk_count": vocab.chunk_count,
                "chunk_rows": vocab.chunk_rows,
                "requested_top_k": int(top_k),
            }
        return result
