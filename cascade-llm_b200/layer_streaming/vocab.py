"""Row lookup and the chunked (vocabulary-streamed) LM head.

Same API as ``layer_streaming/vocab.py:11-300`` of the reference:

* :func:`merge_topk` - exact top-k of the union of two candidate sets
  (``vocab.py:11-32``), computed by the ``cascade.topk_merge`` kernel;
* :class:`VocabStreamingRuntime` - shares the transformer runtime's two
  device slots and streams; ``embedding`` gathers the requested rows on the
  CPU and copies them to the GPU (``vocab.py:100-131``); ``lm_head_topk``
  streams the LM head in ``chunk_rows`` slices (7 x 16,384 + 13,568 rows)
  and runs ONE fused kernel per slice (logits + per-CTA top-k + in-kernel
  merge, ``cascade.lm_head_topk``), then one k-way merge of all slices
  (``vocab.py:207-266``).

Ties: the reference's ``torch.topk`` leaves the order of equal logits
unspecified; these kernels rank larger values first, then smaller indices.
"""

import time

import torch

from . import ops
from .weight_store import WeightStoreMode


def merge_topk(current_values, current_indices, candidate_values, candidate_indices, top_k):
    """Merge two candidate sets exactly (CUDA tensors, one row)."""

    if candidate_values.device.type != "cuda":
        raise RuntimeError("merge_topk runs on the GPU (cascade.topk_merge); got CPU tensors")
    lead = candidate_values.shape[:-1]
    if candidate_values.numel() != candidate_values.shape[-1]:
        raise ValueError("merge_topk supports a single row (batch 1)")
    b_v = candidate_values.reshape(-1).float().contiguous()
    b_i = candidate_indices.reshape(-1).to(torch.int64).contiguous()
    a_v = a_i = None
    total = b_v.numel()
    if current_values is not None:
        a_v = current_values.reshape(-1).float().contiguous()
        a_i = current_indices.reshape(-1).to(torch.int64).contiguous()
        total += a_v.numel()
    keep = min(int(top_k), total)
    out_v = torch.empty(lead + (keep,), dtype=torch.float32, device=b_v.device)
    out_i = torch.empty(lead + (keep,), dtype=torch.int64, device=b_v.device)
    ops.topk_merge(a_v, a_i, b_v, b_i, keep, out_v.view(-1), out_i.view(-1))
    return out_v, out_i


class VocabStreamingRuntime:
    """Share transformer slots for embedding lookup and LM-head chunks."""

    def __init__(self, plan, store, transformer_runtime, embedding_staging_rows=256, profile=False):
        if plan.vocab is None:
            raise ValueError("plan does not enable vocabulary streaming")
        self.plan = plan
        self.vocab = plan.vocab
        self.store = store
        self.transformer_runtime = transformer_runtime
        self.device = transformer_runtime.device
        self.device_slots = transformer_runtime.device_slots
        self.copy_stream = transformer_runtime.copy_stream
        self.compute_stream = transformer_runtime.compute_stream
        self.coordinator = transformer_runtime.coordinator
        self.profile = bool(profile)
        self.last_profile = None
        self.last_embedding_bytes = 0
        self.embedding_staging_rows = int(embedding_staging_rows)
        if self.embedding_staging_rows < 1:
            raise ValueError("embedding_staging_rows must be positive")
        if len(self.device_slots) != 2:
            raise ValueError("vocabulary streaming requires two GPU slots")
        if self.device_slots[0].numel() < self.vocab.chunk_elements:
            raise ValueError("shared GPU slot is smaller than vocab chunk")
        self.embedding_staging = torch.empty(
            (self.embedding_staging_rows, self.vocab.hidden_size), dtype=torch.bfloat16, pin_memory=True
        )
        self.head_staging_slots = None
        if self.store.mode == WeightStoreMode.PINNED_STAGING:
            self.head_staging_slots = [
                torch.empty(self.vocab.chunk_elements, dtype=torch.bfloat16, pin_memory=True)
                for _ in range(2)
            ]
        self._workspace = None
        self._ticket = None
        self._cand = None

    @property
    def gpu_slot_bytes(self):
        return sum(slot.numel() * slot.element_size() for slot in self.device_slots)

    @property
    def extra_pinned_cpu_bytes(self):
        total = self.embedding_staging.numel() * self.embedding_staging.element_size()
        if self.head_staging_slots is not None:
            total += sum(s.numel() * s.element_size() for s in self.head_staging_slots)
        return total

    def embedding(self, input_ids):
        """Gather only the requested CPU rows and copy them to the GPU."""

        shape = tuple(input_ids.shape)
        ids = input_ids.detach().reshape(-1).to(device="cpu", dtype=torch.long)
        table = self.store.tensor(self.vocab.embedding_key)
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.vocab.vocab_size):
            raise IndexError("token id out of vocabulary range")
        out = torch.empty((ids.numel(), self.vocab.hidden_size), dtype=torch.bfloat16, device=self.device)
        self.last_embedding_bytes = ids.numel() * self.vocab.hidden_size * 2
        for start in range(0, ids.numel(), self.embedding_staging_rows):
            end = min(start + self.embedding_staging_rows, ids.numel())
            staging = self.embedding_staging[:end - start]
            torch.index_select(table, 0, ids[start:end], out=staging)
            with torch.cuda.stream(self.copy_stream):
                ops.memcpy_h2d_async(out[start:end], staging)
            # the staging rows are reused by the next group
            self.copy_stream.synchronize()
        return out.view(shape + (self.vocab.hidden_size,))

    def _head_source(self, start_row, end_row, slot_index, ready_event):
        source = self.store.tensor(self.vocab.lm_head_key)[start_row:end_row].reshape(-1)
        if self.head_staging_slots is None:
            if not source.is_pinned():
                raise RuntimeError("full_pinned LM-head source unexpectedly is not pinned")
            return source
        if ready_event is not None:
            ready_event.synchronize()
        target = self.head_staging_slots[slot_index][:source.numel()]
        target.copy_(source)
        return target

    def _buffers(self, top_k):
        need = self.vocab.chunk_count * top_k
        if self._cand is None or self._cand[0].numel() < need:
            self._cand = (
                torch.empty(need, dtype=torch.float32, device=self.device),
                torch.empty(need, dtype=torch.int64, device=self.device),
            )
        if self._workspace is None or self._workspace[0] < top_k:
            ws = torch.empty(ops.lm_head_workspace_bytes(top_k), dtype=torch.uint8, device=self.device)
            self._workspace = (top_k, ws)
        if self._ticket is None:
            self._ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._cand, self._workspace[1]

    def lm_head_topk(self, hidden_states, top_k=10, return_full_logits=False):
        """Stream the head in row chunks and keep an exact global top-k.

        ``hidden_states``: the final-normalised last token ``[1, 1, hidden]``
        (bf16, on the GPU). Returns ``{"values", "indices", "logits"}`` like
        the reference; ``logits`` is fp32 ``[1, 1, vocab]`` when requested.
        """

        if hidden_states.shape[-1] != self.vocab.hidden_size:
            raise ValueError("hidden state width does not match vocabulary")
        if top_k < 1 or top_k > self.vocab.vocab_size:
            raise ValueError("top_k is outside vocabulary range")
        if top_k > 64:
            raise ValueError("the fused LM-head kernel supports top_k <= 64")
        if hidden_states.numel() != self.vocab.hidden_size:
            raise ValueError("lm_head_topk expects one token row")
        hidden = hidden_states.reshape(-1)
        if not hidden.is_contiguous():
            raise ValueError("hidden_states must be contiguous")
        wall_started = time.perf_counter()
        chunks = self.vocab.chunk_count
        timing = dict(enable_timing=True)
        ready = [torch.cuda.Event() for _ in range(chunks)]
        free = [torch.cuda.Event() for _ in range(chunks)]
        if self.profile:
            pipe_start, pipe_end = torch.cuda.Event(**timing), torch.cuda.Event(**timing)
            copy_ev = [(torch.cuda.Event(**timing), torch.cuda.Event(**timing)) for _ in range(chunks)]
            comp_ev = [(torch.cuda.Event(**timing), torch.cuda.Event(**timing)) for _ in range(chunks)]
            pipe_start.record(self.coordinator)
            self.copy_stream.wait_event(pipe_start)
            self.compute_stream.wait_event(pipe_start)
        else:
            self.copy_stream.wait_stream(self.coordinator)
            self.compute_stream.wait_stream(self.coordinator)
        (cand_v, cand_i), workspace = self._buffers(top_k)
        logits = None
        if return_full_logits:
            logits = torch.empty(
                hidden_states.shape[:-1] + (self.vocab.vocab_size,), dtype=torch.float32, device=self.device
            )
        flat_logits = None if logits is None else logits.view(-1)
        transferred = 0
        filled = 0
        for c in range(chunks):
            slot_index = c % 2
            start, end = self.vocab.chunk_range(c)
            rows = end - start
            source = self._head_source(start, end, slot_index, ready[c - 2] if c >= 2 else None)
            slot = self.device_slots[slot_index]
            if c >= 2:
                self.copy_stream.wait_event(free[c - 2])
            with torch.cuda.stream(self.copy_stream):
                if self.profile:
                    copy_ev[c][0].record(self.copy_stream)
                ops.memcpy_h2d_async(slot[:rows * self.vocab.hidden_size], source)
                if self.profile:
                    copy_ev[c][1].record(self.copy_stream)
                ready[c].record(self.copy_stream)
            transferred += rows * self.vocab.hidden_size * 2
            self.compute_stream.wait_event(ready[c])
            with torch.cuda.stream(self.compute_stream):
                if self.profile:
                    comp_ev[c][0].record(self.compute_stream)
                k = min(top_k, rows)
                weight = slot[:rows * self.vocab.hidden_size].view(rows, self.vocab.hidden_size)
                ops.lm_head_topk(
                    hidden, None, 0.0, weight, start, k,
                    None if flat_logits is None else flat_logits[start:end],
                    cand_v[filled:filled + k], cand_i[filled:filled + k], workspace, self._ticket,
                )
                filled += k
                if self.profile:
                    comp_ev[c][1].record(self.compute_stream)
                free[c].record(self.compute_stream)
        keep = min(top_k, filled)
        values = torch.empty(hidden_states.shape[:-1] + (keep,), dtype=torch.float32, device=self.device)
        indices = torch.empty(hidden_states.shape[:-1] + (keep,), dtype=torch.int64, device=self.device)
        with torch.cuda.stream(self.compute_stream):
            ops.topk_merge(None, None, cand_v[:filled], cand_i[:filled], keep, values.view(-1), indices.view(-1))
            free[-1].record(self.compute_stream)
        self.coordinator.wait_event(free[-1])
        if self.profile:
            pipe_end.record(self.coordinator)
        self.coordinator.synchronize()
        if self.profile:
            h2d_ms = sum(a.elapsed_time(b) for a, b in copy_ev)
            self.last_profile = {
                "wall_ms": (time.perf_counter() - wall_started) * 1000.0,
                "pipeline_ms": pipe_start.elapsed_time(pipe_end),
                "h2d_event_sum_ms": h2d_ms,
                "compute_event_sum_ms": sum(a.elapsed_time(b) for a, b in comp_ev),
                "h2d_bytes": transferred,
                "h2d_effective_gbps": (transferred / 1e9) / (h2d_ms / 1000.0),
                "chunk_count": chunks,
                "chunk_rows": self.vocab.chunk_rows,
                "requested_top_k": int(top_k),
            }
        return {"values": values, "indices": indices, "logits": logits}
