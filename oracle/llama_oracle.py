"""Restatement of the reference's Llama-3.1-8B decode math (TEST INFRASTRUCTURE ONLY).

Each function restates one step of the reference's hot path with the same
torch ops and the same BF16 rounding points, so that it runs on the CPU here
and on a GPU box (where the reference itself cannot travel). It is the
checker for the CUDA engine and the timed stand-in for the reference's CPU
path; the product never imports it. ``tests/test_oracle_golden.py`` pins it
against vectors produced by the reference's own code.

Rounding points mirrored (all from ``layer_streaming/llama31.py``):
  * RMSNorm: fp32 mean-square and rsqrt, cast to bf16, then ``w * x`` in bf16
    (``:21-25``);
  * every projection is a bf16 ``F.linear`` (fp32 accumulate, bf16 out)
    (``:241-280``);
  * RoPE: cos/sin computed in fp32 and cast to bf16, then
    ``q*cos + rotate_half(q)*sin`` in bf16 (transformers
    ``modeling_llama.py:124-168``);
  * residual adds, SiLU and ``gate*up`` round to bf16 (``:246-280``);
  * LM head: bf16 ``F.linear`` then ``.float()`` (``:330-334``), top-k on fp32.
"""

import math

import torch
import torch.nn.functional as F

HIDDEN = 4096
HEADS = 32
KV_HEADS = 8
HEAD_DIM = 128
FFN = 14336
VOCAB = 128256
LAYERS = 32
EPS = 1e-5
ROPE_THETA = 500000.0
ROPE_SCALING = {
    "factor": 8.0,
    "low_freq_factor": 1.0,
    "high_freq_factor": 4.0,
    "original_max_position_embeddings": 8192,
}


def rms_norm(hidden, weight, eps=EPS):
    """``layer_streaming/llama31.py:21-25``."""

    variance = hidden.float().pow(2).mean(-1, keepdim=True)
    normalized = hidden.float() * torch.rsqrt(variance + eps)
    return weight * normalized.to(hidden.dtype)


def llama3_inv_freq(theta=ROPE_THETA, dim=HEAD_DIM, scaling=None, device=None):
    """Llama-3 scaled inverse frequencies, fp32 ``[dim // 2]``.

    Restates transformers ``modeling_rope_utils.py:550-626``
    (``_compute_llama3_parameters``), which the reference reaches through
    ``LlamaRotaryEmbedding`` (``layer_streaming/llama31.py:125``).
    """

    scaling = dict(ROPE_SCALING if scaling is None else scaling)
    exponents = torch.arange(0, dim, 2, dtype=torch.int64).to(
        device=device, dtype=torch.float
    )
    inv_freq = 1.0 / (theta ** (exponents / dim))
    factor = scaling["factor"]
    low = scaling["low_freq_factor"]
    high = scaling["high_freq_factor"]
    old_len = scaling["original_max_position_embeddings"]
    low_wavelen = old_len / low
    high_wavelen = old_len / high
    wavelen = 2 * math.pi / inv_freq
    scaled = torch.where(wavelen > low_wavelen, inv_freq / factor, inv_freq)
    smooth = (old_len / wavelen - low) / (high - low)
    smoothed = (1 - smooth) * scaled / factor + smooth * scaled
    medium = ~(wavelen < high_wavelen) * ~(wavelen > low_wavelen)
    return torch.where(medium, smoothed, scaled)


def rope_cos_sin(positions, inv_freq, dtype=torch.bfloat16):
    """cos/sin ``[1, M, 128]`` for int64 ``positions [1, M]``.

    Restates transformers ``modeling_llama.py:124-135``: an fp32 outer
    product, ``cat((f, f))``, ``cos``/``sin`` in fp32, then a cast to the
    activation dtype (attention scaling is 1.0 for llama3).
    """

    inv = inv_freq[None, :, None].float().expand(positions.shape[0], -1, 1)
    pos = positions[:, None, :].float()
    freqs = (inv.float() @ pos.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(q, k, cos, sin):
    """transformers ``modeling_llama.py:138-168`` (unsqueeze_dim=1)."""

    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


def attention(query, key, value, causal):
    """GQA attention, ``layer_streaming/llama31.py:182-234``.

    query ``[1, 32, M, 128]``; key/value ``[1, 8, L, 128]`` (the whole cache
    including the new tokens). K/V are repeated 4x (``_repeat_kv :28-31``)
    and SDPA runs with the default scale 1/sqrt(128); the mask is causal only
    for the first multi-token call.
    """

    groups = query.shape[1] // key.shape[1]
    key = key.repeat_interleave(groups, dim=1)
    value = value.repeat_interleave(groups, dim=1)
    out = F.scaled_dot_product_attention(
        query, key, value, dropout_p=0.0, is_causal=causal
    )
    batch, _, length, _ = out.shape
    return out.transpose(1, 2).contiguous().view(batch, length, HEADS * HEAD_DIM)


def merge_topk(cur_values, cur_indices, values, indices, top_k):
    """``layer_streaming/vocab.py:11-32``: exact top-k of the union."""

    if cur_values is not None:
        values = torch.cat((cur_values, values), dim=-1)
        indices = torch.cat((cur_indices, indices), dim=-1)
    keep = min(int(top_k), values.shape[-1])
    best, positions = torch.topk(values, k=keep, dim=-1)
    return best, torch.gather(indices, dim=-1, index=positions)


def layer_key(layer, name):
    block = "self_attn" if name in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
    return "model.layers.{}.{}.{}.weight".format(layer, block, name)


class OracleDecoder:
    """The reference executor's per-token flow as one function per step.

    Mirrors ``Llama31DecodeExecutor.begin/__call__/finish``
    (``layer_streaming/llama31.py:128-154, 236-283, 324-349``) over a plain
    ``weights`` mapping (reference tensor names -> bf16 tensors on one device).
    ``vocab_chunk_rows`` selects the streamed LM head of
    ``layer_streaming/vocab.py:207-266`` (per-chunk topk + merge_topk);
    ``None`` is the resident head (one F.linear + topk).
    """

    def __init__(self, weights, top_k=10, vocab_chunk_rows=None, rope_scaling=None):
        self.weights = weights
        self.top_k = int(top_k)
        self.vocab_chunk_rows = vocab_chunk_rows
        device = weights["model.norm.weight"].device
        self.inv_freq = llama3_inv_freq(scaling=rope_scaling, device=device)
        self.cache = [None] * LAYERS
        self.length = 0

    def reset(self):
        self.cache = [None] * LAYERS
        self.length = 0

    def _layer(self, index, hidden, positions):
        w = self.weights
        prefix = "model.layers.{}".format(index)
        residual = hidden
        normed = rms_norm(hidden, w[prefix + ".input_layernorm.weight"])
        q = F.linear(normed, w[layer_key(index, "q_proj")])
        k = F.linear(normed, w[layer_key(index, "k_proj")])
        v = F.linear(normed, w[layer_key(index, "v_proj")])
        batch, length, _ = q.shape
        q = q.view(batch, length, HEADS, HEAD_DIM).transpose(1, 2)
        k = k.view(batch, length, KV_HEADS, HEAD_DIM).transpose(1, 2)
        v = v.view(batch, length, KV_HEADS, HEAD_DIM).transpose(1, 2)
        cos, sin = rope_cos_sin(positions, self.inv_freq, dtype=v.dtype)
        q, k = apply_rope(q, k, cos, sin)
        had_past = self.cache[index] is not None
        if had_past:
            k = torch.cat((self.cache[index][0], k), dim=-2)
            v = torch.cat((self.cache[index][1], v), dim=-2)
        self.cache[index] = (k, v)
        attn = attention(q, k, v, causal=(not had_past and length > 1))
        hidden = residual + F.linear(attn, w[layer_key(index, "o_proj")])
        residual = hidden
        normed = rms_norm(hidden, w[prefix + ".post_attention_layernorm.weight"])
        gate = F.silu(F.linear(normed, w[layer_key(index, "gate_proj")]))
        up = F.linear(normed, w[layer_key(index, "up_proj")])
        return residual + F.linear(gate * up, w[layer_key(index, "down_proj")])

    def head(self, hidden, return_full_logits=False):
        """Final norm + LM head + top-k (``llama31.py:324-349``)."""

        normed = rms_norm(hidden, self.weights["model.norm.weight"])
        head = self.weights["lm_head.weight"]
        if self.vocab_chunk_rows is None:
            logits = F.linear(normed, head).float()
            values, indices = torch.topk(logits[:, -1:, :], k=self.top_k, dim=-1)
            return {"values": values, "indices": indices, "logits": logits}
        last = normed[:, -1:, :]
        values = indices = None
        full = [] if return_full_logits else None
        for start in range(0, VOCAB, self.vocab_chunk_rows):
            stop = min(start + self.vocab_chunk_rows, VOCAB)
            part = F.linear(last, head[start:stop]).float()
            local_v, local_i = torch.topk(part, k=min(self.top_k, stop - start), dim=-1)
            values, indices = merge_topk(values, indices, local_v, local_i + start, self.top_k)
            if full is not None:
                full.append(part)
        logits = torch.cat(full, dim=-1) if full is not None else None
        return {"values": values, "indices": indices, "logits": logits}

    def step(self, input_ids, return_full_logits=False):
        """One executor pass: ``begin`` + all layers + ``finish``."""

        if input_ids.ndim != 2 or input_ids.shape[0] != 1:
            raise ValueError("oracle supports one unpadded request")
        if self.length and input_ids.shape[1] != 1:
            raise ValueError("after prefill only one-token steps are supported")
        length = input_ids.shape[1]
        positions = torch.arange(
            self.length, self.length + length, dtype=torch.long, device=input_ids.device
        ).unsqueeze(0)
        hidden = F.embedding(input_ids, self.weights["model.embed_tokens.weight"])
        for index in range(LAYERS):
            hidden = self._layer(index, hidden, positions)
        self.length += length
        return self.head(hidden, return_full_logits=return_full_logits)
