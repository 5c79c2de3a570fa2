"""Host logic of tensor-parallel decode, on CPU (no GPU needed).

* the shard rules cover every tensor of the model, split each sharded
  dimension evenly and give a query head's GQA KV head to the same rank;
* one Llama block computed by two ``gloo`` ranks from their shards (column
  partials of o_proj / down_proj all-reduced before the residual add, as the
  decoder does) equals the block computed from the full weights (fp32);
* the vocabulary-sharded top-k (each rank's exact top-k with global ids,
  all-gathered, merged) equals the global top-k.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from layer_streaming import tensor_parallel as tp
from oracle import llama_oracle as lo

# Llama-3.1-8B block dimensions (the shard rules are written for them)
H, FFN, HEADS, KV, D = 4096, 14336, 32, 8, 128


def test_shard_rules_cover_the_model():
    for world in tp.WORLD_SIZES:
        for key in tp.model_keys():
            shape = tp.full_shape(key)
            pieces = [tp.shard_spec(key, world, r) for r in range(world)]
            if pieces[0] is None:
                assert all(p is None for p in pieces)
                assert key.endswith("norm.weight") or key == "model.embed_tokens.weight"
                continue
            dim = pieces[0][0]
            assert all(p[0] == dim for p in pieces)
            # contiguous, disjoint, covering, equal
            assert pieces[0][1] == 0 and pieces[-1][2] == shape[dim]
            for a, b in zip(pieces, pieces[1:]):
                assert a[2] == b[1]
            sizes = {p[2] - p[1] for p in pieces}
            assert len(sizes) == 1
            size = sizes.pop()
            name = key.split(".")[-2]
            if name in ("q_proj", "o_proj"):
                assert size % D == 0  # whole heads
            if name in ("k_proj", "v_proj"):
                assert size % D == 0
            if key == "lm_head.weight":
                assert size % 2 == 0  # the LM-head kernel pairs rows
    with pytest.raises(ValueError):
        tp.shard_spec("lm_head.weight", 3, 0)


def test_gqa_heads_stay_on_their_rank():
    for world in tp.WORLD_SIZES:
        for r in range(world):
            _, q0, q1 = tp.shard_spec(lo.layer_key(0, "q_proj"), world, r)
            _, k0, k1 = tp.shard_spec(lo.layer_key(0, "k_proj"), world, r)
            q_heads = range(q0 // D, q1 // D)
            kv_heads = range(k0 // D, k1 // D)
            assert all(h // (HEADS // KV) in kv_heads for h in q_heads)
            _, o0, o1 = tp.shard_spec(lo.layer_key(0, "o_proj"), world, r)
            assert (o0, o1) == (q0, q1)  # o_proj columns = this rank's attention output
            _, g0, g1 = tp.shard_spec(lo.layer_key(0, "gate_proj"), world, r)
            _, d0, d1 = tp.shard_spec(lo.layer_key(0, "down_proj"), world, r)
            assert (g0, g1) == (d0, d1)


def _block_weights(seed=5):
    gen = torch.Generator().manual_seed(seed)
    w = {}
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
        key = lo.layer_key(0, name)
        w[key] = torch.randn(tp.full_shape(key), generator=gen) * 0.02
    w["in_norm"] = 1.0 + 0.1 * torch.randn(H, generator=gen)
    w["post_norm"] = 1.0 + 0.1 * torch.randn(H, generator=gen)
    return w


def _block(x, w, heads, kv_heads, positions, all_reduce):
    """One Llama block in fp32 over `heads` query heads (any shard)."""

    m = x.shape[0]
    inv_freq = lo.llama3_inv_freq()
    normed = lo.rms_norm(x, w["in_norm"])
    q = (normed @ w[lo.layer_key(0, "q_proj")].T).view(1, m, heads, D).transpose(1, 2)
    k = (normed @ w[lo.layer_key(0, "k_proj")].T).view(1, m, kv_heads, D).transpose(1, 2)
    v = (normed @ w[lo.layer_key(0, "v_proj")].T).view(1, m, kv_heads, D).transpose(1, 2)
    cos, sin = lo.rope_cos_sin(positions.view(1, -1), inv_freq, dtype=torch.float32)
    q, k = lo.apply_rope(q, k, cos, sin)
    k = k.repeat_interleave(heads // kv_heads, dim=1)
    v = v.repeat_interleave(heads // kv_heads, dim=1)
    attn = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(m, heads * D)
    o = attn @ w[lo.layer_key(0, "o_proj")].T
    x = x + all_reduce(o)
    normed = lo.rms_norm(x, w["post_norm"])
    act = F.silu(normed @ w[lo.layer_key(0, "gate_proj")].T) * (normed @ w[lo.layer_key(0, "up_proj")].T)
    return x + all_reduce(act @ w[lo.layer_key(0, "down_proj")].T)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        full = _block_weights()
        x = torch.randn(5, H, generator=torch.Generator().manual_seed(9)) * 0.5
        positions = torch.arange(3, 8)
        shards = {key: tp.shard_tensor(value, key, world, rank) if key.startswith("model.") else value
                  for key, value in full.items()}

        def reduce(t):
            t = t.clone()
            dist.all_reduce(t)
            return t

        got = _block(x, shards, HEADS // world, KV // world, positions, reduce)
        want = _block(x, full, HEADS, KV, positions, lambda t: t)
        block_err = float((got - want).abs().max() / want.abs().max())

        # vocabulary-sharded top-k with global ids, gathered and merged
        logits = torch.randn(tp.VOCAB, generator=torch.Generator().manual_seed(3))
        logits[1000] = logits[77777] = logits.max() + 1.0  # a tie across shards
        _, lo_row, hi_row = tp.shard_spec("lm_head.weight", world, rank)
        local_v, local_i = torch.topk(logits[lo_row:hi_row], 10)
        local_i = local_i + lo_row
        all_v = [torch.empty_like(local_v) for _ in range(world)]
        all_i = [torch.empty_like(local_i) for _ in range(world)]
        dist.all_gather(all_v, local_v)
        dist.all_gather(all_i, local_i)
        merged_v, merged_i = lo.merge_topk(None, None, torch.cat(all_v), torch.cat(all_i), 10)
        want_v, want_i = torch.topk(logits, 10)
        topk_ok = torch.equal(merged_v, want_v) and set(merged_i[2:].tolist()) == set(want_i[2:].tolist()) \
            and set(merged_i[:2].tolist()) == {1000, 77777}
        results[rank] = (block_err, topk_ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_block_and_vocab_topk_match_full(world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for rank in range(world):
        block_err, topk_ok = results[rank]
        assert block_err < 1e-5, block_err
        assert topk_ok


def test_shard_arena_units_are_the_rank_slices():
    """The streamed shard arena: 4 units per layer in stream order, 256-byte
    aligned, each piece exactly this rank's slice of the full tensor."""

    full = {}
    gen = torch.Generator().manual_seed(11)
    for name in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
        key = lo.layer_key(0, name)
        full[key] = torch.randint(-100, 100, tp.full_shape(key), generator=gen).to(torch.bfloat16)
    for world in (2, 4):
        for rank in range(world):
            arena = tp.ShardArena(world, rank, layers=1, pin=False)
            assert [u[1] for u in arena.units] == ["qkv", "o_proj", "gate_up", "down_proj"]
            for key, value in full.items():
                arena.host_view(key).copy_(tp.shard_tensor(value, key, world, rank))
            spans = arena.spans()
            for (layer, name, offset, elements, pieces), (addr, nbytes) in zip(arena.units, spans):
                assert offset % tp.ShardArena.ALIGN == 0 and nbytes == 2 * elements
                assert addr == arena.storage.data_ptr() + 2 * offset
                flat = arena.storage.narrow(0, offset, elements)
                for key, inner, rows, cols in pieces:
                    want = tp.shard_tensor(full[key], key, world, rank)
                    assert want.shape == (rows, cols)
                    assert torch.equal(flat.narrow(0, inner, rows * cols).view(rows, cols), want)
            # unit views over a "device slot" (here a host tensor) see the same bytes
            slot = torch.empty(arena.unit_elements, dtype=torch.bfloat16)
            _, _, offset, elements, _ = arena.units[2]
            slot[:elements].copy_(arena.storage.narrow(0, offset, elements))
            views = arena.views(2, slot)
            assert torch.equal(views[lo.layer_key(0, "up_proj")],
                               tp.shard_tensor(full[lo.layer_key(0, "up_proj")], lo.layer_key(0, "up_proj"),
                                               world, rank))


def _stream_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _block_weights()
        arena = tp.ShardArena(world, rank, layers=1, pin=False)
        for key, value in full.items():
            if key.startswith("model."):
                arena.host_view(key).copy_(tp.shard_tensor(value, key, world, rank).to(torch.bfloat16))
        # stream the four units through one "slot" in order, as the decoder does
        slot = torch.empty(arena.unit_elements, dtype=torch.bfloat16)
        mats = {}
        for index, (_, _, offset, elements, _) in enumerate(arena.units):
            slot[:elements].copy_(arena.storage.narrow(0, offset, elements))
            mats.update({k: v.float().clone() for k, v in arena.views(index, slot).items()})
        mats["in_norm"], mats["post_norm"] = full["in_norm"], full["post_norm"]
        x = torch.randn(5, H, generator=torch.Generator().manual_seed(9)) * 0.5

        def reduce(t):
            t = t.clone()
            dist.all_reduce(t)
            return t

        got = _block(x, mats, HEADS // world, KV // world, torch.arange(3, 8), reduce)
        ref = {k: (v.to(torch.bfloat16).float() if k.startswith("model.") else v) for k, v in full.items()}
        want = _block(x, ref, HEADS, KV, torch.arange(3, 8), lambda t: t)
        results[rank] = float((got - want).abs().max() / want.abs().max())
    finally:
        dist.destroy_process_group()


def test_streamed_shards_give_the_full_block_over_gloo():
    """Two gloo ranks, each streaming only its shard arena's units, all-reduce
    to the block of the full (bf16) weights."""

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_stream_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert all(results[r] < 1e-5 for r in range(2)), dict(results)
