"""One rank of the two-GPU tensor-parallel parity check (run by torchrun
from test_gpu_tensor_parallel.py; prints TP-PARITY-OK on rank 0 when every
check passes).

Each rank generates its shards of the seeded model (BASELINE config 0
weights), decodes the 6-token seeded prompt + 8 greedy steps through the
peer-memory exchange and through NCCL, and checks that
  * all ranks hold the same top-k bits after every step,
  * both exchange paths give the same greedy tokens and top-k values within
    rtol/atol 2e-2,
  * the greedy tokens and top-k values reproduce the reference's golden run
    (tests/golden/config0.json) within the same tolerance.
"""

import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for path in (REPO, os.path.join(REPO, "cascade-llm_b200")):
    if path not in sys.path:
        sys.path.insert(0, path)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle.seeded import prompt_ids  # noqa: E402


class Config:
    hidden_size = 4096
    intermediate_size = 14336
    num_hidden_layers = 32
    num_attention_heads = 32
    num_key_value_heads = 8
    vocab_size = 128256
    rms_norm_eps = 1e-5
    rope_parameters = {
        "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192, "rope_theta": 500000.0,
    }


def greedy(decoder, ids, steps):
    out = []
    with torch.inference_mode():
        for _ in range(steps):
            state = decoder(ids)
            out.append((state.topk_values.reshape(-1).clone(), state.topk_indices.reshape(-1).clone()))
            ids = state.topk_indices[..., 0].reshape(1, 1)
    decoder.check_errors()
    return out


def main():
    from layer_streaming.tensor_parallel import TensorParallelDecoder, TensorParallelWeights

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    world, rank = dist.get_world_size(), dist.get_rank()
    meta = json.load(open(os.path.join(HERE, "golden", "config0.json")))
    weights = TensorParallelWeights.seeded(world, rank, device, seed=meta["weight_seed"])
    ids = prompt_ids(6, seed=meta["prompt_seed"]).view(1, -1).to(device)
    runs = {}
    for exchange in ("peer", "nccl"):
        decoder = TensorParallelDecoder(Config(), weights, top_k=meta["top_k"], exchange=exchange)
        runs[exchange] = greedy(decoder, ids, 1 + meta["decode_steps"])
        decoder.close()
    failures = []
    for exchange, run in runs.items():
        for step, (values, indices) in enumerate(run):
            both = torch.cat([values.view(torch.int32).to(torch.int64), indices])
            gathered = torch.empty((world,) + tuple(both.shape), dtype=both.dtype, device=device)
            dist.all_gather_into_tensor(gathered, both)
            if not all(torch.equal(gathered[0], gathered[q]) for q in range(world)):
                failures.append("{} step {}: ranks disagree".format(exchange, step))
    if rank == 0:
        for exchange, run in runs.items():
            for step, ((values, indices), record) in enumerate(zip(run, meta["steps"])):
                ref = torch.tensor(record["topk_values"])
                if not torch.allclose(values.cpu(), ref, rtol=2e-2, atol=2e-2):
                    failures.append("{} step {}: top-k values {} vs golden {}".format(
                        exchange, step, values.cpu().tolist(), ref.tolist()))
                if step < 8 and int(indices[0]) != meta["greedy_ids"][step]:
                    failures.append("{} step {}: greedy id {} vs golden {}".format(
                        exchange, step, int(indices[0]), meta["greedy_ids"][step]))
        same_bits = all(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
                        for a, b in zip(runs["peer"], runs["nccl"]))
        print("world {}: peer and NCCL exchanges bit-identical: {}".format(world, same_bits))
        for line in failures:
            print("FAIL", line)
        if not failures:
            print("TP-PARITY-OK")
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
