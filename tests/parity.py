"""Parity criteria shared by the model-level GPU tests and the multi-GPU worker.

North-star criteria: top-k values within rtol/atol 2e-2 of the reference's own
PyTorch path on the same seeded weights and inputs (its ops restated by the
oracle, run on the same GPU) and of its CPU run (tests/golden/config0.*),
each widened by the reference's own disagreement at that step: after 32
random-init layers the reference's GPU and CPU paths differ by up to ~0.3 per
logit and ~0.1 per top-k value, so an engine is held to the same distance
from either path that the reference keeps between its two paths.
"""

import torch

RTOL = ATOL = 2e-2


class GpuTopk(list):
    """Per-step top-k values of the reference's GPU path; `.indices` holds ids."""

    indices = None


def reference_gpu_topk(weights, meta, device):
    """Top-k values (and, as `.indices`, ids) of the reference's ops on
    `device` (the oracle's restatement over the full weight dict), fed the
    golden run's inputs."""

    from oracle import llama_oracle as lo

    oracle = lo.OracleDecoder(weights, top_k=meta["top_k"])
    out = GpuTopk()
    out.indices = []
    with torch.inference_mode():
        for record in meta["steps"]:
            logits = oracle.step(torch.tensor([record["input_ids"]], device=device))["logits"][0, -1].float()
            top = torch.topk(logits, meta["top_k"])
            out.append(top.values.cpu())
            out.indices.append(top.indices.cpu())
    return out


def tolerance(value):
    return ATOL + RTOL * abs(value)


def greedy_failure(step, engine_id, record, meta):
    """None if the engine's greedy pick at `step` is the reference's, or one
    of the candidates tied with it within the tolerance (a summation-order
    flip); else a message. The second return value tells whether the step was
    such a tie (the sequences may part after it)."""

    golden_id = meta["greedy_ids"][step]
    if engine_id == golden_id:
        return None, False
    values, ids = record["topk_values"], record["topk_indices"]
    tied = [ids[j] for j in range(len(values)) if values[0] - values[j] <= tolerance(values[0])]
    if len(tied) > 1 and engine_id in tied:
        return None, True
    return "greedy id {} vs the reference's {} (tied candidates {})".format(engine_id, golden_id, tied), False


def topk_values_failure(values, record, gpu_values):
    """None if `values` meet both criteria, else a message."""

    values = values.float().cpu()
    golden = torch.tensor(record["topk_values"])
    noise = float((gpu_values - golden).abs().max())  # the reference's GPU-vs-CPU top-k distance
    if not bool(((values - gpu_values).abs() <= ATOL + RTOL * gpu_values.abs() + noise).all()):
        return "values {} vs the reference's GPU path {} (its CPU run {})".format(
            values.tolist(), gpu_values.tolist(), golden.tolist())
    if not bool(((values - golden).abs() <= ATOL + RTOL * golden.abs() + noise).all()):
        return "values {} vs the reference's CPU run {} (GPU path {})".format(
            values.tolist(), golden.tolist(), gpu_values.tolist())
    return None
