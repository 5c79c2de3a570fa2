#!/usr/bin/env python3
"""Decode benchmark: Llama-3.1-8B architecture, batch 1, 2K context, B200.

Metric: decode ms/token at bs=1 with a 2K context, plus the
achieved HBM bandwidth against the measured peak. One "step" is one greedy
decode token through the engine's public API (executor.begin -> runtime.run
-> executor.finish) with all weights resident in HBM.

Workload: seeded random-init BF16 weights (N(0,0.02), norms 1; no network
for checkpoints), a 2048-token prefill of uniform random ids fills the KV
cache, then W warm-up and K timed decode steps. The weights (16 GB) exceed
L2 (126 MB), so no L2 flush is needed between steps.

  value          device time per token (CUDA events, max over ranks)
  e2e            the same step with the token id copied in from pinned host
                 memory and the top-k read back every step
  roofline       the dominant kernel (gate+up GEMV with SwiGLU), timed live
  step_roofline  algorithmic bytes of the whole step / ms per token
  cpu_baseline   the reference's algorithm (oracle restatement, torch CPU)
                 on this host's cores, a bounded sample of decode steps

--impl reference times that CPU path alone (rank 0) on the same config.
"""

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "cascade-llm_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode ms/token, Llama-3.1-8B arch bs=1 (2K ctx)"
LAYER_BYTES = 32 * 436_207_616
HEAD_BYTES = 1_050_673_152
NORM_BYTES = 532_480
GATE_UP_BYTES = 234_881_024
# dram__bytes_read.sum + dram__bytes_write.sum of one gate+up launch, from an ncu
# capture (--set full) of `bench.py --micro gate_up` (bytes per launch)
GATE_UP_TRAFFIC = 239_350_000


# algorithmic bytes per launch of the kernels timed by --micro
MICRO_BYTES = {
    "qkv": 6144 * 4096 * 2,
    "o_proj": 4096 * 4096 * 2,
    "gate_up": GATE_UP_BYTES,
    "down_proj": 4096 * 14336 * 2,
    "lm_head": HEAD_BYTES,
    "attention": 8 * 2048 * 128 * 2 * 2,
    # int8 weight-only GEMVs: int8 rows + one fp32 scale per row
    "gate_up_i8": 28672 * 4096 + 28672 * 4,
    "down_proj_i8": 4096 * 14336 + 4096 * 4,
    "lm_head_i8": 128256 * 4096 + 128256 * 4,
}


# prefill GEMMs timed by --micro: (out features, in features) of one layer's
# projection at M = --tokens rows
GEMM_SHAPES = {
    "gemm_qkv": (6144, 4096),
    "gemm_o_proj": (4096, 4096),
    "gemm_gate_up": (28672, 4096),
    "gemm_down_proj": (4096, 14336),
}


def step_bytes(context):
    """Algorithmic HBM bytes of one decode token at `context` cached positions."""

    return LAYER_BYTES + HEAD_BYTES + NORM_BYTES + 8192 + 131_072 * (context + 1) + 131_072


# int8 weight-only decode: half the weight bytes plus one fp32 scale per row
# (32 layers x (6144 + 4096 + 28672 + 4096) rows, LM head 128256 rows)
SCALE_BYTES = 4 * (32 * (6144 + 4096 + 28672 + 4096) + 128256)


def step_bytes_i8(context):
    """Algorithmic HBM bytes of one int8 decode token (bf16 KV cache, norms, embedding)."""

    return step_bytes(context) - (LAYER_BYTES + HEAD_BYTES) // 2 + SCALE_BYTES


def parse_args():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--context", type=int, default=2048)
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--tokens", type=int, default=512, help="rows of the --micro gemm_* cases")
    parser.add_argument("--prefill-chunk", type=int, default=2048,
                        help="tokens per prefill step of the context fill (the prefill line's chunk)")
    parser.add_argument("--sweep", action="store_true",
                        help="BASELINE config 3: each projection at M in {1, 6, 64, 512}, HBM-resident and "
                             "H2D-streamed through two slots (one JSON line per case)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-int8", action="store_true",
                        help="skip the int8 weight-only decode measurement (a reduced-precision side line)")
    parser.add_argument("--no-streamed", action="store_true", help="skip the H2D-streamed mode measurement")
    parser.add_argument("--profile-range", action="store_true",
                        help="after warm-up, run --steps decode steps between cudaProfilerStart/Stop "
                             "(for `ncu --profile-from-start off`) and exit")
    parser.add_argument("--trace", action="store_true",
                        help="after warm-up, record the per-CTA %%globaltimer timeline (cb_set_trace) of "
                             "--steps decode steps and print per-kernel-role phase medians as JSON, then exit")
    parser.add_argument("--micro",
                        choices=sorted(MICRO_BYTES) + sorted(GEMM_SHAPES) + ["prefill_attention", "exchange"],
                        help="time one kernel alone on a small footprint (rotating copies > L2)")
    parser.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                        help="N>1: tensor-parallel exchange through peer memory inside the projection "
                             "kernels (default) or NCCL collectives between kernels")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    return args


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


def measured_peak(key="hbm_gbs"):
    """(peak, "measured"|"fallback"): HBM GB/s, or dense bf16 TFLOP/s for
    key="bf16_tflops" (burst) / "bf16_tflops_sustained"."""

    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}[key]
    try:
        with open(path) as source:
            return float(json.load(source)[key]), "measured"
    except (OSError, KeyError, ValueError):
        return fallback, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(r[1]) for r in rows)
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, flag in zip(names, r[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": sm[len(sm) // 2],
            "sm_max_mhz": float(rows[0][2]),
            "samples": len(rows),
            "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "", 1).isdigit()) if rows else None,
            "reasons": sorted(reasons),
        }


def random_ids(count, seed):
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, 128256, (1, count), generator=gen)


def build_engine(device, context, extra):
    import layer_streaming as ls

    plan = ls.build_llama31_8b_plan("matrix_group")
    store = ls.create_weight_store(plan, "full_pinned")
    store.fill_seeded(seed=0, device=device)
    resident = ls.ResidentDeviceArena(plan, store, device)
    runtime = ls.DoubleBufferRuntime(plan, store, resident, device, weights="hbm")
    executor = ls.Llama31DecodeExecutor(
        Config(), resident, top_k=10, max_length=context + extra, allow_chunked_prefill=True
    )
    return plan, store, resident, runtime, executor


def step(executor, runtime, ids):
    state = executor.begin(ids)
    state = runtime.run(executor, state)
    return executor.finish(state)


def prefill(executor, runtime, device, context, chunk=512):
    """Chunked prefill of `context` random ids; returns (next token, ms)."""

    ids = random_ids(context, seed=1).to(device)
    state = None
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.inference_mode():
        start.record()
        for begin in range(0, context, chunk):
            state = step(executor, runtime, ids[:, begin:begin + chunk])
        end.record()
    torch.cuda.synchronize(device)
    executor.check_errors()
    return state.topk_indices[..., 0], start.elapsed_time(end)


def time_decode(executor, runtime, token, steps, warmup, barrier):
    with torch.inference_mode():
        for _ in range(warmup):
            token = step(executor, runtime, token).topk_indices[..., 0]
        torch.cuda.synchronize()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            token = step(executor, runtime, token).topk_indices[..., 0]
        end.record()
        torch.cuda.synchronize()
        barrier()
    return start.elapsed_time(end) / steps, token


TRACE_ROLES = ("qkv", "attention", "o_proj", "gate_up", "down_proj")


def trace_decode(executor, runtime, token, steps, warmup):
    """Per-CTA launch timeline of `steps` decode steps (cb_set_trace).

    Each traced CTA records its start, the return of its dependency wait,
    the end of its main loop (attention: of its sub-chunk loop) and its end
    (%globaltimer ns); the LM head also the end of its own top-k and of its
    ticket. Launches are grouped per step in issue order (per layer QKV,
    attention, o_proj, gate+up, down; then the LM head). Reported per role,
    as medians over layers and steps, in us: `interval` from the previous
    launch's last CTA end to this launch's last CTA end, `wait_release` from
    the previous launch's end to this launch's first released wait, `loop`
    from its last released wait to its last main-loop end, `loop_spread`
    between its first and last main-loop end, and `tail` from the last
    main-loop end to the last CTA end."""

    from layer_streaming import _native

    lib = _native.lib()
    per_step = 32 * 1500 + 400  # 32 x (4 GEMV grids of 296 CTAs + 256 attention CTAs) + the LM head
    cap = per_step * steps
    buf = torch.zeros(8 * (cap + 1), dtype=torch.int64, device=executor.device)
    buf[1] = cap
    _native.check(lib.cb_set_trace(buf.data_ptr()), "cb_set_trace")
    executor._graphs.clear()  # recapture: a captured launch keeps the trace pointer it was captured with
    try:
        with torch.inference_mode():
            for _ in range(warmup):
                token = step(executor, runtime, token).topk_indices[..., 0]
            torch.cuda.synchronize()
            buf[0] = 0
            for _ in range(steps):
                token = step(executor, runtime, token).topk_indices[..., 0]
            torch.cuda.synchronize()
    finally:
        _native.check(lib.cb_set_trace(None), "cb_set_trace")
        executor._graphs.clear()
    count = min(int(buf[0].item()), cap)
    rec = buf[8:8 * (count + 1)].view(count, 8).cpu().numpy()
    summary = summarize_trace(rec)
    summary["context"] = executor.kv_cache.length
    return summary


def summarize_trace(rec, layers=32):
    """Phase medians of trace records (rows of 8 int64 words as cb_set_trace
    writes them) of whole decode steps; see trace_decode for the phases."""

    tags = rec[:, 0] >> 32
    launches = []
    for tag in np.unique(tags):
        rows = rec[tags == tag]
        rows = rows[np.argsort(rows[:, 2])]
        # a captured launch replays its tag once per step: split at gaps of > 0.5 ms
        cuts = np.where(np.diff(rows[:, 2]) > 500_000)[0] + 1
        launches.extend(np.split(rows, cuts))
    launches.sort(key=lambda r: int(r[:, 2].min()))
    layer_launches = len(TRACE_ROLES) * layers
    roles = {name: {"interval": [], "wait_release": [], "loop": [], "loop_spread": [], "tail": []}
             for name in TRACE_ROLES + ("lm_head",)}
    head_phases = {"topk": [], "ticket": [], "merge": []}
    spans = []
    i = 0
    while i + layer_launches < len(launches):
        group = launches[i:i + layer_launches + 1]
        i += layer_launches + 1
        prev_end = None
        for j, r in enumerate(group):
            name = TRACE_ROLES[j % len(TRACE_ROLES)] if j < layer_launches else "lm_head"
            end, wait_min, wait_max = r[:, 5].max(), r[:, 3].min(), r[:, 3].max()
            loop_min, loop_max = r[:, 4].min(), r[:, 4].max()
            d = roles[name]
            if prev_end is not None:
                d["interval"].append((end - prev_end) / 1e3)
                d["wait_release"].append((wait_min - prev_end) / 1e3)
            d["loop"].append((loop_max - wait_max) / 1e3)
            d["loop_spread"].append((loop_max - loop_min) / 1e3)
            d["tail"].append((end - loop_max) / 1e3)
            prev_end = end
        head = group[-1]
        head_phases["topk"].append((head[:, 6].max() - head[:, 4].max()) / 1e3)
        head_phases["ticket"].append((head[:, 7].max() - head[:, 6].max()) / 1e3)
        head_phases["merge"].append((head[:, 5].max() - head[:, 7].max()) / 1e3)
        spans.append((group[-1][:, 5].max() - group[0][:, 2].min()) / 1e3)
    med = lambda v: round(float(np.median(v)), 2) if v else None
    return {"trace": "decode step, per-CTA %globaltimer", "steps": len(spans),
            "step_us": [round(x, 1) for x in spans],
            "roles_us": {name: {k: med(v) for k, v in d.items()} for name, d in roles.items()},
            "lm_head_tail_us": {k: med(v) for k, v in head_phases.items()},
            "note": "tracing adds a few %globaltimer reads and one atomic per CTA; compare shares"}


def time_int8(resident, runtime, device, context, steps, warmup):
    """The optional int8 weight-only mode on the same workload (own executor
    and KV cache, same seeded weights quantized on the device): a
    reduced-precision side measurement, never the line's value."""

    import layer_streaming as ls

    executor = ls.Llama31DecodeExecutor(Config(), resident, top_k=10, max_length=context + warmup + steps + 72,
                                        allow_chunked_prefill=True, decode_weights="int8")
    token, _ = prefill(executor, runtime, device, context)
    ms, _ = time_decode(executor, runtime, token, steps, warmup, lambda: None)
    executor.check_errors()
    cached = executor.kv_cache.length - steps - 1
    nbytes = step_bytes_i8(cached)
    del executor
    torch.cuda.empty_cache()
    return {"ms_per_token": round(ms, 4), "bytes_per_token": nbytes,
            "achieved_gbs": round(nbytes / (ms / 1000.0) / 1e9, 1),
            "note": "decode_weights='int8' (per-row symmetric int8 weights, fp32 scales; bf16 activations, "
                    "KV cache and prefill): reduced precision, outside the bf16 parity contract"}


def time_e2e(executor, runtime, token, steps):
    """Host-driven loop: id H2D from pinned memory, top-k D2H every step."""

    ids_host = torch.empty((1, 1), dtype=torch.int64).pin_memory()
    ids_host[0, 0] = int(token.reshape(-1)[0])
    h2d = ids_host.numel() * ids_host.element_size()
    d2h = 0
    values_host = indices_host = None
    with torch.inference_mode():
        torch.cuda.synchronize()
        started = time.perf_counter()
        for _ in range(steps):
            state = step(executor, runtime, ids_host)
            if values_host is None:
                values_host = torch.empty(state.topk_values.shape, dtype=state.topk_values.dtype).pin_memory()
                indices_host = torch.empty(state.topk_indices.shape, dtype=state.topk_indices.dtype).pin_memory()
            # both results copied asynchronously, one wait for the step
            values_host.copy_(state.topk_values, non_blocking=True)
            indices_host.copy_(state.topk_indices, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            d2h = values_host.numel() * values_host.element_size() + indices_host.numel() * indices_host.element_size()
            ids_host[0, 0] = int(indices_host.reshape(-1)[0])
        elapsed = time.perf_counter() - started
    return {"value": elapsed * 1000.0 / steps, "unit": "ms/token", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h}


def time_streamed(plan, store, resident, executor, device, token, steps=3, transfer="bf16"):
    """The reference's own mode on this GPU: every decode token streams the 15 GB
    of layer weights H2D from the pinned host arena through two 224 MiB slots
    (copy stream overlapped with the compute stream), same kernels. With
    transfer="int8" the units cross PCIe as int8 rows + fp32 scales (about
    half the bytes; reduced precision)."""

    import layer_streaming as ls

    runtime = ls.DoubleBufferRuntime(plan, store, resident, device, weights="streamed", profile=True,
                                     transfer=transfer)
    with torch.inference_mode():
        token = step(executor, runtime, token).topk_indices[..., 0]  # warm-up
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            token = step(executor, runtime, token).topk_indices[..., 0]
        end.record()
        torch.cuda.synchronize()
    profile = runtime.last_profile or {}
    return {"ms_per_token": round(start.elapsed_time(end) / steps, 2), "steps": steps,
            "h2d_bytes_per_token": int(profile.get("h2d_bytes", plan.stream_bytes_per_token)),
            "h2d_effective_gbps": round(float(profile.get("h2d_effective_gbps", 0.0)), 2),
            "note": "weights='streamed'{}: H2D-bound (PCIe); the timed value is the HBM-resident mode".format(
                ", transfer='int8' (int8 rows + fp32 scales, reduced precision)" if transfer == "int8" else "")}


def time_gate_up(executor, runtime, plan, reps=4):
    """Live timing of the dominant kernel: the 32 gate+up GEMVs back to back
    (one per layer, so the 7.5 GB they read cannot come from L2)."""

    from layer_streaming import ops

    x = executor._x[0]
    out = executor._mlp[0]
    mats = []
    for index, unit in enumerate(plan.units):
        if unit.operation == "gate_up":
            views = runtime.unit_views(index)
            layer = unit.layer_index
            mats.append((
                views["model.layers.{}.mlp.gate_proj.weight".format(layer)],
                views["model.layers.{}.mlp.up_proj.weight".format(layer)],
                executor.resident["model.layers.{}.post_attention_layernorm.weight".format(layer)],
            ))
    stream = torch.cuda.current_stream()
    for wg, wu, norm in mats:  # warm-up
        ops.gate_up_swiglu(x, norm, 1e-5, wg, wu, out)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        for wg, wu, norm in mats:
            ops.gate_up_swiglu(x, norm, 1e-5, wg, wu, out)
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / (reps * len(mats))


def cpu_decode_ms(weights, context, threads, budget_s, max_steps=20):
    """ms/token of the reference's decode step (the oracle's restatement of
    its executor, torch CPU ops) on `threads` host threads, over a
    `context`-token KV cache of seeded random post-RoPE K/V (a CPU prefill
    of the context would be ~33 TFLOP; attention cost does not depend on the
    cached values). Steps run until `budget_s` is spent (at most
    `max_steps`); the first step is excluded as warm-up."""

    from oracle import llama_oracle as lo

    previous = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        oracle = lo.OracleDecoder(weights, top_k=10)
        gen = torch.Generator().manual_seed(2)
        oracle.cache = [
            tuple(torch.randn((1, 8, context, 128), generator=gen).to(torch.bfloat16) for _ in range(2))
            for _ in range(32)
        ]
        oracle.length = context
        token = torch.tensor([[1]])
        times = []
        with torch.inference_mode():
            while len(times) < max_steps and (len(times) < 3 or sum(times[1:]) < budget_s):
                started = time.perf_counter()
                token = oracle.step(token)["indices"][..., 0]
                times.append(time.perf_counter() - started)
    finally:
        torch.set_num_threads(previous)
    steady = times[1:]
    return 1000.0 * sum(steady) / len(steady), len(steady)


def cpu_baseline(weights, context, budget_s):
    """The reference's CPU path on this host: all cores (the reported value)
    and 8 threads, the same sample for both arms of the benchmark."""

    cores = len(os.sched_getaffinity(0)) or 1  # the host threads this process may use
    full, steps_full = cpu_decode_ms(weights, context, cores, budget_s)
    eight, steps_eight = cpu_decode_ms(weights, context, min(8, cores), budget_s)
    return {
        "value": round(full, 3),
        "unit": "ms/token",
        "cores": cores,
        "kind": "port",
        "sample": "{} decode steps (after 1 warm-up) at a {}-token context of seeded random K/V; "
                  "oracle/llama_oracle.py restates the reference executor's torch ops".format(steps_full, context),
        "threads_8": {"value": round(eight, 3), "unit": "ms/token", "cores": min(8, cores), "steps": steps_eight},
    }


def bench_config(args):
    """The config both arms report (the driver compares them)."""

    return {
        "workload": "llama31-8b decode bs=1, {}-token context".format(args.context),
        "context": args.context,
        "model": "Llama-3.1-8B architecture, seeded random-init bf16 weights (seed 0)",
        "plan": "matrix_group, resident vocab",
        "flush": "none needed: weights (16 GB) larger than L2 (126 MB)",
        "parallelism": "single GPU" if args.gpus == 1 else "tp{}".format(args.gpus),
    }


def micro_gemm(args, device):
    """One prefill projection GEMM of a layer (tcgen05), back to back over the
    weights of 8 layers (> L2), at M = --tokens rows: TFLOP/s vs the measured
    dense bf16 peak."""

    from layer_streaming import _native, ops

    lib = _native.lib()
    _native.check(lib.cb_prepare(), "cb_prepare")
    bf = torch.bfloat16
    name = args.micro
    n, k = GEMM_SHAPES[name]
    m = args.tokens
    # the executor's split-K registration for short chunks
    split_ws = torch.empty(4 << 20, dtype=torch.float32, device=device)
    split_tickets = torch.zeros(1024, dtype=torch.int32, device=device)
    _native.check(lib.cb_set_gemm_workspace(split_ws.data_ptr(), 16 << 20, split_tickets.data_ptr(), 1024),
                  "cb_set_gemm_workspace")
    gen = torch.Generator(device=device).manual_seed(5)
    a = (torch.randn((m, k), generator=gen, device=device)).to(bf)
    layers = 8
    if name == "gemm_gate_up":
        mats = [((torch.randn((n // 2, k), generator=gen, device=device) * 0.02).to(bf),
                 (torch.randn((n // 2, k), generator=gen, device=device) * 0.02).to(bf)) for _ in range(layers)]
        out = torch.empty((m, n // 2), dtype=bf, device=device)
        run = lambda w: ops.gemm_swiglu(a, w[0], w[1], out)
    elif name == "gemm_qkv":
        mats = [tuple((torch.randn((r, k), generator=gen, device=device) * 0.02).to(bf) for r in (4096, 1024, 1024))
                for _ in range(layers)]
        inv = torch.ones(64, device=device)
        pos = torch.zeros(1, dtype=torch.int32, device=device)
        q = torch.empty((m, 4096), dtype=bf, device=device)
        kc = torch.empty((8, m, 128), dtype=bf, device=device)
        vc = torch.empty_like(kc)
        run = lambda w: ops.prefill_qkv_rope(a, w[0], w[1], w[2], inv, pos, q, kc, vc)
    else:
        mats = [(torch.randn((n, k), generator=gen, device=device) * 0.02).to(bf) for _ in range(layers)]
        res = torch.randn((m, n), generator=gen, device=device).to(bf)
        run = lambda w: ops.gemm_residual(a, w, res, res)
    for i in range(args.warmup * layers):
        run(mats[i % layers])
    torch.cuda.synchronize()
    launches = args.steps * layers
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(launches):
        run(mats[i % layers])
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1000.0 / launches
    flops = 2.0 * m * n * k
    tflops = flops / (us * 1e-6) / 1e12
    peak, kind = measured_peak("bf16_tflops")
    k_split = lib.cb_gemm_split_k(m, k, n // 2 if name == "gemm_gate_up" else n, 1 if name == "gemm_gate_up" else 0)
    lib.cb_set_gemm_workspace(None, 0, None, 0)
    print(json.dumps({"micro": name, "tokens": m, "k_split": k_split, "us_per_launch": round(us, 3),
                      "flop_per_launch": flops,
                      "achieved_tflops": round(tflops, 1), "peak_tflops": peak, "peak_kind": kind,
                      "frac": round(tflops / peak, 4), "weight_gbs": round(n * k * 2 / (us * 1e-6) / 1e9, 1),
                      "launches": launches}), flush=True)


def micro_prefill_attention(args, device):
    """Causal prefill attention of a --tokens chunk at the end of a --context
    cache (8 KV heads), back to back over the caches of 8 layers: TFLOP/s
    (QK^T and PV of the causal triangle) vs the measured dense bf16 peak."""

    from layer_streaming import _native, ops

    _native.check(_native.lib().cb_prepare(), "cb_prepare")
    bf = torch.bfloat16
    m, length = args.tokens, args.context
    gen = torch.Generator(device=device).manual_seed(6)
    caches = [tuple(torch.randn((8, length, 128), generator=gen, device=device).to(bf) for _ in range(2))
              for _ in range(8)]
    q = torch.randn((m, 32 * 128), generator=gen, device=device).to(bf)
    out = torch.empty_like(q)
    pos = torch.tensor([length - m], dtype=torch.int32, device=device)
    run = lambda c: ops.prefill_attention(q, c[0], c[1], pos, out)
    for i in range(args.warmup * 8):
        run(caches[i % 8])
    torch.cuda.synchronize()
    launches = args.steps * 8
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(launches):
        run(caches[i % 8])
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1000.0 / launches
    keys = sum(length - m + t + 1 for t in range(m))  # causal (query, key) pairs per head
    flops = 4.0 * 32 * keys * 128
    tflops = flops / (us * 1e-6) / 1e12
    peak, kind = measured_peak("bf16_tflops")
    print(json.dumps({"micro": "prefill_attention", "tokens": m, "context": length, "us_per_launch": round(us, 3),
                      "flop_per_launch": flops, "achieved_tflops": round(tflops, 1), "peak_tflops": peak,
                      "peak_kind": kind, "frac": round(tflops / peak, 4), "launches": launches}), flush=True)


def sweep(args, device):
    """Matrix-group projections (QKV + RoPE, O + residual, gate+up + SwiGLU,
    down + residual) at M rows (GEMV kernel for M = 1, tcgen05 GEMM above):
    HBM-resident over 8 rotating weight copies (> L2), and H2D-streamed from
    pinned host memory through two device slots (copy stream overlapped with
    the compute stream), as the reference's runtime streams its units."""

    from layer_streaming import _native, ops

    lib = _native.lib()
    _native.check(lib.cb_prepare(), "cb_prepare")
    # the executor's split-K registration for chunks of <= 128 tokens
    split_ws = torch.empty(48 << 18, dtype=torch.float32, device=device)
    split_tickets = torch.zeros(1024, dtype=torch.int32, device=device)
    _native.check(lib.cb_set_gemm_workspace(split_ws.data_ptr(), 48 << 20, split_tickets.data_ptr(), 1024),
                  "cb_set_gemm_workspace")
    bf = torch.bfloat16
    gen = torch.Generator(device=device).manual_seed(9)
    rnd = lambda *shape: (torch.randn(shape, generator=gen, device=device) * 0.02).to(bf)
    shapes = {"qkv": [(4096, 4096), (1024, 4096), (1024, 4096)], "o_proj": [(4096, 4096)],
              "gate_up": [(14336, 4096), (14336, 4096)], "down_proj": [(4096, 14336)]}
    inv = torch.ones(64, device=device)
    pos = torch.zeros(1, dtype=torch.int32, device=device)
    kc = torch.zeros((8, 600, 128), dtype=bf, device=device)
    vc = torch.zeros_like(kc)
    for name, mats in shapes.items():
        k_in = mats[0][1]
        x = (torch.randn((512, k_in), generator=gen, device=device)).to(bf)
        res = torch.randn((512, 4096), generator=gen, device=device).to(bf)
        q = torch.empty((512, 4096), dtype=bf, device=device)
        mlp = torch.empty((512, 14336), dtype=bf, device=device)

        def run(w, m, name=name, x=x, res=res, q=q, mlp=mlp):
            if name == "qkv":
                if m == 1:
                    ops.qkv_rope(x[0], None, 1e-5, w[0], w[1], w[2], inv, pos, 0, q[0], kc, vc)
                else:
                    ops.prefill_qkv_rope(x[:m], w[0], w[1], w[2], inv, pos, q[:m], kc, vc)
            elif name == "gate_up":
                if m == 1:
                    ops.gate_up_swiglu(x[0], None, 1e-5, w[0], w[1], mlp[0])
                else:
                    ops.gemm_swiglu(x[:m], w[0], w[1], mlp[:m])
            elif m == 1:
                ops.proj_residual(x[0], w[0], res[0], res[0])
            else:
                ops.gemm_residual(x[:m], w[0], res[:m], res[:m])

        copies = [[rnd(*s) for s in mats] for _ in range(8)]
        host = [torch.empty(s, dtype=bf).pin_memory() for s in mats]
        for h, d in zip(host, copies[0]):
            h.copy_(d.cpu())
        slots = [[torch.empty(s, dtype=bf, device=device) for s in mats] for _ in range(2)]
        nbytes = sum(a * b * 2 for a, b in mats)
        flop_per_row = 2 * sum(a * b for a, b in mats)
        copy_stream = torch.cuda.Stream(device)
        for m in (1, 6, 64, 512):
            for i in range(16):
                run(copies[i % 8], m)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(32):
                run(copies[i % 8], m)
            e1.record()
            torch.cuda.synchronize()
            resident_us = e0.elapsed_time(e1) * 1000.0 / 32
            # streamed: unit i is copied into slot i % 2 while unit i - 1 computes
            ready = [torch.cuda.Event() for _ in range(2)]
            free = [torch.cuda.Event() for _ in range(2)]
            compute = torch.cuda.current_stream(device)
            for f in free:
                f.record(compute)
            torch.cuda.synchronize()
            started = time.perf_counter()
            n = 16
            for i in range(n):
                sl = i % 2
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_event(free[sl])
                    for h, d in zip(host, slots[sl]):
                        ops.memcpy_h2d_async(d, h)
                    ready[sl].record(copy_stream)
                compute.wait_event(ready[sl])
                run(slots[sl], m)
                free[sl].record(compute)
            torch.cuda.synchronize()
            streamed_us = (time.perf_counter() - started) * 1e6 / n
            n_out = sum(a for a, _ in mats)
            k_split = 1 if m == 1 else lib.cb_gemm_split_k(m, k_in, mats[0][0] if name == "gate_up" else n_out,
                                                          1 if name == "gate_up" else 0)
            print(json.dumps({
                "sweep": name, "M": m, "weight_bytes": nbytes, "k_split": k_split,
                "resident_us": round(resident_us, 2),
                "resident_gbs": round(nbytes / (resident_us * 1e-6) / 1e9, 1),
                "resident_tflops": round(flop_per_row * m / (resident_us * 1e-6) / 1e12, 1),
                "streamed_us": round(streamed_us, 2),
                "streamed_h2d_gbs": round(nbytes / (streamed_us * 1e-6) / 1e9, 2),
            }), flush=True)
        del copies, host, slots
    lib.cb_set_gemm_workspace(None, 0, None, 0)


def micro(args, device):
    """One kernel, back to back over rotating weight copies (> L2 in total)."""

    from layer_streaming import _native, ops
    from layer_streaming.llama31 import attention_split

    _native.check(_native.lib().cb_prepare(), "cb_prepare")
    bf = torch.bfloat16
    name = args.micro
    if name in GEMM_SHAPES:
        return micro_gemm(args, device)
    if name == "prefill_attention":
        return micro_prefill_attention(args, device)
    copies = {"lm_head": 2, "gate_up": 2, "lm_head_i8": 3, "gate_up_i8": 4}.get(name, 6)

    def rnd(*shape, std=0.02):
        return (torch.randn(shape, device=device) * std).to(bf)

    x = rnd(4096, std=1.0)
    norm = torch.ones(4096, dtype=bf, device=device)
    if name == "qkv":
        mats = [(rnd(4096, 4096), rnd(1024, 4096), rnd(1024, 4096)) for _ in range(copies)]
        inv = torch.ones(64, device=device)
        pos = torch.zeros(1, dtype=torch.int32, device=device)
        q = torch.empty(4096, dtype=bf, device=device)
        kc = torch.empty((8, 64, 128), dtype=bf, device=device)
        vc = torch.empty_like(kc)
        run = lambda m: ops.qkv_rope(x, norm, 1e-5, m[0], m[1], m[2], inv, pos, 0, q, kc, vc)
    elif name in ("o_proj", "down_proj"):
        k = 4096 if name == "o_proj" else 14336
        xin = rnd(k, std=1.0)
        mats = [rnd(4096, k) for _ in range(copies)]
        res = rnd(4096, std=1.0)
        run = lambda m: ops.proj_residual(xin, m, res, res)
    elif name == "gate_up":
        mats = [(rnd(14336, 4096), rnd(14336, 4096)) for _ in range(copies)]
        out = torch.empty(14336, dtype=bf, device=device)
        run = lambda m: ops.gate_up_swiglu(x, norm, 1e-5, m[0], m[1], out)
    elif name.endswith("_i8"):
        rows, k = {"gate_up_i8": (28672, 4096), "down_proj_i8": (4096, 14336), "lm_head_i8": (128256, 4096)}[name]

        def quantized():
            w = rnd(rows, k)
            q = torch.empty((rows, k), dtype=torch.int8, device=device)
            sc = torch.empty(rows, dtype=torch.float32, device=device)
            ops.quantize_rows_i8(w, q, sc)
            return q, sc

        mats = [quantized() for _ in range(copies)]
        if name == "gate_up_i8":
            out = torch.empty(14336, dtype=bf, device=device)
            run = lambda m: ops.gate_up_swiglu_i8(x, norm, 1e-5, m[0][:14336], m[1][:14336], m[0][14336:],
                                                  m[1][14336:], out)
        elif name == "down_proj_i8":
            xin = rnd(14336, std=1.0)
            res = rnd(4096, std=1.0)
            run = lambda m: ops.proj_residual_i8(xin, m[0], m[1], res, res)
        else:
            values = torch.empty(10, device=device)
            indices = torch.empty(10, dtype=torch.int64, device=device)
            ws = torch.empty(ops.lm_head_workspace_bytes(10), dtype=torch.uint8, device=device)
            ticket = torch.zeros(1, dtype=torch.int32, device=device)
            run = lambda m: ops.lm_head_topk_i8(x, norm, 1e-5, m[0], m[1], 10, None, values, indices, ws, ticket)
    elif name == "lm_head":
        mats = [rnd(128256, 4096) for _ in range(copies)]
        values = torch.empty(10, device=device)
        indices = torch.empty(10, dtype=torch.int64, device=device)
        ws = torch.empty(ops.lm_head_workspace_bytes(10), dtype=torch.uint8, device=device)
        ticket = torch.zeros(1, dtype=torch.int32, device=device)
        run = lambda m: ops.lm_head_topk(x, norm, 1e-5, m, 0, 10, None, values, indices, ws, ticket)
    else:  # attention, one decode token at args.context positions
        cap = args.context + 64
        mats = [(rnd(8, cap, 128, std=1.0), rnd(8, cap, 128, std=1.0)) for _ in range(64)]
        q = rnd(4096, std=1.0)
        pos = torch.tensor([args.context - 1], dtype=torch.int32, device=device)
        splits, chunk = attention_split(1, args.context, torch.cuda.get_device_properties(device).multi_processor_count)
        ws = torch.empty(ops.attention_workspace_bytes(1, splits), dtype=torch.uint8, device=device)
        tickets = torch.zeros(8, dtype=torch.int32, device=device)
        out = torch.empty(4096, dtype=bf, device=device)
        run = lambda m: ops.attention(q, m[0], m[1], pos, splits, chunk, out, ws, tickets)
    for i in range(args.warmup * len(mats)):
        run(mats[i % len(mats)])
    torch.cuda.synchronize()
    launches = args.steps * len(mats)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(launches):
        run(mats[i % len(mats)])
    end.record()
    torch.cuda.synchronize()
    us = start.elapsed_time(end) * 1000.0 / launches
    nbytes = MICRO_BYTES[name] if name != "attention" else 8 * args.context * 128 * 2 * 2
    peak, kind = measured_peak()
    gbs = nbytes / (us * 1e-6) / 1e9
    print(json.dumps({"micro": name, "us_per_launch": round(us, 3), "bytes_per_launch": nbytes,
                      "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "peak_kind": kind,
                      "frac": round(gbs / peak, 4), "launches": launches, "copies": len(mats)}), flush=True)


def micro_exchange(args, world, rank, local, device):
    """--micro exchange (any N, under torchrun for N > 1): a rank's o_proj and
    down_proj shards (K = 4096/N and 14336/N columns) as the local projection
    (cb_proj_residual) and as the fused projection + peer-memory all-reduce
    (cb_proj_allreduce_residual), back to back over rotating weight copies;
    CUDA events, max over ranks. The difference is the exchange's cost."""

    import ctypes
    import datetime

    import torch.distributed as dist

    from layer_streaming import _native, ops
    from layer_streaming.tensor_parallel import SLOTS, ExchangeBuffers, _Group

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    lib = _native.lib()
    _native.check(lib.cb_prepare(), "cb_prepare")
    group = _Group.of(None)
    buffers = ExchangeBuffers(group, device)
    epoch = torch.zeros(1, dtype=torch.int32, device=device)
    bf = torch.bfloat16
    results = {}
    stream = _native.stream_ptr(device)
    for name, full_k in (("o_proj", 4096), ("down_proj", 14336)):
        k = full_k // world
        copies = [(torch.randn((4096, k), device=device) * 0.02).to(bf) for _ in range(8)]
        xin = torch.randn(k, device=device).to(bf)
        res = torch.randn(4096, device=device).to(bf)
        out = torch.empty_like(res)

        def local_proj(w):
            ops.proj_residual(xin, w, res, out)

        slot = [0]

        def fused(w):
            s = slot[0]
            _native.check(lib.cb_proj_allreduce_residual(
                xin.data_ptr(), k, w.data_ptr(), 4096, res.data_ptr(), out.data_ptr(), buffers.pointers,
                group.rank, group.world, s, SLOTS, epoch.data_ptr(), stream), "cb_proj_allreduce_residual")
            slot[0] = s + 1
            if slot[0] == SLOTS:  # one "step": advance the epoch as the decoder does
                slot[0] = 0
                ops.position_advance(epoch, 1)

        for label, fn in (("local", local_proj), ("exchange", fused)):
            for i in range(args.warmup * len(copies)):
                fn(copies[i % len(copies)])
            torch.cuda.synchronize()
            group.barrier()
            launches = args.steps * SLOTS
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(launches):
                fn(copies[i % len(copies)])
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / launches], device=device)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            results[name + "_" + label + "_us"] = round(float(t), 3)
        results[name + "_exchange_cost_us"] = round(results[name + "_exchange_us"] - results[name + "_local_us"], 3)
        results[name + "_weight_bytes_per_rank"] = 4096 * k * 2
        results[name + "_nvlink_bytes_per_rank"] = 2 * 4096 * 8 * (world - 1)  # tagged fp32 partials pushed
        del copies
    buffers.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"micro": "exchange", "n_gpus": world, "launches_per_case": args.steps * SLOTS,
                          **results}), flush=True)


def reference_arm(args, rank):
    """--impl reference: the reference's CPU algorithm on this host's cores."""

    if rank != 0:
        return None
    from layer_streaming.plan import build_llama31_8b_plan
    from oracle.seeded import fill_model

    plan = build_llama31_8b_plan("matrix_group")
    weights = {k: torch.empty(s.shape, dtype=torch.bfloat16) for k, s in plan.tensors.items()}
    fill_model(sorted(weights), weights.__getitem__, seed=0)
    baseline = cpu_baseline(weights, args.context, args.cpu_seconds)
    value = baseline["value"]
    return {
        "metric": METRIC, "value": value, "unit": "ms/token", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": value,
        "higher_is_better": False, "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded random-init weights, random token ids)",
        "config": bench_config(args),
        "impl": "reference",
        "cpu_baseline": baseline,
        "e2e": {"value": value, "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def tp_streamed(args, world, rank, device, barrier, steps=3):
    """The reference's H2D-streamed mode under tensor parallelism: every rank
    streams only its layer shards (13.96 GB / N per token) from its own pinned
    shard arena through two device slots; a short prompt, then timed decode
    steps (max over ranks)."""

    import torch.distributed as dist

    from layer_streaming.tensor_parallel import TensorParallelDecoder, TensorParallelWeights

    weights = TensorParallelWeights.seeded(world, rank, device, seed=0, stream_layers=True)
    decoder = TensorParallelDecoder(Config(), weights, top_k=10, max_length=256, profile=True)
    with torch.inference_mode():
        token = decoder(random_ids(64, seed=1).to(device)).topk_indices[..., 0].reshape(1, 1)
        token = decoder(token).topk_indices[..., 0].reshape(1, 1)  # warm-up
        torch.cuda.synchronize()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            token = decoder(token).topk_indices[..., 0].reshape(1, 1)
        end.record()
        torch.cuda.synchronize()
        barrier()
    prof = decoder.last_stream
    gbps = prof["h2d_bytes"] / 1e9 / (prof["h2d_event_sum_ms"] / 1000.0)
    t = torch.tensor([start.elapsed_time(end) / steps, -gbps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    decoder.close()
    return {"ms_per_token": round(float(t[0]), 2), "steps": steps,
            "h2d_bytes_per_token_per_rank": int(prof["h2d_bytes"]),
            "h2d_gbps_per_rank_min": round(-float(t[1]), 2),
            "note": "stream_layers shards: each rank streams its own 1/N of the layer weights (PCIe-bound)"}


def tensor_parallel(args, world, rank, local, device):
    """N>1: one request decoded by all ranks (tensor parallelism over heads,
    FFN rows and vocabulary), strong scaling of the same workload."""

    import datetime

    import torch.distributed as dist

    from layer_streaming import ops
    from layer_streaming.tensor_parallel import TensorParallelDecoder, TensorParallelWeights

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    weights = TensorParallelWeights.seeded(world, rank, device, seed=0)
    extra = args.warmup + args.steps * 2 + 72
    decoder = TensorParallelDecoder(Config(), weights, top_k=10, max_length=args.context + extra,
                                    exchange=args.exchange)
    ids = random_ids(args.context, seed=1).to(device)
    torch.cuda.synchronize(device)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.inference_mode():
        p0.record()
        for start in range(0, args.context, 512):
            state = decoder(ids[:, start:start + 512])
        p1.record()
    torch.cuda.synchronize(device)
    decoder.check_errors()
    t = torch.tensor([p0.elapsed_time(p1)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    prefill_ms = float(t.item())
    token = state.topk_indices[..., 0].reshape(1, 1)

    def barrier():
        dist.barrier(device_ids=[local])

    clocks = ClockSampler(local)
    clocks.start()
    with torch.inference_mode():
        for _ in range(args.warmup):
            token = decoder(token).topk_indices[..., 0].reshape(1, 1)
        torch.cuda.synchronize()
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            token = decoder(token).topk_indices[..., 0].reshape(1, 1)
        end.record()
        torch.cuda.synchronize()
        barrier()
    clock_info = clocks.stop()
    decoder.check_errors()
    t = torch.tensor([start.elapsed_time(end) / args.steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # end to end: the token id from pinned host memory, the top-k read back
    ids_host = torch.empty((1, 1), dtype=torch.int64).pin_memory()
    ids_host[0, 0] = int(token.reshape(-1)[0])
    with torch.inference_mode():
        torch.cuda.synchronize()
        barrier()
        started = time.perf_counter()
        values = indices = None
        for _ in range(args.steps):
            state = decoder(ids_host)
            if values is None:
                values = torch.empty(state.topk_values.shape, dtype=state.topk_values.dtype).pin_memory()
                indices = torch.empty(state.topk_indices.shape, dtype=state.topk_indices.dtype).pin_memory()
            values.copy_(state.topk_values, non_blocking=True)  # both results, one wait per step
            indices.copy_(state.topk_indices, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            ids_host[0, 0] = int(indices.reshape(-1)[0])
        e2e_ms = (time.perf_counter() - started) * 1000.0 / args.steps
    t = torch.tensor([e2e_ms], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e = {"value": round(float(t.item()), 4), "unit": "ms/token", "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": values.numel() * 4 + indices.numel() * 8}

    # dominant kernel on this rank: the gate+up GEMV over its FFN rows
    x, out = decoder._x[0], decoder._mlp[0]
    mats = [(weights["model.layers.{}.mlp.gate_proj.weight".format(i)],
             weights["model.layers.{}.mlp.up_proj.weight".format(i)],
             weights["model.layers.{}.post_attention_layernorm.weight".format(i)]) for i in range(32)]
    for wg, wu, norm in mats:
        ops.gate_up_swiglu(x, norm, 1e-5, wg, wu, out)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(4):
        for wg, wu, norm in mats:
            ops.gate_up_swiglu(x, norm, 1e-5, wg, wu, out)
    end.record(stream)
    end.synchronize()
    gate_up_ms = start.elapsed_time(end) / (4 * len(mats))
    gate_up_bytes = GATE_UP_BYTES // world
    streamed = None if args.no_streamed else tp_streamed(args, world, rank, device, barrier)
    peak, peak_kind = measured_peak()
    achieved = gate_up_bytes / (gate_up_ms / 1000.0) / 1e9
    context = decoder.kv_cache.length - args.steps - 1
    rank_bytes = (LAYER_BYTES + HEAD_BYTES) // world + NORM_BYTES + (131_072 * (context + 1)) // world
    rank_gbs = rank_bytes / (ms / 1000.0) / 1e9
    line = {
        "metric": METRIC,
        "value": round(ms, 4),
        "unit": "ms/token",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, random token ids)",
        "config": bench_config(args),
        "weights": "hbm-resident shards (heads, FFN rows, vocabulary), {:.1f} GB per rank; {} exchange".format(
            weights.nbytes / 1e9, args.exchange),
        "tokens_per_s": round(1000.0 / ms, 2),
        "e2e": e2e,
        "roofline": {
            "bound": "hbm", "kernel": "gemv gate_up_swiglu shard (K=4096, N=2x{})".format(14336 // world),
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": GATE_UP_TRAFFIC // world,
            "traffic_note": "single-GPU capture scaled by the rows a rank streams",
            "ms_per_launch": round(gate_up_ms, 5), "bytes_per_launch": gate_up_bytes,
        },
        "step_roofline": {
            "achieved_per_rank": round(rank_gbs, 1), "peak": peak, "unit": "GB/s",
            "frac": round(rank_gbs / peak, 4), "bytes_per_token_per_rank": rank_bytes,
        },
        "cpu_baseline": None,
        "streamed_mode": streamed,
        "prefill": {"tokens": args.context, "chunk": 512, "ms": round(prefill_ms, 2),
                    "tokens_per_s": round(args.context / (prefill_ms / 1000.0), 1)},
        "gpu_launches": (1 + 32 * 5 + 1 + 2) * args.steps if args.exchange == "peer" else None,
        "clocks": clock_info,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    decoder.close()
    barrier()
    dist.destroy_process_group()


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = reference_arm(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.micro == "exchange":
        micro_exchange(args, world, rank, local, device)
        return
    if args.micro:
        micro(args, device)
        return
    if args.sweep:
        sweep(args, device)
        return
    if world > 1:
        tensor_parallel(args, world, rank, local, device)
        return

    def barrier():
        pass

    extra = args.warmup + args.steps * 2 + 72
    plan, store, resident, runtime, executor = build_engine(device, args.context, extra)
    token, prefill_ms = prefill(executor, runtime, device, args.context, chunk=args.prefill_chunk)
    if args.trace:
        print(json.dumps(trace_decode(executor, runtime, token, args.steps, args.warmup)), flush=True)
        return
    if args.profile_range:
        with torch.inference_mode():
            for _ in range(args.warmup):
                token = step(executor, runtime, token).topk_indices[..., 0]
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()
            for _ in range(args.steps):
                token = step(executor, runtime, token).topk_indices[..., 0]
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps({"profile_range": args.steps, "context": args.context}), flush=True)
        return
    clocks = ClockSampler(local)
    clocks.start()
    ms, token = time_decode(executor, runtime, token, args.steps, args.warmup, barrier)
    clock_info = clocks.stop()
    executor.check_errors()
    e2e = time_e2e(executor, runtime, token, args.steps)
    gate_up_ms = time_gate_up(executor, runtime, plan)
    streamed = None if args.no_streamed else time_streamed(plan, store, resident, executor, device, token)
    streamed_i8 = None
    if not args.no_streamed and not args.no_int8:
        streamed_i8 = time_streamed(plan, store, resident, executor, device, token, transfer="int8")
    int8 = None if args.no_int8 else time_int8(resident, runtime, device, args.context, args.steps, args.warmup)
    peak, peak_kind = measured_peak()
    context = executor.kv_cache.length - args.steps - 1  # mean cached length over the timed steps
    achieved = GATE_UP_BYTES / (gate_up_ms / 1000.0) / 1e9
    step_gbs = step_bytes(context) / (ms / 1000.0) / 1e9
    baseline = None
    if rank == 0 and not args.no_cpu_baseline:
        baseline = cpu_baseline({key: store.tensor(key) for key in store.required_keys()}, args.context,
                                args.cpu_seconds)
    kernels_per_step = 1 + 32 * 5 + 1 + 1  # embedding, 5 per layer, position advance, LM head
    line = {
        "metric": METRIC,
        "value": round(ms, 4),
        "unit": "ms/token",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, random token ids)",
        "config": bench_config(args),
        "weights": "hbm-resident (every transfer unit in HBM), one CUDA graph per decode step",
        "tokens_per_s": round(1000.0 / ms, 2),
        "e2e": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in e2e.items()},
        "roofline": {
            "bound": "hbm", "kernel": "gemv gate_up_swiglu (K=4096, N=2x14336)",
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": GATE_UP_TRAFFIC,
            "ms_per_launch": round(gate_up_ms, 5), "bytes_per_launch": GATE_UP_BYTES,
        },
        "step_roofline": {
            "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(step_gbs / peak, 4),
            "frac_of_8tbs": round(step_gbs / 8000.0, 4), "bytes_per_token": step_bytes(context),
        },
        "cpu_baseline": baseline,
        "streamed_mode": streamed,
        "streamed_int8_mode": streamed_i8,
        "int8_mode": int8,
        "prefill": {
            "tokens": args.context, "chunk": args.prefill_chunk, "ms": round(prefill_ms, 2),
            "tokens_per_s": round(args.context / (prefill_ms / 1000.0), 1),
            "note": "first (cold) prefill through the API: tcgen05 GEMMs + split-KV attention per chunk",
        },
        "gpu_launches": kernels_per_step * args.steps,
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
