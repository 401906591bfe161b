"""Decode throughput of the B200 resident Qwen2 FP32 path.

Workload: 24-layer Qwen2.5-0.5B-architecture FP32 model,
vocab 151936 (tied LM head), random-init weights N(0, 0.02) (seed 1), a
32-token random prompt (seed 1 + rank), 128 greedy tokens per step at batch 1.
One step = one resident launch that decodes the 128 tokens after the prompt
(positions 31..158). The prompt is ingested before timing.

Reported (one JSON line, rank 0):
  value       tokens/s over all ranks, device-timed (CUDA events on the
              runtime's default queue), inputs resident in HBM
  e2e         the same through lrq_generate (host hidden in, host tokens out)
  roofline    algorithmic weight + KV bytes per launch / launch time vs the
              measured HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline  the CPU oracle (reference algorithm restated) on the host
              cores, bounded sample
  long_context  BASELINE config 3 on the same model: KV cache rows 0..4095
              N(0, 1), 256 decode tokens at positions 4096..4351, one
              resident launch, device-timed, with its HBM roofline
  prefill     BASELINE config 5 on the same model: a 512-token prompt
              (seed 3) through the 3xTF32 tensor-core prefill (511 rows),
              device-timed, against the 3xTF32 tensor roof; then 256 greedy
              decode tokens after it
  batched     BASELINE config 4: 32 streams at context 1024 (seed 2),
              32/N per GPU decoded as one batch per GPU, 128 tokens each;
              aggregate tokens/s over all ranks (max-over-ranks time)
  scheduler_floor  the control-only resident kernel (the reference's
              scheduler-profile workload: Programs, stages and grid barriers
              with only the state-changing tasks) on the same 128-token run:
              microseconds per token and per grid barrier
Weights (2 GB) exceed L2 (126 MB), so no flush is needed between steps.

--profile-case prefill|batch|long runs one of the profiler workloads instead (the
measured launches inside cuProfilerStart/Stop, for
`ncu --profile-from-start off`), and prints no bench line.

--impl reference times the reference's CPU implementation of the path (the
oracle port; the reference's own code is HIP for AMD gfx1101 and cannot run
here) on the same workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "light-rocm-runtime_b200"))

LAYERS, VOCAB, PROMPT, NEW_TOKENS = 24, 151936, 32, 128
PREFILL_PROMPT, PREFILL_DECODE = 512, 256              # config 5
STREAMS, STREAM_CONTEXT, STREAM_TOKENS = 32, 1024, 128  # config 4
LONG_CONTEXT, LONG_TOKENS = 4096, 256                  # config 3
BATCH_CAPACITY = STREAM_CONTEXT + STREAM_TOKENS + 8    # KV positions per batched stream
CAPACITY = LONG_CONTEXT + LONG_TOKENS + 8              # model RoPE rows / KV positions
SEED = 1
KV_BYTES_PER_LAYER_POSITION = 128 * 4 * 2  # K and V rows of one position
METRIC = "decode tokens/s, Qwen2.5-0.5B-arch FP32, batch 1 (config 2: 24 layers, 128 new tokens)"


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--cpu-seconds", type=float, default=12.0,
                        help="CPU baseline sample length")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--new-tokens", type=int, default=NEW_TOKENS,
                        help="tokens per step (smaller only for profiler captures)")
    parser.add_argument("--no-extra", action="store_true",
                        help="skip the config-5 prefill and config-4 batched lines")
    parser.add_argument("--profile-case", choices=["prefill", "batch", "long"],
                        help="run a profiler workload instead of the bench")
    parser.add_argument("--layers", type=int, default=LAYERS, help="profile cases only")
    parser.add_argument("--prompt", type=int, default=PREFILL_PROMPT, help="profile cases only")
    parser.add_argument("--streams", type=int, default=STREAMS, help="profile cases only")
    parser.add_argument("--context", type=int, default=STREAM_CONTEXT,
                        help="profile cases only")
    parser.add_argument("--case-steps", type=int, default=2, help="profile cases only")
    parser.add_argument("--vocab", type=int, default=VOCAB, help="profile cases only")
    return parser.parse_args()


def algorithmic_bytes_per_launch(weight_bytes: int, first_position: int, tokens: int) -> int:
    """Weights once per token plus, per layer, the KV rows read (p+1) and the
    row written at each position p."""
    total = 0
    for p in range(first_position, first_position + tokens):
        total += weight_bytes + LAYERS * KV_BYTES_PER_LAYER_POSITION * (p + 2)
    return total


def measured_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s from MEASURED_PEAKS.json (burst figure: the prefill
    is timed alone), else the pool's fallback measurement."""
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def profiled_traffic_per_token():
    """DRAM bytes per decode token of the compiled kernel from the committed
    ncu summary (profiles/), or None when no capture has been summarised."""
    path = REPO / "profiles" / "qwen_compiled_kernel_dram.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_token:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.process = None

    def __enter__(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.process = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.process is not None:
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()

    def summary(self):
        self.file.flush()
        rows = [line.split(",") for line in Path(self.file.name).read_text().splitlines()
                if line.strip()]
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].strip() else None,
                "reasons": reasons, "samples": len(rows)}


def max_over_ranks(values, dist):
    """Element-wise maximum of per-rank timings (the job takes as long as its
    slowest rank). The tensor lives where the process group's backend wants
    it: on the rank's GPU for NCCL, on the host for gloo."""
    import torch
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def rank_seeds(rank: int):
    """(weight seed, prompt seed) of a replica: every rank holds the same
    model and decodes its own prompt, so the replicas are independent streams."""
    return SEED, SEED + rank


def stream_slice(rank: int, world: int) -> list[int]:
    """Config-4 streams decoded by `rank` of `world`: 32 / world consecutive
    streams starting at rank * 32 / world (world divides 32)."""
    if world <= 0 or STREAMS % world != 0 or not 0 <= rank < world:
        raise ValueError(f"{world} ranks cannot split {STREAMS} streams evenly")
    per_rank = STREAMS // world
    return [rank * per_rank + local for local in range(per_rank)]


def make_weights(rank: int):
    from lrrt_b200 import synthetic as S
    weight_seed, prompt_seed = rank_seeds(rank)
    weights, tail = S.model(weight_seed, LAYERS, VOCAB)
    prompt = S.prompt(prompt_seed, PROMPT, VOCAB)
    return weights, tail, prompt


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def oracle_decoder(weights, tail, prompt, threads: int):
    """The CPU oracle with the bench's prompt ingested (positions 0..30), and
    a function decoding `count` greedy tokens from position 31 (the GPU arm's
    workload: positions 31..158 for 128 tokens)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O
    O.set_threads(threads)
    model = O.OracleModel(weights, tail, PROMPT + NEW_TOKENS, 32, workers=148,
                          max_tokens=NEW_TOKENS, keep_logits=False)
    for position, token in enumerate(prompt[:-1]):
        model.decode(model.embedding(int(token)), position, 1)
    start_hidden = model.embedding(int(prompt[-1]))

    def decode(count: int) -> None:
        model.decode(start_hidden, PROMPT - 1, count)

    return decode


def cpu_tokens_per_second(decode, seconds: float):
    """Tokens/s of the oracle on the GPU arm's workload (positions 31..),
    repeating decodes of up to 128 tokens for about `seconds`."""
    tokens, start = 0, time.perf_counter()
    count = 4
    while True:
        decode(count)
        tokens += count
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
        count = min(NEW_TOKENS, count * 2)
    return tokens / elapsed, tokens, elapsed


def reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    weights, tail, prompt = make_weights(0)
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle as O
    threads = O.max_threads()
    decode = oracle_decoder(weights, tail, prompt, threads)
    # Each step decodes the GPU arm's workload from position 31, as many of
    # its 128 tokens as keep the whole run to about four minutes.
    probe = time.perf_counter()
    decode(4)
    rate = 4 / (time.perf_counter() - probe)
    per_step_tokens = int(max(4, min(NEW_TOKENS, 240.0 * rate / max(1, args.steps + args.warmup))))
    for _ in range(args.warmup):
        decode(per_step_tokens)
    start = time.perf_counter()
    for _ in range(args.steps):
        decode(per_step_tokens)
    elapsed = time.perf_counter() - start
    value = per_step_tokens * args.steps / elapsed
    sample = (f"greedy decode of the GPU arm's workload (prompt ingested, positions "
              f"31..{31 + per_step_tokens - 1}, {per_step_tokens} of its 128 tokens per step) "
              f"on {threads} host threads of {cpu_model()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * elapsed / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2: 24-layer Qwen2.5-0.5B-arch FP32 greedy decode, "
                               "batch 1", "global_batch": 1, "seq_len": PROMPT + NEW_TOKENS},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference implementation of this path is HIP for AMD gfx1101; its "
                "CPU restatement (oracle/) is timed instead",
    }
    print(json.dumps(line), flush=True)


def prefill_flops(rows: int) -> int:
    """Algorithmic FLOPs of one prefill pass over `rows` prompt rows: the
    four projections (2 * rows * weight elements) plus causal attention
    (S = Q.K^T and P.V: 2 * 2 * 64 FLOPs per (row, head, key), keys 1..row+1)."""
    h, kv, i = 896, 128, 4864
    per_layer_weights = h * (h + 2 * kv) + h * h + 2 * i * h + i * h
    attention = 4 * 64 * 14 * rows * (rows + 1) // 2
    return LAYERS * (2 * rows * per_layer_weights + attention)


def extra_configs(model, Q, S, rank: int, world: int, dist, warmup: int):
    """Config 3 (long context), config 5 (prefill) and config 4 (batched
    streams) on the bench's model."""
    timer = Q.EventTimer(model.device)
    # Config 3: KV rows 0..4095 ~ N(0, 1), then 256 tokens in one launch.
    for layer, (keys, values) in enumerate(S.kv_prefill(SEED, LAYERS, LONG_CONTEXT)):
        model.set_kv(layer, 0, keys, values)
    model.set_hidden(S.hidden(SEED))
    long_request = model.request(LONG_CONTEXT, LONG_TOKENS)
    for _ in range(max(1, min(warmup, 2))):
        model.launch(long_request)
    model.synchronize()
    timer.record_start()
    model.launch(long_request)
    timer.record_end()
    model.synchronize()
    long_s = timer.elapsed_ns() / 1e9
    state = model.read_state()
    if state.status != 2 or state.generated_tokens != LONG_TOKENS:
        raise RuntimeError(f"long-context decode failed: status {state.status}")
    long_bytes = algorithmic_bytes_per_launch(int(model.info.weight_bytes_per_token),
                                              LONG_CONTEXT, LONG_TOKENS)
    hbm_peak, _ = measured_peaks()
    model.enable_prefill(1024)
    # Config 5: seed-3 prompt of 512 tokens, 3xTF32 prefill of rows 0..510.
    prompt5 = [int(t) for t in S.prompt(3, PREFILL_PROMPT, VOCAB)]
    for _ in range(max(1, warmup)):
        model.prefill(prompt5, Q.PREFILL_TF32X3)
    times = []
    for _ in range(3):
        model.synchronize()
        timer.record_start()
        model.prefill(prompt5, Q.PREFILL_TF32X3)
        timer.record_end()
        model.synchronize()
        times.append(timer.elapsed_ns() / 1e9)
    prefill_s = min(times)
    timer.record_start()
    state, _ = model.decode(PREFILL_PROMPT - 1, PREFILL_DECODE)
    timer.record_end()
    decode_s = timer.elapsed_ns() / 1e9
    if state.status != 2 or state.generated_tokens != PREFILL_DECODE:
        raise RuntimeError(f"decode after prefill failed: status {state.status}")
    peak_bf16, _ = measured_tensor_peak()
    roof = peak_bf16 / 2.0 / 3.0  # TF32 runs at half the bf16 rate; 3 products per FP32 product
    flops = prefill_flops(PREFILL_PROMPT - 1)
    achieved = flops / prefill_s / 1e12
    # Config 4: streams [rank * per_rank, ...) of 32, each a 1025-token prompt
    # (context 1024), one batch per GPU, 128 greedy tokens per stream.
    mine = stream_slice(rank, world)
    per_rank = len(mine)
    all_prompts = S.prompt(2, STREAMS * (STREAM_CONTEXT + 1), VOCAB).reshape(STREAMS, -1)
    with Q.Batch(model, per_rank, BATCH_CAPACITY, STREAM_TOKENS) as batch:
        for local, stream in enumerate(mine):
            batch.prefill(local, [int(t) for t in all_prompts[stream]])
        batch.decode(4)  # graph capture and warm-up
        model.synchronize()
        timer.record_start()
        tokens, _ = batch.decode(STREAM_TOKENS - 4)
        timer.record_end()
        model.synchronize()
        batch_s = timer.elapsed_ns() / 1e9
    steps = STREAM_TOKENS - 4
    if world > 1:
        long_s, prefill_s, decode_s, batch_s = max_over_ranks(
            [long_s, prefill_s, decode_s, batch_s], dist)
    return {
        "long_context": {
            "workload": "config3: KV cache rows 0..4095 N(0,1), 256 greedy tokens at positions "
                        "4096..4351 in one resident launch, batch 1",
            "value": world * LONG_TOKENS / long_s, "unit": "tokens/s",
            "ms_per_token": 1000.0 * long_s / LONG_TOKENS,
            "roofline": {"bound": "hbm", "achieved": long_bytes / long_s / 1e9,
                         "peak": hbm_peak, "unit": "GB/s",
                         "frac": long_bytes / long_s / 1e9 / hbm_peak,
                         "algorithmic_bytes_per_launch": long_bytes},
        },
        "prefill": {
            "workload": "config5: 512-token prompt (seed 3), prefill of rows 0..510 through "
                        "24 layers, 3xTF32 tcgen05 GEMMs + causal attention",
            "ms": 1000.0 * prefill_s, "rows": PREFILL_PROMPT - 1,
            "algorithmic_flops": flops, "achieved_tflops": achieved,
            "roof_tflops": roof, "frac": achieved / roof,
            "roof": "3xTF32 roof = measured bf16 dense peak / 2 (TF32) / 3",
            "decode_after": {"tokens": PREFILL_DECODE, "positions": "511..766",
                             "tokens_per_s": PREFILL_DECODE / decode_s},
        },
        "batched": {
            "workload": f"config4: {STREAMS} streams at context {STREAM_CONTEXT} (seed 2), "
                        f"{per_rank} per GPU decoded as one batch (3xTF32 GEMMs, one CUDA "
                        f"graph per step), {steps} timed greedy steps",
            "value": world * per_rank * steps / batch_s, "unit": "tokens/s",
            "streams_per_gpu": per_rank, "ms_per_step": 1000.0 * batch_s / steps,
            "n_gpus": world,
        },
    }


def our_arm(args, rank: int, world: int, local_rank: int):
    from lrrt_b200 import qwen as Q

    weights, tail, prompt = make_weights(rank)
    config = Q.ModelConfig(layer_count=LAYERS, vocab_size=VOCAB, cache_capacity=CAPACITY,
                           max_tokens_per_run=max(NEW_TOKENS, PREFILL_DECODE))
    model = Q.Model(config, device_index=local_rank)
    for i, w in enumerate(weights):
        model.set_layer(i, w)
    model.set_tail(tail["final_norm"], tail["lm_head"])
    model.ingest_prompt([int(t) for t in prompt])
    start_position = PROMPT - 1
    request = model.request(start_position, NEW_TOKENS)

    def check(state):
        if state.status != 2 or state.generated_tokens != NEW_TOKENS:
            raise RuntimeError(f"decode run failed: status {state.status} error "
                               f"{state.error_code}")

    for _ in range(args.warmup):
        model.launch(request)
    model.synchronize()
    check(model.read_state())
    assert model.read_state().fused_path == 1

    dist = None
    if world > 1:
        import torch.distributed as dist_module
        dist = dist_module
        dist.barrier()
    timer = Q.EventTimer(model.device)
    per_launch = []
    launch_timer = Q.EventTimer(model.device)
    with ClockSampler(local_rank) as clocks:
        model.synchronize()
        timer.record_start()
        for _ in range(args.steps):
            model.launch(request)
        timer.record_end()
        model.synchronize()
        total_ns = timer.elapsed_ns()
        # Per-launch durations (separately bracketed) for the roofline.
        for _ in range(min(args.steps, 3)):
            launch_timer.record_start()
            model.launch(request)
            launch_timer.record_end()
            model.synchronize()
            per_launch.append(launch_timer.elapsed_ns())
    check(model.read_state())
    clock_summary = clocks.summary()

    # Scheduler floor: the control-only kernel over the same 128-token run
    # (every stage ends with a grid barrier: 9 per layer + 4 per token).
    floor_request = model.request(start_position, NEW_TOKENS, path=Q.PATH_SCHEDULER_PROFILE)
    model.launch(floor_request)
    model.synchronize()
    floor_times = []
    for _ in range(3):
        launch_timer.record_start()
        model.launch(floor_request)
        launch_timer.record_end()
        model.synchronize()
        floor_times.append(launch_timer.elapsed_ns())
    floor_state = model.read_state()
    if floor_state.status != 2 or floor_state.generated_tokens != NEW_TOKENS:
        raise RuntimeError(f"scheduler-floor run failed: status {floor_state.status}")
    floor_ns = statistics.median(floor_times)
    barriers_per_token = LAYERS * 9 + 4
    scheduler_floor = {
        "kernel": "qwen_stateful_graph_scheduler_profile_kernel",
        "us_per_token": floor_ns / 1e3 / NEW_TOKENS,
        "barriers_per_token": barriers_per_token,
        "us_per_barrier": floor_ns / 1e3 / NEW_TOKENS / barriers_per_token,
        "workers": model.info.worker_count,
    }

    # End to end through the C ABI: host hidden in, host tokens out.
    hidden_host = tail["lm_head"][int(prompt[-1])].copy()
    tokens_host = np.zeros(NEW_TOKENS, np.uint32)
    for _ in range(max(1, min(args.warmup, 2))):
        model.generate(start_position, NEW_TOKENS, hidden=hidden_host, tokens=tokens_host)
    e2e_start = time.perf_counter()
    for _ in range(args.steps):
        state, _ = model.generate(start_position, NEW_TOKENS, hidden=hidden_host,
                                  tokens=tokens_host)
        check(state)
    e2e_seconds = time.perf_counter() - e2e_start

    elapsed_s = total_ns / 1e9
    if world > 1:
        elapsed_s, e2e_seconds = max_over_ranks([elapsed_s, e2e_seconds], dist)

    info = model.info
    weight_bytes = int(info.weight_bytes_per_token)
    algorithmic = algorithmic_bytes_per_launch(weight_bytes, start_position, NEW_TOKENS)
    launch_s = statistics.median(per_launch) / 1e9
    peak, peak_kind = measured_peaks()
    achieved = algorithmic / launch_s / 1e9
    traffic_per_token = profiled_traffic_per_token()
    roofline = {
        "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
        "frac": achieved / peak, "peak_source": peak_kind,
        "traffic": traffic_per_token * NEW_TOKENS if traffic_per_token else None,
        "algorithmic_bytes_per_launch": algorithmic,
        "kernel": "qwen_stateful_graph_compiled_kernel",
    }
    tokens_total = world * NEW_TOKENS * args.steps
    line = {
        "metric": METRIC, "value": tokens_total / elapsed_s, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * elapsed_s / args.steps,
        "ms_per_token": 1000.0 * elapsed_s / args.steps / NEW_TOKENS,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights N(0,0.02), seeded prompt)",
        "config": {"workload": "config2: 24-layer Qwen2.5-0.5B-arch FP32 greedy decode, "
                               "batch 1, 32-token prompt, 128 new tokens per step",
                   "global_batch": world, "seq_len": PROMPT + NEW_TOKENS,
                   "parallelism": f"dp{world} (independent replicas, no collective)",
                   "l2": "weights 2 GB > L2 126 MB, no flush needed",
                   "workers": info.worker_count},
        "e2e": {"value": tokens_total / e2e_seconds, "unit": "tokens/s",
                "h2d_bytes_per_step": 896 * 4, "d2h_bytes_per_step": NEW_TOKENS * 4},
        "gpu_launches": args.steps,
        "roofline": roofline,
        "clocks": clock_summary,
        "scheduler_floor": scheduler_floor,
    }
    if not args.no_extra:
        from lrrt_b200 import synthetic as S
        line.update(extra_configs(model, Q, S, rank, world, dist, args.warmup))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle as O
        threads = O.max_threads()
        decode = oracle_decoder(weights, tail, prompt, threads)
        tps, tokens, seconds = cpu_tokens_per_second(decode, args.cpu_seconds)
        O.set_threads(1)
        tps1, tokens1, seconds1 = cpu_tokens_per_second(decode, args.cpu_seconds / 2)
        line["cpu_baseline"] = {
            "value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{tokens} greedy tokens of the same workload (prompt ingested, "
                      f"decodes from position 31; {seconds:.1f} s, OpenMP over rows, "
                      f"reference reduction order)",
            "one_core": {"value": tps1, "unit": "tokens/s", "cores": 1,
                         "sample": f"{tokens1} tokens in {seconds1:.1f} s"}}
    model.close()
    if rank == 0:
        print(json.dumps(line), flush=True)


def profile_case(args) -> None:
    """Profiler workloads of the prefill and batched-decode paths: warm-up
    outside the profiler range, the measured launches inside
    cuProfilerStart/Stop (for `ncu --profile-from-start off`). Small sizes
    keep `--set full` captures to a few hundred MB of device memory."""
    import ctypes

    from lrrt_b200 import qwen as Q
    from lrrt_b200 import synthetic as S

    def build(capacity: int, max_tokens: int, chunk: int):
        weights, tail = S.model(3, args.layers, args.vocab, True)
        model = Q.Model(Q.ModelConfig(layer_count=args.layers, vocab_size=args.vocab,
                                      cache_capacity=capacity, max_tokens_per_run=max_tokens))
        for i, w in enumerate(weights):
            model.set_layer(i, w)
        model.set_tail(tail["final_norm"], tail["lm_head"])
        model.enable_prefill(chunk)
        return model

    cuda = ctypes.CDLL("libcuda.so.1")
    if args.profile_case == "long":
        # Config 3's resident decode: KV rows 0..context-1 pre-filled, one
        # warm-up launch, then --case-steps tokens at positions context...
        weights, tail = S.model(SEED, args.layers, args.vocab, True)
        model = Q.Model(Q.ModelConfig(layer_count=args.layers, vocab_size=args.vocab,
                                      cache_capacity=args.context + 2 * args.case_steps + 8,
                                      max_tokens_per_run=args.case_steps))
        for i, w in enumerate(weights):
            model.set_layer(i, w)
        model.set_tail(tail["final_norm"], tail["lm_head"])
        for layer, (keys, values) in enumerate(S.kv_prefill(SEED, args.layers, args.context)):
            model.set_kv(layer, 0, keys, values)
        model.set_hidden(S.hidden(SEED))
        model.decode(args.context, args.case_steps)
        model.set_hidden(S.hidden(SEED))
        cuda.cuProfilerStart()
        state, _ = model.decode(args.context, args.case_steps)
        cuda.cuProfilerStop()
        if state.status != 2 or state.fused_path != 1:
            raise RuntimeError(f"long-context case: status {state.status}")
    elif args.profile_case == "prefill":
        model = build(args.prompt, 1, args.prompt)
        prompt = S.prompt(3, args.prompt, args.vocab)
        model.prefill(prompt, Q.PREFILL_TF32X3)  # warm-up: weight split, maps
        model.synchronize()
        cuda.cuProfilerStart()
        model.prefill(prompt, Q.PREFILL_TF32X3)
        model.synchronize()
        cuda.cuProfilerStop()
    else:
        capacity = args.context + args.case_steps + 8
        model = build(capacity, args.case_steps + 4, max(args.streams, args.context))
        prompts = S.prompt(2, args.streams * (args.context + 1), args.vocab)
        with Q.Batch(model, args.streams, capacity, args.case_steps + 4) as batch:
            for s in range(args.streams):
                batch.prefill(s, prompts[s * (args.context + 1):(s + 1) * (args.context + 1)])
            batch.decode(4)  # graph capture, warm-up
            cuda.cuProfilerStart()
            batch.decode(args.case_steps)
            cuda.cuProfilerStop()
    model.close()
    print("profile case done")


def main():
    global NEW_TOKENS
    args = parse_args()
    NEW_TOKENS = args.new_tokens
    if args.profile_case:
        profile_case(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and "RANK" in os.environ:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            reference_arm(args, rank, world)
        else:
            our_arm(args, rank, world, local_rank)
    finally:
        if world > 1 and "RANK" in os.environ:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
