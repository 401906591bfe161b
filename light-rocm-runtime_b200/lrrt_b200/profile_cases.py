"""Profiler workloads of the prefill and batched-decode paths.

Each case builds a synthetic model (random-init weights N(0, 0.02), seeded
prompts), runs its warm-up outside a profiler range and the measured work
inside one (cuProfilerStart/Stop), so that

    ncu --profile-from-start off --clock-control none ... \\
        python -m lrrt_b200.profile_cases <case> [options]

captures only the measured launches. Small sizes keep `--set full` captures
to a few hundred MB of device memory; the defaults are the BASELINE shapes.

  prefill   one 3xTF32 prefill of a `--prompt`-token prompt (rows 0..n-2)
  batch     `--streams` streams at context `--context`, `--steps` greedy steps
"""
from __future__ import annotations

import argparse
import ctypes

from . import qwen as Q
from . import synthetic as S


def _model(layers: int, vocab: int, capacity: int, max_tokens: int, chunk: int) -> Q.Model:
    weights, tail = S.model(3, layers, vocab, True)
    model = Q.Model(Q.ModelConfig(layer_count=layers, vocab_size=vocab, cache_capacity=capacity,
                                  max_tokens_per_run=max_tokens))
    for i, w in enumerate(weights):
        model.set_layer(i, w)
    model.set_tail(tail["final_norm"], tail["lm_head"])
    model.enable_prefill(chunk)
    return model


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("case", choices=["prefill", "batch"])
    parser.add_argument("--layers", type=int, default=24)
    parser.add_argument("--vocab", type=int, default=151936)
    parser.add_argument("--prompt", type=int, default=512)
    parser.add_argument("--streams", type=int, default=32)
    parser.add_argument("--context", type=int, default=1024)
    parser.add_argument("--steps", type=int, default=2)
    args = parser.parse_args()
    cuda = ctypes.CDLL("libcuda.so.1")
    if args.case == "prefill":
        model = _model(args.layers, args.vocab, args.prompt, 1, args.prompt)
        prompt = S.prompt(3, args.prompt, args.vocab)
        model.prefill(prompt, Q.PREFILL_TF32X3)  # warm-up: weight split, maps
        model.synchronize()
        cuda.cuProfilerStart()
        model.prefill(prompt, Q.PREFILL_TF32X3)
        model.synchronize()
        cuda.cuProfilerStop()
    else:
        capacity = args.context + args.steps + 8
        model = _model(args.layers, args.vocab, capacity, args.steps + 4,
                       max(args.streams, args.context))
        prompts = S.prompt(2, args.streams * (args.context + 1), args.vocab)
        with Q.Batch(model, args.streams, capacity, args.steps + 4) as batch:
            for s in range(args.streams):
                batch.prefill(s, prompts[s * (args.context + 1):(s + 1) * (args.context + 1)])
            batch.decode(4)  # graph capture, warm-up
            cuda.cuProfilerStart()
            batch.decode(args.steps)
            cuda.cuProfilerStop()
    model.close()
    print("ok")


if __name__ == "__main__":
    main()
