"""Shared helpers: build a device model and an oracle model from the same
seeded synthetic weights, and compare their outputs."""
from __future__ import annotations

import numpy as np

import oracle as O
from lrrt_b200 import qwen as Q
from lrrt_b200 import synthetic as S

# Floating-point tolerance (north star: max relative logit error <= 1e-4).
# Intermediate activations are compared with the same relative bound scaled by
# the vector's magnitude, plus a small absolute floor for near-zero entries.
LOGIT_RTOL = 1.0e-4


def max_relative_error(actual: np.ndarray, expected: np.ndarray) -> float:
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    scale = max(float(np.max(np.abs(expected))), 1.0e-30)
    return float(np.max(np.abs(actual - expected)) / scale)


def elementwise_relative_error(actual: np.ndarray, expected: np.ndarray,
                               floor: float = 1.0e-2) -> float:
    """max |actual - expected| / max(|expected|, floor), element by element:
    relative for every value whose magnitude exceeds `floor`, absolute
    (scaled by floor) below it, where cancellation makes any reordered FP32
    sum differ by more than a relative 1e-4."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    return float(np.max(np.abs(actual - expected) / np.maximum(np.abs(expected), floor)))


def build_pair(seed: int, layers: int, vocab: int, capacity: int, max_tokens: int,
               partitions: int = 0, distinct_layers: bool = True, fused: bool = True,
               worker_count: int = 0):
    layer_weights, tail = S.model(seed, layers, vocab, distinct_layers)
    config = Q.ModelConfig(layer_count=layers, vocab_size=vocab, cache_capacity=capacity,
                           lm_head_partitions=partitions, worker_count=worker_count,
                           max_tokens_per_run=max_tokens,
                           disable_fused_path=not fused)
    model = Q.Model(config)
    for i, w in enumerate(layer_weights):
        model.set_layer(i, w)
    model.set_tail(tail["final_norm"], tail["lm_head"])
    oracle = O.OracleModel(layer_weights, tail, capacity, model.info.lm_head_partitions,
                           workers=model.info.worker_count, max_tokens=max_tokens)
    return model, oracle, layer_weights, tail


def prefill_kv(model, oracle, seed: int, layers: int, positions: int):
    for layer, (keys, values) in enumerate(S.kv_prefill(seed, layers, positions)):
        model.set_kv(layer, 0, keys, values)
        oracle.set_kv(layer, 0, keys, values)


def ingest_prompt(model, oracle, prompt):
    """Positions 0..n-2 through single-token decodes on both sides."""
    model.ingest_prompt([int(t) for t in prompt])
    for i, token in enumerate(prompt[:-1]):
        oracle.decode(oracle.embedding(int(token)), i, 1)
