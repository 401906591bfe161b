"""Seeded synthetic Qwen2.5-0.5B-architecture FP32 weights and inputs.

No checkpoint is available offline, so every workload uses random-init weights
of the real shapes: projection weights and biases ~ N(0, 0.02), RMSNorm gains
1.0, tied embedding / LM head table ~ N(0, 0.02) (numpy default_rng(seed)).
"""
from __future__ import annotations

import numpy as np

from .qwen import HEAD_DIM, HIDDEN, INTERMEDIATE, KV

SCALE = np.float32(0.02)

LAYER_SHAPES = {
    "attention_norm": (HIDDEN,),
    "q": (HIDDEN, HIDDEN),
    "k": (KV, HIDDEN),
    "v": (KV, HIDDEN),
    "q_bias": (HIDDEN,),
    "k_bias": (KV,),
    "v_bias": (KV,),
    "o": (HIDDEN, HIDDEN),
    "mlp_norm": (HIDDEN,),
    "gate": (INTERMEDIATE, HIDDEN),
    "up": (INTERMEDIATE, HIDDEN),
    "down": (HIDDEN, INTERMEDIATE),
}


def normal(rng: np.random.Generator, shape, scale=SCALE) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float32)


def layer(rng: np.random.Generator) -> dict:
    weights = {}
    for name, shape in LAYER_SHAPES.items():
        if name.endswith("norm"):
            weights[name] = np.ones(shape, np.float32)
        else:
            weights[name] = normal(rng, shape)
    return weights


def tail(rng: np.random.Generator, vocab: int) -> dict:
    return {"final_norm": np.ones(HIDDEN, np.float32),
            "lm_head": normal(rng, (vocab, HIDDEN))}


def model(seed: int, layers: int, vocab: int, distinct_layers: bool = True):
    """(list of layer dicts, tail dict). With distinct_layers False every layer
    shares one set of arrays (the device still stores each layer separately)."""
    rng = np.random.default_rng(seed)
    first = layer(rng)
    stack = [first] + [layer(rng) if distinct_layers else first for _ in range(layers - 1)]
    return stack, tail(rng, vocab)


def kv_prefill(seed: int, layers: int, positions: int):
    """KV cache rows ~ N(0, 1): list of (keys, values), each [positions][128]."""
    rng = np.random.default_rng(seed + 1000)
    return [(rng.standard_normal((positions, KV), dtype=np.float32),
             rng.standard_normal((positions, KV), dtype=np.float32)) for _ in range(layers)]


def hidden(seed: int) -> np.ndarray:
    return np.random.default_rng(seed + 2000).standard_normal(HIDDEN, dtype=np.float32)


def prompt(seed: int, length: int, vocab: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, vocab, length, dtype=np.int64).astype(
        np.uint32)


__all__ = ["layer", "tail", "model", "kv_prefill", "hidden", "prompt", "LAYER_SHAPES",
           "HEAD_DIM"]
