"""Writers of the FP32 weight-bundle formats the decode path loads (the
manifest + data-file layout of light-rocm-runtime's tools/convert_qwen_layer.py
and executor/qwen/weight_bundle.hpp; the C++ loader and writer are in
include/lrrt/qwen/weight_bundle.hpp).

A decoder layer bundle is <dir>/weights.json + <dir>/<data>, the data file
holding the float32 tensors below end to end in this order; a tail bundle
holds token_embeddings (rows of `token_ids`), final_norm_weight and
lm_head_weight.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

LAYER_TENSORS = ("attention_norm_weight", "mlp_norm_weight", "q_weight", "k_weight",
                 "v_weight", "q_bias", "k_bias", "v_bias", "out_weight", "gate_weight",
                 "up_weight", "down_weight")
# lrrt_b200.synthetic / Model.set_layer field names of the same tensors.
LAYER_FIELDS = {"attention_norm_weight": "attention_norm", "mlp_norm_weight": "mlp_norm",
                "q_weight": "q", "k_weight": "k", "v_weight": "v", "q_bias": "q_bias",
                "k_bias": "k_bias", "v_bias": "v_bias", "out_weight": "o",
                "gate_weight": "gate", "up_weight": "up", "down_weight": "down"}


def _write(manifest: Path, data_name: str, header: dict, tensors) -> None:
    if Path(data_name).name != data_name or data_name in ("", ".", ".."):
        raise ValueError("the data file must be a plain file name")
    manifest = Path(manifest)
    manifest.parent.mkdir(parents=True, exist_ok=True)
    entries, offset = [], 0
    with (manifest.parent / data_name).open("wb") as data:
        for name, array in tensors:
            payload = np.ascontiguousarray(array, dtype="<f4").tobytes()
            entries.append({"name": name, "offset": offset, "count": len(payload) // 4})
            data.write(payload)
            offset += len(payload)
    manifest.write_text(json.dumps({**header, "data": data_name, "tensors": entries},
                                   indent=2) + "\n")


def write_layer_bundle(manifest, weights: dict, keys: int, rope_theta: float = 1.0e6,
                       data_name: str = "weights.bin", heads: int = 14, kv_heads: int = 2,
                       head_dim: int = 64) -> None:
    """`weights` uses the Model.set_layer names (q, k, v, o, gate, ...)."""
    hidden = int(np.asarray(weights["attention_norm"]).shape[0])
    intermediate = int(np.asarray(weights["gate"]).shape[0])
    header = {"format": "lrrt.mini_decoder_weights", "version": 2, "dtype": "f32",
              "keys": keys, "hidden": hidden, "heads": heads, "kv_heads": kv_heads,
              "head_dim": head_dim, "intermediate": intermediate,
              "rope_theta": float(rope_theta)}
    _write(manifest, data_name, header,
           [(name, weights[LAYER_FIELDS[name]]) for name in LAYER_TENSORS])


def write_tail_bundle(manifest, final_norm, lm_head, token_ids=None, token_embeddings=None,
                      data_name: str = "weights.bin") -> None:
    """token_ids defaults to every row of lm_head (with the LM head rows as
    the embeddings, i.e. a tied model)."""
    lm_head = np.asarray(lm_head, np.float32)
    vocab, hidden = lm_head.shape
    if token_ids is None:
        token_ids = list(range(vocab))
        token_embeddings = lm_head
    header = {"format": "lrrt.mini_model_tail_weights", "version": 1, "dtype": "f32",
              "hidden": int(hidden), "vocab": int(vocab), "token_ids": [int(t) for t in token_ids]}
    _write(manifest, data_name, header,
           [("token_embeddings", token_embeddings), ("final_norm_weight", final_norm),
            ("lm_head_weight", lm_head)])
