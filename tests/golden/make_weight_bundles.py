"""Generates tests/golden/weight_bundles/: one small decoder-layer bundle
("lrrt.mini_decoder_weights" v2) and one model-tail bundle
("lrrt.mini_model_tail_weights" v1), written by light-rocm-runtime's own
converter functions (tools/convert_qwen_layer.py write_bundle :421-466 and
_write_tail_bundle :469-539), so the loader is checked against files the
reference produces.

Values follow a formula the C++ test recomputes: element i of the k-th
tensor (in manifest order) is float32(k + 1 + 0.001 * (i % 97)).

Run once, in an environment that has the reference checkout:
  python tests/golden/make_weight_bundles.py <path to the reference checkout>
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("weight_bundles")


def values(k: int, count: int) -> np.ndarray:
    i = np.arange(count, dtype=np.float64)
    return (k + 1 + 0.001 * (i % 97)).astype(np.float32)


def main(reference: Path) -> None:
    sys.path.insert(0, str(reference / "tools"))
    import convert_qwen_layer as C  # the reference's converter

    shape = C.DecoderLayerShape(keys=4, hidden=8, heads=2, kv_heads=1, head_dim=4,
                                intermediate=12)
    tensors = {}
    for k, mapping in enumerate(C.tensor_mappings(0, shape)):
        count = int(np.prod(mapping.shape))
        tensors[mapping.bundle_name] = values(k, count).reshape(mapping.shape)
    C.write_bundle(OUT / "layer_0" / "weights.json", "weights.bin", shape, tensors,
                   rope_theta=1000000.0)

    hidden, vocab, token_ids = 8, 10, [1, 5, 7]
    C._write_tail_bundle(OUT / "model_tail" / "weights.json", "weights.bin", hidden, token_ids,
                         values(0, len(token_ids) * hidden).reshape(len(token_ids), hidden),
                         values(1, hidden), values(2, vocab * hidden).reshape(vocab, hidden))


if __name__ == "__main__":
    main(Path(sys.argv[1]))
