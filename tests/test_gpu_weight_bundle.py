"""A model loaded from FP32 weight bundles (lrrt_b200.weight_bundle writer,
C++ loader) decodes exactly like one whose weights were uploaded from
arrays: same tokens, bit-identical logits and hidden state."""
import numpy as np
import pytest

from lrrt_b200 import qwen as Q
from lrrt_b200 import synthetic as S
from lrrt_b200 import weight_bundle as WB


@pytest.mark.gpu
def test_bundle_loaded_model_decodes_like_array_loaded(gpu, tmp_path):
    layers, vocab, capacity = 2, 4096, 40
    weights, tail = S.model(21, layers, vocab)
    config = Q.ModelConfig(layer_count=layers, vocab_size=vocab, cache_capacity=capacity,
                           max_tokens_per_run=16)
    for i, w in enumerate(weights):
        WB.write_layer_bundle(tmp_path / f"layer_{i}" / "weights.json", w, keys=capacity)
    WB.write_tail_bundle(tmp_path / "model_tail" / "weights.json", tail["final_norm"],
                         tail["lm_head"])
    from_arrays = Q.Model(config)
    from_bundles = Q.Model(config)
    try:
        for i, w in enumerate(weights):
            from_arrays.set_layer(i, w)
            from_bundles.load_layer_bundle(i, tmp_path / f"layer_{i}" / "weights.json")
        from_arrays.set_tail(tail["final_norm"], tail["lm_head"])
        from_bundles.load_tail_bundle(tmp_path / "model_tail" / "weights.json")
        prompt = [int(t) for t in S.prompt(21, 8, vocab)]
        runs = []
        for model in (from_arrays, from_bundles):
            model.ingest_prompt(prompt)
            state, tokens = model.decode(len(prompt) - 1, 12)
            assert state.status == 2
            runs.append((tokens.tolist(), state.sampled_logit, model.read("hidden")))
        assert runs[0][0] == runs[1][0]
        assert np.float32(runs[0][1]).tobytes() == np.float32(runs[1][1]).tobytes()
        assert np.array_equal(runs[0][2], runs[1][2])
    finally:
        from_arrays.close()
        from_bundles.close()
