"""Batched multi-stream decode (BASELINE config 4's per-GPU batch) against
single-stream decoding: every stream of a batch must produce the tokens its
own single-stream decode produces (the oracle's on the small model, the GPU
decode path's at full size), with logits and KV rows within 1e-4."""
import numpy as np
import pytest

from helpers import LOGIT_RTOL, build_pair, max_relative_error
from lrrt_b200 import native as N
from lrrt_b200 import qwen as Q
from lrrt_b200 import synthetic as S

KV_RTOL = 1.0e-4


@pytest.mark.gpu
def test_batch_streams_match_oracle(gpu):
    """Five streams with prompts of 1..40 tokens (ragged positions, one
    stream never prefilled beyond its single token), 12 greedy steps; each
    stream against the oracle's single-stream run."""
    layers, vocab, steps = 2, 4096, 12
    model, oracle, _, _ = build_pair(seed=31, layers=layers, vocab=vocab, capacity=96,
                                     max_tokens=steps)
    model.enable_prefill(64)
    lengths = [3, 17, 1, 40, 9]
    prompts = [S.prompt(100 + i, n, vocab) for i, n in enumerate(lengths)]
    with Q.Batch(model, len(prompts), 96, steps) as batch:
        for stream, prompt in enumerate(prompts):
            batch.prefill(stream, prompt)
        tokens, logits = batch.decode(steps)
        for stream, prompt in enumerate(prompts):
            start = len(prompt) - 1
            assert batch.position(stream) == start + steps
            for cache in oracle.key_cache + oracle.value_cache:
                cache[:] = 0  # fresh caches for this stream
            for i, token in enumerate(prompt[:-1]):
                oracle.decode(oracle.embedding(int(token)), i, 1)
            oracle.decode(oracle.embedding(int(prompt[-1])), start, steps)
            want = oracle.output_tokens[:steps].tolist()
            assert tokens[stream].tolist() == want, stream
            d = oracle.decode_state
            assert abs(logits[stream] - d.sampled_logit) <= LOGIT_RTOL * max(1.0, abs(d.sampled_logit))
            # Cache rows 0..start+steps-1 were written (the last token's row
            # is written by the step that consumes it, one past the run).
            rows = start + steps
            for layer in range(layers):
                keys, values = batch.read_cache(stream, layer, rows)
                assert max_relative_error(keys, oracle.key_cache[layer][:rows]) <= KV_RTOL
                assert max_relative_error(values, oracle.value_cache[layer][:rows]) <= KV_RTOL
        # A second decode call continues every stream.
        more, _ = batch.decode(4)
        assert all(batch.position(s) == len(p) - 1 + steps + 4 for s, p in enumerate(prompts))
    model.close()


@pytest.mark.gpu
def test_config4_shape_streams_match_oracle(gpu):
    """BASELINE config 4's shape: the 24-layer, vocab-151936 model, four
    streams whose caches hold 1024 positions of N(0, 1) rows (written
    directly, no prompt), 8 greedy tokens each, against the oracle's
    single-stream decode of the same context: tokens, last logit, new KV rows."""
    import oracle as O
    O.set_threads(O.max_threads())
    layers, vocab, context, steps, streams = 24, 151936, 1024, 8, 4
    model, oracle, _, _ = build_pair(seed=1, layers=layers, vocab=vocab,
                                     capacity=context + 16, max_tokens=steps)
    model.enable_prefill(64)
    first_tokens = S.prompt(2, streams, vocab)
    contexts = [S.kv_prefill(200 + s, layers, context) for s in range(streams)]
    with Q.Batch(model, streams, context + 16, steps) as batch:
        for stream in range(streams):
            for layer, (keys, values) in enumerate(contexts[stream]):
                batch.write_cache(stream, layer, 0, keys, values)
            batch.set_next(stream, context, int(first_tokens[stream]))
        tokens, logits = batch.decode(steps)
        for stream in range(streams):
            for layer, (keys, values) in enumerate(contexts[stream]):
                oracle.set_kv(layer, 0, keys, values)
            oracle.decode(oracle.embedding(int(first_tokens[stream])), context, steps)
            assert tokens[stream].tolist() == oracle.output_tokens[:steps].tolist(), stream
            d = oracle.decode_state
            assert abs(logits[stream] - d.sampled_logit) <= \
                LOGIT_RTOL * max(1.0, abs(d.sampled_logit))
            rows = context + steps
            for layer in range(layers):
                keys, values = batch.read_cache(stream, layer, rows)
                assert max_relative_error(keys[context:], oracle.key_cache[layer][context:rows]) \
                    <= KV_RTOL
                assert max_relative_error(values[context:],
                                          oracle.value_cache[layer][context:rows]) <= KV_RTOL
    O.set_threads(1)
    model.close()


@pytest.mark.gpu
def test_batch_argument_errors(gpu):
    model, _, _, _ = build_pair(seed=3, layers=1, vocab=1024, capacity=64, max_tokens=4)
    with pytest.raises(N.LrrtError, match="not enabled"):
        Q.Batch(model, 2, 64, 4)
    model.enable_prefill(8)
    with pytest.raises(N.LrrtError, match="streams"):
        Q.Batch(model, 9, 64, 4)          # more streams than the prefill chunk
    with pytest.raises(N.LrrtError, match="capacity"):
        Q.Batch(model, 2, 65, 4)          # beyond the model's RoPE rows
    with Q.Batch(model, 2, 16, 8) as batch:
        batch.prefill(0, [1] * 10)
        with pytest.raises(N.LrrtError, match="capacity"):
            batch.decode(8)               # 9 + 8 > 16
        with pytest.raises(N.LrrtError, match="out of range"):
            batch.prefill(1, [1, 1024])
        tokens, _ = batch.decode(6)
        assert tokens.shape == (2, 6)
    model.close()


@pytest.mark.gpu
def test_batch_of_40_streams_runs_the_wide_gemms(gpu):
    """More than 32 streams run the 128-row-band GEMM kernels instead of the
    narrow ones: 40 streams with prompts of 1..40 tokens, 6 greedy steps;
    three streams against the oracle's single-stream runs."""
    layers, vocab, steps = 2, 4096, 6
    model, oracle, _, _ = build_pair(seed=37, layers=layers, vocab=vocab, capacity=64,
                                     max_tokens=steps)
    model.enable_prefill(64)
    prompts = [S.prompt(300 + i, 1 + i, vocab) for i in range(40)]
    with Q.Batch(model, len(prompts), 64, steps) as batch:
        for stream, prompt in enumerate(prompts):
            batch.prefill(stream, prompt)
        tokens, logits = batch.decode(steps)
    for stream in (0, 17, 39):
        prompt = prompts[stream]
        start = len(prompt) - 1
        for cache in oracle.key_cache + oracle.value_cache:
            cache[:] = 0
        for i, token in enumerate(prompt[:-1]):
            oracle.decode(oracle.embedding(int(token)), i, 1)
        oracle.decode(oracle.embedding(int(prompt[-1])), start, steps)
        assert tokens[stream].tolist() == oracle.output_tokens[:steps].tolist(), stream
        d = oracle.decode_state
        assert abs(logits[stream] - d.sampled_logit) <= LOGIT_RTOL * max(1.0, abs(d.sampled_logit))
    model.close()


@pytest.mark.gpu
def test_config4_batch_32_streams_context_1024(gpu):
    """BASELINE config 4 on one GPU: 32 streams, each with a 1025-token random
    prompt (seed 2; context 1024), 128 greedy tokens per stream. Streams 0, 13
    and 31 must equal single-stream decoding of the same prompt on the GPU
    decode path (itself checked against the oracle by the config-2 test)."""
    layers, tail = S.model(2, 24, 151936, True)
    config = Q.ModelConfig(layer_count=24, vocab_size=151936, cache_capacity=1152,
                           max_tokens_per_run=128)
    model = Q.Model(config)
    for i, w in enumerate(layers):
        model.set_layer(i, w)
    model.set_tail(tail["final_norm"], tail["lm_head"])
    model.enable_prefill(1024)
    prompts = [S.prompt(2000 + s, 1025, 151936) for s in range(32)]
    with Q.Batch(model, 32, 1152, 128) as batch:
        for stream, prompt in enumerate(prompts):
            batch.prefill(stream, prompt)
        tokens, logits = batch.decode(128)
    for stream in (0, 13, 31):
        model.prefill(prompts[stream])
        state, single = model.decode(1024, 128)
        assert state.status == 2
        mismatch = np.nonzero(single != tokens[stream])[0]
        assert mismatch.size == 0, (stream, int(mismatch[0]))
        assert abs(logits[stream] - state.sampled_logit) <= \
            LOGIT_RTOL * max(1.0, abs(state.sampled_logit))
    model.close()
