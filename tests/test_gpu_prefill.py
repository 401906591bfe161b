"""Batched prompt prefill against token-by-token ingestion.

The prefill computes positions 0..n-2 of a prompt with GEMMs over all prompt
rows (FP32 SIMT tiles, or 3xTF32 on the tcgen05 tensor cores); the oracle
ingests the same prompt one decode step at a time on the CPU. K/V rows are
compared with the activation tolerance (the summation order differs, so the
match is to FP32 rounding, not bit for bit), and the greedy decode that
follows must produce the oracle's tokens with logits within 1e-4."""
import numpy as np
import pytest

import oracle as O
from helpers import LOGIT_RTOL, build_pair, ingest_prompt, max_relative_error, prefill_kv
from lrrt_b200 import native as N
from lrrt_b200 import qwen as Q
from lrrt_b200 import synthetic as S

KV_RTOL = 1.0e-4
PATHS = [pytest.param(Q.PREFILL_SIMT, id="simt"), pytest.param(Q.PREFILL_TF32X3, id="tf32x3")]


def compare_kv(model, oracle, positions, first=0):
    worst = 0.0
    for layer in range(oracle.layers):
        for name, cache in (("key_cache", oracle.key_cache), ("value_cache", oracle.value_cache)):
            got = model.read(name, layer).reshape(-1, 128)[first:positions]
            error = max_relative_error(got, cache[layer][first:positions])
            worst = max(worst, error)
            assert error <= KV_RTOL, (name, layer, error)
    return worst


def decode_matches(model, oracle, start, count):
    state, tokens = model.decode(start, count)
    assert state.status == 2 and state.error_code == 0
    assert tokens.tolist() == oracle.output_tokens[:count].tolist()
    d = oracle.decode_state
    assert (state.token_position, state.kv_length, state.sampled_token) == (
        d.token_position, d.kv_length, d.sampled_token)
    assert abs(state.sampled_logit - d.sampled_logit) <= LOGIT_RTOL * max(1.0, abs(d.sampled_logit))


@pytest.mark.gpu
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("prompt_length,chunk", [(41, 512), (41, 16), (300, 512), (2, 512)])
def test_prefill_matches_oracle_ingest(gpu, path, prompt_length, chunk):
    """Ragged row counts (40, 299 rows: partial 128-row tiles, several M
    tiles), chunked prompts (16-token chunks attend across chunks) and the
    one-row case; then 8 greedy tokens identical to the oracle."""
    model, oracle, _, _ = build_pair(seed=11, layers=2, vocab=4096, capacity=320, max_tokens=8)
    model.enable_prefill(chunk)
    prompt = S.prompt(11, prompt_length, 4096)
    model.prefill(prompt, path)
    for i, token in enumerate(prompt[:-1]):
        oracle.decode(oracle.embedding(int(token)), i, 1)
    worst = compare_kv(model, oracle, prompt_length - 1)
    print(f"prefill path {path} rows {prompt_length - 1} chunk {chunk}: kv error {worst:.2e}")
    start = prompt_length - 1
    oracle.decode(oracle.embedding(int(prompt[-1])), start, 8)
    decode_matches(model, oracle, start, 8)
    model.close()


@pytest.mark.gpu
@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("cached", [64, 2100])
def test_prefill_at_continues_a_cached_context(gpu, path, cached):
    """prefill_at on top of `cached` cache rows written by set_kv: the next 36
    rows from tokens, earlier rows untouched, decode continues after them.
    Past 2048 keys the attention chunks grow to 256 keys (four 64-key
    sub-tiles per block on the tensor-core path)."""
    model, oracle, _, _ = build_pair(seed=12, layers=2, vocab=4096, capacity=cached + 64,
                                     max_tokens=4)
    model.enable_prefill(512)
    prefill_kv(model, oracle, seed=12, layers=2, positions=cached)
    before = [model.read("key_cache", layer).reshape(-1, 128)[:cached].copy()
              for layer in range(2)]
    tokens = S.prompt(13, 37, 4096)
    model.prefill_at(tokens[:-1], cached, path)
    for i, token in enumerate(tokens[:-1]):
        oracle.decode(oracle.embedding(int(token)), cached + i, 1)
    for layer in range(2):
        assert np.array_equal(model.read("key_cache", layer).reshape(-1, 128)[:cached],
                              before[layer])
    compare_kv(model, oracle, cached + 36, first=cached)
    model.set_hidden_from_token(int(tokens[-1]))
    oracle.decode(oracle.embedding(int(tokens[-1])), cached + 36, 4)
    decode_matches(model, oracle, cached + 36, 4)
    model.close()


@pytest.mark.gpu
def test_prefill_argument_errors(gpu):
    model, _, _, _ = build_pair(seed=3, layers=1, vocab=1024, capacity=64, max_tokens=2)
    with pytest.raises(N.LrrtError, match="not enabled"):
        model.prefill([1, 2, 3])
    model.enable_prefill(32)
    with pytest.raises(N.LrrtError, match="out of range"):
        model.prefill([1, 1024, 3])
    with pytest.raises(N.LrrtError, match="capacity"):
        model.prefill_at([1] * 10, 60)
    with pytest.raises(N.LrrtError, match="unknown prefill path"):
        model.prefill([1, 2, 3], path=7)
    model.prefill([5], Q.PREFILL_TF32X3)  # one token: nothing to prefill, hidden staged
    model.close()


@pytest.mark.gpu
def test_prefill_refreshes_split_weights_after_upload(gpu):
    """The TF32 weight copies follow a later set_layer: prefill after the
    upload matches a fresh model built with the new weights."""
    model, _, _, _ = build_pair(seed=21, layers=1, vocab=1024, capacity=64, max_tokens=2)
    model.enable_prefill(64)
    prompt = S.prompt(21, 20, 1024)
    model.prefill(prompt, Q.PREFILL_TF32X3)
    layers, tail = S.model(22, 1, 1024, True)
    model.set_layer(0, layers[0])
    model.set_tail(tail["final_norm"], tail["lm_head"])
    model.prefill(prompt, Q.PREFILL_TF32X3)
    fresh, _, _, _ = build_pair(seed=22, layers=1, vocab=1024, capacity=64, max_tokens=2)
    fresh.enable_prefill(64)
    fresh.prefill(prompt, Q.PREFILL_TF32X3)
    a = model.read("key_cache", 0).reshape(-1, 128)[:19]
    b = fresh.read("key_cache", 0).reshape(-1, 128)[:19]
    assert np.array_equal(a, b)
    model.close()
    fresh.close()


@pytest.mark.gpu
def test_config5_prefill_512_then_256_tokens(gpu):
    """24 layers, vocab 151936, 512-token prompt (seed 3).
    3xTF32 prefill against single-token ingestion of the same prompt on the
    GPU (itself checked against the oracle by the config-2 test): every
    layer's K/V rows agree to the activation tolerance, and the 256 greedy
    tokens that follow are identical."""
    layers, tail = S.model(3, 24, 151936, True)
    config = Q.ModelConfig(layer_count=24, vocab_size=151936, cache_capacity=768,
                           max_tokens_per_run=256)
    prompt = S.prompt(3, 512, 151936)
    runs = {}
    for name in ("ingest", "prefill"):
        model = Q.Model(config)
        for i, w in enumerate(layers):
            model.set_layer(i, w)
        model.set_tail(tail["final_norm"], tail["lm_head"])
        if name == "ingest":
            model.ingest_prompt([int(t) for t in prompt])
        else:
            model.enable_prefill(512)
            model.prefill(prompt, Q.PREFILL_TF32X3)
        kv = [(model.read("key_cache", l).reshape(-1, 128)[:511].copy(),
               model.read("value_cache", l).reshape(-1, 128)[:511].copy()) for l in range(24)]
        state, tokens = model.decode(511, 256)
        assert state.status == 2 and state.error_code == 0
        runs[name] = (kv, tokens, state.sampled_logit)
        model.close()
    worst = 0.0
    for (k0, v0), (k1, v1) in zip(runs["ingest"][0], runs["prefill"][0]):
        worst = max(worst, max_relative_error(k1, k0), max_relative_error(v1, v0))
    print(f"config5: worst K/V relative error {worst:.2e}")
    assert worst <= KV_RTOL
    mismatch = np.nonzero(runs["ingest"][1] != runs["prefill"][1])[0]
    assert mismatch.size == 0, f"first differing step {int(mismatch[0])}"


# ---- the prefill GEMMs alone, against float64 on the host -----------------

GEMM_RTOL = 2.0e-5  # FP32 accumulation over K <= 4864 (3xTF32 keeps FP32 products)


@pytest.fixture(scope="module")
def gemm_model(gpu):
    model, _, _, _ = build_pair(seed=5, layers=1, vocab=256, capacity=16, max_tokens=1)
    model.enable_prefill(16)
    yield model
    model.close()


def _silu(x):
    return x / (1.0 + np.exp(-x))


@pytest.mark.gpu
@pytest.mark.parametrize("tile", [0, 192, 224, 256, 288])
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["bias", "residual", "swiglu"])
@pytest.mark.parametrize("m,n,k", [(40, 448, 896), (300, 896, 4864), (512, 4864, 896),
                                   (512, 9728, 896)])
def test_prefill_gemm_matches_float64(gemm_model, tile, mode, m, n, k):
    """Every tile width and epilogue: split-K only (40 rows), several 128-row
    bands with a long K (300 x 896 x 4864), and tile counts past one wave
    that are not a multiple of the 148 SMs: full waves plus a split-K
    remainder (512 x 4864: 152 tiles of 128 x 256; 512 x 9728: 152 to 304
    tiles, up to two full waves)."""
    if tile == 288 and mode != 2:
        pytest.skip("288-column tiles are gate/up pairs (144 + 144)")
    if mode == 2 and tile not in (0, 288) and (n % (tile // 2) != 0 or tile == 224):
        pytest.skip("swiglu tiles: 192 or 256 columns whose halves divide n")
    _check_gemm(gemm_model, tile, mode, m, n, k)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1, 2], ids=["bias", "residual", "swiglu"])
@pytest.mark.parametrize("m,n,k", [(1, 1152, 896), (17, 480, 4864), (32, 4864, 896),
                                   (32, 896, 4864), (32, 19072, 896)])
def test_narrow_gemm_matches_float64(gemm_model, mode, m, n, k):
    """At most 32 rows run the swapped-operand kernels (weights as the MMA's
    A operand, 128 output columns per tile, gate/up pairs in two
    accumulators) under the same split-K schedule: one row, a ragged last
    column tile (480 = 3.75 x 128) with a long K, a 32-row swiglu of
    Qwen2-0.5B's MLP width, the down projection's shape, and 149 tiles (more
    than one wave: the two-CTAs-per-SM kernel, then a split-K remainder)."""
    _check_gemm(gemm_model, 256, mode, m, n, k)


def _check_gemm(gemm_model, tile, mode, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k + mode)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (rng.standard_normal((2 * n if mode == 2 else n, k), dtype=np.float32) * 0.02)
    c = rng.standard_normal((m, n), dtype=np.float32)
    bias = rng.standard_normal(n, dtype=np.float32)
    got = gemm_model.prefill_gemm_check(tile, mode, a, b, c, bias if mode == 0 else None)
    acc = a.astype(np.float64) @ b.astype(np.float64).T
    if mode == 0:
        want = acc + bias
    elif mode == 1:
        want = c.astype(np.float64) + acc
    else:
        want = _silu(acc[:, :n]) * acc[:, n:]
    error = max_relative_error(got, want)
    assert error <= GEMM_RTOL, error


@pytest.mark.gpu
def test_decode_rearms_state_after_many_short_runs(gpu):
    """A decode whose (max_steps, stop_value) differ from the previous
    launch's rewrites the executor's State image with lr_memcpy; that copy
    must have landed before the queue re-arms State from it. Hundreds of
    one-token ingestion launches, prefills and alternating step limits, each
    decode then generates all of its tokens."""
    model, _, _, _ = build_pair(seed=9, layers=2, vocab=4096, capacity=400, max_tokens=16)
    model.enable_prefill(512)
    prompt = [int(t) for t in S.prompt(9, 300, 4096)]
    model.ingest_prompt(prompt[:64])
    model.prefill(prompt, Q.PREFILL_TF32X3)
    model.ingest_prompt(prompt)
    for max_steps in (0, 10_000, 0, 777):
        state, tokens = model.decode(299, 16, max_steps=max_steps)
        assert (state.status, state.error_code, state.generated_tokens) == (2, 0, 16), max_steps
    model.close()
