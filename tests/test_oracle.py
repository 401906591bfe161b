"""CPU tests of the oracle itself against the reference's known answers."""
import ctypes as C
import json
from pathlib import Path

import numpy as np

import oracle as O
from lrrt_b200 import synthetic as S

GOLDEN = Path(__file__).parent / "golden"


def run_fixture():
    golden = json.loads((GOLDEN / "scheduler_fixture.json").read_text())
    g = golden["graph"]
    values = np.zeros(8, np.uint32)
    checksums = np.zeros(8, np.uint32)
    branch_steps = np.zeros(8, np.uint32)
    executions = np.zeros(5, np.uint32)
    calls = np.zeros(1, np.uint32)
    context = O.FixtureContext(0x53504754, 8, values.ctypes.data, checksums.ctypes.data,
                               branch_steps.ctypes.data, executions.ctypes.data,
                               calls.ctypes.data)
    state = O.initial_state(g["initial_program"], g["max_steps"], g["stop_value"],
                            g["workers"])
    O.run_graph(state, [tuple(t) for t in g["tasks"]], [tuple(p) for p in g["programs"]],
                g["phase_state_count"], O.library().or_fixture_workload(),
                C.cast(C.pointer(context), C.c_void_p))
    return golden, state, values, checksums, branch_steps, executions, calls


def test_scheduler_fixture_matches_reference_goldens(built):
    golden, state, values, checksums, branch_steps, executions, calls = run_fixture()
    for key, want in golden["expected_state"].items():
        assert getattr(state, key) == want, key
    assert values.tolist() == golden["expected_values"]
    assert checksums.tolist() == golden["expected_checksums"]
    assert branch_steps.tolist() == golden["expected_branch_steps"]
    assert executions.tolist() == golden["expected_task_executions"]
    assert calls[0] == 1


def tiny_oracle(max_tokens=4, vocab=64):
    layers, tail = S.model(11, 1, vocab)
    return O.OracleModel(layers, tail, 16, 4, workers=8, max_tokens=max_tokens)


def test_oracle_executes_64_task_chain(built):
    """qwen_stateful_graph.cpp:1272-1291: 64 chained residual_advance tasks use
    both mask words; predicate, step and executed count all reach 64/1/64."""
    model = tiny_oracle()
    tasks = [O.make_task(9, 0 if i == 0 else 1 << (i - 1), 0, 1, 1) for i in range(64)]
    programs = [(0, 64, 0, 1 | 2, 0)]
    model.decode_state.maximum_tokens = 1
    state = O.initial_state(0, 1, 64, 8)
    O.run_graph(state, tasks, programs, 16, O.library().or_qwen_workload(),
                C.cast(model.contexts, C.c_void_p))
    assert (state.status, state.step, state.predicate_value, state.executed_tasks) == (2, 1, 64, 64)


def test_oracle_rejects_cyclic_decode_graph(built):
    """qwen_stateful_graph.cpp:1293-1311: the attention root made dependent on
    the last attention task closes a cycle -> invalid_program, error 1."""
    model = tiny_oracle()
    tasks = list(model.tasks)
    mask = 1 << 24
    tasks[0] = tasks[0][:1] + (mask & 0xFFFFFFFF,) + tasks[0][2:6] + (mask >> 32, 0)
    model.decode_state.maximum_tokens = 4
    state = O.initial_state(0, 16, 1, 8)
    O.run_graph(state, tasks, model.programs, 64, O.library().or_qwen_workload(),
                C.cast(model.contexts, C.c_void_p))
    assert (state.status, state.error_code) == (4, 1)


def test_oracle_stops_at_eos(built):
    """qwen_stateful_graph.cpp:1314-1340: EOS = the first greedy token stops
    the run after one token at step == layers."""
    model = tiny_oracle(max_tokens=4)
    hidden = S.hidden(11)
    model.decode(hidden, 0, 1)
    first = int(model.decode_state.sampled_token)
    state = model.decode(hidden, 0, 4, eos=first)
    assert state.status == 2 and state.step == 1
    assert model.decode_state.generated_tokens == 1
    assert model.decode_state.stop_reason == 2
    assert model.decode_state.sampled_token == first


def test_oracle_final_state_bookkeeping(built):
    """qwen_stateful_graph.cpp:1619-1632: executed_tasks and phase generation
    after `steps` tokens."""
    model = tiny_oracle(max_tokens=4)
    state = model.decode(S.hidden(3), 0, 4)
    layers, steps, partitions = 1, 4, 4
    assert state.status == 2 and state.step == steps * layers
    assert state.executed_tasks == steps * layers * 79 + steps * (partitions + 3)
    assert state.phase >> 8 == steps * (2 * layers + 1) - 1
    assert state.phase & 0xFF == 2
    assert model.decode_state.generated_tokens == 4
    assert model.decode_state.token_position == 3


def test_oracle_matches_transformers_golden(built):
    """Greedy decode of the oracle equals HF transformers' Qwen2ForCausalLM on
    the committed fixture; last-step logits within 1e-4 of max |logit|."""
    golden = np.load(GOLDEN / "hf_qwen2_decode.npz")
    seed, layers, vocab = int(golden["seed"]), int(golden["layers"]), int(golden["vocab"])
    prompt = golden["prompt"]
    weights, tail = S.model(seed, layers, vocab)
    new_tokens = len(golden["tokens"])
    model = O.OracleModel(weights, tail, 64, 32, workers=148, max_tokens=new_tokens)
    for i, token in enumerate(prompt[:-1]):
        model.decode(model.embedding(int(token)), i, 1)
    state = model.decode(model.embedding(int(prompt[-1])), len(prompt) - 1, new_tokens)
    assert state.status == 2
    assert model.output_tokens[:new_tokens].tolist() == golden["tokens"].tolist()
    last = golden["last_logits"].astype(np.float64)
    error = np.max(np.abs(model.logits - last)) / np.max(np.abs(last))
    assert error <= 1.0e-4, error
    assert abs(model.decode_state.sampled_logit - golden["max_logits"][-1]) <= \
        1.0e-4 * abs(golden["max_logits"][-1])


def test_oracle_matches_transformers_config1_logits(built):
    """BASELINE config 1 (one layer, vocab 151936, KV rows 0..127 ~ N(0, 1),
    hidden ~ N(0, 1)): every logit of the step at position 128 within 1e-4
    of transformers' (element by element, relative above 1e-2 in magnitude)."""
    golden = np.load(GOLDEN / "hf_qwen2_config1.npz")
    weights, tail = S.model(0, 1, 151936)
    model = O.OracleModel(weights, tail, 136, 32, workers=148, max_tokens=1)
    keys, values = S.kv_prefill(0, 1, 128)[0]
    model.set_kv(0, 0, keys, values)
    O.set_threads(O.max_threads())
    state = model.decode(S.hidden(0), 128, 1)
    O.set_threads(1)
    assert state.status == 2
    want = golden["logits"].astype(np.float64)
    error = np.max(np.abs(model.logits - want) / np.maximum(np.abs(want), 1.0e-2))
    assert error <= 1.0e-4, error
    assert model.decode_state.sampled_token == int(np.argmax(want))


def test_oracle_matches_transformers_config2_tokens(built):
    """BASELINE config 2 (24 layers, vocab 151936, the 32-token seed-1
    prompt): the first 32 greedy tokens equal transformers' and each chosen
    logit is within 1e-4."""
    golden = np.load(GOLDEN / "hf_qwen2_config2.npz")
    weights, tail = S.model(1, 24, 151936)
    prompt = golden["prompt"]
    count = len(golden["tokens"])
    model = O.OracleModel(weights, tail, 64, 32, workers=148, max_tokens=count,
                          keep_logits=False)
    O.set_threads(O.max_threads())
    for i, token in enumerate(prompt[:-1]):
        model.decode(model.embedding(int(token)), i, 1)
    state = model.decode(model.embedding(int(prompt[-1])), len(prompt) - 1, count)
    O.set_threads(1)
    assert state.status == 2
    assert model.output_tokens[:count].tolist() == golden["tokens"].tolist()
    assert abs(model.decode_state.sampled_logit - golden["max_logits"][-1]) <= \
        1.0e-4 * max(1.0, abs(golden["max_logits"][-1]))


def test_wave_dot_reduction_order(built):
    """The dot product follows the lane-strided order and shfl_down tree."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal(896).astype(np.float32)
    w = rng.standard_normal(896).astype(np.float32)
    lanes = np.zeros(32, np.float32)
    for c in range(0, 896, 32):
        for lane in range(32):
            lanes[lane] = np.float32(np.float64(x[c + lane]) * np.float64(w[c + lane]) +
                                     np.float64(lanes[lane]))
    offset = 16
    while offset:
        lanes[:offset] = lanes[:offset] + lanes[offset:2 * offset]
        offset //= 2
    assert O.wave_dot(x, w) == lanes[0]
