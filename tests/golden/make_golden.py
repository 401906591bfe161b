"""Generates tests/golden/hf_qwen2_decode.npz: greedy decode vectors from
Hugging Face transformers' Qwen2ForCausalLM (FP32, eager attention), the
model-level oracle light-rocm-runtime itself uses
(tools/run_qwen_e2e.py:313-419). transformers is a third-party dependency of
that tool, not vendored in the reference; the version used is recorded in the
file.

The model is the Qwen2.5-0.5B architecture (hidden 896, 14/2 heads, head_dim
64, intermediate 4864, RMSNorm eps 1e-6, RoPE theta 1e6, tied embeddings)
with a reduced depth and vocabulary so the fixture stays small; weights come
from lrrt_b200.synthetic.model(SEED, LAYERS, VOCAB) and are regenerated
bit-identically by the tests from the same seed.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "light-rocm-runtime_b200"))
from lrrt_b200 import synthetic  # noqa: E402

SEED, LAYERS, VOCAB, PROMPT, NEW_TOKENS = 7, 2, 4096, 6, 8
OUT = Path(__file__).with_name("hf_qwen2_decode.npz")


def build_hf(layers, tail):
    import transformers
    from transformers import Qwen2Config, Qwen2ForCausalLM

    config = Qwen2Config(vocab_size=VOCAB, hidden_size=896, intermediate_size=4864,
                         num_hidden_layers=LAYERS, num_attention_heads=14,
                         num_key_value_heads=2, rope_theta=1.0e6, rms_norm_eps=1.0e-6,
                         tie_word_embeddings=True, max_position_embeddings=4096,
                         attn_implementation="eager")
    model = Qwen2ForCausalLM(config).float().eval()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(t(tail["lm_head"]))
        model.model.norm.weight.copy_(t(tail["final_norm"]))
        for layer, w in zip(model.model.layers, layers):
            layer.input_layernorm.weight.copy_(t(w["attention_norm"]))
            layer.post_attention_layernorm.weight.copy_(t(w["mlp_norm"]))
            a = layer.self_attn
            for proj, key in ((a.q_proj, "q"), (a.k_proj, "k"), (a.v_proj, "v")):
                proj.weight.copy_(t(w[key]))
                proj.bias.copy_(t(w[key + "_bias"]))
            a.o_proj.weight.copy_(t(w["o"]))
            layer.mlp.gate_proj.weight.copy_(t(w["gate"]))
            layer.mlp.up_proj.weight.copy_(t(w["up"]))
            layer.mlp.down_proj.weight.copy_(t(w["down"]))
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    return model, transformers.__version__


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    layers, tail = synthetic.model(SEED, LAYERS, VOCAB)
    prompt = synthetic.prompt(SEED, PROMPT, VOCAB)
    model, version = build_hf(layers, tail)
    sequence = torch.tensor([prompt.astype(np.int64)])
    tokens, maxima = [], []
    with torch.no_grad():
        for _ in range(NEW_TOKENS):
            logits = model(sequence).logits[0, -1]
            token = int(torch.argmax(logits))
            tokens.append(token)
            maxima.append(float(logits[token]))
            last = logits.numpy().astype(np.float32)
            sequence = torch.cat([sequence, torch.tensor([[token]])], dim=1)
    np.savez_compressed(OUT, seed=SEED, layers=LAYERS, vocab=VOCAB, prompt=prompt,
                        tokens=np.array(tokens, np.uint32),
                        max_logits=np.array(maxima, np.float32), last_logits=last,
                        transformers_version=np.array(version))
    print(f"wrote {OUT}: tokens {tokens}")


if __name__ == "__main__":
    main()
