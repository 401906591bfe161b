"""Generates the Hugging Face golden fixtures under tests/golden/: decode
vectors from transformers' Qwen2ForCausalLM (FP32, eager attention), the
model-level oracle light-rocm-runtime itself uses
(tools/run_qwen_e2e.py:313-419). transformers is a third-party dependency of
that tool, not vendored in the reference; the version used is recorded in
each file.

Every model is the Qwen2.5-0.5B architecture (hidden 896, 14/2 heads,
head_dim 64, intermediate 4864, RMSNorm eps 1e-6, RoPE theta 1e6, tied
embeddings); weights come from lrrt_b200.synthetic.model(seed, layers, vocab)
and are regenerated bit-identically by the tests from the same seed.

  hf_qwen2_decode.npz   2 layers, vocab 4096: 8 greedy tokens after a
                        6-token prompt, last-step logits
  hf_qwen2_config1.npz  BASELINE config 1: one layer, vocab 151936, KV cache
                        rows 0..127 ~ N(0, 1) (seed 0), hidden ~ N(0, 1):
                        all 151936 logits of the step at position 128
  hf_qwen2_config2.npz  BASELINE config 2: 24 layers, vocab 151936, the
                        32-token seed-1 prompt: the first 32 greedy tokens and
                        the logit of each

Run: python tests/golden/make_golden.py [decode|config1|config2 ...]
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
CONFIG1 = Path(__file__).with_name("hf_qwen2_config1.npz")
CONFIG2 = Path(__file__).with_name("hf_qwen2_config2.npz")


def build_hf(layers, tail):
    import transformers
    from transformers import Qwen2Config, Qwen2ForCausalLM

    config = Qwen2Config(vocab_size=tail["lm_head"].shape[0], hidden_size=896,
                         intermediate_size=4864,
                         num_hidden_layers=len(layers), num_attention_heads=14,
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


def make_decode() -> None:
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


def make_config1() -> None:
    """One decoder step at position 128 over a cache prefilled with N(0, 1)
    rows. The cache rows are post-RoPE keys and values ([position][2 heads x
    64]), which is also what a transformers KV cache holds."""
    from transformers import DynamicCache

    layers, tail = synthetic.model(0, 1, 151936)
    keys, values = synthetic.kv_prefill(0, 1, 128)[0]
    hidden = synthetic.hidden(0)
    model, version = build_hf(layers, tail)
    cache = DynamicCache()
    as_heads = lambda a: torch.from_numpy(a.reshape(128, 2, 64).transpose(1, 0, 2)[None].copy())  # noqa: E731
    cache.update(as_heads(keys), as_heads(values), 0)
    with torch.no_grad():
        out = model(inputs_embeds=torch.from_numpy(hidden)[None, None],
                    past_key_values=cache, position_ids=torch.tensor([[128]]),
                    cache_position=torch.tensor([128]), use_cache=True)
    logits = out.logits[0, -1].numpy().astype(np.float32)
    np.savez_compressed(CONFIG1, logits=logits, transformers_version=np.array(version))
    print(f"wrote {CONFIG1}: argmax {int(np.argmax(logits))}")


def make_config2(count: int = 32) -> None:
    layers, tail = synthetic.model(1, 24, 151936)
    prompt = synthetic.prompt(1, 32, 151936)
    model, version = build_hf(layers, tail)
    tokens, maxima = [], []
    with torch.no_grad():
        out = model(torch.tensor([prompt.astype(np.int64)]), use_cache=True)
        for _ in range(count):
            logits = out.logits[0, -1]
            token = int(torch.argmax(logits))
            tokens.append(token)
            maxima.append(float(logits[token]))
            out = model(torch.tensor([[token]]), past_key_values=out.past_key_values,
                        use_cache=True)
    np.savez_compressed(CONFIG2, prompt=prompt, tokens=np.array(tokens, np.uint32),
                        max_logits=np.array(maxima, np.float32),
                        transformers_version=np.array(version))
    print(f"wrote {CONFIG2}: tokens {tokens}")


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    which = sys.argv[1:] or ["decode", "config1", "config2"]
    for name in which:
        {"decode": make_decode, "config1": make_config1, "config2": make_config2}[name]()


if __name__ == "__main__":
    main()
