"""Generates the golden fixtures that pin the Qwen3 decoder oracle (oracle/qwen3.py).

Two sources, both the reference's own:

1. ``qwen3_tiny_reference.npz`` -- the tiny bf16 checkpoint and the expected logits of the reference's model tests
   (tests/models/qwen3/qwen3_model_test.cpp:59-320: a 2-layer model with hidden 6, 2 query / 1 key-value heads of
   4, MLP 10, vocab 13; forward of [1, 5, 3, 2] and the cached forward of [1, 5, 3] then [2]), read from the test
   source as text. The reference accepts its own model within 0.05 of these values (its
   expect_float_values_near tolerance).
2. ``qwen3_hf_small.npz`` -- logits of Hugging Face ``Qwen3ForCausalLM`` in bf16 with eager attention, the oracle
   the reference generates its model goldens with (tests/models/qwen3/qwen3_model_oracle.py), on a small random
   checkpoint with the Qwen3-0.6B head geometry (head_dim 128, 2:1 grouped-query attention). The weights are
   ``cppinf_b200.qwen3.random_weights(config, seed)``, so only the logits are stored.

Run from the repository root:  python tests/golden/make_decoder_golden.py [path-to-reference-checkout]
(transformers 5.5 and torch 2.11 here; the reference pins transformers 4.52.3 for its oracle.)
"""

from __future__ import annotations

import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from cppinf_b200.qwen3 import Qwen3Config, f32_to_bf16_bits, random_weights  # noqa: E402

NUMBER = re.compile(r"-?\d+(?:\.\d*)?(?:e-?\d+)?f")

TINY = Qwen3Config(vocab_size=13, hidden_size=6, intermediate_size=10, num_hidden_layers=2, num_attention_heads=2,
                   num_key_value_heads=1, head_dim=4, rms_norm_eps=1e-6, rope_theta=1_000_000.0)

HF_SMALL = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=128)
HF_SEED = 7
HF_STD = 0.05
HF_TOKENS = [3, 141, 59, 265, 358, 97, 93, 238, 462, 64, 33, 83, 279, 502, 88, 41, 97, 169, 399, 375]


def _balanced(text: str, start: int) -> tuple[str, int]:
    """The brace block starting at text[start] == '{' and the index after it."""
    depth = 0
    for i in range(start, len(text)):
        if text[i] == "{":
            depth += 1
        elif text[i] == "}":
            depth -= 1
            if depth == 0:
                return text[start:i + 1], i + 1
    raise ValueError("unbalanced braces")


def _floats(block: str) -> np.ndarray:
    return np.array([float(m[:-1]) for m in NUMBER.findall(block)], dtype=np.float32)


def parse_tiny(test_source: str) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    for m in re.finditer(r'append_bf16_(matrix|vector)\(\s*header,\s*tensor_data,\s*"([^"]+)",', test_source):
        kind, name = m.group(1), m.group(2)
        block, _ = _balanced(test_source, test_source.index("{", m.end()))
        values = _floats(block)
        if kind == "matrix":
            rows = block.count("{") - 1
            values = values.reshape(rows, -1)
        out[name] = f32_to_bf16_bits(values)
    expected = set(TINY.weight_shapes())
    assert set(out) == expected, sorted(set(out) ^ expected)
    for name, shape in TINY.weight_shapes().items():
        assert out[name].shape == shape, (name, out[name].shape, shape)
    return out


def parse_expected(test_source: str, test_name: str) -> np.ndarray:
    start = test_source.index(test_name)
    call = test_source.index("expect_float_values_near(", start)
    block, _ = _balanced(test_source, test_source.index("{", call))
    return _floats(block)


def make_tiny(reference: Path) -> None:
    src = (reference / "tests/models/qwen3/qwen3_model_test.cpp").read_text()
    weights = parse_tiny(src)
    forward = parse_expected(src, "GivenTinyBf16Checkpoint_WhenRunningForward_ThenExpectedLogitsAreReturned")
    cached = parse_expected(src, "GivenTinyBf16Checkpoint_WhenRunningCachedForward_ThenLastTokenMatchesFullForward")
    assert forward.size == 4 * 13 and cached.size == 13
    np.savez_compressed(HERE / "qwen3_tiny_reference.npz", forward_tokens=np.array([1, 5, 3, 2]),
                        forward_logits=forward.reshape(4, 13), cached_prompt=np.array([1, 5, 3]),
                        cached_next=np.array([2]), cached_logits=cached.reshape(1, 13), tolerance=np.float32(0.05),
                        **{"w:" + k: v for k, v in weights.items()})
    print("wrote", HERE / "qwen3_tiny_reference.npz")


def make_hf_small() -> None:
    import torch
    from transformers import Qwen3Config as HfQwen3Config
    from transformers import Qwen3ForCausalLM

    c = HF_SMALL
    hf_cfg = HfQwen3Config(vocab_size=c.vocab_size, hidden_size=c.hidden_size,
                           intermediate_size=c.intermediate_size, num_hidden_layers=c.num_hidden_layers,
                           num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                           head_dim=c.head_dim, max_position_embeddings=64, rms_norm_eps=c.rms_norm_eps,
                           rope_parameters={"rope_type": "default", "rope_theta": c.rope_theta},
                           tie_word_embeddings=True, use_sliding_window=False,
                           attn_implementation="eager")
    model = Qwen3ForCausalLM(hf_cfg).eval().to(torch.bfloat16)
    weights = random_weights(c, HF_SEED, HF_STD)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name, bits in weights.items():
            t = torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)
            params[name].copy_(t)
        model.tie_weights()
        # Module.to(bfloat16) also rounds the rotary inverse frequencies to bf16, which shifts RoPE angles by up to
        # 2^-9 relative; the reference computes them in f32 (src/nn/rope.cpp), so they are restored in f32.
        rotary = model.model.rotary_emb
        expected = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float32) / c.head_dim))
        assert torch.allclose(rotary.inv_freq.float(), expected, rtol=1e-2), "rope theta not applied"
        rotary.inv_freq = expected
        logits = model(input_ids=torch.tensor([HF_TOKENS]), use_cache=False).logits[0]
    bits = logits.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    np.savez_compressed(HERE / "qwen3_hf_small.npz", tokens=np.array(HF_TOKENS), logits=bits,
                        seed=np.int64(HF_SEED), std=np.float32(HF_STD))
    print("wrote", HERE / "qwen3_hf_small.npz")


if __name__ == "__main__":
    # The reference tree: the first argument, else $CPPINF_REFERENCE_DIR, else where oracle/Makefile compiled it from.
    sys.path.insert(0, str(HERE.parent.parent))
    from oracle.oracle import reference_tree

    reference = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_tree()
    if reference is None:
        sys.exit("usage: make_decoder_golden.py <reference tree> (or set CPPINF_REFERENCE_DIR)")
    make_tiny(reference)
    make_hf_small()
