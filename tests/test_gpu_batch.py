"""Right-padded batches of cached sequences through the device decoder (cppinf_qwen3_forward_batch): the reference's
Qwen3Model::forward_cached(TokenIdBatch, Qwen3Cache&) (src/models/qwen3/qwen3_model.cpp:275-311, packing at
:104-130) and its mixed-length batch test (tests/models/qwen3/qwen3_model_test.cpp:459-486), where each batch row
must equal the standalone forward of its sequence. Here the equality is bit for bit, and the standalone forward is
itself bit-exact to the CPU oracle (test_gpu_decoder.py).
"""

from __future__ import annotations

import numpy as np
import pytest

from _dev import to_host

pytestmark = pytest.mark.gpu


def small_config():
    from cppinf_b200.qwen3 import Qwen3Config

    return Qwen3Config(vocab_size=1000, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=128)


@pytest.fixture(scope="module")
def model(cuda):
    from cppinf_b200.qwen3 import Qwen3Model, random_weights

    cfg = small_config()
    return Qwen3Model(cfg, 700, random_weights(cfg, seed=11, std=0.05))


def bits(t) -> np.ndarray:
    return to_host(t).view(np.uint16)


def test_mixed_length_batch_rows_equal_standalone_forward(model):
    # the reference's case: prompts {1, 5, 3} and {1, 5}, then one more token each
    cache = model.make_cache(2, 4)
    prompt = model.forward_cached_batch([[1, 5, 3], [1, 5]], cache)
    nxt = model.forward_cached_batch([[2], [3]], cache)
    assert tuple(prompt.shape) == (2, 3, model.config.vocab_size)
    assert tuple(nxt.shape) == (2, 1, model.config.vocab_size)
    assert cache.sequence_lengths == [4, 3]
    first = bits(model.forward([1, 5, 3, 2]))
    second = bits(model.forward([1, 5, 3]))
    np.testing.assert_array_equal(bits(nxt[0]), first[3:4])
    np.testing.assert_array_equal(bits(nxt[1]), second[2:3])
    np.testing.assert_array_equal(bits(prompt[0]), first[:3])
    np.testing.assert_array_equal(bits(prompt[1, :2]), second[:2])
    assert not bits(prompt[1, 2]).any()  # right-padded row


def test_batch_spanning_chunks_equals_standalone(model):
    # 300 + 260 + 7 rows: the first chunk takes 300 rows of sequence 0 and 212 of sequence 1, the second chunk the
    # remaining 48 rows of sequence 1 (reading its first 212 from the cache) and sequence 2
    rng = np.random.default_rng(5)
    seqs = [rng.integers(0, model.config.vocab_size, n).tolist() for n in (300, 260, 7)]
    cache = model.make_cache(3, 320)
    got = model.forward_cached_batch(seqs, cache)
    assert cache.sequence_lengths == [300, 260, 7]
    for b, seq in enumerate(seqs):
        want = bits(model.forward(seq))
        np.testing.assert_array_equal(bits(got[b, :len(seq)]), want, err_msg=f"sequence {b}")
        assert not bits(got[b, len(seq):]).any()
    # a decode-like step of every sequence at once, then against the standalone forward's last row
    extra = [[int(rng.integers(0, model.config.vocab_size))] for _ in seqs]
    step = model.forward_cached_batch(extra, cache)
    for b, seq in enumerate(seqs):
        want = bits(model.forward(seq + extra[b]))
        np.testing.assert_array_equal(bits(step[b]), want[-1:], err_msg=f"step of sequence {b}")


def test_batch_equal_lengths_one_lm_head_run(model):
    # equal lengths: the logits rows of all sequences are consecutive, so the LM head runs once per chunk
    rng = np.random.default_rng(6)
    seqs = [rng.integers(0, model.config.vocab_size, 16).tolist() for _ in range(4)]
    cache = model.make_cache(4, 64)
    got = model.forward_cached_batch(seqs, cache)
    for b, seq in enumerate(seqs):
        np.testing.assert_array_equal(bits(got[b]), bits(model.forward(seq)), err_msg=f"sequence {b}")


def test_batch_validation(model):
    cache = model.make_cache(2, 8)
    with pytest.raises(ValueError, match="at least one sequence"):
        model.forward_cached_batch([], cache)
    with pytest.raises(ValueError, match="at least one token"):
        model.forward_cached_batch([[1], []], cache)
    with pytest.raises(ValueError, match="batch size must match"):
        model.forward_cached_batch([[1]], cache)
    with pytest.raises(IndexError, match="vocabulary"):
        model.forward_cached_batch([[1], [model.config.vocab_size]], cache)
    with pytest.raises(IndexError, match="too small"):
        model.forward_cached_batch([[1] * 9, [1]], cache)
    assert cache.sequence_lengths == [0, 0]  # rejected calls leave the cache as it was
    with pytest.raises(ValueError, match="non-zero"):
        model.make_cache(0, 8)
    with pytest.raises(NotImplementedError):
        model.make_cache(1, 701)  # beyond the model's rotary table
