"""Failure detection on the device, without a GPU fault.

The decoder's kernels that stage weights or cached rows by bulk copies wait on a shared-memory barrier with a poll
limit. These tests set the limit to 0 through cppinf_set_wait_poll_limit, so every first wait gives up at once while
the copies still land (the cleanup wait keeps the default limit), and check that the error reaches the host: a
decode step returns CPPINF_ERR_CUDA and the model refuses work until reset. Restoring the limit brings back tokens
equal to the oracle's.
"""

from __future__ import annotations

import numpy as np
import pytest


pytestmark = pytest.mark.gpu


@pytest.fixture()
def capi(cuda):
    from cppinf_b200 import capi as _capi

    yield _capi
    _capi.set_wait_poll_limit(_capi.DEFAULT_POLL_LIMIT)


def test_poll_limit_setter_returns_previous(capi):
    assert capi.set_wait_poll_limit(5) == capi.DEFAULT_POLL_LIMIT
    assert capi.set_wait_poll_limit(capi.DEFAULT_POLL_LIMIT) == 5


def test_decode_wait_that_runs_out_returns_error_until_reset(capi, oracle):
    from cppinf_b200.qwen3 import Qwen3Config, Qwen3Model, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128)
    weights = random_weights(cfg, seed=7, std=0.05)
    prompt = np.random.default_rng(8).integers(0, cfg.vocab_size, 20)
    model = Qwen3Model(cfg, 64, weights)
    try:
        want = OracleQwen3(cfg, weights, 64, oracle).generate(prompt, 6)
        assert model.generate(prompt, 6) == want  # captures the step graph with the default limit
        model.reset()
        capi.set_wait_poll_limit(0)
        model.forward_cached(prompt, logits=None)
        with pytest.raises(RuntimeError, match="poll limit"):
            model.decode(3)  # the step graph is captured again with limit 0
        with pytest.raises(RuntimeError, match="reset"):
            model.decode(1)
        with pytest.raises(RuntimeError, match="reset"):
            model.forward_cached(prompt[:2], logits=None)
        capi.set_wait_poll_limit(capi.DEFAULT_POLL_LIMIT)
        model.reset()
        assert model.generate(prompt, 6) == want
    finally:
        model.close()
