"""The decoder oracle (oracle/qwen3.py over oracle/oracle.c) pinned to the reference's golden logits and to Hugging
Face Qwen3, plus the host-side validation of the decoder's C ABI. CPU only.

Pins:
- tests/golden/qwen3_tiny_reference.npz: the reference's own tiny bf16 checkpoint and expected logits
  (tests/models/qwen3/qwen3_model_test.cpp:295-345), accepted within the reference's tolerance of 0.05;
- tests/golden/qwen3_hf_small.npz: Hugging Face Qwen3ForCausalLM (bf16, eager attention; the reference's model
  oracle, tests/models/qwen3/qwen3_model_oracle.py) at the Qwen3-0.6B head geometry, within 2 bf16 ulps at the
  logits' magnitude (0.0625) and 0.01 on average.
The fixed accumulation orders (linear, attention, exp) are checked against float64 restatements.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from oracle.oracle import bf16_to_f32, f32_to_bf16
from oracle.qwen3 import OracleQwen3


def test_pexp_accuracy_and_special_values(oracle):
    x = np.linspace(-103.0, 88.7, 400_001, dtype=np.float32)
    got = oracle.pexp(x).astype(np.float64)
    exact = np.exp(x.astype(np.float64))
    normal = exact > 1.2e-38
    ulp = np.spacing(exact[normal].astype(np.float32)).astype(np.float64)
    assert (np.abs(got[normal] - exact[normal]) / ulp).max() <= 1.25
    special = oracle.pexp(np.array([0.0, -0.0, 89.0, -105.0, np.inf, -np.inf, np.nan], np.float32))
    assert special[0] == 1.0 and special[1] == 1.0
    assert np.isinf(special[2]) and special[3] == 0.0 and np.isinf(special[4]) and special[5] == 0.0
    assert np.isnan(special[6])


def test_linear_canonical_close_to_exact_and_row_independent(oracle):
    rng = np.random.default_rng(0)
    x = f32_to_bf16(rng.standard_normal((70, 1024)).astype(np.float32))
    w = f32_to_bf16((rng.standard_normal((96, 1024)) * 0.05).astype(np.float32))
    y = oracle.linear_canonical(x, w)
    exact = bf16_to_f32(x).astype(np.float64) @ bf16_to_f32(w).astype(np.float64).T
    # one bf16 rounding of an f32 sum: within 1 bf16 ulp of the exact value (+ f32 accumulation slack)
    assert (np.abs(bf16_to_f32(y) - exact) <= np.abs(exact) * 2.0 ** -8 + 1e-4).all()
    # the single-row path and the 64-row blocks give identical bits
    for r in (0, 63, 64, 69):
        assert (oracle.linear_canonical(x[r:r + 1], w) == y[r:r + 1]).all()
    # K not a multiple of 8: one element per lane step
    xs, ws = x[:, :13].copy(), w[:, :13].copy()
    ys = oracle.linear_canonical(xs, ws)
    exact = bf16_to_f32(xs).astype(np.float64) @ bf16_to_f32(ws).astype(np.float64).T
    assert (np.abs(bf16_to_f32(ys) - exact) <= np.abs(exact) * 2.0 ** -8 + 1e-6).all()


def attention_f64(q, kc, vc, pos0):
    t, hq, d = q.shape
    hkv = kc.shape[1]
    qf, kf, vf = (bf16_to_f32(a).astype(np.float64) for a in (q, kc, vc))
    out = np.zeros((t, hq, d))
    for i in range(t):
        n = pos0 + i + 1
        for h in range(hq):
            g = h // (hq // hkv)
            s = kf[:n, g] @ qf[i, h] / math.sqrt(d)
            p = np.exp(s - s.max())
            out[i, h] = (p / p.sum()) @ vf[:n, g]
    return out


@pytest.mark.parametrize("t,pos0,hq,hkv,d", [(1, 0, 2, 1, 128), (1, 50, 4, 2, 128), (6, 10, 4, 2, 64),
                                             (3, 0, 2, 1, 4)])
def test_decoder_attention_close_to_exact(oracle, t, pos0, hq, hkv, d):
    rng = np.random.default_rng(t + pos0 + d)
    cap = pos0 + t + 3
    q = f32_to_bf16(rng.standard_normal((t, hq, d)).astype(np.float32))
    kc = f32_to_bf16(rng.standard_normal((cap, hkv, d)).astype(np.float32))
    vc = f32_to_bf16(rng.standard_normal((cap, hkv, d)).astype(np.float32))
    got = bf16_to_f32(oracle.decoder_attention(q, kc, vc, pos0))
    want = attention_f64(q, kc, vc, pos0)
    # bf16 probabilities and a bf16 result: a few bf16 ulps of the largest |v|
    assert np.abs(got - want).max() <= 0.03


def tiny_model(golden, oracle):
    from golden.make_decoder_golden import TINY

    fx = golden("qwen3_tiny_reference")
    weights = {k[2:]: v for k, v in fx.items() if k.startswith("w:")}
    return fx, OracleQwen3(TINY, weights, 8, oracle)


def test_tiny_reference_forward_logits(golden, oracle):
    # tests/models/qwen3/qwen3_model_test.cpp:295-320
    fx, model = tiny_model(golden, oracle)
    logits = bf16_to_f32(model.forward_cached(fx["forward_tokens"], all_logits=True))
    assert logits.shape == (4, 13)
    assert np.abs(logits - fx["forward_logits"]).max() <= float(fx["tolerance"])


def test_tiny_reference_cached_forward(golden, oracle):
    # tests/models/qwen3/qwen3_model_test.cpp:322-345: [1, 5, 3] then [2]; the last row matches the full forward
    fx, model = tiny_model(golden, oracle)
    model.forward_cached(fx["cached_prompt"])
    nxt = bf16_to_f32(model.forward_cached(fx["cached_next"]))
    assert model.length == 4
    assert np.abs(nxt - fx["cached_logits"]).max() <= float(fx["tolerance"])


def test_hf_small_logits(golden, oracle):
    from cppinf_b200.qwen3 import random_weights
    from golden.make_decoder_golden import HF_SMALL

    fx = golden("qwen3_hf_small")
    weights = random_weights(HF_SMALL, int(fx["seed"]), float(fx["std"]))
    model = OracleQwen3(HF_SMALL, weights, 32, oracle)
    got = bf16_to_f32(model.forward_cached(fx["tokens"], all_logits=True))
    want = bf16_to_f32(fx["logits"])
    diff = np.abs(got - want)
    assert diff.max() <= 0.0625 and diff.mean() <= 0.01
    # the cached path (prefill 12, then one token at a time) gives the same bits as the full forward
    model.reset()
    rows = [model.forward_cached(fx["tokens"][:12], all_logits=True)]
    rows += [model.forward_cached([t]) for t in fx["tokens"][12:]]
    assert (np.concatenate(rows) == f32_to_bf16(got)).all()


def test_random_weights_reproducible():
    from cppinf_b200.qwen3 import Qwen3Config, random_weights

    cfg = Qwen3Config(vocab_size=50, hidden_size=16, intermediate_size=24, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=8)
    a, b = random_weights(cfg, 3), random_weights(cfg, 3)
    assert set(a) == set(cfg.weight_shapes()) and all((a[k] == b[k]).all() for k in a)
    assert (a["model.norm.weight"] == 0x3F80).all()
    assert abs(bf16_to_f32(a["model.embed_tokens.weight"]).std() - 0.02) < 0.003
    assert Qwen3Config.qwen3_0_6b().parameter_count() == 596_049_920


# ---- C ABI host-side validation (no device work is issued) ---------------------------------------------------


@pytest.fixture(scope="module")
def capi():
    from cppinf_b200 import capi as _capi

    _capi.load()
    return _capi


def test_linear_validation(capi):
    lib = capi.load()
    assert lib.cppinf_linear(None, 12, None, None, 2, 12, 4, None) == capi.ERR_UNSUPPORTED
    assert "multiple of 8" in capi.last_error()
    assert lib.cppinf_linear(None, 8, None, None, 2, 0, 4, None) == capi.ERR_INVALID_ARGUMENT
    assert lib.cppinf_linear(None, 8, None, None, 0, 8, 4, None) == capi.OK
    assert lib.cppinf_linear(None, 8, None, None, 2, 8, 4, None) == capi.ERR_INVALID_ARGUMENT
    assert lib.cppinf_linear(None, 8192, None, None, 2, 8192, 4, None) == capi.ERR_UNSUPPORTED
    assert lib.cppinf_linear_argmax_scratch_bytes(151936, 1024) >= 16 + 8


def test_attention_validation(capi):
    lib = capi.load()
    assert lib.cppinf_decoder_attention(None, None, None, None, 1, 3, 2, 128, 0, 8, None) == capi.ERR_INVALID_ARGUMENT
    assert lib.cppinf_decoder_attention(None, None, None, None, 1, 4, 2, 96, 0, 8, None) == capi.ERR_UNSUPPORTED
    assert lib.cppinf_decoder_attention(None, None, None, None, 4, 4, 2, 128, 5, 8, None) == capi.ERR_OUT_OF_RANGE
    assert lib.cppinf_decoder_attention(None, None, None, None, 0, 4, 2, 128, 5, 8, None) == capi.OK


def test_qwen3_create_validation(capi):
    lib = capi.load()
    handle = ctypes.c_void_p()

    def create(**kw):
        base = dict(vocab_size=100, hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                    num_attention_heads=2, num_key_value_heads=1, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6)
        base.update(kw)
        cfg = capi.Qwen3ConfigC(*base.values())
        return lib.cppinf_qwen3_create(ctypes.byref(cfg), 16, ctypes.byref(handle))

    assert create(num_attention_heads=3, num_key_value_heads=2) == capi.ERR_INVALID_ARGUMENT
    assert "divide" in capi.last_error()
    assert create(num_hidden_layers=0) == capi.ERR_INVALID_ARGUMENT
    assert create(head_dim=4) == capi.ERR_UNSUPPORTED
    assert create(hidden_size=6) == capi.ERR_UNSUPPORTED
    assert handle.value is None
