"""The reference's attention and decoder-block goldens (tests/nn/qwen_attention_test.cpp:30-189,
tests/nn/qwen_decoder_block_test.cpp:33-213; values from its Hugging Face oracles) through this library's device ops.

Each block is composed the way the reference composes it -- linear_project (src/nn/qwen_common.cpp:15-37: matmul of
the rows by the transposed weight), per-head ops::rms_norm, apply_rope_batched (src/nn/qwen_attention.cpp:136-162),
fused_causal_attention (:237-333: permutes, GQA repeat, f32 scores, the position-causal softmax, probabilities cast
to the input dtype, P·V, permute back), the o_proj projection, and for the decoder block
(src/nn/qwen_decoder_block.cpp:65-90) the input RMSNorm, residual adds and the MLP (src/nn/qwen_mlp.cpp:58-66:
gate/up projections, ops::silu, ops::mul, down projection) -- with every op running on the device kernels
(cppinf_b200.ops: matmul, rms_norm, apply_rope, scaled_position_causal_softmax_last_dim, cast, add, silu, mul and the
strided gather for the layout changes). The cases have head sizes 4 and 2 and hidden size 6, so they exercise the
generic (non-vector) paths of those kernels. Tolerances are the reference tests' own.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _dev import to_dev, to_host
from oracle.oracle import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda):
    from cppinf_b200 import ops as _ops

    return _ops


def load_cases(golden):
    data = golden("ref_blocks")
    names = sorted({k.split("/")[0] for k in data})
    return {n: {k.split("/", 1)[1]: v for k, v in data.items() if k.startswith(n + "/")} for n in names}


def device_tensor(arr: np.ndarray, bf16: bool) -> torch.Tensor:
    return to_dev(f32_to_bf16(arr) if bf16 else arr.astype(np.float32))


def linear_project(ops, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    b, t, h = x.shape
    return ops.matmul(x.reshape(b * t, h), w.t()).reshape(b, t, w.shape[0])


def attention(ops, x, wts, heads, kv_heads, head_dim, eps):
    b, t, _ = x.shape
    q = linear_project(ops, x, wts["q_proj_weight"]).reshape(b, t, heads, head_dim)
    k = linear_project(ops, x, wts["k_proj_weight"]).reshape(b, t, kv_heads, head_dim)
    v = linear_project(ops, x, wts["v_proj_weight"]).reshape(b, t, kv_heads, head_dim)
    q = ops.rms_norm(q, wts["q_norm_weight"], eps)
    k = ops.rms_norm(k, wts["k_norm_weight"], eps)
    # apply_rope_batched: batch row i rotated at offset cache_length[i] (0: an empty cache), sequence axis 0. The
    # reference's cases are all one batch row.
    assert b == 1
    q = ops.apply_rope(q[0], 0, 1e6, 0).unsqueeze(0)
    k = ops.apply_rope(k[0], 0, 1e6, 0).unsqueeze(0)
    # An empty cache of capacity t takes the t new rows, so the cached keys/values are k and v themselves.
    rep = heads // kv_heads
    q_bh = ops.materialize(q.permute(0, 2, 1, 3)).reshape(b * heads, t, head_dim)
    k_bh = ops.materialize(k.permute(0, 2, 3, 1).unsqueeze(2).expand(b, kv_heads, rep, head_dim, t)
                           ).reshape(b * heads, head_dim, t)
    v_bh = ops.materialize(v.permute(0, 2, 1, 3).unsqueeze(2).expand(b, kv_heads, rep, t, head_dim)
                           ).reshape(b * heads, t, head_dim)
    scores = ops.matmul(q_bh, k_bh, output_dtype=torch.float32).reshape(b, heads, t, t)
    probs = ops.scaled_position_causal_softmax_last_dim(scores, 1.0 / math.sqrt(head_dim), [0] * b, [t] * b,
                                                        [t] * b)
    if x.dtype != torch.float32:
        probs = ops.cast(probs, x.dtype)
    ctx = ops.matmul(probs.reshape(b * heads, t, t), v_bh).reshape(b, heads, t, head_dim)
    ctx = ops.materialize(ctx.permute(0, 2, 1, 3)).reshape(b, t, heads * head_dim)
    return linear_project(ops, ctx, wts["o_proj_weight"])


def decoder_block(ops, x, wts, heads, kv_heads, head_dim, eps):
    h = ops.add(x, attention(ops, ops.rms_norm(x, wts["input_layernorm_weight"], eps), wts, heads, kv_heads,
                             head_dim, eps))
    m = ops.rms_norm(h, wts["post_attention_layernorm_weight"], eps)
    gated = ops.mul(ops.silu(linear_project(ops, m, wts["gate_proj_weight"])),
                    linear_project(ops, m, wts["up_proj_weight"]))
    return ops.add(h, linear_project(ops, gated, wts["down_proj_weight"]))


CASE_NAMES = [
    "GivenHfQwen3OracleF32Inputs_WhenApplyingQwenAttention_ThenExpectedValuesAreReturned",
    "GivenHfQwen3OracleGroupedKvInputs_WhenApplyingQwenAttention_ThenExpectedValuesAreReturned",
    "GivenHfQwen3OracleBf16Inputs_WhenApplyingQwenAttention_ThenExpectedValuesAreReturned",
    "GivenHfQwen3OracleF32Inputs_WhenApplyingQwenDecoderBlock_ThenExpectedValuesAreReturned",
    "GivenHfQwen3OracleBf16Inputs_WhenApplyingQwenDecoderBlock_ThenExpectedValuesAreReturned",
]


@pytest.mark.parametrize("name", CASE_NAMES)
def test_reference_block_golden_through_device_ops(ops, golden, name):
    case = load_cases(golden)[name]
    kind, dtype, heads, kv_heads, head_dim, seq, eps, tol = case["meta"]
    bf16 = dtype == 1
    wts = {k: device_tensor(v, bf16) for k, v in case.items() if k not in ("meta", "expected")}
    x = wts.pop("hidden_states")
    assert x.shape[1] == int(seq)
    block = attention if kind == 0 else decoder_block
    out = block(ops, x, wts, int(heads), int(kv_heads), int(head_dim), float(eps))
    got = to_host(out[0])
    got = bf16_to_f32(got) if bf16 else got
    np.testing.assert_allclose(got.ravel(), case["expected"], rtol=0, atol=float(tol))


def test_block_golden_fixture_holds_every_reference_case(golden):
    cases = load_cases(golden)
    assert sorted(cases) == sorted(CASE_NAMES)
    for c in cases.values():
        assert c["expected"].size == c["hidden_states"].shape[1] * c["hidden_states"].shape[2]
