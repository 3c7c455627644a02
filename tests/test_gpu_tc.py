"""The tensor-core projections (cppinf_linear_tc: tcgen05.mma with TMA-staged tiles) against the CUDA-core ones
(cppinf_linear / _residual / _silu_mul, bit-exact to the oracle's restated order).

The tensor cores accumulate in f32 in an order of their own, so the comparison is to tolerance. Two f32 sums of the
same K products, in any two orders, differ by at most 2 K u sum|x_i w_i| (u = 2^-24), and bf16 rounding is monotone,
so the bounds per epilogue are (ulp() = bf16 spacing at that magnitude, S = 2 K u sum|x_i w_i| of the output):
- store:    |tc - ref| <= S + ulp(ref);
- residual: |tc - ref| <= S + ulp(bf16(x w^T)) + ulp(ref);
- SiLU*up:  with g, u the two projections and s = silu(g) (|silu'| <= 1.1):
            |tc - ref| <= |u| (1.1 (S_g + ulp(g)) + ulp(s)) + |s| (S_u + ulp(u)) + ulp(ref).
The share of bit-identical elements is checked too (the orders agree to ~1e-6 relative on these inputs).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _dev import seeded_bf16, to_dev, to_host
from oracle.oracle import bf16_to_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi(cuda):
    from cppinf_b200 import capi as _capi

    return _capi


def ulp(x: np.ndarray) -> np.ndarray:
    """bf16 unit in the last place at magnitude |x| (the spacing of bf16 values there)."""
    a = np.maximum(np.abs(x.astype(np.float32)), np.float32(2.0 ** -126))
    return np.exp2(np.floor(np.log2(a)) - 7).astype(np.float32)


def run(capi, epi, x, w0, w1=None, residual=None, error=None):
    rows, k = x.shape
    n = w0.shape[0]
    y = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    capi.call("cppinf_linear_tc", epi, x.data_ptr(), k, w0.data_ptr(), 0 if w1 is None else w1.data_ptr(),
              0 if residual is None else residual.data_ptr(), y.data_ptr(), rows, k, n,
              0 if error is None else error.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return y


def reference(capi, epi, x, w0, w1=None, residual=None):
    rows, k = x.shape
    n = w0.shape[0]
    y = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    if epi == 0:
        capi.call("cppinf_linear", x.data_ptr(), k, w0.data_ptr(), y.data_ptr(), rows, k, n, s)
    elif epi == 1:
        capi.call("cppinf_linear_residual", x.data_ptr(), k, w0.data_ptr(), residual.data_ptr(), y.data_ptr(), rows, k,
                  n, s)
    else:
        capi.call("cppinf_linear_silu_mul", x.data_ptr(), k, w0.data_ptr(), w1.data_ptr(), y.data_ptr(), rows, k, n, s)
    return y


# (rows, out, in): the smallest tile, a K tail (136 = 2 * 64 + 8), an M tail of a prompt chunk, and the Qwen3-0.6B
# prefill shapes of each epilogue (512 rows: q|k|v 1024 -> 4096, o_proj 2048 -> 1024, gate/up 1024 -> 3072,
# down 3072 -> 1024).
SHAPES = {
    0: [(128, 32, 64), (200, 96, 136), (88, 1024, 1024), (512, 4096, 1024)],
    1: [(128, 64, 64), (88, 1024, 3072), (512, 1024, 2048), (512, 1024, 3072)],
    2: [(128, 32, 64), (200, 96, 136), (512, 3072, 1024)],
}


@pytest.mark.parametrize("epi,rows,n,k", [(e, *s) for e, shapes in SHAPES.items() for s in shapes])
def test_linear_tc_matches_cuda_core_within_tolerance(capi, epi, rows, n, k):
    rng = np.random.default_rng(rows * 7 + n * 3 + k + epi)
    x = to_dev(seeded_bf16(rng, (rows, k), 0, 1))
    w0 = to_dev(seeded_bf16(rng, (n, k), 0, 0.05))
    w1 = to_dev(seeded_bf16(rng, (n, k), 0, 0.05)) if epi == 2 else None
    res = to_dev(seeded_bf16(rng, (rows, n), 0, 1)) if epi == 1 else None
    got = bf16_to_f32(to_host(run(capi, epi, x, w0, w1, res)))
    want = bf16_to_f32(to_host(reference(capi, epi, x, w0, w1, res)))
    assert np.isfinite(got).all()
    err = np.abs(got - want)

    def order_bound(w):  # 2 K u sum |x_i w_i| per output
        return (2 * k * 2.0 ** -24) * (x.float().abs() @ w.float().abs().T).cpu().numpy()

    if epi == 0:
        bound = order_bound(w0) + ulp(want)
    elif epi == 1:
        prod = bf16_to_f32(to_host(reference(capi, 0, x, w0)))
        bound = order_bound(w0) + ulp(prod) + ulp(want)
    else:
        g = bf16_to_f32(to_host(reference(capi, 0, x, w0)))
        u = bf16_to_f32(to_host(reference(capi, 0, x, w1)))
        sg = g / (1.0 + np.exp(-g.astype(np.float64)))
        bound = (np.abs(u) * (1.1 * (order_bound(w0) + ulp(g)) + ulp(sg)) + np.abs(sg) * (order_bound(w1) + ulp(u))
                 + ulp(want))
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"at {worst}: tc {got[worst]} vs {want[worst]}, bound {bound[worst]}"
    assert (got == want).mean() > 0.8


def test_linear_tc_in_place_residual(capi):
    rng = np.random.default_rng(5)
    x = to_dev(seeded_bf16(rng, (256, 512), 0, 1))
    w = to_dev(seeded_bf16(rng, (256, 512), 0, 0.05))
    h = to_dev(seeded_bf16(rng, (256, 256), 0, 1))
    want = bf16_to_f32(to_host(reference(capi, 1, x, w, residual=h)))
    capi.call("cppinf_linear_tc", 1, x.data_ptr(), 512, w.data_ptr(), 0, h.data_ptr(), h.data_ptr(), 256, 512, 256, 0,
              torch.cuda.current_stream().cuda_stream)
    got = bf16_to_f32(to_host(h))
    prod = bf16_to_f32(to_host(reference(capi, 0, x, w)))
    order = (2 * 512 * 2.0 ** -24) * (x.float().abs() @ w.float().abs().T).cpu().numpy()
    assert (np.abs(got - want) <= order + ulp(prod) + ulp(want)).all()


def test_linear_tc_rejects_unsupported_layouts(capi):
    x = torch.zeros((128, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((48, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):
        run(capi, 0, x, w)  # 48 outputs: not a multiple of 32
    with pytest.raises(ValueError):
        run(capi, 3, x, w)


def test_linear_tc_wait_that_runs_out_sets_error(capi):
    rng = np.random.default_rng(9)
    x = to_dev(seeded_bf16(rng, (256, 1024), 0, 1))
    w = to_dev(seeded_bf16(rng, (512, 1024), 0, 0.05))
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    capi.set_wait_poll_limit(0)
    try:
        run(capi, 0, x, w, error=error)
        torch.cuda.synchronize()
    finally:
        capi.set_wait_poll_limit(capi.DEFAULT_POLL_LIMIT)
    assert int(error.item()) == 1
    error.zero_()
    got = bf16_to_f32(to_host(run(capi, 0, x, w, error=error)))
    want = bf16_to_f32(to_host(reference(capi, 0, x, w)))
    assert int(error.item()) == 0
    order = (2 * 1024 * 2.0 ** -24) * (x.float().abs() @ w.float().abs().T).cpu().numpy()
    assert (np.abs(got - want) <= order + ulp(want)).all()


def test_model_prefill_on_tensor_cores_within_logit_tolerance(cuda, oracle):
    # Prompt projections on the tensor cores: every logit row within 0.0625 of the oracle's (the bound the reference's
    # Hugging Face model oracle uses for bf16 logits, tests/models/qwen3/qwen3_model_oracle.py; its tiny-model test
    # uses 0.05 at logits about ten times smaller); switching back restores the bit-exact default.
    from cppinf_b200.qwen3 import Qwen3Config, Qwen3Model, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128)
    w = random_weights(cfg, seed=31, std=0.05)
    tokens = np.random.default_rng(6).integers(0, cfg.vocab_size, 300)
    model = Qwen3Model(cfg, 400, w)
    try:
        model.set_prefill("tensor_cores")
        got = bf16_to_f32(to_host(model.forward(tokens)))
        ref = OracleQwen3(cfg, w, 400, oracle)
        want = bf16_to_f32(ref.forward_cached(tokens, all_logits=True))
        assert np.abs(got - want).max() <= 0.0625, np.abs(got - want).max()
        model.set_prefill("cuda_cores")
        model.reset()
        assert np.array_equal(bf16_to_f32(to_host(model.forward(tokens))), want)  # the default is bit-exact again
        with pytest.raises(ValueError):
            model.set_prefill("fp8")
    finally:
        model.close()


def attention_inputs(rng, t, pos, cap, hq, hkv):
    q = to_dev(seeded_bf16(rng, (t, hq, 128), 0, 1))
    kc = to_dev(seeded_bf16(rng, (cap, hkv, 128), 0, 1))
    vc = to_dev(seeded_bf16(rng, (cap, hkv, 128), 0, 1))
    return q, kc, vc


def run_attention(capi, name, q, kc, vc, t, pos, cap, hq, hkv, error=None):
    ctx = torch.empty((t, hq, 128), dtype=torch.bfloat16, device="cuda")
    args = [q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ctx.data_ptr(), t, hq, hkv, 128, pos, cap]
    if name == "cppinf_decoder_attention_tc":
        args.append(0 if error is None else error.data_ptr())
    capi.call(name, *args, torch.cuda.current_stream().cuda_stream)
    return bf16_to_f32(to_host(ctx))


# (queries, position of query 0, cache rows, q heads, kv heads): the 512-query prompt chunk of Qwen3-0.6B, the second
# chunk of a 600-token prompt, one query, odd sizes across key tiles, and 4:1 grouped-query heads.
ATTN_SHAPES = [(512, 0, 640, 16, 8), (88, 512, 640, 16, 8), (1, 100, 256, 16, 8), (130, 37, 300, 4, 2),
               (200, 0, 200, 8, 2)]


@pytest.mark.parametrize("t,pos,cap,hq,hkv", ATTN_SHAPES)
def test_attention_tc_matches_restated_attention_within_tolerance(capi, t, pos, cap, hq, hkv):
    # Contexts are weighted means of bf16 V rows; the tensor cores' score sums, the running softmax sum and bf16
    # probabilities that round the other way move them by a few bf16 ulps at most. Bound: 0.02, the reference's own
    # bf16 attention tolerance (tests/nn/qwen_attention_test.cpp:184-189), and a mean error far below it.
    rng = np.random.default_rng(t * 31 + pos)
    q, kc, vc = attention_inputs(rng, t, pos, cap, hq, hkv)
    want = run_attention(capi, "cppinf_decoder_attention", q, kc, vc, t, pos, cap, hq, hkv)
    got = run_attention(capi, "cppinf_decoder_attention_tc", q, kc, vc, t, pos, cap, hq, hkv)
    assert np.isfinite(got).all()
    err = np.abs(got - want)
    assert err.max() <= 0.02, err.max()
    assert err.mean() <= 2e-3, err.mean()


def test_attention_tc_wait_that_runs_out_sets_error_and_completes(capi):
    rng = np.random.default_rng(12)
    q, kc, vc = attention_inputs(rng, 256, 0, 300, 8, 4)
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = run_attention(capi, "cppinf_decoder_attention", q, kc, vc, 256, 0, 300, 8, 4)
    capi.set_wait_poll_limit(0)
    try:
        got = run_attention(capi, "cppinf_decoder_attention_tc", q, kc, vc, 256, 0, 300, 8, 4, error=error)
    finally:
        capi.set_wait_poll_limit(capi.DEFAULT_POLL_LIMIT)
    assert int(error.item()) == 1
    # every wait then waits again with the default limit, so the protocol completes and the result stands
    assert np.abs(got - want).max() <= 0.02
