"""Parity of the device decoder (projections, attention, the Qwen3 model) with the CPU oracle, through the C ABI.

The oracle restates the device decoder's accumulation orders (oracle/oracle.c: oracle_linear_canonical,
oracle_decoder_attention, oracle_pexp) and is pinned to the reference's tiny-model golden logits and to Hugging
Face Qwen3 logits (tests/test_decoder_oracle.py). Every comparison here is bit for bit: logits, contexts and greedy
tokens.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _dev import seeded_bf16, to_dev, to_host
from oracle.oracle import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda):
    from cppinf_b200 import ops as _ops

    return _ops


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str):
    assert got.shape == want.shape, (got.shape, want.shape)
    bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
    assert bad.size == 0, (f"{what}: {bad.size} of {want.size} differ; first at {bad[0]}: "
                           f"{bf16_to_f32(got.reshape(-1)[bad[:4]])} vs {bf16_to_f32(want.reshape(-1)[bad[:4]])}")


# ---------------------------------------------------------------------------------------------------------------
# Projections
# ---------------------------------------------------------------------------------------------------------------

LINEAR_SHAPES = [
    (1, 1024, 4096),   # decode q|k|v
    (1, 2048, 1024),   # decode o_proj
    (1, 3072, 1024),   # decode down_proj
    (1, 8, 5),         # one chunk
    (1, 264, 77),      # chunks not a multiple of 32 lanes
    (3, 1024, 300),
    (16, 512, 64),
    (37, 3072, 128),   # partial tile
    (512, 1024, 256),  # prefill
    (21, 1024, 77),    # odd number of outputs: a warp's second weight row is past the end
    (20, 4096, 33),    # K past the f32 tile: bf16 staging
]


@pytest.mark.parametrize("m,k,n", LINEAR_SHAPES)
def test_linear_bit_exact(ops, oracle, m, k, n):
    rng = np.random.default_rng(1000 + m + k + n)
    x = seeded_bf16(rng, (m, k))
    w = seeded_bf16(rng, (n, k), std=0.05)
    got = to_host(ops.linear(to_dev(x), to_dev(w)))
    assert_bits_equal(got, oracle.linear_canonical(x, w), "linear")


@pytest.mark.parametrize("m,k,n", [(1, 1024, 64), (16, 1024, 64), (1, 264, 9)])
def test_linear_subnormal_products_bit_exact(ops, oracle, m, k, n):
    # Operands scaled by 2^-70: every product lies near 2^-140, where a separately rounded product would lose bits
    # and only the fused multiply-add keeps them. Device (fma.rn.f32.bf16) and oracle (fmaf) still agree bit for
    # bit, in the bf16 projection and in the f32 output of the generic matmul.
    rng = np.random.default_rng(31 + m + k)
    scale = np.float32(2.0**-70)
    x = f32_to_bf16(bf16_to_f32(seeded_bf16(rng, (m, k))) * scale)
    w = f32_to_bf16(bf16_to_f32(seeded_bf16(rng, (n, k))) * scale)
    assert_bits_equal(to_host(ops.linear(to_dev(x), to_dev(w))), oracle.linear_canonical(x, w), "tiny linear")
    got = to_host(ops.matmul(to_dev(x), to_dev(w).t(), output_dtype=torch.float32))
    want = oracle.linear_canonical(x, w, f32_out=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.any(want != 0) and np.all(np.abs(want) < 2.0**-120)  # the case is really in the subnormal range


def test_linear_strided_rows(ops, oracle):
    rng = np.random.default_rng(7)
    big = seeded_bf16(rng, (9, 1032))
    w = seeded_bf16(rng, (40, 1024), std=0.05)
    got = to_host(ops.linear(to_dev(big)[:, 8:], to_dev(w)))  # materialised, then dense rows
    assert_bits_equal(got, oracle.linear_canonical(np.ascontiguousarray(big[:, 8:]), w), "strided linear")


@pytest.mark.parametrize("m,k,n", [(1, 1024, 1024), (1, 3072, 1024), (19, 2048, 256), (5, 1024, 131)])
def test_linear_residual_bit_exact(ops, oracle, m, k, n):
    rng = np.random.default_rng(m * 7 + k)
    x = seeded_bf16(rng, (m, k))
    w = seeded_bf16(rng, (n, k), std=0.03)
    res = seeded_bf16(rng, (m, n))
    want = oracle.add(res, oracle.linear_canonical(x, w))
    got = to_host(ops.linear_residual(to_dev(x), to_dev(w), to_dev(res)))
    assert_bits_equal(got, want, "linear_residual")
    # in place on the residual, as the decoder uses it
    r = to_dev(res)
    ops.linear_residual(to_dev(x), to_dev(w), r, out=r)
    assert_bits_equal(to_host(r), want, "linear_residual in place")


@pytest.mark.parametrize("m,k,n", [(1, 1024, 3072), (1, 256, 100), (24, 1024, 512)])
def test_linear_silu_mul_bit_exact(ops, oracle, m, k, n):
    rng = np.random.default_rng(m + 3 * n)
    x = seeded_bf16(rng, (m, k))
    g = seeded_bf16(rng, (n, k), std=0.08)
    u = seeded_bf16(rng, (n, k), std=0.08)
    want = oracle.silu_mul_pexp(oracle.linear_canonical(x, g), oracle.linear_canonical(x, u))
    got = to_host(ops.linear_silu_mul(to_dev(x), to_dev(g), to_dev(u)))
    assert_bits_equal(got, want, "linear_silu_mul")


@pytest.mark.parametrize("k,n", [(1024, 151936), (1024, 1000), (64, 7), (256, 40000)])
def test_linear_argmax_matches_oracle(ops, oracle, k, n):
    rng = np.random.default_rng(k + n)
    x = seeded_bf16(rng, (1, k))
    w = seeded_bf16(rng, (n, k), std=0.02)
    logits = oracle.linear_canonical(x, w)
    token, got_logits = ops.linear_argmax(to_dev(x), to_dev(w), with_logits=True)
    assert_bits_equal(to_host(got_logits), logits[0], "argmax logits")
    assert int(token.item()) == int(oracle.row_argmax(logits)[0])
    assert int(ops.linear_argmax(to_dev(x), to_dev(w)).item()) == int(oracle.row_argmax(logits)[0])


def test_linear_argmax_ties_and_nan(ops, oracle):
    rng = np.random.default_rng(5)
    k, n = 64, 5000
    x = seeded_bf16(rng, (1, k))
    w = seeded_bf16(rng, (n, k), std=0.02)
    w[4321] = w[1234] = f32_to_bf16(np.full(k, 0.5, np.float32) * np.sign(bf16_to_f32(x[0]) + 1e-9))
    logits = oracle.linear_canonical(x, w)
    assert int(oracle.row_argmax(logits)[0]) == 1234  # equal maxima: the lowest index wins
    assert int(ops.linear_argmax(to_dev(x), to_dev(w)).item()) == 1234
    # NaN logits never win, except at index 0, where the reference's scan starts (cli_app.cpp:80-91)
    w_nan = w.copy()
    w_nan[77, 3] = 0x7FC0
    assert int(ops.linear_argmax(to_dev(x), to_dev(w_nan)).item()) == 1234
    w_nan[0, 3] = 0x7FC0
    assert int(ops.linear_argmax(to_dev(x), to_dev(w_nan)).item()) == 0


def test_embedding(ops):
    rng = np.random.default_rng(3)
    table = seeded_bf16(rng, (1000, 256))
    ids = np.array([5, 0, 999, 5, 17], np.int64)
    got = to_host(ops.embedding(to_dev(table), torch.from_numpy(ids)))
    assert (got == table[ids]).all()
    with pytest.raises(IndexError):
        ops.embedding(to_dev(table), torch.tensor([1000]))


# ---------------------------------------------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------------------------------------------


@pytest.mark.parametrize("t,pos,hq,hkv,d", [
    (1, 0, 16, 8, 128),     # first decode position: one key
    (1, 1, 16, 8, 128),
    (1, 7, 16, 8, 128),     # fewer keys than parts
    (1, 100, 16, 8, 128),
    (1, 639, 16, 8, 128),   # last row of a 640-token cache
    (33, 5, 16, 8, 128),    # prefill chunk after a cached prefix
    (64, 0, 4, 4, 64),
    (9, 300, 8, 2, 256),
    (301, 20, 16, 8, 128),  # prompt: clusters take runs of consecutive queries, the last run shorter
    (512, 0, 16, 8, 128),
    (200, 440, 32, 4, 64),
])
def test_decoder_attention_bit_exact(ops, oracle, t, pos, hq, hkv, d):
    rng = np.random.default_rng(t * 1000 + pos + d)
    cap = max(pos + t, 640)
    q = seeded_bf16(rng, (t, hq, d), std=2.0)
    kc = np.zeros((cap, hkv, d), np.uint16)
    vc = np.zeros((cap, hkv, d), np.uint16)
    kc[:pos + t] = seeded_bf16(rng, (pos + t, hkv, d), std=2.0)
    vc[:pos + t] = seeded_bf16(rng, (pos + t, hkv, d))
    want = oracle.decoder_attention(q, kc, vc, pos)
    got = to_host(ops.decoder_attention(to_dev(q), to_dev(kc), to_dev(vc), pos))
    assert_bits_equal(got, want, "decoder attention")


def test_decoder_attention_rejects_overflow(ops):
    q = torch.zeros(2, 2, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(8, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(IndexError):
        ops.decoder_attention(q, kc, kc, 7)
    with pytest.raises(NotImplementedError):
        ops.decoder_attention(q[..., :96], kc[..., :96], kc[..., :96], 0)


# ---------------------------------------------------------------------------------------------------------------
# The model
# ---------------------------------------------------------------------------------------------------------------


def small_config():
    from cppinf_b200.qwen3 import Qwen3Config

    return Qwen3Config(vocab_size=1000, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=128)


@pytest.fixture(scope="module")
def small_pair(cuda):
    from cppinf_b200.qwen3 import Qwen3Model, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = small_config()
    w = random_weights(cfg, seed=11, std=0.05)
    return cfg, Qwen3Model(cfg, 700, w), OracleQwen3(cfg, w, 700)


def test_model_forward_logits_bit_exact(small_pair):
    cfg, model, ref = small_pair
    tokens = np.random.default_rng(1).integers(0, cfg.vocab_size, 40)
    got = to_host(model.forward(tokens))
    ref.reset()
    want = ref.forward_cached(tokens, all_logits=True)
    assert_bits_equal(got, want, "model logits")


def test_model_chunked_prefill_and_decode_tokens(small_pair):
    # 600 prompt tokens: two prefill chunks (512 + 88); then 24 graph-replayed decode steps
    cfg, model, ref = small_pair
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, 600)
    got = model.generate(prompt, 25)
    ref.reset()
    want = ref.generate(prompt, 25)
    assert got == want
    assert model.length == 600 + 24


@pytest.mark.parametrize("head_dim,hq,hkv", [(64, 4, 2), (256, 2, 1)])
def test_model_decode_tokens_other_head_dims(cuda, head_dim, hq, hkv):
    # The decode step's kernels for head_dim 64 and 256 (the staged GEMVs and the 8-warp cluster attention with its
    # TMA-staged K/V tiles and half-row P·V chains): greedy tokens of prefill + graph-replayed decode steps equal
    # the oracle's.
    from cppinf_b200.qwen3 import Qwen3Config, Qwen3Model, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=hq, num_key_value_heads=hkv, head_dim=head_dim)
    w = random_weights(cfg, seed=21 + head_dim, std=0.05)
    model = Qwen3Model(cfg, 200, w)
    ref = OracleQwen3(cfg, w, 200)
    prompt = np.random.default_rng(head_dim).integers(0, cfg.vocab_size, 70)
    got = model.generate(prompt, 40)
    ref.reset()
    assert got == ref.generate(prompt, 40)
    model.close()


def test_model_decode_from_one_token_prompt(small_pair):
    # Decode steps at contexts of 2 .. 41 keys: most of the 8 parts hold zero or one cached row, so some CTAs stage
    # nothing and the new token's part may be the only non-empty one.
    cfg, model, ref = small_pair
    prompt = [int(np.random.default_rng(4).integers(0, cfg.vocab_size))]
    got = model.generate(prompt, 41)
    ref.reset()
    assert got == ref.generate(prompt, 41)


def test_model_cached_logits_match_full_forward(small_pair):
    cfg, model, ref = small_pair
    tokens = np.random.default_rng(3).integers(0, cfg.vocab_size, 12)
    full = to_host(model.forward(tokens))
    model.reset()
    model.forward_cached(tokens[:9], logits=None)
    rows = [to_host(model.forward_cached([t], logits="last")[1]) for t in tokens[9:]]
    assert_bits_equal(np.concatenate(rows), full[9:], "cached rows")


def test_model_validation(small_pair):
    cfg, model, _ = small_pair
    model.reset()
    with pytest.raises(IndexError):
        model.forward_cached([cfg.vocab_size])
    with pytest.raises(ValueError):
        model.decode(1)  # empty cache
    with pytest.raises(IndexError):
        model.forward_cached(np.zeros(701, np.int64))


def test_model_matches_hf_fixture_bit_exact_with_oracle(cuda, golden, oracle):
    # the Hugging Face fixture's model: device logits equal the oracle's bit for bit (the oracle is pinned to the
    # Hugging Face logits in tests/test_decoder_oracle.py)
    from cppinf_b200.qwen3 import Qwen3Model, random_weights
    from golden.make_decoder_golden import HF_SMALL
    from oracle.qwen3 import OracleQwen3

    fx = golden("qwen3_hf_small")
    w = random_weights(HF_SMALL, int(fx["seed"]), float(fx["std"]))
    got = to_host(Qwen3Model(HF_SMALL, 64, w).forward(fx["tokens"]))
    want = OracleQwen3(HF_SMALL, w, 64, oracle).forward_cached(fx["tokens"], all_logits=True)
    assert_bits_equal(got, want, "hf-fixture model logits")
    assert np.abs(bf16_to_f32(got) - bf16_to_f32(fx["logits"])).max() <= 0.0625


def test_qwen3_0_6b_greedy_tokens_bit_exact(cuda, oracle):
    """Random-init Qwen3-0.6B (weights ~N(0, 0.02), norm weights 1): 512-token seeded prompt, then greedy decode;
    every generated token equals the oracle's."""
    from cppinf_b200.qwen3 import Qwen3Config, Qwen3Model, random_weights
    from oracle.qwen3 import OracleQwen3

    cfg = Qwen3Config.qwen3_0_6b()
    w = random_weights(cfg, seed=0)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, 512)
    steps = 24
    model = Qwen3Model(cfg, 512 + steps, w)
    got = model.generate(prompt, steps)
    model.close()
    want = OracleQwen3(cfg, w, 512 + steps, oracle).generate(prompt, steps)
    assert got == want


# ---------------------------------------------------------------------------------------------------------------
# ops::matmul
# ---------------------------------------------------------------------------------------------------------------


def test_matmul_reference_kats(ops):
    # tests/ops/ops_test.cpp:63-110, 219-257: exact small-integer and quarter-step products
    f32 = lambda a: to_dev(np.asarray(a, np.float32))  # noqa: E731
    b16 = lambda a: to_dev(f32_to_bf16(np.asarray(a, np.float32)))  # noqa: E731
    lhs, rhs = [[1, 2, 3], [4, 5, 6]], [[7, 8], [9, 10], [11, 12]]
    assert to_host(ops.matmul(f32(lhs), f32(rhs))).tolist() == [[58, 64], [139, 154]]
    got = ops.matmul(b16(lhs), b16(rhs))
    assert got.dtype == torch.bfloat16 and bf16_to_f32(to_host(got)).tolist() == [[58, 64], [139, 154]]
    bl = [[[1, 2, 3], [4, 5, 6]], [[-1, 0.5, 2], [3, -2, 1]]]
    br = [[[7, 8], [9, 10], [11, 12]], [[2, -1], [0.25, 3.5], [-4, 1.5]]]
    want = [[[58, 64], [139, 154]], [[-9.875, 5.75], [1.5, -8.5]]]
    assert to_host(ops.matmul(f32(bl), f32(br))).tolist() == want
    got = ops.matmul(b16(bl), b16(br), output_dtype=torch.float32)
    assert got.dtype == torch.float32 and to_host(got).tolist() == want
    ml, mr = [[1, -2.5, 3.25], [4.5, 0.5, -1.75]], [[2, -1], [0.25, 3.5], [-4, 1.5]]
    mw = [[-11.625, -4.875], [16.125, -5.375]]
    assert to_host(ops.matmul(f32(ml), b16(mr))).tolist() == mw
    assert to_host(ops.matmul(b16(ml), f32(mr))).tolist() == mw
    assert bf16_to_f32(to_host(ops.matmul(b16(ml), b16(mr)))).tolist() == mw
    strided = f32([[1, 2, 3, 4], [5, 6, 7, 8]]).reshape(2, 2, 2)[:, 1, :]  # narrow + squeeze view
    assert to_host(ops.matmul(strided, f32([[2], [-1]]))).tolist() == [[2], [6]]
    with pytest.raises(ValueError):
        ops.matmul(f32(bl), f32(np.zeros((3, 3, 2))))
    with pytest.raises(ValueError):
        ops.matmul(f32(lhs), f32(rhs), output_dtype=torch.bfloat16)


@pytest.mark.parametrize("b,m,k,n,dx,dw,dy,rhs_layout", [
    (1, 7, 1024, 96, "bf16", "bf16", "bf16", "weight_t"),   # vector path: rhs = transposed weight view
    (1, 1, 2048, 333, "bf16", "bf16", "bf16", "weight_t"),
    (2, 5, 64, 40, "bf16", "bf16", "bf16", "dense"),        # generic path, dense rhs [k, n]
    (3, 4, 13, 6, "f32", "f32", "f32", "dense"),            # k not a multiple of 8
    (1, 9, 200, 17, "f32", "bf16", "f32", "weight_t"),
    (2, 3, 48, 5, "bf16", "f32", "f32", "dense"),
    (4, 16, 128, 33, "bf16", "bf16", "f32", "dense"),       # attention-style scores in f32
])
def test_matmul_bit_exact(ops, oracle, b, m, k, n, dx, dw, dy, rhs_layout):
    rng = np.random.default_rng(b * 1000 + m + k + n)
    def make(shape, dt):
        a = rng.standard_normal(shape).astype(np.float32)
        return f32_to_bf16(a) if dt == "bf16" else a
    lhs = make((b, m, k), dx)
    if rhs_layout == "weight_t":
        w = make((b, n, k), dw)
        rhs_np = np.swapaxes(w, 1, 2)
        rhs_dev = to_dev(w).transpose(1, 2)
    else:
        rhs_np = make((b, k, n), dw)
        rhs_dev = to_dev(rhs_np)
    out_dtype = torch.bfloat16 if dy == "bf16" else torch.float32
    got = to_host(ops.matmul(to_dev(lhs), rhs_dev, output_dtype=out_dtype))
    want = oracle.matmul(lhs, np.ascontiguousarray(rhs_np), np.uint16 if dy == "bf16" else np.float32)
    assert got.shape == want.shape and got.dtype == want.dtype
    assert (got.view(np.uint32 if dy == "f32" else np.uint16) == want.view(np.uint32 if dy == "f32" else np.uint16)).all()


# ---------------------------------------------------------------------------------------------------------------
# Safetensors checkpoints straight to the device
# ---------------------------------------------------------------------------------------------------------------


def test_load_safetensors_matches_set_weight(cuda, tmp_path):
    from cppinf_b200.qwen3 import Qwen3Model, random_weights, write_safetensors

    cfg = small_config()
    w = random_weights(cfg, seed=21, std=0.05)
    extra = dict(w)
    extra["lm_head.weight"] = w["model.embed_tokens.weight"]          # a tied checkpoint's copy: skipped
    extra["model.rotary_emb.inv_freq"] = np.ones(64, np.float32)      # a tensor the model does not use: skipped
    path = tmp_path / "model.safetensors"
    write_safetensors(path, extra, {"format": "pt"})
    tokens = np.random.default_rng(4).integers(0, cfg.vocab_size, 20)
    from_file = Qwen3Model(cfg, 64)
    assert from_file.load_safetensors(path) == 11 * cfg.num_hidden_layers + 2
    want = to_host(Qwen3Model(cfg, 64, w).forward(tokens))
    assert_bits_equal(to_host(from_file.forward(tokens)), want, "safetensors-loaded logits")

    missing = dict(w)
    del missing["model.layers.1.mlp.down_proj.weight"]
    write_safetensors(tmp_path / "missing.safetensors", missing)
    with pytest.raises(IndexError):
        Qwen3Model(cfg, 64).load_safetensors(tmp_path / "missing.safetensors")
    wrong = dict(w)
    wrong["model.norm.weight"] = np.ones(cfg.hidden_size, np.float32)
    write_safetensors(tmp_path / "wrong.safetensors", wrong)
    with pytest.raises(ValueError):
        Qwen3Model(cfg, 64).load_safetensors(tmp_path / "wrong.safetensors")


@pytest.mark.parametrize("name,make,message", [
    # q_proj is [q_dim, hidden] = [512, 256]; its transpose has the same byte count
    ("model.layers.0.self_attn.q_proj.weight", lambda a: np.ascontiguousarray(a.T), "has an unexpected shape"),
    # gate_proj [512, 256] stored as [256, 512] (a swapped layout)
    ("model.layers.1.mlp.gate_proj.weight", lambda a: a.reshape(256, 512), "has an unexpected shape"),
    ("model.layers.0.self_attn.o_proj.weight", lambda a: a.reshape(-1), "must be rank-2"),
    ("model.norm.weight", lambda a: a.reshape(16, 16), "requires a rank-1 weight tensor"),
])
def test_load_safetensors_rejects_wrong_shapes_with_same_bytes(cuda, tmp_path, name, make, message):
    # validate_projection_weight (src/nn/qwen_common.cpp:38-49) and ops::rms_norm's weight checks
    # (src/ops/nn_ops.cpp:150-159): a tensor with the right byte count but the wrong shape is rejected.
    from cppinf_b200.qwen3 import Qwen3Model, random_weights, write_safetensors

    cfg = small_config()
    w = random_weights(cfg, seed=22, std=0.05)
    bad = dict(w)
    bad[name] = make(w[name])
    assert bad[name].nbytes == w[name].nbytes
    write_safetensors(tmp_path / "bad.safetensors", bad)
    model = Qwen3Model(cfg, 64)
    try:
        with pytest.raises(ValueError, match=message):
            model.load_safetensors(tmp_path / "bad.safetensors")
    finally:
        model.close()
