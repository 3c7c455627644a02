"""Generates tests/golden/ref_*.npz: golden vectors produced by the reference's OWN op code, compiled in place from
the reference sources into oracle/_ref/libcppinf_ref.so (see oracle/Makefile), on seeded inputs:

- ops::scaled_causal_softmax_last_dim          (src/ops/nn_ops.cpp:77-138)
- scaled_position_causal_softmax_last_dim      (src/nn/qwen_attention.cpp:164-235), ragged offsets/lengths
- nn::apply_rope, bf16 and f32, seq dim 0 and 1 (src/nn/rope.cpp:58-109)
- apply_rope_batched                           (src/nn/qwen_attention.cpp:136-162)
- ops::add / ops::mul / ops::cast              (src/ops/elementwise_ops.cpp, src/ops/tensor_ops.cpp)
- ops::silu then ops::mul                      (src/nn/qwen_mlp.cpp:65-66)

The oneDNN-backed pieces (add/mul/silu/cast) run through the scalar stand-ins of oracle/ref_shim/one_dnn_shim.cpp.

Run from the repository root after `make -C oracle`:  python tests/golden/make_reference_golden.py
The outputs are committed so that GPU runs need neither the reference tree nor this script.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.oracle import Reference, f32_to_bf16  # noqa: E402

OUT = Path(__file__).resolve().parent


def main() -> None:
    ref = Reference()
    rng = np.random.default_rng(9002)

    x = (rng.standard_normal((3, 48, 48)) * 2.0).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(128.0))
    np.savez_compressed(OUT / "ref_causal_softmax.npz", x=x, y=ref.scaled_causal_softmax(x, float(scale)),
                        scale=scale)

    b, h, qc, kc = 3, 2, 8, 40
    xp = (rng.standard_normal((b, h, qc, kc)) * 2.0).astype(np.float32)
    offsets = np.array([0, 17, 30], dtype=np.int64)
    qlens = np.array([8, 5, 3], dtype=np.int64)
    klens = np.array([8, 22, 33], dtype=np.int64)
    yp = ref.position_causal_softmax(xp, float(scale), offsets, qlens, klens)
    np.savez_compressed(OUT / "ref_position_softmax.npz", x=xp, y=yp, scale=scale, offsets=offsets, qlens=qlens,
                        klens=klens)

    rope_cases = {}
    xr = f32_to_bf16(rng.standard_normal((6, 4, 64)).astype(np.float32))
    rope_cases["bf16_seq1"] = (xr, ref.apply_rope(xr, offset=3, base=1e6, seq_dim=1))
    rope_cases["bf16_seq0"] = (xr, ref.apply_rope(xr, offset=1000, base=1e6, seq_dim=0))
    xf = rng.standard_normal((5, 3, 32)).astype(np.float32)
    rope_cases["f32_seq1"] = (xf, ref.apply_rope(xf, offset=7, base=10000.0, seq_dim=1))
    np.savez_compressed(OUT / "ref_rope.npz", **{f"{k}_x": v[0] for k, v in rope_cases.items()},
                        **{f"{k}_y": v[1] for k, v in rope_cases.items()})

    xb = f32_to_bf16(rng.standard_normal((2, 9, 4, 128)).astype(np.float32))
    boffs = np.array([0, 1234], dtype=np.int64)
    np.savez_compressed(OUT / "ref_rope_batched.npz", x=xb, offsets=boffs, y=ref.apply_rope_batched(xb, boffs))

    n = 4099
    ab = f32_to_bf16((rng.standard_normal(n) * 3).astype(np.float32))
    bb = f32_to_bf16((rng.standard_normal(n) * 3).astype(np.float32))
    af = (rng.standard_normal(n) * 3).astype(np.float32)
    bf = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    gate = f32_to_bf16((rng.standard_normal(n) * 2).astype(np.float32))
    up = f32_to_bf16(rng.standard_normal(n).astype(np.float32))
    np.savez_compressed(
        OUT / "ref_elementwise.npz",
        a_bf16=ab, b_bf16=bb, add_bf16=ref.add(ab, bb), mul_bf16=ref.mul(ab, bb),
        a_f32=af, b_f32=bf, add_f32=ref.add(af, bf), mul_f32=ref.mul(af, bf),
        cast_f32_bf16=ref.cast(af, True), cast_bf16_f32=ref.cast(ab, False),
        gate=gate, up=up, silu_bf16=ref.silu(gate), silu_mul_bf16=ref.silu_mul(gate, up),
        silu_f32=ref.silu(af), silu_mul_f32=ref.silu_mul(af, bf),
    )


if __name__ == "__main__":
    main()
