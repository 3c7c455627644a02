"""Generates tests/golden/torch_*.npz: seeded golden vectors for the hot-path ops, computed with PyTorch 2.11.0 on the
CPU -- the version and formulas the reference pins its op goldens to:

- rms_norm: x * rsqrt(mean(x^2) + eps) * w in f32, cast to bf16 (tests/ops/ops_test.cpp:312-320 comment)
- silu then mul, quantised to bf16 after each op (tests/nn/qwen_mlp_oracle.py:14-31)
- split-half RoPE with inv_freq = 1 / base^(2i/D) (tests/nn/rope_oracle.py:13-24)
- softmax over the last dim (tests/ops/ops_test.cpp:280-286 comment)
- first-index argmax (torch.argmax returns the first maximal index)

Run from the repository root:  python tests/golden/make_golden.py
The outputs are committed; the tests never run torch to produce expected values.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def normal(gen: torch.Generator, shape, mean=0.0, std=1.0) -> torch.Tensor:
    return (torch.randn(shape, generator=gen, dtype=torch.float32) * std + mean).to(torch.bfloat16)


def rms_norm_bf16(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf, wf = x.float(), w.float()
    return (xf * torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps) * wf).to(torch.bfloat16)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope(x: torch.Tensor, base: float, offset: int) -> torch.Tensor:
    """x [T, H, D] f32, positions offset + t."""
    d = x.shape[-1]
    positions = torch.arange(offset, offset + x.shape[0], dtype=torch.float32)
    inv_freq = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = torch.outer(positions, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)[:, None, :]
    return x * emb.cos() + rotate_half(x) * emb.sin()


def main() -> None:
    gen = torch.Generator().manual_seed(20261201)
    eps = 1e-6

    # RMSNorm over hidden (bf16 [64, 1024]).
    x = normal(gen, (64, 1024))
    w = normal(gen, (1024,), 1.0, 0.1)
    np.savez_compressed(OUT / "torch_rms_norm.npz", x=bits(x), w=bits(w), y=bits(rms_norm_bf16(x, w, eps)),
                        eps=np.float32(eps))

    # Residual add + RMSNorm (bf16 [32, 1024]).
    a = normal(gen, (32, 1024))
    b = normal(gen, (32, 1024))
    w2 = normal(gen, (1024,), 1.0, 0.1)
    s = (a.float() + b.float()).to(torch.bfloat16)
    np.savez_compressed(OUT / "torch_add_rms_norm.npz", a=bits(a), b=bits(b), w=bits(w2), sum=bits(s),
                        y=bits(rms_norm_bf16(s, w2, eps)), eps=np.float32(eps))

    # SiLU(gate) * up with per-op bf16 quantisation (bf16 [32, 3072]).
    gate = normal(gen, (32, 3072))
    up = normal(gen, (32, 3072))
    act = torch.nn.functional.silu(gate.float()).to(torch.bfloat16)
    out = (act.float() * up.float()).to(torch.bfloat16)
    np.savez_compressed(OUT / "torch_silu_mul.npz", gate=bits(gate), up=bits(up), out=bits(out))

    # Per-head q/k RMSNorm + RoPE (q [16, 16, 128], k [16, 8, 128], positions 5..20, theta 1e6).
    q = normal(gen, (16, 16, 128))
    k = normal(gen, (16, 8, 128))
    qw = normal(gen, (128,), 1.0, 0.1)
    kw = normal(gen, (128,), 1.0, 0.1)
    offset, base = 5, 1_000_000.0
    q_out = rope(rms_norm_bf16(q, qw, eps).float(), base, offset).to(torch.bfloat16)
    k_out = rope(rms_norm_bf16(k, kw, eps).float(), base, offset).to(torch.bfloat16)
    np.savez_compressed(OUT / "torch_qk_norm_rope.npz", q=bits(q), k=bits(k), qw=bits(qw), kw=bits(kw),
                        q_out=bits(q_out), k_out=bits(k_out), offset=np.int64(offset), base=np.float32(base),
                        eps=np.float32(eps))

    # Causal scaled softmax (f32 [2, 64, 64] ~ N(0, 4), scale 1/sqrt(128)).
    scores = torch.randn((2, 64, 64), generator=gen, dtype=torch.float32) * 2.0
    scale = 1.0 / np.sqrt(128.0)
    mask = torch.triu(torch.ones(64, 64, dtype=torch.bool), diagonal=1)
    probs = torch.softmax((scores * scale).masked_fill(mask, float("-inf")), dim=-1)
    np.savez_compressed(OUT / "torch_causal_softmax.npz", x=scores.numpy(), y=probs.numpy(),
                        scale=np.float32(scale))

    # softmax_last_dim in bf16 ([16, 256]).
    sx = normal(gen, (16, 256), 0.0, 2.0)
    np.savez_compressed(OUT / "torch_softmax.npz", x=bits(sx), y=bits(torch.softmax(sx, dim=-1)))

    # Row argmax over bf16 logits ([8, 4096] ~ N(0, 2)) with planted ties, a -0/+0 pair and NaNs.
    logits = normal(gen, (8, 4096), 0.0, 2.0)
    logits[1, 100] = 50.0
    logits[1, 3000] = 50.0  # tie: the lower index wins
    logits[2, :] = 0.0
    logits[2, 7] = -0.0  # all zeros: index 0 wins
    logits[3, 0] = float("nan")  # NaN at index 0: the reference returns 0
    logits[4, 55] = float("nan")  # NaN elsewhere is skipped
    logits[4, 56] = 40.0
    logits[5, :] = float("-inf")
    logits[5, 4095] = -1e30
    ref = []
    for row in logits.float():
        best, best_id = row[0].item(), 0
        for i in range(1, row.shape[0]):
            if row[i].item() > best:
                best, best_id = row[i].item(), i
        ref.append(best_id)
    np.savez_compressed(OUT / "torch_row_argmax.npz", x=bits(logits), index=np.array(ref, dtype=np.int64),
                        torch_argmax=torch.argmax(torch.nan_to_num(logits.float(), nan=-np.inf), dim=-1).numpy())


if __name__ == "__main__":
    main()
