"""Host <-> device helpers for the tests: numpy bf16 bit arrays and float32 arrays to torch CUDA tensors and back."""

from __future__ import annotations

import numpy as np
import torch


def to_dev(arr: np.ndarray, device="cuda") -> torch.Tensor:
    """uint16 (bf16 bits) -> torch.bfloat16, float32 -> torch.float32, int64 -> torch.int64."""
    arr = np.ascontiguousarray(arr)
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(arr).to(device)


def to_host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def bf16_bits(values) -> np.ndarray:
    from oracle.oracle import f32_to_bf16

    return f32_to_bf16(np.asarray(values, dtype=np.float32))


def seeded_bf16(rng: np.random.Generator, shape, mean=0.0, std=1.0) -> np.ndarray:
    from oracle.oracle import f32_to_bf16

    return f32_to_bf16((rng.standard_normal(shape) * std + mean).astype(np.float32))
