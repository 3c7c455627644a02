"""Qwen3 decoder on the device: configuration, seeded random weights and the model object.

Mirrors the reference's model interface (src/models/qwen3/qwen3_model.h): ``Qwen3Model.forward(token_ids)`` returns
bf16 logits [T, vocab]; ``forward_cached(token_ids)`` appends to the model's cached sequence;
``make_cache(batch, max_sequence_length)`` / ``forward_cached_batch(token_id_batch, cache)`` run right-padded
batches of cached sequences; ``generate`` is the greedy loop of src/cli/cli_app.cpp (temperature 0: argmax of the
last logits row).
The model itself lives in libcppinf_b200.so (cppinf_qwen3_* in include/cppinf_b200.h): weights, KV cache and
activations stay in HBM, and decode steps are replayed from captured CUDA graphs (of eight steps, and of one step
for the remainder) whose kernels read the position and the previous token from device memory.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Qwen3Config:
    """The fields of the reference's HfConfig that the decoder uses (src/loaders/hf/hf_config.h)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0

    @staticmethod
    def qwen3_0_6b() -> "Qwen3Config":
        """Qwen3-0.6B: 28 layers, hidden 1024, 16 query / 8 key-value heads of 128, MLP 3072, vocab 151936."""
        return Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                           num_attention_heads=16, num_key_value_heads=8, head_dim=128)

    def replace(self, **kw) -> "Qwen3Config":
        return dataclasses.replace(self, **kw)

    def weight_shapes(self) -> dict[str, tuple[int, ...]]:
        """Tensor names and shapes of a tied-embedding checkpoint (Hugging Face naming, as the reference loads)."""
        h, d = self.hidden_size, self.head_dim
        shapes: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (self.vocab_size, h)}
        for i in range(self.num_hidden_layers):
            p = f"model.layers.{i}."
            shapes.update({
                p + "input_layernorm.weight": (h,),
                p + "self_attn.q_proj.weight": (self.num_attention_heads * d, h),
                p + "self_attn.k_proj.weight": (self.num_key_value_heads * d, h),
                p + "self_attn.v_proj.weight": (self.num_key_value_heads * d, h),
                p + "self_attn.q_norm.weight": (d,),
                p + "self_attn.k_norm.weight": (d,),
                p + "self_attn.o_proj.weight": (h, self.num_attention_heads * d),
                p + "post_attention_layernorm.weight": (h,),
                p + "mlp.gate_proj.weight": (self.intermediate_size, h),
                p + "mlp.up_proj.weight": (self.intermediate_size, h),
                p + "mlp.down_proj.weight": (h, self.intermediate_size),
            })
        shapes["model.norm.weight"] = (h,)
        return shapes

    def parameter_count(self) -> int:
        return sum(int(np.prod(s)) for s in self.weight_shapes().values())


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = bits + (np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1)))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def random_weights(config: Qwen3Config, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded random initialisation: matrices ~N(0, std) rounded to bf16, norm weights 1.0 (bf16 0x3f80).

    Rows [4096 b, 4096 (b + 1)) of tensor i (in weight_shapes() order) draw from numpy's PCG64 seeded with
    (seed, i, b), so the values do not depend on generation order; the blocks are generated on a thread pool."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    block = 4096
    out: dict[str, np.ndarray] = {}
    jobs = []
    for i, (name, shape) in enumerate(config.weight_shapes().items()):
        if len(shape) == 1:
            out[name] = np.full(shape, 0x3F80, dtype=np.uint16)
            continue
        out[name] = np.empty(shape, dtype=np.uint16)
        jobs += [(name, i, b) for b in range((shape[0] + block - 1) // block)]

    def fill(job):
        name, i, b = job
        dst = out[name][b * block:(b + 1) * block]
        rng = np.random.Generator(np.random.PCG64([seed, i, b]))
        dst[...] = f32_to_bf16_bits(rng.standard_normal(dst.shape, dtype=np.float32) * np.float32(std))

    with ThreadPoolExecutor(max(1, min(16, os.cpu_count() or 1))) as pool:
        list(pool.map(fill, jobs))
    return out


def write_safetensors(path, tensors: dict[str, np.ndarray], metadata: dict[str, str] | None = None) -> None:
    """Writes numpy arrays (uint16 = bf16 bits, float32 = f32) as a safetensors file: 8-byte little-endian header
    length, JSON header (padded with spaces to a multiple of 8), tensor bytes in order."""
    import json
    import struct

    header: dict = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    offset = 0
    blobs = []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        dtype = {np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}[arr.dtype]
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [offset, offset + arr.nbytes]}
        blobs.append(arr.tobytes())
        offset += arr.nbytes
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


class Qwen3Model:
    """Device-resident Qwen3 with one cached sequence (libcppinf_b200.so, cppinf_qwen3_*).

    ``forward(token_ids)`` returns the bf16 logits [T, vocab] of a fresh sequence (Qwen3Model::forward,
    src/models/qwen3/qwen3_model.cpp:202-206); ``forward_cached(token_ids)`` appends to the cached sequence
    (:269-273); ``generate(prompt, steps)`` is greedy decoding (src/cli/cli_app.cpp, temperature 0).
    """

    def __init__(self, config: Qwen3Config, max_sequence_length: int, weights: dict | None = None,
                 device: int | None = None):
        import ctypes

        import torch

        from . import capi

        self.config = config
        self.capacity = int(max_sequence_length)
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self._capi = capi
        lib = capi.load()
        cfg = capi.Qwen3ConfigC(config.vocab_size, config.hidden_size, config.intermediate_size,
                                config.num_hidden_layers, config.num_attention_heads, config.num_key_value_heads,
                                config.head_dim, config.rms_norm_eps, config.rope_theta)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            capi.check(lib.cppinf_qwen3_create(ctypes.byref(cfg), self.capacity, ctypes.byref(handle)),
                       "cppinf_qwen3_create")
        self._handle = handle
        if weights is not None:
            self.load_weights(weights)

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            self._capi.load().cppinf_qwen3_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_weights(self, weights: dict) -> None:
        """Copies checkpoint tensors (numpy uint16 bf16 bits, or torch bf16 tensors on host or device)."""
        import torch

        shapes = self.config.weight_shapes()
        missing = sorted(set(shapes) - set(weights))
        if missing:
            raise ValueError(f"Qwen3Model is missing tensor '{missing[0]}'.")
        with torch.cuda.device(self.device):
            for name, value in weights.items():
                if isinstance(value, np.ndarray):
                    arr = np.ascontiguousarray(value)
                    if arr.dtype != np.uint16 or arr.shape != shapes.get(name, arr.shape):
                        raise ValueError(f"Qwen3Model tensor '{name}' has an unexpected shape or dtype.")
                    self._capi.call("cppinf_qwen3_set_weight", self._handle, name.encode(), arr.ctypes.data,
                                    arr.nbytes, 0)
                else:
                    t = value.contiguous()
                    if t.dtype != torch.bfloat16:
                        raise ValueError(f"Qwen3Model tensor '{name}' must be bf16.")
                    self._capi.call("cppinf_qwen3_set_weight", self._handle, name.encode(), t.data_ptr(),
                                    t.numel() * 2, 1 if t.is_cuda else 0)
            torch.cuda.synchronize(self.device)

    def set_prefill(self, mode: str) -> None:
        """Prompt-row projections on "cuda_cores" (default: bit-exact to the oracle) or "tensor_cores" (tcgen05,
        tolerance parity)."""
        modes = {"cuda_cores": 0, "tensor_cores": 1}
        if mode not in modes:
            raise ValueError(f"prefill mode must be one of {sorted(modes)}")
        self._capi.call("cppinf_qwen3_set_prefill", self._handle, modes[mode])

    def load_safetensors(self, path) -> int:
        """Loads a safetensors checkpoint straight from the mapped file into the model (cppinf_qwen3_load_safetensors);
        returns the number of tensors copied."""
        import ctypes

        import torch

        n = ctypes.c_int64(0)
        with torch.cuda.device(self.device):
            self._capi.call("cppinf_qwen3_load_safetensors", self._handle, str(path).encode(), ctypes.byref(n))
        return int(n.value)

    @property
    def length(self) -> int:
        return int(self._capi.load().cppinf_qwen3_length(self._handle))

    @property
    def step_launches(self) -> int:
        return int(self._capi.load().cppinf_qwen3_step_launches(self._handle))

    def reset(self) -> None:
        import torch

        with torch.cuda.device(self.device):
            self._capi.call("cppinf_qwen3_reset", self._handle, torch.cuda.current_stream().cuda_stream)

    def forward_cached(self, token_ids, logits: str | None = "last"):
        """Appends token_ids; returns (next greedy token, logits) with logits None, the last row [1, vocab] or all
        rows [T, vocab] (bf16 device tensor) for logits=None / "last" / "all"."""
        import ctypes

        import torch

        ids = [int(t) for t in token_ids]
        arr = self._capi.i64_array(ids)
        nxt = ctypes.c_int64(0)
        out = None
        with torch.cuda.device(self.device):
            if logits == "all":
                out = torch.empty(len(ids), self.config.vocab_size, dtype=torch.bfloat16, device=self.device)
            elif logits == "last":
                out = torch.empty(1, self.config.vocab_size, dtype=torch.bfloat16, device=self.device)
            self._capi.call("cppinf_qwen3_forward", self._handle, arr, len(ids),
                            out.data_ptr() if out is not None else None, 1 if logits == "all" else 0,
                            ctypes.byref(nxt), torch.cuda.current_stream().cuda_stream)
        return int(nxt.value), out

    def make_cache(self, batch_size: int, max_sequence_length: int) -> "Qwen3Cache":
        """Qwen3Model::make_cache(batch_size, max_sequence_length) (qwen3_model.cpp:222-245): a batch of empty cached
        sequences for forward_cached_batch, separate from the model's own sequence."""
        return Qwen3Cache(self, batch_size, max_sequence_length)

    def forward_cached_batch(self, token_ids, cache: "Qwen3Cache"):
        """Qwen3Model::forward_cached(TokenIdBatch, Qwen3Cache&) (qwen3_model.cpp:275-311): sequence b appends
        token_ids[b] to its cached rows. Returns bf16 logits [batch, longest, vocab] on the device, right-padded rows
        zero; each row equals the same row of a forward of that sequence alone, bit for bit."""
        import torch

        seqs = [[int(t) for t in seq] for seq in token_ids]
        batch = len(seqs)
        longest = max((len(q) for q in seqs), default=0)
        packed = [0] * max(batch * longest, 1)
        for b, q in enumerate(seqs):
            packed[b * longest:b * longest + len(q)] = q
        out = torch.empty(max(batch, 1), max(longest, 1), self.config.vocab_size, dtype=torch.bfloat16,
                          device=self.device)
        with torch.cuda.device(self.device):
            self._capi.call("cppinf_qwen3_forward_batch", self._handle, cache._handle, self._capi.i64_array(packed),
                            self._capi.i64_array([len(q) for q in seqs]), batch, longest, out.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
        return out

    def forward(self, token_ids):
        """Qwen3Model::forward: logits [T, vocab] of `token_ids` as a fresh sequence."""
        self.reset()
        return self.forward_cached(token_ids, logits="all")[1]

    def decode(self, steps: int) -> list[int]:
        """`steps` greedy decode steps from the cached state (graphs of eight steps, then single steps)."""
        import torch

        if steps <= 0:
            return []
        buf = self._capi.i64_array([0] * steps)
        with torch.cuda.device(self.device):
            self._capi.call("cppinf_qwen3_decode", self._handle, int(steps), buf,
                            torch.cuda.current_stream().cuda_stream)
        return [int(buf[i]) for i in range(steps)]

    def generate(self, prompt, steps: int) -> list[int]:
        """Greedy generation: prefill `prompt` as a fresh sequence, then `steps` tokens in total (the first from the
        prompt's last logits row, the rest from decode steps)."""
        self.reset()
        first, _ = self.forward_cached(prompt, logits=None)
        return [first] + self.decode(steps - 1)


class Qwen3Cache:
    """A batch of cached sequences on the model's device (cppinf_qwen3_cache_*): per layer and sequence K and V
    [capacity, kv_heads, head_dim]; ``sequence_lengths`` mirrors Qwen3Cache::sequence_lengths."""

    def __init__(self, model: Qwen3Model, batch_size: int, max_sequence_length: int):
        import ctypes

        import torch

        self._capi = model._capi
        handle = ctypes.c_void_p()
        with torch.cuda.device(model.device):
            self._capi.call("cppinf_qwen3_cache_create", model._handle, int(batch_size), int(max_sequence_length),
                            ctypes.byref(handle))
        self._handle = handle
        self.capacity = int(max_sequence_length)

    @property
    def batch_size(self) -> int:
        return int(self._capi.load().cppinf_qwen3_cache_batch(self._handle))

    @property
    def sequence_lengths(self) -> list[int]:
        n = self.batch_size
        arr = self._capi.i64_array([0] * n)
        self._capi.call("cppinf_qwen3_cache_lengths", self._handle, arr)
        return [int(arr[i]) for i in range(n)]

    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            self._capi.load().cppinf_qwen3_cache_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
