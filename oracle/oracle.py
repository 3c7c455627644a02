"""numpy interface to the CPU checkers. TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use this module, and only as the checker
(or the timed CPU baseline): the product path never imports it.

- ``Oracle`` wraps ``oracle/_build/liboracle.so``, the C restatement of the reference ops (oracle/oracle.c).
- ``Reference`` wraps ``oracle/_ref/libcppinf_ref.so``, the reference's own sources compiled in place
  (oracle/Makefile); it is absent where the reference tree was not available at build time.

bf16 arrays are numpy uint16 bit patterns; f32 arrays are numpy float32.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIB = ORACLE_DIR / "_build" / "liboracle.so"
REFERENCE_LIB = ORACLE_DIR / "_ref" / "libcppinf_ref.so"

BF16 = 0
F32 = 1

_p = ctypes.c_void_p
_i = ctypes.c_int
_l = ctypes.c_int64
_f = ctypes.c_float


def dtype_code(arr: np.ndarray) -> int:
    if arr.dtype == np.uint16:
        return BF16
    if arr.dtype == np.float32:
        return F32
    raise TypeError(f"oracle arrays are uint16 (bf16 bits) or float32, got {arr.dtype}")


def _ptr(arr: np.ndarray):
    assert arr.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return arr.ctypes.data_as(_p)


def _i64(values) -> ctypes.Array:
    arr = (_l * max(len(values), 1))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even as src/tensors/bfloat16.cpp:8-15 (vectorised numpy restatement)."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bits = bits + 0x7FFF + ((bits >> 16) & 1)
    return ((bits >> 16) & 0xFFFF).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def as_float(arr: np.ndarray) -> np.ndarray:
    return bf16_to_f32(arr) if arr.dtype == np.uint16 else arr.astype(np.float32)


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two bf16 bit arrays (monotone integer mapping; +0 and -0 are 0 apart)."""

    def ordered(b):
        b = b.astype(np.int64)
        return np.where(b & 0x8000, -(b & 0x7FFF), b)

    return np.abs(ordered(a_bits) - ordered(b_bits))


def cpu_has_fma() -> bool:
    """True when the host CPU has FMA3 (read from /proc/cpuinfo; assumed present where that file does not exist)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return "fma" in line.split()
    except OSError:
        return True
    return True


class Oracle:
    """The C restatement (oracle/oracle.c)."""

    def __init__(self, path: Path | str | None = None):
        path = Path(path or os.environ.get("CPPINF_ORACLE_LIB", ORACLE_LIB))
        if not path.exists():
            raise RuntimeError(f"oracle library missing at {path}; build it with `make -C oracle`")
        if not cpu_has_fma():
            raise RuntimeError("the oracle is built with FMA3 instructions (its fmaf dot products); this CPU lacks them")
        self.lib = ctypes.CDLL(str(path))
        sig = {
            "oracle_f32_to_bf16": [_p, _p, _l],
            "oracle_bf16_to_f32": [_p, _p, _l],
            "oracle_cast": [_i, _p, _i, _p, _l],
            "oracle_add": [_i, _p, _p, _p, _l],
            "oracle_mul": [_i, _p, _p, _p, _l],
            "oracle_silu": [_i, _p, _p, _l],
            "oracle_silu_mul": [_i, _p, _p, _p, _p, _l],
            "oracle_rms_norm": [_i, _p, _l, _p, _p, _l, _l, _f, _i],
            "oracle_add_rms_norm": [_i, _p, _p, _p, _p, _p, _l, _l, _f, _i],
            "oracle_softmax_last_dim": [_i, _p, _p, _l, _l],
            "oracle_scaled_causal_softmax": [_p, _p, _l, _l, _l, _f],
            "oracle_position_causal_softmax": [_p, _p, _l, _l, _l, _l, _f, _p, _p, _p],
            "oracle_rope_table": [_f, _l, _l, _p],
            "oracle_rope": [_i, _p, _l, _l, _l, _l, _l, _l, _l, _l, _f, _p],
            "oracle_qk_norm_rope": [_i, _p, _p, _p, _p, _p, _p, _l, _l, _l, _l, _l, _f, _f, _i],
            "oracle_row_argmax": [_i, _p, _l, _l, _l, _p],
            "oracle_linear": [_i, _p, _p, _p, _l, _l, _l],
            "oracle_pexp_array": [_p, _p, _l],
            "oracle_silu_mul_pexp": [_p, _p, _p, _l],
            "oracle_linear_canonical": [_p, _l, _p, _l, _l, _l, _p, _p],
            "oracle_decoder_attention": [_p, _p, _p, _p, _l, _l, _l, _l, _l],
            "oracle_matmul_canonical": [_i, _p, _p, _i, _p, _p, _i, _p, _l, _l, _l, _l],
        }
        for name, args in sig.items():
            fn = getattr(self.lib, name)
            fn.argtypes = args
            fn.restype = None

    # -- elementwise --
    def cast(self, x: np.ndarray, to_bf16: bool) -> np.ndarray:
        x = np.ascontiguousarray(x)
        out = np.empty(x.shape, dtype=np.uint16 if to_bf16 else np.float32)
        self.lib.oracle_cast(dtype_code(x), _ptr(x), dtype_code(out), _ptr(out), x.size)
        return out

    def add(self, a, b):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        out = np.empty_like(a)
        self.lib.oracle_add(dtype_code(a), _ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def mul(self, a, b):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        out = np.empty_like(a)
        self.lib.oracle_mul(dtype_code(a), _ptr(a), _ptr(b), _ptr(out), a.size)
        return out

    def silu(self, x):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        self.lib.oracle_silu(dtype_code(x), _ptr(x), _ptr(out), x.size)
        return out

    def silu_mul(self, gate, up, with_alternative: bool = False):
        gate, up = np.ascontiguousarray(gate), np.ascontiguousarray(up)
        out = np.empty_like(gate)
        alt = np.empty_like(gate) if with_alternative else None
        self.lib.oracle_silu_mul(dtype_code(gate), _ptr(gate), _ptr(up), _ptr(out),
                                 _ptr(alt) if alt is not None else None, gate.size)
        return (out, alt) if with_alternative else out

    # -- reductions --
    @staticmethod
    def canonical_chunk(arr: np.ndarray, width: int, vector_path: bool = True) -> int:
        """Elements per lane step of the device reduction: a 16-byte vector, or 1 on the scalar path (operands not
        16-byte aligned, or a width that is not a whole number of vectors)."""
        vec = 8 if arr.dtype == np.uint16 else 4
        if not vector_path or width % vec != 0:
            return 1
        return vec

    def rms_norm(self, x, w, eps: float, chunk: int | None = None, row_stride: int | None = None):
        width = w.shape[0]
        rows = x.size // width if row_stride is None else (x.size - width) // row_stride + 1
        stride = width if row_stride is None else row_stride
        x = np.ascontiguousarray(x)
        out = np.empty((rows, width), dtype=x.dtype)
        chunk = self.canonical_chunk(x, width, row_stride is None or row_stride % (8 if x.dtype == np.uint16 else 4) == 0) if chunk is None else chunk
        self.lib.oracle_rms_norm(dtype_code(x), _ptr(x), stride, _ptr(np.ascontiguousarray(w)), _ptr(out), rows,
                                 width, eps, chunk)
        return out.reshape(x.shape) if row_stride is None else out

    def add_rms_norm(self, a, b, w, eps: float, chunk: int | None = None):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        width = w.shape[0]
        s = np.empty_like(a)
        y = np.empty_like(a)
        chunk = self.canonical_chunk(a, width) if chunk is None else chunk
        self.lib.oracle_add_rms_norm(dtype_code(a), _ptr(a), _ptr(b), _ptr(np.ascontiguousarray(w)), _ptr(s),
                                     _ptr(y), a.size // width, width, eps, chunk)
        return s, y

    def softmax_last_dim(self, x):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        width = x.shape[-1]
        self.lib.oracle_softmax_last_dim(dtype_code(x), _ptr(x), _ptr(out), x.size // width, width)
        return out

    def scaled_causal_softmax(self, x: np.ndarray, scale: float):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q, k = x.shape[-2], x.shape[-1]
        out = np.empty_like(x)
        self.lib.oracle_scaled_causal_softmax(_ptr(x), _ptr(out), x.size // (q * k), q, k, scale)
        return out

    def position_causal_softmax(self, x, scale, query_offsets, query_lengths, key_lengths):
        x = np.ascontiguousarray(x, dtype=np.float32)
        b, h, q, k = x.shape
        out = np.empty_like(x)
        self.lib.oracle_position_causal_softmax(_ptr(x), _ptr(out), b, h, q, k, scale, _i64(query_offsets),
                                                _i64(query_lengths), _i64(key_lengths))
        return out

    # -- RoPE --
    def rope_table(self, base: float, head_dim: int, positions: int):
        table = np.empty((positions, head_dim), dtype=np.float32)
        self.lib.oracle_rope_table(base, head_dim, positions, _ptr(table))
        return table

    def rope(self, x, offset: int = 0, base: float = 1e6, seq_dim: int = 1):
        """nn::apply_rope on an array [d0, d1, D] (any numpy strides; element strides are passed through)."""
        d0, d1, d = x.shape
        itemsize = x.itemsize
        s0, s1, s2 = (s // itemsize for s in x.strides)
        out = np.empty((d0, d1, d), dtype=x.dtype)
        self.lib.oracle_rope(dtype_code(x), x.ctypes.data_as(_p), d0, d1, d, s0, s1, s2, seq_dim, offset, base,
                             _ptr(out))
        return out

    def qk_norm_rope(self, q, k, qw, kw, eps, offset=0, base=1e6, chunk: int | None = None):
        q, k = np.ascontiguousarray(q), np.ascontiguousarray(k)
        t, hq, d = q.shape
        hk = k.shape[1]
        q_out, k_out = np.empty_like(q), np.empty_like(k)
        chunk = self.canonical_chunk(q, d) if chunk is None else chunk
        self.lib.oracle_qk_norm_rope(dtype_code(q), _ptr(q), _ptr(k), _ptr(np.ascontiguousarray(qw)),
                                     _ptr(np.ascontiguousarray(kw)), _ptr(q_out), _ptr(k_out), t, hq, hk, d, offset,
                                     eps, base, chunk)
        return q_out, k_out

    def row_argmax(self, x):
        x = np.ascontiguousarray(x)
        rows, cols = x.shape
        out = np.empty(rows, dtype=np.int64)
        self.lib.oracle_row_argmax(dtype_code(x), _ptr(x), rows, cols, cols, _ptr(out))
        return out

    def linear(self, x, weight):
        x, weight = np.ascontiguousarray(x), np.ascontiguousarray(weight)
        rows, fin = x.shape
        fout = weight.shape[0]
        out = np.empty((rows, fout), dtype=x.dtype)
        self.lib.oracle_linear(dtype_code(x), _ptr(x), _ptr(weight), _ptr(out), rows, fin, fout)
        return out

    # -- decoder (fixed-order restatements of the device decoder) --
    def pexp(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.oracle_pexp_array(_ptr(x), _ptr(out), x.size)
        return out

    def silu_mul_pexp(self, gate, up):
        gate, up = np.ascontiguousarray(gate), np.ascontiguousarray(up)
        out = np.empty_like(gate)
        self.lib.oracle_silu_mul_pexp(_ptr(gate), _ptr(up), _ptr(out), gate.size)
        return out

    def linear_canonical(self, x, weight, f32_out: bool = False):
        """x [M, K] bf16 times weight [N, K] bf16 transposed, canonical lane order; bf16 [M, N] (or f32)."""
        x, weight = np.ascontiguousarray(x), np.ascontiguousarray(weight)
        m, k = x.shape
        n = weight.shape[0]
        out = np.empty((m, n), dtype=np.float32 if f32_out else np.uint16)
        self.lib.oracle_linear_canonical(_ptr(x), k, _ptr(weight), m, k, n, None if f32_out else _ptr(out),
                                         _ptr(out) if f32_out else None)
        return out

    def matmul(self, lhs, rhs, out_dtype=None):
        """ops::matmul in the device order: lhs [.., m, k], rhs [.., k, n] numpy arrays of any strides (uint16 = bf16,
        float32 = f32); out_dtype np.uint16 / np.float32 (default: the reference's rule)."""
        if out_dtype is None:
            out_dtype = lhs.dtype if lhs.dtype == rhs.dtype else np.float32
        l3 = lhs if lhs.ndim == 3 else lhs[None]
        r3 = rhs if rhs.ndim == 3 else rhs[None]
        b, m, k = l3.shape
        n = r3.shape[2]
        xs = _i64([st // l3.itemsize for st in l3.strides])
        ws = _i64([st // r3.itemsize for st in r3.strides])
        out = np.empty((b, m, n), dtype=out_dtype)
        self.lib.oracle_matmul_canonical(dtype_code(l3), l3.ctypes.data_as(_p), xs, dtype_code(r3), r3.ctypes.data_as(_p),
                                         ws, dtype_code(out), _ptr(out), b, m, k, n)
        return out if lhs.ndim == 3 else out[0]

    def decoder_attention(self, q, k_cache, v_cache, pos0: int):
        """q [T, Hq, D], caches [cap, Hkv, D] (bf16); query t at position pos0 + t. Returns ctx [T, Hq, D]."""
        q = np.ascontiguousarray(q)
        k_cache, v_cache = np.ascontiguousarray(k_cache), np.ascontiguousarray(v_cache)
        t, hq, d = q.shape
        hkv = k_cache.shape[1]
        out = np.empty_like(q)
        self.lib.oracle_decoder_attention(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), t, hq, hkv, d, pos0)
        return out


class ReferenceUnavailable(RuntimeError):
    """The reference function needs a oneDNN primitive, which this environment does not have."""


class Reference:
    """The reference's own op sources compiled in place (oracle/_ref/libcppinf_ref.so)."""

    def __init__(self, path: Path | str | None = None):
        path = Path(path or os.environ.get("CPPINF_REFERENCE_LIB", REFERENCE_LIB))
        if not path.exists():
            raise RuntimeError(f"reference library missing at {path}; build it with `make -C oracle`")
        self.lib = ctypes.CDLL(str(path))
        sig = {
            "ref_f32_to_bf16": ([_p, _p, _l], None),
            "ref_scaled_causal_softmax": ([_p, _p, _l, _l, _l, _f], _i),
            "ref_position_causal_softmax": ([_p, _p, _l, _l, _l, _l, _f, _p, _p, _p], _i),
            "ref_apply_rope": ([_i, _p, _l, _l, _l, _l, _f, _l, _p], _i),
            "ref_apply_rope_batched": ([_i, _p, _l, _l, _l, _l, _p, _f, _p], _i),
            "ref_add": ([_i, _p, _p, _p, _l], _i),
            "ref_mul": ([_i, _p, _p, _p, _l], _i),
            "ref_silu": ([_i, _p, _p, _l], _i),
            "ref_silu_mul": ([_i, _p, _p, _p, _l], _i),
            "ref_cast": ([_i, _p, _i, _p, _l], _i),
            "ref_rms_norm": ([_i, _p, _p, _p, _l, _l, _f], _i),
            "ref_rms_norm_validate": ([_i, _l, _p, _i, _l, _p, _f], _i),
            "ref_last_error": ([], ctypes.c_char_p),
        }
        for name, (args, res) in sig.items():
            fn = getattr(self.lib, name)
            fn.argtypes = args
            fn.restype = res

    def _check(self, status: int) -> None:
        if status == 0:
            return
        msg = self.lib.ref_last_error().decode()
        if status == -1:
            raise ValueError(msg)
        if status == -2:
            raise IndexError(msg)
        if status == -3:
            raise OverflowError(msg)
        if status == -6:
            raise ReferenceUnavailable(msg)
        raise RuntimeError(msg)

    def f32_to_bf16(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.ref_f32_to_bf16(_ptr(x), _ptr(out), x.size)
        return out

    def scaled_causal_softmax(self, x, scale):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q, k = x.shape[-2], x.shape[-1]
        out = np.empty_like(x)
        self._check(self.lib.ref_scaled_causal_softmax(_ptr(x), _ptr(out), x.size // (q * k), q, k, scale))
        return out

    def position_causal_softmax(self, x, scale, query_offsets, query_lengths, key_lengths):
        x = np.ascontiguousarray(x, dtype=np.float32)
        b, h, q, k = x.shape
        out = np.empty_like(x)
        self._check(self.lib.ref_position_causal_softmax(_ptr(x), _ptr(out), b, h, q, k, scale, _i64(query_offsets),
                                                         _i64(query_lengths), _i64(key_lengths)))
        return out

    def apply_rope(self, x, offset=0, base=1e6, seq_dim=1):
        x = np.ascontiguousarray(x)
        d0, d1, d = x.shape
        out = np.empty_like(x)
        self._check(self.lib.ref_apply_rope(dtype_code(x), _ptr(x), d0, d1, d, offset, base, seq_dim, _ptr(out)))
        return out

    def apply_rope_batched(self, x, offsets, base=1e6):
        x = np.ascontiguousarray(x)
        b, s, h, d = x.shape
        out = np.empty_like(x)
        self._check(self.lib.ref_apply_rope_batched(dtype_code(x), _ptr(x), b, s, h, d, _i64(offsets), base,
                                                    _ptr(out)))
        return out

    def add(self, a, b):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        out = np.empty_like(a)
        self._check(self.lib.ref_add(dtype_code(a), _ptr(a), _ptr(b), _ptr(out), a.size))
        return out

    def mul(self, a, b):
        a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
        out = np.empty_like(a)
        self._check(self.lib.ref_mul(dtype_code(a), _ptr(a), _ptr(b), _ptr(out), a.size))
        return out

    def silu(self, x):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        self._check(self.lib.ref_silu(dtype_code(x), _ptr(x), _ptr(out), x.size))
        return out

    def silu_mul(self, gate, up):
        gate, up = np.ascontiguousarray(gate), np.ascontiguousarray(up)
        out = np.empty_like(gate)
        self._check(self.lib.ref_silu_mul(dtype_code(gate), _ptr(gate), _ptr(up), _ptr(out), gate.size))
        return out

    def cast(self, x, to_bf16: bool):
        x = np.ascontiguousarray(x)
        out = np.empty(x.shape, dtype=np.uint16 if to_bf16 else np.float32)
        self._check(self.lib.ref_cast(dtype_code(x), _ptr(x), dtype_code(out), _ptr(out), x.size))
        return out

    def rms_norm(self, x, w, eps):
        x = np.ascontiguousarray(x)
        out = np.empty_like(x)
        width = w.shape[0]
        self._check(self.lib.ref_rms_norm(dtype_code(x), _ptr(x), _ptr(np.ascontiguousarray(w)), _ptr(out),
                                          x.size // width, width, eps))
        return out

    def rms_norm_validate(self, x_dtype: int, x_dims, w_dtype: int, w_dims, eps: float) -> None:
        """Runs the reference's rms_norm validation; raises what it raises (ReferenceUnavailable once it passes)."""
        self._check(self.lib.ref_rms_norm_validate(x_dtype, len(x_dims), _i64(x_dims), w_dtype, len(w_dims),
                                                   _i64(w_dims), eps))


def reference_available() -> bool:
    return REFERENCE_LIB.exists()


def reference_tree() -> Path | None:
    """The reference's source tree, when it is on this machine: $CPPINF_REFERENCE_DIR, else the directory that
    oracle/Makefile compiled oracle/_ref from (recorded in oracle/_ref/reference_dir.txt). None when neither exists."""
    candidates = [os.environ.get("CPPINF_REFERENCE_DIR")]
    recorded = ORACLE_DIR / "_ref" / "reference_dir.txt"
    if recorded.exists():
        candidates.append(recorded.read_text().strip())
    for c in candidates:
        if c and (Path(c) / "src").is_dir():
            return Path(c)
    return None
