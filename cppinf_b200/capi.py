"""ctypes binding of the cppinf_b200 C ABI (include/cppinf_b200.h).

The shared library is built in-tree (``make -C cppinf_b200``) into ``cppinf_b200/_lib/libcppinf_b200.so``. Loading
fails loudly when it is missing: there is no CPU fallback behind these entry points.

Every wrapper takes raw integers for device pointers and streams, checks the returned status and raises the Python
counterpart of the exception the reference throws for the same condition:

    CPPINF_ERR_INVALID_ARGUMENT -> ValueError      (std::invalid_argument)
    CPPINF_ERR_OUT_OF_RANGE     -> IndexError      (std::out_of_range)
    CPPINF_ERR_OVERFLOW         -> OverflowError   (std::overflow_error)
    CPPINF_ERR_UNSUPPORTED      -> NotImplementedError
    CPPINF_ERR_CUDA             -> RuntimeError
"""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
LIB_PATH = PACKAGE_DIR / "_lib" / "libcppinf_b200.so"
HEADER_PATH = REPO_ROOT / "include" / "cppinf_b200.h"

DTYPE_BF16 = 0
DTYPE_F32 = 1

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_OUT_OF_RANGE = -2
ERR_OVERFLOW = -3
ERR_UNSUPPORTED = -4
ERR_CUDA = -5

_EXCEPTIONS = {
    ERR_INVALID_ARGUMENT: ValueError,
    ERR_OUT_OF_RANGE: IndexError,
    ERR_OVERFLOW: OverflowError,
    ERR_UNSUPPORTED: NotImplementedError,
    ERR_CUDA: RuntimeError,
}

_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_ptr = ctypes.c_void_p
_int = ctypes.c_int

# name -> argument types; every entry point returns int unless listed in _RESTYPES.
_SIGNATURES = {
    "cppinf_abi_version": [],
    "cppinf_last_error": [],
    "cppinf_status_name": [_int],
    "cppinf_launch_count": [],
    "cppinf_set_wait_poll_limit": [ctypes.c_uint32],
    "cppinf_add": [_int, _ptr, _ptr, _ptr, _i64, _ptr],
    "cppinf_mul": [_int, _ptr, _ptr, _ptr, _i64, _ptr],
    "cppinf_silu": [_int, _ptr, _ptr, _i64, _ptr],
    "cppinf_cast": [_int, _ptr, _int, _ptr, _i64, _ptr],
    "cppinf_silu_mul": [_int, _ptr, _ptr, _ptr, _i64, _ptr],
    "cppinf_strided_copy": [_int, _ptr, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64), _ptr, _ptr],
    "cppinf_rms_norm": [_int, _ptr, _i64, _ptr, _ptr, _i64, _i64, _f32, _ptr],
    "cppinf_add_rms_norm": [_int, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _f32, _ptr],
    "cppinf_softmax_last_dim": [_int, _ptr, _ptr, _i64, _i64, _ptr],
    "cppinf_scaled_causal_softmax_f32": [_ptr, _ptr, _i64, _i64, _i64, _f32, _ptr],
    "cppinf_scaled_position_causal_softmax_f32": [
        _ptr, _ptr, _i64, _i64, _i64, _i64, _f32,
        ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64), _ptr,
    ],
    "cppinf_row_argmax": [_int, _ptr, _i64, _i64, _i64, _ptr, _ptr],
    "cppinf_rope_table": [_f32, _i64, _i64, ctypes.POINTER(_f32)],
    "cppinf_rope": [_int, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _i64, _ptr, _ptr],
    "cppinf_qk_norm_rope": [
        _int, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _f32, _ptr, _i64, _ptr,
    ],
    "cppinf_matmul": [_int, _ptr, ctypes.POINTER(_i64), _int, _ptr, ctypes.POINTER(_i64), _int, _ptr, _i64, _i64, _i64,
                      _i64, _ptr],
    "cppinf_linear": [_ptr, _i64, _ptr, _ptr, _i64, _i64, _i64, _ptr],
    "cppinf_linear_residual": [_ptr, _i64, _ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr],
    "cppinf_linear_silu_mul": [_ptr, _i64, _ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr],
    "cppinf_linear_tc": [_int, _ptr, _i64, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr, _ptr],
    "cppinf_linear_argmax": [_ptr, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr],
    "cppinf_linear_argmax_scratch_bytes": [_i64, _i64],
    "cppinf_linear_argmax_noalloc": [_ptr, _ptr, _ptr, _i64, _i64, _ptr, _ptr],
    "cppinf_decoder_attention": [_ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr],
    "cppinf_decoder_attention_tc": [_ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr],
    "cppinf_embedding": [_ptr, _i64, _i64, _ptr, _i64, _ptr, _ptr],
    "cppinf_qwen3_create": [ctypes.c_void_p, _i64, ctypes.POINTER(_ptr)],
    "cppinf_qwen3_destroy": [_ptr],
    "cppinf_qwen3_set_weight": [_ptr, ctypes.c_char_p, _ptr, _i64, _int],
    "cppinf_qwen3_forward": [_ptr, ctypes.POINTER(_i64), _i64, _ptr, _int, ctypes.POINTER(_i64), _ptr],
    "cppinf_qwen3_decode": [_ptr, _i64, ctypes.POINTER(_i64), _ptr],
    "cppinf_qwen3_load_safetensors": [_ptr, ctypes.c_char_p, ctypes.POINTER(_i64)],
    "cppinf_safetensors_info": [ctypes.c_char_p, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "cppinf_qwen3_reset": [_ptr, _ptr],
    "cppinf_qwen3_set_prefill": [_ptr, _int],
    "cppinf_qwen3_length": [_ptr],
    "cppinf_qwen3_step_launches": [_ptr],
    "cppinf_qwen3_cache_create": [_ptr, _i64, _i64, ctypes.POINTER(_ptr)],
    "cppinf_qwen3_cache_destroy": [_ptr],
    "cppinf_qwen3_cache_batch": [_ptr],
    "cppinf_qwen3_cache_lengths": [_ptr, ctypes.POINTER(_i64)],
    "cppinf_qwen3_forward_batch": [_ptr, _ptr, ctypes.POINTER(_i64), ctypes.POINTER(_i64), _i64, _i64, _ptr, _ptr],
}
_RESTYPES = {
    "cppinf_last_error": ctypes.c_char_p,
    "cppinf_status_name": ctypes.c_char_p,
    "cppinf_launch_count": ctypes.c_uint64,
    "cppinf_set_wait_poll_limit": ctypes.c_uint32,
    "cppinf_linear_argmax_scratch_bytes": _i64,
    "cppinf_qwen3_destroy": None,
    "cppinf_qwen3_length": _i64,
    "cppinf_qwen3_step_launches": _i64,
    "cppinf_qwen3_cache_destroy": None,
    "cppinf_qwen3_cache_batch": _i64,
}


class Qwen3ConfigC(ctypes.Structure):
    """cppinf_qwen3_config."""

    _fields_ = [
        ("vocab_size", _i64),
        ("hidden_size", _i64),
        ("intermediate_size", _i64),
        ("num_hidden_layers", _i64),
        ("num_attention_heads", _i64),
        ("num_key_value_heads", _i64),
        ("head_dim", _i64),
        ("rms_norm_eps", _f32),
        ("rope_theta", _f32),
    ]

_lib: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Names of every entry point declared in include/cppinf_b200.h."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"CPPINF_API\s+[\w\s\*]+?\b(cppinf_\w+)\s*\(", text)))


def load() -> ctypes.CDLL:
    """Loads the kernel library once and declares every signature. Raises if the library was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("CPPINF_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"cppinf_b200 kernel library not found at {path}; build it with `make -C cppinf_b200` "
            "(there is no CPU fallback for these ops)"
        )
    lib = ctypes.CDLL(str(path))
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().cppinf_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    """Raises the mapped exception for a non-zero status."""
    if status == OK:
        return
    exc = _EXCEPTIONS.get(status, RuntimeError)
    name = load().cppinf_status_name(status).decode()
    raise exc(f"{last_error()} [{name}{' in ' + what if what else ''}]")


def launch_count() -> int:
    return int(load().cppinf_launch_count())


def set_wait_poll_limit(polls: int) -> int:
    """Sets the process-wide poll limit of the kernels' first wait on staged copies; returns the previous one."""
    return int(load().cppinf_set_wait_poll_limit(int(polls)))


DEFAULT_POLL_LIMIT = 1 << 24


def call(name: str, *args) -> None:
    """Calls an entry point and raises on failure."""
    fn = getattr(load(), name)
    check(fn(*args), name)


def i64_array(values) -> ctypes.Array:
    arr = (_i64 * max(len(values), 1))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def rope_table(base: float, head_dim: int, positions: int):
    """Host-built RoPE angle table [positions, head_dim] (float32 numpy array), see cppinf_rope_table."""
    import numpy as np

    table = np.zeros((positions, head_dim), dtype=np.float32)
    call("cppinf_rope_table", float(base), int(head_dim), int(positions),
         table.ctypes.data_as(ctypes.POINTER(_f32)))
    return table


def safetensors_info(path) -> tuple[int, int]:
    """(tensor count, data offset) of a safetensors file, parsed by the library (cppinf_safetensors_info)."""
    count = _i64(0)
    offset = _i64(0)
    call("cppinf_safetensors_info", str(path).encode(), ctypes.byref(count), ctypes.byref(offset))
    return int(count.value), int(offset.value)
