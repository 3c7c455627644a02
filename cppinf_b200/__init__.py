"""cppinf_b200: sm_100a kernels for the tensor-op hot path of cppinf's Qwen3 decoder.

Layers:
    include/cppinf_b200.h        the C ABI (device pointers, sizes, a stream); the drop-in boundary
    cppinf_b200/csrc/            the CUDA kernels and the C ABI implementation (libcppinf_b200.so)
    cppinf_b200/cpp/             the C++20 drop-in of cppinf's tensors/ops API on top of the C ABI (libcppinf_ops.so)
    cppinf_b200.capi             ctypes binding of the C ABI
    cppinf_b200.ops              Python mirror of the op interface over torch CUDA tensors
    cppinf_b200.shard            row partitioning across GPUs (one process per GPU)
"""

from . import capi  # noqa: F401

__all__ = ["capi"]
