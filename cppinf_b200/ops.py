"""Python mirror of cppinf's op interface (src/ops/nn_ops.h, src/ops/elementwise_ops.h, src/ops/tensor_ops.h:15,
src/nn/rope.h) running on the sm_100a kernels of the C ABI.

Tensors are torch CUDA tensors, used only as device memory (``data_ptr``) and for the current stream; the arithmetic
is the library's. Argument meaning, validation order and messages follow the reference functions cited on each op.
Non-contiguous inputs are materialised with the library's own strided-gather kernel before the op runs.

Also exposed: the fused forms the Qwen3 decoder block uses (residual add + RMSNorm, SiLU(gate)*up, per-head q/k
RMSNorm + RoPE), the row argmax of the greedy sampler, and the position-aware causal softmax of attention.
"""

from __future__ import annotations

import math
import threading

import torch

from . import capi

_DTYPES = {torch.bfloat16: capi.DTYPE_BF16, torch.float32: capi.DTYPE_F32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(t: torch.Tensor, op: str) -> int:
    # ops::detail::validate_supported_float_dtype, src/ops/op_utils.h:18-27
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise ValueError(f"{op} received an unsupported dtype.")
    return code


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("cppinf_b200 ops take CUDA tensors; copy host data with .to('cuda') first.")


def materialize(t: torch.Tensor) -> torch.Tensor:
    """Dense copy of a strided view made by the library's gather kernel (no-op for contiguous tensors)."""
    if t.is_contiguous():
        return t
    code = _dtype_code(t, "materialize")
    out = torch.empty(t.shape, dtype=t.dtype, device=t.device)
    dims = capi.i64_array(list(t.shape))
    strides = capi.i64_array(list(t.stride()))
    capi.call("cppinf_strided_copy", code, t.data_ptr(), t.dim(), dims, strides, out.data_ptr(), _stream())
    return out


# ---- elementwise ------------------------------------------------------------------------------------------------


def _validate_elementwise(lhs: torch.Tensor, rhs: torch.Tensor, op: str) -> int:
    # validate_elementwise_inputs, src/ops/elementwise_ops.cpp:14-24
    if lhs.dtype != rhs.dtype:
        raise ValueError(f"{op} requires matching tensor dtypes.")
    if lhs.shape != rhs.shape:
        raise ValueError(f"{op} requires matching tensor shapes.")
    return _dtype_code(lhs, op)


def add(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """ops::add, src/ops/elementwise_ops.h:10."""
    code = _validate_elementwise(lhs, rhs, "add")
    _require_cuda(lhs, rhs)
    lhs, rhs = materialize(lhs), materialize(rhs)
    out = torch.empty_like(lhs)
    capi.call("cppinf_add", code, lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(), lhs.numel(), _stream())
    return out


def mul(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    """ops::mul, src/ops/elementwise_ops.h:14."""
    code = _validate_elementwise(lhs, rhs, "mul")
    _require_cuda(lhs, rhs)
    lhs, rhs = materialize(lhs), materialize(rhs)
    out = torch.empty_like(lhs)
    capi.call("cppinf_mul", code, lhs.data_ptr(), rhs.data_ptr(), out.data_ptr(), lhs.numel(), _stream())
    return out


def silu(input: torch.Tensor) -> torch.Tensor:
    """ops::silu, src/ops/nn_ops.h:9."""
    code = _dtype_code(input, "silu")
    _require_cuda(input)
    x = materialize(input)
    out = torch.empty_like(x)
    capi.call("cppinf_silu", code, x.data_ptr(), out.data_ptr(), x.numel(), _stream())
    return out


def cast(input: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """ops::cast, src/ops/tensor_ops.h:15."""
    src = _dtype_code(input, "cast")
    if dtype not in _DTYPES:
        raise ValueError("cast received an unsupported dtype.")
    _require_cuda(input)
    x = materialize(input)
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    capi.call("cppinf_cast", src, x.data_ptr(), _DTYPES[dtype], out.data_ptr(), x.numel(), _stream())
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """ops::mul(ops::silu(gate), up) in one pass, as qwen_mlp calls them (src/nn/qwen_mlp.cpp:65-66)."""
    code = _validate_elementwise(gate, up, "mul")
    _require_cuda(gate, up)
    gate, up = materialize(gate), materialize(up)
    out = torch.empty_like(gate)
    capi.call("cppinf_silu_mul", code, gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(), _stream())
    return out


# ---- row reductions ---------------------------------------------------------------------------------------------


def _validate_last_dim(input: torch.Tensor, op: str) -> int:
    # validate_last_dim_operation_input, src/ops/nn_ops.cpp:30-40
    code = _dtype_code(input, op)
    if input.dim() == 0:
        raise ValueError(f"{op} requires a tensor with rank at least 1.")
    if input.shape[-1] == 0:
        raise ValueError(f"{op} requires a non-empty last dimension.")
    return code


def _validate_rms(input: torch.Tensor, weight: torch.Tensor, epsilon: float) -> int:
    # src/ops/nn_ops.cpp:140-159
    code = _validate_last_dim(input, "rms_norm")
    if epsilon < 0.0:
        raise ValueError("rms_norm requires a non-negative epsilon.")
    if input.dtype != weight.dtype:
        raise ValueError("rms_norm requires matching tensor dtypes.")
    if weight.dim() != 1:
        raise ValueError("rms_norm requires a rank-1 weight tensor.")
    if weight.shape[0] != input.shape[-1]:
        raise ValueError("rms_norm weight size must match the input last dimension.")
    return code


def rms_norm(input: torch.Tensor, weight: torch.Tensor, epsilon: float) -> torch.Tensor:
    """ops::rms_norm, src/ops/nn_ops.h:22. Row-strided inputs (a uniform stride between rows, dense rows) are read in
    place; other views are materialised first."""
    code = _validate_rms(input, weight, epsilon)
    _require_cuda(input, weight)
    width = input.shape[-1]
    rows = input.numel() // width
    x = input
    row_stride = width
    if not x.is_contiguous():
        # A 2-D row-strided view is consumed directly, anything else is gathered to dense first.
        if x.dim() == 2 and x.stride(1) == 1 and x.stride(0) >= width:
            row_stride = x.stride(0)
        else:
            x = materialize(x)
    w = materialize(weight)
    out = torch.empty(input.shape, dtype=input.dtype, device=input.device)
    capi.call("cppinf_rms_norm", code, x.data_ptr(), row_stride, w.data_ptr(), out.data_ptr(), rows, width,
              float(epsilon), _stream())
    return out


def add_rms_norm(a: torch.Tensor, b: torch.Tensor, weight: torch.Tensor, epsilon: float,
                 out_sum: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Residual add then RMSNorm (src/nn/qwen_decoder_block.cpp:80-84): returns (a + b, rms_norm(a + b))."""
    code = _validate_elementwise(a, b, "add")
    _validate_rms(a, weight, epsilon)
    _require_cuda(a, b, weight)
    a, b, w = materialize(a), materialize(b), materialize(weight)
    width = a.shape[-1]
    rows = a.numel() // width
    s = torch.empty_like(a) if out_sum is None else out_sum
    y = torch.empty_like(a)
    capi.call("cppinf_add_rms_norm", code, a.data_ptr(), b.data_ptr(), w.data_ptr(), s.data_ptr(), y.data_ptr(),
              rows, width, float(epsilon), _stream())
    return s, y


def softmax_last_dim(input: torch.Tensor) -> torch.Tensor:
    """ops::softmax_last_dim, src/ops/nn_ops.h:13."""
    code = _validate_last_dim(input, "softmax_last_dim")
    _require_cuda(input)
    x = materialize(input)
    width = x.shape[-1]
    out = torch.empty_like(x)
    capi.call("cppinf_softmax_last_dim", code, x.data_ptr(), out.data_ptr(), x.numel() // width, width, _stream())
    return out


def scaled_causal_softmax_last_dim(input: torch.Tensor, scale: float) -> torch.Tensor:
    """ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.h:17 (f32 result, like the reference)."""
    op = "scaled_causal_softmax_last_dim"
    _validate_last_dim(input, op)
    if input.dim() < 2:
        raise ValueError(f"{op} requires a tensor with rank at least 2.")
    if not math.isfinite(scale):
        raise ValueError(f"{op} requires a finite scale.")
    q, k = input.shape[-2], input.shape[-1]
    if q == 0 or k == 0:
        raise ValueError(f"{op} requires non-empty attention dimensions.")
    if q != k:
        raise ValueError(f"{op} requires square attention score matrices.")
    _require_cuda(input)
    x = materialize(input)
    if x.dtype != torch.float32:
        x = cast(x, torch.float32)
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    capi.call("cppinf_scaled_causal_softmax_f32", x.data_ptr(), out.data_ptr(), x.numel() // (q * k), q, k,
              float(scale), _stream())
    return out


def scaled_position_causal_softmax_last_dim(input: torch.Tensor, scale: float, query_position_offsets,
                                            query_lengths, key_lengths) -> torch.Tensor:
    """The attention softmax of src/nn/qwen_attention.cpp:164-235 on f32 [batch, heads, Qcap, Kcap]."""
    if input.dim() != 4:
        raise ValueError("qwen_attention batched softmax requires a rank-4 tensor.")
    if not math.isfinite(scale):
        raise ValueError("qwen_attention batched softmax requires a finite scale.")
    batch = input.shape[0]
    for name, seq in (("query offsets", query_position_offsets), ("query lengths", query_lengths),
                      ("key lengths", key_lengths)):
        if len(seq) != batch:
            raise ValueError(f"qwen_attention {name} sequence_lengths must match the batch size.")
    _require_cuda(input)
    x = materialize(input)
    if x.dtype != torch.float32:
        x = cast(x, torch.float32)
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    capi.call("cppinf_scaled_position_causal_softmax_f32", x.data_ptr(), out.data_ptr(), batch, x.shape[1],
              x.shape[2], x.shape[3], float(scale), capi.i64_array(query_position_offsets),
              capi.i64_array(query_lengths), capi.i64_array(key_lengths), _stream())
    return out


def row_argmax(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token pick of src/cli/cli_app.cpp:72-94 for every row of [rows, vocab] logits (int64 [rows])."""
    code = _dtype_code(logits, "row_argmax")
    if logits.dim() != 2:
        raise ValueError("CLI generation requires rank-2 logits.")
    _require_cuda(logits)
    rows, cols = logits.shape
    x = logits
    if x.stride(-1) != 1:
        x = materialize(x)
    row_stride = x.stride(0) if rows > 1 else cols
    out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    capi.call("cppinf_row_argmax", code, x.data_ptr(), rows, cols, row_stride, out.data_ptr(), _stream())
    return out


# ---- RoPE -------------------------------------------------------------------------------------------------------

_table_lock = threading.Lock()
_tables: dict[tuple[float, int, int], torch.Tensor] = {}


def rope_table(rope_base: float, head_dim: int, positions: int, device: torch.device | int | None = None):
    """Device copy of the host-built angle table (cppinf_rope_table), cached per (base, head_dim, device) and grown
    to cover `positions` (rounded up to a power of two)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    key = (float(rope_base), int(head_dim), dev.index)
    with _table_lock:
        table = _tables.get(key)
        if table is None or table.shape[0] < positions:
            n = 1 << max(int(positions - 1).bit_length(), 6)
            host = capi.rope_table(rope_base, head_dim, n)
            table = torch.from_numpy(host).to(dev)
            _tables[key] = table
    return table


def apply_rope(input: torch.Tensor, sequence_position_offset: int = 0, rope_base: float = 1000000.0,
               sequence_dimension: int = 1) -> torch.Tensor:
    """nn::apply_rope, src/nn/rope.h:12-13, on a rank-3 tensor."""
    # validate_rope_input, src/nn/rope.cpp:33-54
    code = _dtype_code(input, "apply_rope")
    if input.dim() != 3:
        raise ValueError("apply_rope requires a rank-3 tensor.")
    if not math.isfinite(rope_base) or rope_base <= 0.0:
        raise ValueError("apply_rope requires a positive finite rope base.")
    if sequence_dimension > 1:
        raise ValueError("apply_rope requires the sequence dimension to be 0 or 1.")
    d0, d1, d = input.shape
    for name, v in (("rope dim 0", d0), ("rope dim 1", d1), ("rope head size", d)):
        if v == 0:
            raise ValueError(f"{name} must be non-zero.")
    if d % 2 != 0:
        raise ValueError("apply_rope requires an even head size.")
    _require_cuda(input)
    seq = input.shape[sequence_dimension]
    table = rope_table(rope_base, d, sequence_position_offset + seq, input.device)
    out = torch.empty(input.shape, dtype=input.dtype, device=input.device)
    s0, s1, s2 = input.stride()
    capi.call("cppinf_rope", code, input.data_ptr(), d0, d1, d, s0, s1, s2, sequence_dimension,
              sequence_position_offset, table.data_ptr(), table.shape[0], out.data_ptr(), _stream())
    return out


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 epsilon: float, position_offset: int = 0, rope_base: float = 1000000.0,
                 out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head RMSNorm of q [T, Hq, D] and k [T, Hk, D] followed by RoPE at positions position_offset + t
    (src/nn/qwen_attention.cpp:383-390), one kernel for both tensors."""
    code = _validate_rms(q, q_weight, epsilon)
    _validate_rms(k, k_weight, epsilon)
    if q.dtype != k.dtype:
        raise ValueError("qk_norm_rope requires matching tensor dtypes.")
    if q.dim() != 3 or k.dim() != 3 or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError("qk_norm_rope requires q [T, Hq, D] and k [T, Hk, D].")
    _require_cuda(q, k, q_weight, k_weight)
    q, k = materialize(q), materialize(k)
    tokens, hq, d = q.shape
    hk = k.shape[1]
    table = rope_table(rope_base, d, position_offset + tokens, q.device)
    q_out, k_out = out if out is not None else (torch.empty_like(q), torch.empty_like(k))
    capi.call("cppinf_qk_norm_rope", code, q.data_ptr(), k.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(),
              q_out.data_ptr(), k_out.data_ptr(), tokens, hq, hk, d, position_offset, float(epsilon),
              table.data_ptr(), table.shape[0], _stream())
    return q_out, k_out


# ---- decoder: projections and attention ---------------------------------------------------------------------------


def matmul(lhs: torch.Tensor, rhs: torch.Tensor, output_dtype: torch.dtype | None = None) -> torch.Tensor:
    """ops::matmul, src/ops/matmul.cpp:85-114: rank-2 [m, k] x [k, n] or rank-3 [b, m, k] x [b, k, n], f32/bf16, any
    strides (views are read in place). Output dtype as the reference resolves it (:14-24) and validated as
    :26-60."""
    code_l = _dtype_code(lhs, "matmul")
    code_r = _dtype_code(rhs, "matmul")
    out = output_dtype if output_dtype is not None else (lhs.dtype if lhs.dtype == rhs.dtype else torch.float32)
    code_o = _dtype_code(torch.empty(0, dtype=out), "matmul")
    if lhs.dtype == rhs.dtype:
        if out != lhs.dtype and (lhs.dtype != torch.bfloat16 or out != torch.float32):
            raise ValueError("matmul output dtype must match the input dtype, except BF16 inputs may request an F32 "
                             "result.")
    elif out != torch.float32:
        raise ValueError("matmul requires an F32 result when input dtypes differ.")
    if lhs.dim() != rhs.dim():
        raise ValueError("matmul requires tensors with matching rank.")
    if lhs.dim() not in (2, 3):
        raise ValueError("matmul requires rank-2 or rank-3 tensors.")
    if lhs.dim() == 3 and lhs.shape[0] != rhs.shape[0]:
        raise ValueError("matmul requires matching batch dimensions.")
    if lhs.shape[-1] != rhs.shape[-2]:
        raise ValueError("matmul inner dimensions must match.")
    _require_cuda(lhs, rhs)
    l3 = lhs if lhs.dim() == 3 else lhs.unsqueeze(0)
    r3 = rhs if rhs.dim() == 3 else rhs.unsqueeze(0)
    b, m, k = l3.shape
    n = r3.shape[2]
    y = torch.empty(b, m, n, dtype=out, device=lhs.device)
    capi.call("cppinf_matmul", code_l, l3.data_ptr(), capi.i64_array(l3.stride()), code_r, r3.data_ptr(),
              capi.i64_array(r3.stride()), code_o, y.data_ptr(), b, m, k, n, _stream())
    return y if lhs.dim() == 3 else y[0]


def _validate_linear(input: torch.Tensor, weight: torch.Tensor, op: str) -> tuple[torch.Tensor, int, int, int]:
    # validate_projection_weight, src/nn/qwen_common.cpp:39-49, and matmul's dtype rules, src/ops/matmul.cpp:28-45
    if input.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError(f"{op} requires bf16 input and weight.")
    if weight.dim() != 2:
        raise ValueError(f"{op} weight must be rank-2.")
    if input.dim() < 1 or input.shape[-1] != weight.shape[1]:
        raise ValueError("matmul inner dimensions must match.")
    _require_cuda(input, weight)
    x = materialize(input).reshape(-1, input.shape[-1])
    return x, x.shape[0], weight.shape[1], weight.shape[0]


def linear(input: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """nn::detail::linear_project, src/nn/qwen_common.cpp:15-37: input [..., in] times weight [out, in]^T, bf16."""
    x, rows, fin, fout = _validate_linear(input, weight, "linear")
    out = torch.empty(*input.shape[:-1], fout, dtype=torch.bfloat16, device=input.device)
    capi.call("cppinf_linear", x.data_ptr(), fin, materialize(weight).data_ptr(), out.data_ptr(), rows, fin, fout,
              _stream())
    return out


def linear_residual(input: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """residual + linear(input, weight) (src/nn/qwen_decoder_block.cpp:80-89); `out` may be `residual`."""
    x, rows, fin, fout = _validate_linear(input, weight, "linear_residual")
    if residual.dtype != torch.bfloat16 or residual.shape != (*input.shape[:-1], fout):
        raise ValueError("add requires matching tensor shapes.")
    residual = materialize(residual)
    out = torch.empty_like(residual) if out is None else out
    capi.call("cppinf_linear_residual", x.data_ptr(), fin, materialize(weight).data_ptr(), residual.data_ptr(),
              out.data_ptr(), rows, fin, fout, _stream())
    return out


def linear_silu_mul(input: torch.Tensor, gate_weight: torch.Tensor, up_weight: torch.Tensor) -> torch.Tensor:
    """silu(linear(input, gate)) * linear(input, up), the MLP front of src/nn/qwen_mlp.cpp:58-66."""
    x, rows, fin, fout = _validate_linear(input, gate_weight, "linear_silu_mul")
    if up_weight.shape != gate_weight.shape or up_weight.dtype != torch.bfloat16:
        raise ValueError("qwen_mlp up_proj_weight has an unexpected shape.")
    out = torch.empty(*input.shape[:-1], fout, dtype=torch.bfloat16, device=input.device)
    capi.call("cppinf_linear_silu_mul", x.data_ptr(), fin, materialize(gate_weight).data_ptr(),
              materialize(up_weight).data_ptr(), out.data_ptr(), rows, fin, fout, _stream())
    return out


def linear_argmax(input: torch.Tensor, weight: torch.Tensor, with_logits: bool = False):
    """Greedy token of one row's logits input @ weight^T, computed without materialising the logits unless asked
    (the LM head of src/models/qwen3/qwen3_model.cpp:306-311 and src/cli/cli_app.cpp:72-94). Returns an int64
    device tensor [1] (and the bf16 logits [out] when with_logits)."""
    x, rows, fin, fout = _validate_linear(input, weight, "linear_argmax")
    if rows != 1:
        raise ValueError("linear_argmax takes a single row.")
    nbytes = int(capi.load().cppinf_linear_argmax_scratch_bytes(fout, fin))
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=input.device)
    token = torch.empty(1, dtype=torch.int64, device=input.device)
    logits = torch.empty(fout, dtype=torch.bfloat16, device=input.device) if with_logits else None
    capi.call("cppinf_linear_argmax", x.data_ptr(), materialize(weight).data_ptr(),
              logits.data_ptr() if logits is not None else None, fin, fout, token.data_ptr(), scratch.data_ptr(),
              _stream())
    return (token, logits) if with_logits else token


def linear_argmax_noalloc(input: torch.Tensor, weight: torch.Tensor, with_logits: bool = False):
    """linear_argmax with the library's static per-device scratch (cppinf_linear_argmax_noalloc): no scratch tensor
    is allocated. Calls on one device must not overlap in time (one stream, or synchronised)."""
    x, rows, fin, fout = _validate_linear(input, weight, "linear_argmax")
    if rows != 1:
        raise ValueError("linear_argmax takes a single row.")
    token = torch.empty(1, dtype=torch.int64, device=input.device)
    logits = torch.empty(fout, dtype=torch.bfloat16, device=input.device) if with_logits else None
    capi.call("cppinf_linear_argmax_noalloc", x.data_ptr(), materialize(weight).data_ptr(),
              logits.data_ptr() if logits is not None else None, fin, fout, token.data_ptr(), _stream())
    return (token, logits) if with_logits else token


def decoder_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, position: int) -> torch.Tensor:
    """Causal GQA attention of one sequence (src/nn/qwen_attention.cpp:236-333): q [T, Hq, D] at positions
    position .. position + T - 1, caches [capacity, Hkv, D]; returns the bf16 context [T, Hq, D]."""
    if q.dim() != 3 or k_cache.dim() != 3 or v_cache.shape != k_cache.shape:
        raise ValueError("qwen_attention requires rank-4 query, key, and value tensors.")
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("qwen_attention requires matching tensor dtypes.")
    if q.shape[2] != k_cache.shape[2]:
        raise ValueError("qwen_attention requires matching query/key/value head sizes.")
    _require_cuda(q, k_cache, v_cache)
    q, k_cache, v_cache = materialize(q), materialize(k_cache), materialize(v_cache)
    ctx = torch.empty_like(q)
    capi.call("cppinf_decoder_attention", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), ctx.data_ptr(),
              q.shape[0], q.shape[1], k_cache.shape[1], q.shape[2], int(position), k_cache.shape[0], _stream())
    return ctx


def embedding(table: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
    """Embedding lookup, src/models/qwen3/qwen3_model.cpp:132-165 (ids must be in range; they are checked here)."""
    if table.dim() != 2:
        raise ValueError("embedding_lookup requires a rank-2 embedding table.")
    ids = token_ids.to(device=table.device, dtype=torch.int64).contiguous()
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= table.shape[0]):
        raise IndexError("Qwen3Model token id is out of vocabulary range.")
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    capi.call("cppinf_embedding", materialize(table).data_ptr(), table.shape[0], table.shape[1], ids.data_ptr(),
              ids.numel(), out.data_ptr(), _stream())
    return out.reshape(*token_ids.shape, table.shape[1])
