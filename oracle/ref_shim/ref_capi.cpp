// C entry points into the reference's own op code, compiled from the reference sources where they lie (see
// oracle/Makefile). TEST INFRASTRUCTURE ONLY: the parity tests use these to pin the CPU oracle to the reference and,
// where the reference code runs without oneDNN, as a second checker; bench.py may time them as the reference CPU
// baseline.
//
// Including the reference's attention translation unit gives this file access to the position-aware causal softmax
// and the batched RoPE, which the reference keeps in an anonymous namespace (src/nn/qwen_attention.cpp:136-235).
//
// Return codes: 0 ok, -1 std::invalid_argument, -2 std::out_of_range, -3 std::overflow_error, -6 the reference code
// needs a oneDNN primitive (unavailable here), -7 any other exception. ref_last_error() holds the message.
#include "nn/qwen_attention.cpp"

#include <cstdint>
#include <cstring>
#include <span>
#include <string>
#include <vector>

#include "nn/rope.h"
#include "ops/elementwise_ops.h"
#include "ops/nn_ops.h"
#include "ops/tensor_ops.h"
#include "tensors/bfloat16.h"

namespace {

using cppinf::tensors::DType;
using cppinf::tensors::Shape;
using cppinf::tensors::Tensor;
using cppinf::tensors::TensorInfo;

thread_local std::string g_error;

DType to_dtype(int code) {
    return code == 0 ? DType::BF16 : DType::F32;
}

Tensor make_input(int dtype, std::vector<std::int64_t> dims, const void* data) {
    TensorInfo info{.name = "input", .dtype = to_dtype(dtype), .shape = Shape(std::move(dims)), .byte_offset = 0};
    const auto bytes = info.byte_size();
    std::vector<std::byte> storage(bytes);
    if (bytes != 0) {
        std::memcpy(storage.data(), data, bytes);
    }
    return Tensor(std::move(info), std::move(storage));
}

void copy_out(const Tensor& t, void* out) {
    if (t.byte_size() != 0) {
        std::memcpy(out, t.data().data(), t.byte_size());
    }
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        g_error.clear();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return -1;
    } catch (const std::out_of_range& e) {
        g_error = e.what();
        return -2;
    } catch (const std::overflow_error& e) {
        g_error = e.what();
        return -3;
    } catch (const dnnl::error& e) {
        g_error = e.what();
        return -6;
    } catch (const std::runtime_error& e) {
        g_error = e.what();
        return std::string(e.what()).find("oneDNN is not available") != std::string::npos ? -6 : -7;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -7;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error(void) {
    return g_error.c_str();
}

// tensors::float_to_bfloat16_bits, src/tensors/bfloat16.cpp:8-15
void ref_f32_to_bf16(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        y[i] = cppinf::tensors::float_to_bfloat16_bits(x[i]);
    }
}

// ops::scaled_causal_softmax_last_dim, src/ops/nn_ops.cpp:77-138
int ref_scaled_causal_softmax(const float* x, float* y, int64_t matrices, int64_t query_len, int64_t key_len,
                              float scale) {
    return guarded([&] {
        const auto in = make_input(1, {matrices, query_len, key_len}, x);
        copy_out(cppinf::ops::scaled_causal_softmax_last_dim(in.view(), scale), y);
    });
}

// scaled_position_causal_softmax_last_dim, src/nn/qwen_attention.cpp:164-235
int ref_position_causal_softmax(const float* x, float* y, int64_t batch, int64_t heads, int64_t query_cap,
                                int64_t key_cap, float scale, const int64_t* query_offsets,
                                const int64_t* query_lengths, const int64_t* key_lengths) {
    return guarded([&] {
        const auto in = make_input(1, {batch, heads, query_cap, key_cap}, x);
        std::vector<std::size_t> offsets(query_offsets, query_offsets + batch);
        std::vector<std::size_t> qlens(query_lengths, query_lengths + batch);
        std::vector<std::size_t> klens(key_lengths, key_lengths + batch);
        copy_out(cppinf::nn::scaled_position_causal_softmax_last_dim(in.view(), scale, offsets, qlens, klens), y);
    });
}

// nn::apply_rope, src/nn/rope.cpp:58-109, on a dense [d0, d1, head_dim] tensor.
int ref_apply_rope(int dtype, const void* x, int64_t d0, int64_t d1, int64_t head_dim, int64_t offset, float base,
                   int64_t seq_dim, void* y) {
    return guarded([&] {
        const auto in = make_input(dtype, {d0, d1, head_dim}, x);
        copy_out(cppinf::nn::apply_rope(in.view(), static_cast<std::size_t>(offset), base,
                                        static_cast<std::size_t>(seq_dim)),
                 y);
    });
}

// apply_rope_batched, src/nn/qwen_attention.cpp:136-162, on a dense [batch, seq, heads, head_dim] tensor.
int ref_apply_rope_batched(int dtype, const void* x, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                           const int64_t* offsets, float base, void* y) {
    return guarded([&] {
        const auto in = make_input(dtype, {batch, seq, heads, head_dim}, x);
        std::vector<std::size_t> offs(offsets, offsets + batch);
        copy_out(cppinf::nn::apply_rope_batched(in.view(), offs, base, "ref_rope"), y);
    });
}

// ops::add / ops::mul, src/ops/elementwise_ops.cpp:28-36
int ref_add(int dtype, const void* a, const void* b, void* out, int64_t n) {
    return guarded([&] {
        const auto ta = make_input(dtype, {n}, a);
        const auto tb = make_input(dtype, {n}, b);
        copy_out(cppinf::ops::add(ta.view(), tb.view()), out);
    });
}

int ref_mul(int dtype, const void* a, const void* b, void* out, int64_t n) {
    return guarded([&] {
        const auto ta = make_input(dtype, {n}, a);
        const auto tb = make_input(dtype, {n}, b);
        copy_out(cppinf::ops::mul(ta.view(), tb.view()), out);
    });
}

// ops::silu, src/ops/nn_ops.cpp:44-48
int ref_silu(int dtype, const void* x, void* y, int64_t n) {
    return guarded([&] {
        const auto t = make_input(dtype, {n}, x);
        copy_out(cppinf::ops::silu(t.view()), y);
    });
}

// The Qwen MLP's gate product, src/nn/qwen_mlp.cpp:65-66: ops::mul(ops::silu(gate), up).
int ref_silu_mul(int dtype, const void* gate, const void* up, void* out, int64_t n) {
    return guarded([&] {
        const auto g = make_input(dtype, {n}, gate);
        const auto u = make_input(dtype, {n}, up);
        const auto activated = cppinf::ops::silu(g.view());
        copy_out(cppinf::ops::mul(activated.view(), u.view()), out);
    });
}

// ops::cast, src/ops/tensor_ops.cpp:138-143
int ref_cast(int src_dtype, const void* x, int dst_dtype, void* y, int64_t n) {
    return guarded([&] {
        const auto t = make_input(src_dtype, {n}, x);
        copy_out(cppinf::ops::cast(t.view(), to_dtype(dst_dtype)), y);
    });
}

// ops::rms_norm, src/ops/nn_ops.cpp:140-201. Needs oneDNN's reduction primitive: returns -6 here.
int ref_rms_norm(int dtype, const void* x, const void* w, void* y, int64_t rows, int64_t width, float eps) {
    return guarded([&] {
        const auto tx = make_input(dtype, {rows, width}, x);
        const auto tw = make_input(dtype, {width}, w);
        copy_out(cppinf::ops::rms_norm(tx.view(), tw.view(), eps), y);
    });
}

// ops::rms_norm validation only: calls the reference with the given shapes and reports the exception it throws
// before any arithmetic (or -6 once validation passed and oneDNN would be needed).
int ref_rms_norm_validate(int x_dtype, int64_t x_rank, const int64_t* x_dims, int w_dtype, int64_t w_rank,
                          const int64_t* w_dims, float eps) {
    return guarded([&] {
        std::vector<std::int64_t> xd(x_dims, x_dims + x_rank);
        std::vector<std::int64_t> wd(w_dims, w_dims + w_rank);
        TensorInfo xi{.name = "input", .dtype = to_dtype(x_dtype), .shape = Shape(xd), .byte_offset = 0};
        TensorInfo wi{.name = "weight", .dtype = to_dtype(w_dtype), .shape = Shape(wd), .byte_offset = 0};
        std::vector<std::byte> xb(xi.byte_size());
        std::vector<std::byte> wb(wi.byte_size());
        const Tensor tx(xi, xb);
        const Tensor tw(wi, wb);
        copy_out(cppinf::ops::rms_norm(tx.view(), tw.view(), eps), nullptr);
    });
}

}  // extern "C"
