// C++ tests of the drop-in op API. They follow the reference's own tests (tests/ops/ops_test.cpp,
// tests/nn/rope_test.cpp, tests/tensors/tensor_test.cpp) case by case: same inputs, same expected values and
// tolerances, same whole-tensor equality where the reference uses it. Host tensors go through the GPU; the Device*
// cases keep tensors resident on the GPU. HOST_TEST cases (metadata, views, validation) need no GPU.
#include <array>
#include <cstdint>
#include <cstring>
#include <initializer_list>
#include <stdexcept>
#include <string>
#include <vector>

#include "nn/rope.h"
#include "ops/elementwise_ops.h"
#include "ops/matmul.h"
#include "ops/nn_ops.h"
#include "ops/tensor_ops.h"
#include "tensors/bfloat16.h"
#include "tensors/tensor_utils.h"
#include "test_harness.h"

using cppinf::tensors::Device;
using cppinf::tensors::DType;
using cppinf::tensors::Shape;
using cppinf::tensors::Tensor;
using cppinf::tensors::TensorInfo;
using cppinf::tensors::TensorView;

namespace {

Shape shape(std::initializer_list<std::int64_t> dims) {
    return Shape(std::vector<std::int64_t>(dims));
}

Tensor f32(std::string_view name, std::initializer_list<std::int64_t> dims, std::initializer_list<float> values) {
    return cppinf::tensors::make_f32_tensor(name, shape(dims), std::span<const float>(values.begin(), values.size()));
}

Tensor bf16(std::string_view name, std::initializer_list<std::int64_t> dims, std::initializer_list<float> values) {
    return cppinf::tensors::make_bf16_tensor(name, shape(dims), std::span<const float>(values.begin(), values.size()));
}

Tensor bf16_bits(std::string_view name, std::initializer_list<std::int64_t> dims,
                 std::initializer_list<std::uint16_t> values) {
    return cppinf::tensors::make_bf16_bits_tensor(name, shape(dims),
                                                  std::span<const std::uint16_t>(values.begin(), values.size()));
}

std::vector<float> values_of(const Tensor& tensor) {
    const auto host = tensor.to(Device::host());
    const auto& info = host.tensor_info();
    std::vector<float> out(info.shape.num_elements());
    for (std::size_t i = 0; i < out.size(); ++i) {
        if (info.dtype == DType::BF16) {
            std::uint16_t bits = 0;
            std::memcpy(&bits, host.bytes().data() + 2 * i, 2);
            out[i] = cppinf::tensors::bfloat16_bits_to_float(bits);
        } else {
            std::memcpy(&out[i], host.bytes().data() + 4 * i, 4);
        }
    }
    return out;
}

void expect_values_near(const Tensor& tensor, std::initializer_list<float> expected, float tolerance) {
    const auto actual = values_of(tensor);
    ASSERT_EQ(actual.size(), expected.size());
    std::size_t i = 0;
    for (const float e : expected) {
        EXPECT_NEAR(e, actual[i], tolerance);
        ++i;
    }
}

Tensor on_gpu(const Tensor& t) {
    return t.to(Device::cuda(0));
}

} // namespace

// ---- tests/ops/ops_test.cpp --------------------------------------------------------------------------------------

TEST(OpsTest, GivenMatchingTensors_WhenAdding_ThenElementwiseSumIsReturned) {
    const auto lhs = f32("lhs", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    const auto rhs = f32("rhs", {2, 2}, {10.0f, 20.0f, 30.0f, 40.0f});
    EXPECT_TRUE(f32("add_result", {2, 2}, {11.0f, 22.0f, 33.0f, 44.0f}) == cppinf::ops::add(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenMatchingTensors_WhenMultiplying_ThenElementwiseProductIsReturned) {
    const auto lhs = f32("lhs", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    const auto rhs = f32("rhs", {2, 2}, {10.0f, 20.0f, 30.0f, 40.0f});
    EXPECT_TRUE(f32("mul_result", {2, 2}, {10.0f, 40.0f, 90.0f, 160.0f}) == cppinf::ops::mul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenF32Tensor_WhenCastingToBf16_ThenExpectedBitsAreReturned) {
    const auto input = f32("input", {2, 2}, {1.5f, -2.25f, 0.5f, -0.75f});
    EXPECT_TRUE(bf16_bits("cast_result", {2, 2}, {0x3fc0U, 0xc010U, 0x3f00U, 0xbf40U}) ==
                cppinf::ops::cast(input.view(), DType::BF16));
}

TEST(OpsTest, GivenBf16Tensor_WhenCastingToF32_ThenExpectedValuesAreReturned) {
    const auto input = bf16_bits("input", {2, 2}, {0x3fc0U, 0xc010U, 0x3f00U, 0xbf40U});
    EXPECT_TRUE(f32("cast_result", {2, 2}, {1.5f, -2.25f, 0.5f, -0.75f}) == cppinf::ops::cast(input.view(), DType::F32));
}

HOST_TEST(OpsTest, GivenTensorView_WhenReshaping_ThenMetadataChangesOnly) {
    const auto input = f32("input", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    const auto reshaped = cppinf::ops::reshape(input.view(), shape({4}));
    EXPECT_EQ(std::string("input"), reshaped.tensor_info().name);
    EXPECT_TRUE(shape({4}) == reshaped.tensor_info().shape);
    EXPECT_EQ(std::size_t{0}, reshaped.tensor_info().byte_offset);
    EXPECT_TRUE(input.view().data().data() == reshaped.data().data());
}

HOST_TEST(OpsTest, GivenIncompatibleShape_WhenReshaping_ThenItThrows) {
    const auto input = f32("input", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    EXPECT_THROW(cppinf::ops::reshape(input.view(), shape({3})), std::invalid_argument);
}

TEST(OpsTest, GivenRank2Tensor_WhenTransposing_ThenExpectedResultIsReturned) {
    const auto input = f32("input", {2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f});
    EXPECT_TRUE(f32("transpose_2d_result", {3, 2}, {1.0f, 4.0f, 2.0f, 5.0f, 3.0f, 6.0f}) ==
                cppinf::ops::transpose_2d(input.view()));
}

TEST(OpsTest, GivenRank3Tensor_WhenTransposingLastTwoDims_ThenExpectedResultIsReturned) {
    const auto input =
        f32("input", {2, 2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, -1.0f, 0.5f, 2.0f, 3.0f, -2.0f, 1.0f});
    EXPECT_TRUE(f32("transpose_last_two_dims_result", {2, 3, 2},
                    {1.0f, 4.0f, 2.0f, 5.0f, 3.0f, 6.0f, -1.0f, 3.0f, 0.5f, -2.0f, 2.0f, 1.0f}) ==
                cppinf::ops::transpose_last_two_dims(input.view()));
}

TEST(OpsTest, GivenRank3Tensor_WhenPermutingAxes_ThenExpectedResultIsReturned) {
    const auto input =
        f32("input", {2, 2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, 7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f});
    const std::array<std::size_t, 3> axes = {1, 2, 0};
    EXPECT_TRUE(f32("permute_result", {2, 3, 2},
                    {1.0f, 7.0f, 2.0f, 8.0f, 3.0f, 9.0f, 4.0f, 10.0f, 5.0f, 11.0f, 6.0f, 12.0f}) ==
                cppinf::ops::permute(input.view(), axes));
}

TEST(OpsTest, GivenTensor_WhenRepeatingInterleavedDimension_ThenExpectedResultIsReturned) {
    const auto input = f32("input", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    EXPECT_TRUE(f32("repeat_interleave_result", {4, 2}, {1.0f, 2.0f, 1.0f, 2.0f, 3.0f, 4.0f, 3.0f, 4.0f}) ==
                cppinf::ops::repeat_interleave(input.view(), 0, 2));
}

HOST_TEST(OpsTest, GivenTensorView_WhenNarrowingFirstDimension_ThenSubspanIsReturned) {
    const auto input = f32("input", {3, 2}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f});
    const auto narrowed = cppinf::ops::narrow(input.view(), 0, 1, 2);
    EXPECT_EQ(std::string("input"), narrowed.tensor_info().name);
    EXPECT_TRUE(shape({2, 2}) == narrowed.tensor_info().shape);
    EXPECT_EQ(std::size_t{2 * sizeof(float)}, narrowed.tensor_info().byte_offset);
    EXPECT_TRUE(input.view().data().data() + 2 * sizeof(float) == narrowed.data().data());
}

HOST_TEST(OpsTest, GivenStridedTensorView_WhenReshaping_ThenItThrows) {
    const auto input = f32("input", {2, 4}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, 7.0f, 8.0f});
    const auto reshaped = cppinf::ops::reshape(input.view(), shape({2, 2, 2}));
    EXPECT_THROW(cppinf::ops::reshape(cppinf::ops::narrow(reshaped, 1, 1, 1), shape({2, 2})), std::invalid_argument);
}

TEST(OpsTest, GivenUnitDimension_WhenSqueezing_ThenStridedValuesAreRead) {
    // tests/ops/ops_test.cpp:203-210: the squeezed narrow view is strided; a strided device gather reads it.
    const auto input = f32("input", {2, 4}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, 7.0f, 8.0f});
    const auto reshaped = cppinf::ops::reshape(input.view(), shape({2, 2, 2}));
    const auto squeezed = cppinf::ops::squeeze(cppinf::ops::narrow(reshaped, 1, 1, 1), 1);
    EXPECT_TRUE(shape({2, 2}) == squeezed.tensor_info().shape);
    const auto ones = f32("ones", {2, 2}, {1.0f, 1.0f, 1.0f, 1.0f});
    expect_values_near(cppinf::ops::mul(squeezed, ones.view()), {3.0f, 4.0f, 7.0f, 8.0f}, 0.0f);
    const auto device = on_gpu(input);
    const auto dview = cppinf::ops::squeeze(
        cppinf::ops::narrow(cppinf::ops::reshape(device.view(), shape({2, 2, 2})), 1, 1, 1), 1);
    expect_values_near(cppinf::ops::mul(dview, on_gpu(ones).view()), {3.0f, 4.0f, 7.0f, 8.0f}, 0.0f);
}

TEST(OpsTest, GivenMatchingBf16Tensors_WhenAdding_ThenElementwiseSumIsReturned) {
    const auto lhs = bf16("lhs", {2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
    const auto rhs = bf16("rhs", {2, 2}, {10.0f, 20.0f, 30.0f, 40.0f});
    EXPECT_TRUE(bf16("add_result", {2, 2}, {11.0f, 22.0f, 33.0f, 44.0f}) == cppinf::ops::add(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenTorchOracleBf16Tensor_WhenApplyingSilu_ThenExpectedValuesAreReturned) {
    const auto input = bf16("input", {2, 4}, {-1.5f, -0.25f, 0.5f, 2.0f, 3.0f, -4.5f, 1.25f, 0.75f});
    const auto result = cppinf::ops::silu(input.view());
    EXPECT_EQ(std::string("silu_result"), result.tensor_info().name);
    EXPECT_TRUE(DType::BF16 == result.tensor_info().dtype);
    EXPECT_TRUE(shape({2, 4}) == result.tensor_info().shape);
    expect_values_near(result,
                       {-0.2734375f, -0.109375f, 0.310546875f, 1.7578125f, 2.859375f, -0.0495605469f, 0.97265625f,
                        0.5078125f},
                       1e-6f);
}

TEST(OpsTest, GivenTorchOracleBf16Tensor_WhenApplyingSoftmaxLastDim_ThenExpectedValuesAreReturned) {
    const auto input = bf16("input", {2, 4}, {1.0f, -2.5f, 3.25f, 0.75f, 4.5f, 0.5f, -1.75f, 2.25f});
    const auto result = cppinf::ops::softmax_last_dim(input.view());
    EXPECT_EQ(std::string("softmax_last_dim_result"), result.tensor_info().name);
    EXPECT_TRUE(DType::BF16 == result.tensor_info().dtype);
    expect_values_near(result,
                       {0.0883789062f, 0.0026702881f, 0.83984375f, 0.0688476562f, 0.88671875f, 0.0162353516f,
                        0.0017166138f, 0.09375f},
                       1e-6f);
}

TEST(OpsTest, GivenAttentionScores_WhenApplyingScaledCausalSoftmax_ThenFuturePositionsAreMasked) {
    const auto input = f32("input", {1, 2, 2}, {1.0f, 1000.0f, 3.0f, 4.0f});
    const auto result = cppinf::ops::scaled_causal_softmax_last_dim(input.view(), 1.0f);
    EXPECT_EQ(std::string("scaled_causal_softmax_last_dim_result"), result.tensor_info().name);
    EXPECT_TRUE(DType::F32 == result.tensor_info().dtype);
    EXPECT_TRUE(shape({1, 2, 2}) == result.tensor_info().shape);
    expect_values_near(result, {1.0f, 0.0f, 0.2689414322f, 0.7310585976f}, 1e-6f);
}

TEST(OpsTest, GivenTorchOracleBf16Tensor_WhenApplyingRmsNorm_ThenExpectedValuesAreReturned) {
    const auto input = bf16("input", {2, 4}, {-1.5f, -0.25f, 0.5f, 2.0f, 3.0f, -4.5f, 1.25f, 0.75f});
    const auto weight = bf16("weight", {4}, {1.0f, 0.5f, -1.5f, 2.0f});
    const auto result = cppinf::ops::rms_norm(input.view(), weight.view(), 1e-5f);
    EXPECT_EQ(std::string("rms_norm_result"), result.tensor_info().name);
    EXPECT_TRUE(DType::BF16 == result.tensor_info().dtype);
    EXPECT_TRUE(shape({2, 4}) == result.tensor_info().shape);
    expect_values_near(result,
                       {-1.171875f, -0.09765625f, -0.5859375f, 3.125f, 1.0703125f, -0.8046875f, -0.66796875f,
                        0.53515625f},
                       1e-6f);
}

HOST_TEST(OpsTest, GivenMismatchedTensorDtypes_WhenAdding_ThenItThrows) {
    const auto lhs = f32("lhs", {4}, {1.0f, 2.0f, 3.0f, 4.0f});
    const auto rhs = bf16("rhs", {4}, {5.0f, 6.0f, 7.0f, 8.0f});
    EXPECT_THROW(cppinf::ops::add(lhs.view(), rhs.view()), std::invalid_argument);
}

HOST_TEST(OpsTest, GivenInvalidRmsNormArguments_WhenNormalizing_ThenReferenceErrorsAreThrown) {
    const auto input = bf16("input", {2, 4}, {1, 2, 3, 4, 5, 6, 7, 8});
    const auto weight = bf16("weight", {4}, {1, 1, 1, 1});
    const auto weight_f32 = f32("weight", {4}, {1, 1, 1, 1});
    const auto weight_3 = bf16("weight", {3}, {1, 1, 1});
    EXPECT_THROW(cppinf::ops::rms_norm(input.view(), weight.view(), -1.0f), std::invalid_argument);
    EXPECT_THROW(cppinf::ops::rms_norm(input.view(), weight_f32.view(), 1e-6f), std::invalid_argument);
    EXPECT_THROW(cppinf::ops::rms_norm(input.view(), weight_3.view(), 1e-6f), std::invalid_argument);
    EXPECT_THROW(cppinf::ops::rms_norm(input.view(), input.view(), 1e-6f), std::invalid_argument);
    const auto rect = f32("input", {1, 2, 3}, {1, 2, 3, 4, 5, 6});
    EXPECT_THROW(cppinf::ops::scaled_causal_softmax_last_dim(rect.view(), 1.0f), std::invalid_argument);
    EXPECT_THROW(cppinf::ops::permute(rect.view(), std::array<std::size_t, 2>{0, 1}), std::invalid_argument);
    EXPECT_THROW(cppinf::ops::permute(rect.view(), std::array<std::size_t, 3>{0, 1, 5}), std::out_of_range);
    EXPECT_THROW(cppinf::ops::repeat_interleave(rect.view(), 3, 2), std::out_of_range);
}

HOST_TEST(OpsTest, GivenHostAndDeviceInputs_WhenAdding_ThenItThrows) {
    // Fabricated device view (never dereferenced): placement is checked before any CUDA call.
    const auto lhs = f32("lhs", {4}, {1.0f, 2.0f, 3.0f, 4.0f});
    const TensorView device_view(lhs.tensor_info(), lhs.data(), {}, 0, Device::cuda(0));
    EXPECT_THROW(cppinf::ops::add(lhs.view(), device_view), std::invalid_argument);
}

// ---- device-resident tensors -------------------------------------------------------------------------------------

TEST(DeviceOpsTest, GivenDeviceTensors_WhenRunningDecoderBlockOps_ThenResultsStayOnDeviceAndMatchHostPath) {
    const auto x = bf16("x", {2, 8}, {1, -2, 3, -4, 5, -6, 7, -8, 0.5f, 0.25f, -0.75f, 1.5f, 2, -1, 0, 3});
    const auto r = bf16("r", {2, 8}, {0.1f, 0.2f, 0.3f, 0.4f, 0.5f, 0.6f, 0.7f, 0.8f, 1, 1, 1, 1, 1, 1, 1, 1});
    const auto w = bf16("w", {8}, {1, 0.5f, -1, 2, 1, 1, 1, 1});
    const auto dx = on_gpu(x);
    const auto dr = on_gpu(r);
    const auto dw = on_gpu(w);
    const auto [dsum, dnorm] = cppinf::ops::add_rms_norm(dx.view(), dr.view(), dw.view(), 1e-6f);
    EXPECT_TRUE(dsum.device().is_cuda());
    EXPECT_TRUE(dnorm.device().is_cuda());
    const auto host_sum = cppinf::ops::add(x.view(), r.view());
    EXPECT_TRUE(dsum.to(Device::host()) == host_sum);
    EXPECT_TRUE(dnorm.to(Device::host()) == cppinf::ops::rms_norm(host_sum.view(), w.view(), 1e-6f));
    const auto gated = cppinf::ops::silu_mul(dx.view(), dr.view());
    EXPECT_TRUE(gated.to(Device::host()) ==
                cppinf::ops::mul(cppinf::ops::silu(x.view()).view(), r.view()));
}

TEST(DeviceOpsTest, GivenDeviceLogits_WhenSelectingArgmax_ThenLowestMaximalIndexIsReturned) {
    const auto logits = bf16("logits", {2, 6}, {1, 5, 5, -2, 0, 3, -1, -1, -1, -1, -1, -1});
    const auto ids = cppinf::ops::row_argmax(on_gpu(logits).view());
    ASSERT_EQ(ids.size(), std::size_t{2});
    EXPECT_EQ(ids[0], std::int64_t{1});
    EXPECT_EQ(ids[1], std::int64_t{0});
}

TEST(DeviceOpsTest, GivenQkHeads_WhenFusingNormAndRope_ThenResultMatchesTwoStepSequence) {
    std::vector<float> qv(3 * 4 * 64);
    std::vector<float> kv(3 * 2 * 64);
    for (std::size_t i = 0; i < qv.size(); ++i) {
        qv[i] = static_cast<float>((i * 37) % 17) / 8.0f - 1.0f;
    }
    for (std::size_t i = 0; i < kv.size(); ++i) {
        kv[i] = static_cast<float>((i * 11) % 13) / 6.0f - 1.0f;
    }
    std::vector<float> wv(64, 1.0f);
    wv[3] = 0.5f;
    const auto q = cppinf::tensors::make_bf16_tensor("q", shape({3, 4, 64}), qv);
    const auto k = cppinf::tensors::make_bf16_tensor("k", shape({3, 2, 64}), kv);
    const auto w = cppinf::tensors::make_bf16_tensor("w", shape({64}), wv);
    const auto dq = on_gpu(q);
    const auto dk = on_gpu(k);
    const auto dw = on_gpu(w);
    const auto [fq, fk] = cppinf::nn::qk_norm_rope(dq.view(), dk.view(), dw.view(), dw.view(), 1e-6f, 7);
    const auto sq = cppinf::nn::apply_rope(cppinf::ops::rms_norm(q.view(), w.view(), 1e-6f).view(), 7, 1e6f, 0);
    const auto sk = cppinf::nn::apply_rope(cppinf::ops::rms_norm(k.view(), w.view(), 1e-6f).view(), 7, 1e6f, 0);
    EXPECT_TRUE(fq.to(Device::host()).bytes() == sq.bytes());
    EXPECT_TRUE(fk.to(Device::host()).bytes() == sk.bytes());
}

// ---- tests/nn/rope_test.cpp --------------------------------------------------------------------------------------

TEST(RopeTest, GivenZeroPositionOffset_WhenApplyingRope_ThenValuesStayTheSame) {
    const auto input = f32("input", {1, 1, 4}, {1.0f, -0.5f, 0.25f, 1.5f});
    EXPECT_TRUE(f32("rope_result", {1, 1, 4}, {1.0f, -0.5f, 0.25f, 1.5f}) == cppinf::nn::apply_rope(input.view()));
}

TEST(RopeTest, GivenTorchOracleBf16Inputs_WhenApplyingRope_ThenExpectedValuesAreReturned) {
    const auto input = bf16("input", {2, 3, 4},
                            {1.0f, -0.5f, 0.25f, 1.5f, -1.25f, 0.75f, 1.0f, -0.25f, 0.5f, 1.25f, -0.75f, 0.5f,
                             -0.5f, 1.0f, 1.5f, -1.25f, 0.75f, -1.5f, 0.5f, 1.0f, 1.25f, 0.25f, -1.0f, 0.75f});
    const auto result = cppinf::nn::apply_rope(input.view(), 2);
    EXPECT_EQ(std::string("rope_result"), result.tensor_info().name);
    EXPECT_TRUE(DType::BF16 == result.tensor_info().dtype);
    expect_values_near(result,
                       {-0.64453125f, -0.50390625f, 0.8046875f, 1.5f, 1.09375f, 0.75f, -1.1640625f, -0.248046875f,
                        -0.89453125f, 1.25f, 0.11181640625f, 0.50390625f, -1.15625f, 1.0f, -1.078125f, -1.25f,
                        -0.8125f, -1.5f, -0.388671875f, 0.99609375f, -1.5703125f, 0.2470703125f, -0.29296875f, 0.75f},
                       1e-6f);
    const auto device_result = cppinf::nn::apply_rope(on_gpu(input).view(), 2);
    EXPECT_TRUE(device_result.device().is_cuda());
    EXPECT_TRUE(device_result.to(Device::host()) == result);
}

HOST_TEST(RopeTest, GivenOddHeadSize_WhenApplyingRope_ThenItThrows) {
    const auto input = f32("input", {1, 2, 3}, {1.0f, -0.5f, 0.25f, 0.75f, -1.0f, 0.5f});
    EXPECT_THROW(cppinf::nn::apply_rope(input.view()), std::invalid_argument);
}

// ---- tests/tensors/tensor_test.cpp -------------------------------------------------------------------------------

HOST_TEST(TensorTest, GivenFloatValue_WhenConvertingThroughBf16_ThenExpectedBitsRoundTrip) {
    EXPECT_EQ(1.5f, cppinf::tensors::bfloat16_bits_to_float(cppinf::tensors::float_to_bfloat16_bits(1.5f)));
}

HOST_TEST(TensorTest, GivenShape_WhenQueryingRankAndElements_ThenCountsAreReturned) {
    const Shape s({2, 3, 4});
    EXPECT_EQ(std::size_t{3}, s.rank());
    EXPECT_EQ(std::size_t{24}, s.num_elements());
    EXPECT_EQ(std::string("[2, 3, 4]"), cppinf::tensors::to_string(s));
}

HOST_TEST(TensorTest, GivenNegativeDimension_WhenConstructingShape_ThenItThrows) {
    EXPECT_THROW(Shape({1, -1}), std::invalid_argument);
}

HOST_TEST(TensorTest, GivenTensorInfo_WhenFormattingMetadata_ThenStringMatches) {
    const TensorInfo info{.name = "model.embed_tokens.weight", .dtype = DType::BF16, .shape = Shape({2, 4}),
                          .byte_offset = 128};
    EXPECT_EQ(std::size_t{16}, info.byte_size());
    EXPECT_EQ(std::string("TensorInfo(name=\"model.embed_tokens.weight\", dtype=bf16, shape=[2, 4], offset=128, "
                          "bytes=16)"),
              cppinf::tensors::to_string(info));
}

HOST_TEST(TensorTest, GivenNonZeroOffset_WhenCreatingTensor_ThenItThrows) {
    EXPECT_THROW(Tensor(TensorInfo{.name = "a", .dtype = DType::F32, .shape = Shape({2, 2}), .byte_offset = 16},
                        std::vector<std::byte>(16)),
                 std::invalid_argument);
}

HOST_TEST(TensorTest, GivenMismatchedBytes_WhenCreatingTensorView_ThenItThrows) {
    const TensorInfo info{.name = "w", .dtype = DType::BF16, .shape = Shape({2, 4}), .byte_offset = 128};
    const std::array<std::byte, 8> wrong{};
    EXPECT_THROW(TensorView(info, wrong), std::invalid_argument);
}

TEST(TensorTest, GivenHostTensor_WhenRoundTrippingThroughDevice_ThenBytesAreUnchanged) {
    const auto t = bf16("t", {3, 5}, {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15});
    const auto d = t.to(Device::cuda(0));
    EXPECT_TRUE(d.device().is_cuda());
    EXPECT_TRUE(d.to(Device::host()) == t);
    EXPECT_THROW(d.bytes(), std::logic_error);
}

int main(int argc, char** argv) {
    return test_harness::run_all(argc, argv);
}

// ---- ops::matmul: tests/ops/ops_test.cpp:63-110, 219-257, 341-357 ------------------------------------------------

TEST(OpsTest, GivenCompatibleMatrices_WhenMultiplying_ThenMatmulResultIsReturned) {
    const auto lhs = f32("lhs", {2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f});
    const auto rhs = f32("rhs", {3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f});
    EXPECT_TRUE(f32("matmul_result", {2, 2}, {58.0f, 64.0f, 139.0f, 154.0f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenCompatibleBatchedMatrices_WhenMultiplying_ThenBatchedMatmulResultIsReturned) {
    const auto lhs = f32("lhs", {2, 2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, -1.0f, 0.5f, 2.0f, 3.0f, -2.0f, 1.0f});
    const auto rhs =
        f32("rhs", {2, 3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f, 2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f});
    EXPECT_TRUE(f32("matmul_result", {2, 2, 2}, {58.0f, 64.0f, 139.0f, 154.0f, -9.875f, 5.75f, 1.5f, -8.5f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenCompatibleBatchedBf16Matrices_WhenMultiplyingToF32_ThenF32MatmulResultIsReturned) {
    const auto lhs =
        bf16("lhs", {2, 2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, -1.0f, 0.5f, 2.0f, 3.0f, -2.0f, 1.0f});
    const auto rhs =
        bf16("rhs", {2, 3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f, 2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f});
    const auto result =
        cppinf::ops::matmul(lhs.view(), rhs.view(), cppinf::ops::MatmulOptions{.output_dtype = DType::F32});
    EXPECT_EQ(std::string("matmul_result"), result.tensor_info().name);
    EXPECT_TRUE(result.tensor_info().dtype == DType::F32);
    EXPECT_TRUE(result.tensor_info().shape == shape({2, 2, 2}));
    expect_values_near(result, {58.0f, 64.0f, 139.0f, 154.0f, -9.875f, 5.75f, 1.5f, -8.5f}, 0.0f);
}

TEST(OpsTest, GivenF32AndBf16Matrices_WhenMultiplying_ThenF32MatmulResultIsReturned) {
    const auto lhs = f32("lhs", {2, 3}, {1.0f, -2.5f, 3.25f, 4.5f, 0.5f, -1.75f});
    const auto rhs = bf16("rhs", {3, 2}, {2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f});
    EXPECT_TRUE(f32("matmul_result", {2, 2}, {-11.625f, -4.875f, 16.125f, -5.375f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenBf16AndF32Matrices_WhenMultiplying_ThenF32MatmulResultIsReturned) {
    const auto lhs = bf16("lhs", {2, 3}, {1.0f, -2.5f, 3.25f, 4.5f, 0.5f, -1.75f});
    const auto rhs = f32("rhs", {3, 2}, {2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f});
    EXPECT_TRUE(f32("matmul_result", {2, 2}, {-11.625f, -4.875f, 16.125f, -5.375f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenStridedTensorView_WhenMultiplying_ThenMatmulUsesLogicalLayout) {
    const auto input = f32("input", {2, 4}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, 7.0f, 8.0f});
    const auto rhs = f32("rhs", {2, 1}, {2.0f, -1.0f});
    const auto reshaped = cppinf::ops::reshape(input.view(), shape({2, 2, 2}));
    const auto strided_lhs = cppinf::ops::squeeze(cppinf::ops::narrow(reshaped, 1, 1, 1), 1);
    EXPECT_TRUE(f32("matmul_result", {2, 1}, {2.0f, 6.0f}) == cppinf::ops::matmul(strided_lhs, rhs.view()));
}

TEST(OpsTest, GivenCompatibleBf16Matrices_WhenMultiplying_ThenMatmulResultIsReturned) {
    const auto lhs = bf16("lhs", {2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f});
    const auto rhs = bf16("rhs", {3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f});
    EXPECT_TRUE(bf16("matmul_result", {2, 2}, {58.0f, 64.0f, 139.0f, 154.0f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(OpsTest, GivenTorchOracleBf16Matrices_WhenMultiplying_ThenExpectedResultIsReturned) {
    const auto lhs = bf16("lhs", {2, 3}, {1.0f, -2.5f, 3.25f, 4.5f, 0.5f, -1.75f});
    const auto rhs = bf16("rhs", {3, 2}, {2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f});
    EXPECT_TRUE(bf16("matmul_result", {2, 2}, {-11.625f, -4.875f, 16.125f, -5.375f}) ==
                cppinf::ops::matmul(lhs.view(), rhs.view()));
}

TEST(DeviceOpsTest, GivenDeviceTransposedWeightView_WhenMultiplying_ThenVectorPathMatchesHostPath) {
    // linear_project's use (src/nn/qwen_common.cpp:15-37): hidden [3, 16] times transpose_2d(weight [8, 16]).
    std::vector<float> xs(3 * 16);
    std::vector<float> ws(8 * 16);
    for (std::size_t i = 0; i < xs.size(); ++i) {
        xs[i] = static_cast<float>(static_cast<int>(i % 7) - 3) * 0.5f;
    }
    for (std::size_t i = 0; i < ws.size(); ++i) {
        ws[i] = static_cast<float>(static_cast<int>(i % 5) - 2) * 0.25f;
    }
    const auto x = cppinf::tensors::make_bf16_tensor("x", shape({3, 16}), xs);
    const auto w = cppinf::tensors::make_bf16_tensor("w", shape({8, 16}), ws);
    const auto host = cppinf::ops::matmul(x.view(), cppinf::ops::transpose_2d(w.view()).view());
    const auto dx = x.to(Device::cuda(0));
    const auto dw = w.to(Device::cuda(0));
    const auto dwt = TensorView(TensorInfo{"w_t", DType::BF16, shape({16, 8})}, dw.view().data(), {2, 32}, 0,
                                Device::cuda(0));
    const auto dev = cppinf::ops::matmul(dx.view(), dwt);
    EXPECT_TRUE(dev.device().is_cuda());
    EXPECT_TRUE(host == dev.to(Device::host()));
}

HOST_TEST(OpsTest, GivenMismatchedBatchDimensions_WhenMultiplying_ThenMatmulThrows) {
    const auto lhs = f32("lhs", {2, 2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, -1.0f, 0.5f, 2.0f, 3.0f, -2.0f, 1.0f});
    const auto rhs = f32("rhs", {3, 3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f, 2.0f, -1.0f, 0.25f, 3.5f, -4.0f, 1.5f,
                                            0.5f, 1.5f, -2.0f, 0.25f, 3.0f, -0.5f});
    EXPECT_THROW(cppinf::ops::matmul(lhs.view(), rhs.view()), std::invalid_argument);
}

HOST_TEST(OpsTest, GivenF32InputsAndBf16OutputRequest_WhenMultiplying_ThenMatmulThrows) {
    const auto lhs = f32("lhs", {2, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f});
    const auto rhs = f32("rhs", {3, 2}, {7.0f, 8.0f, 9.0f, 10.0f, 11.0f, 12.0f});
    EXPECT_THROW(cppinf::ops::matmul(lhs.view(), rhs.view(), cppinf::ops::MatmulOptions{.output_dtype = DType::BF16}),
                 std::invalid_argument);
}
