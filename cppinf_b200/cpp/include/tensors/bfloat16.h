#pragma once

#include <cstdint>

namespace cppinf::tensors {

// Round-to-nearest-even f32 -> bf16 bits and the exact inverse (src/tensors/bfloat16.h:7-8).
std::uint16_t float_to_bfloat16_bits(float value);
float bfloat16_bits_to_float(std::uint16_t bits);

} // namespace cppinf::tensors
