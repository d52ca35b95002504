// Minimal stand-in for Gufo core's GGML dequantisation helpers, restating
// the GGML formats the reference reads: fp16 -> fp32 widening and Q8_0
// blocks {fp16 d; int8 qs[32]} decoded as d * q (the rule the reference's
// own GPU embedding kernel uses, hip/ops.hip:865-867). TEST INFRASTRUCTURE
// ONLY: lets weights.cpp compile unmodified for the CPU oracle in oracle/_ref.
#ifndef LFM3_ORACLE_STUB_GGML_DEQUANT_HPP_
#define LFM3_ORACLE_STUB_GGML_DEQUANT_HPP_
#include <cstddef>
#include <cstdint>
#include <cstring>

#include "../gguf_reader.hpp"
namespace gufo::quant {
struct block_q8_0 {
  std::uint16_t d;
  std::int8_t qs[32];
};
static_assert(sizeof(block_q8_0) == 34);
inline float Fp16ToFloat(std::uint16_t bits) {
  const std::uint32_t sign = std::uint32_t(bits & 0x8000u) << 16;
  const std::uint32_t e = (bits >> 10) & 0x1fu, m = bits & 0x3ffu;
  std::uint32_t x;
  float f;
  if (e == 0x1f)
    x = sign | 0x7f800000u | (m << 13);
  else if (e)
    x = sign | ((e + 112) << 23) | (m << 13);
  else if (!m)
    x = sign;
  else {
    f = float(m) * 5.9604644775390625e-8f;
    std::memcpy(&x, &f, 4);
    x |= sign;
  }
  std::memcpy(&f, &x, 4);
  return f;
}
inline std::size_t QuantizedBlockElements(core::GgmlType type) {
  return type == core::GgmlType::kQ8_0 ? 32 : 0;
}
inline std::size_t EncodedSizeBytes(core::GgmlType type, std::size_t count) {
  switch (type) {
    case core::GgmlType::kF32:
      return count * 4;
    case core::GgmlType::kF16:
    case core::GgmlType::kBF16:
      return count * 2;
    case core::GgmlType::kQ8_0:
      return count % 32 ? 0 : count / 32 * 34;
  }
  return 0;
}
inline void DequantizeQ8_0(const void* data, float* out, std::size_t count) {
  const auto* blocks = static_cast<const unsigned char*>(data);
  for (std::size_t b = 0; b < count / 32; ++b) {
    std::uint16_t d;
    std::memcpy(&d, blocks + b * 34, 2);
    const float scale = Fp16ToFloat(d);
    for (std::size_t j = 0; j < 32; ++j)
      out[b * 32 + j] =
          float(static_cast<std::int8_t>(blocks[b * 34 + 2 + j])) * scale;
  }
}
}  // namespace gufo::quant
#endif
