// pvlc_checkpoint_oracle.cpp -- CPU restatement of the reference's BF16 -> F16
// checkpoint payload conversion.  TEST INFRASTRUCTURE: only tests/ and the
// bench's CPU legs call it, as the checker of the device conversion; the
// product never links it.
//
// Follows crates/pvlc-safetensors/src/fp16.rs:
//   :171-210 finite_bf16_to_f16_bits -- IEEE binary16, round to nearest, ties
//            to even; NaN / infinity and finite values beyond the f16 range
//            have no result;
//   :212-276 stream_bf16_payload_to_f16 -- converts a little-endian payload in
//            order and stops at the first element without a result, naming its
//            index and whether it was non-finite (exponent 0xff) or out of range.
// Pinned by the reference's known-answer table and rejection list
// (crates/pvlc-safetensors/tests/fp16_checkpoint_conversion_contract.rs:57-87).

#include <cstddef>
#include <cstdint>

namespace {

// Returns 0 and writes *out, or 1 (non-finite) / 2 (out of range).
int finite_bf16_to_f16_bits(uint16_t bits, uint16_t* out) {
  const uint16_t sign = bits & 0x8000u;
  const uint16_t exponent = (bits >> 7) & 0xffu;
  const uint16_t fraction = bits & 0x007fu;
  if (exponent == 0xffu) return 1;
  if (exponent == 0) {
    *out = sign;
    return 0;
  }
  const int32_t unbiased = (int32_t)exponent - 127;
  if (unbiased > 15) return 2;
  if (unbiased >= -14) {
    *out = (uint16_t)(sign | ((uint16_t)(unbiased + 15) << 10) | (uint16_t)(fraction << 3));
    return 0;
  }
  const uint16_t significand = (uint16_t)(0x0080u | fraction);
  const int32_t shift = -(unbiased + 17);
  if (shift <= 0) {
    *out = (uint16_t)(sign | (uint16_t)(significand << (uint32_t)(-shift)));
    return 0;
  }
  if (shift > 8) {
    *out = sign;
    return 0;
  }
  uint16_t rounded = (uint16_t)(significand >> shift);
  const uint16_t mask = (uint16_t)((1u << shift) - 1u);
  const uint16_t remainder = significand & mask;
  const uint16_t halfway = (uint16_t)(1u << (shift - 1));
  if (remainder > halfway || (remainder == halfway && (rounded & 1u) != 0)) rounded += 1;
  *out = (uint16_t)(sign | rounded);
  return 0;
}

}  // namespace

extern "C" {

// Element-wise: status[i] = 0 (dst[i] written), 1 (non-finite) or 2 (out of range).
void pvlc_oracle_bf16_to_f16_bits(const uint16_t* src, uint16_t* dst, uint8_t* status,
                                  uint64_t count) {
  for (uint64_t i = 0; i < count; ++i) {
    uint16_t out = 0;
    status[i] = (uint8_t)finite_bf16_to_f16_bits(src[i], &out);
    dst[i] = out;
  }
}

// Stream form: converts in order and stops at the first rejected element.
// Returns 0 when every element converted, else 1 / 2 with *rejected_index set.
int pvlc_oracle_stream_bf16_to_f16(const uint16_t* src, uint16_t* dst, uint64_t count,
                                   uint64_t* rejected_index) {
  for (uint64_t i = 0; i < count; ++i) {
    const int status = finite_bf16_to_f16_bits(src[i], &dst[i]);
    if (status != 0) {
      *rejected_index = i;
      return status;
    }
  }
  return 0;
}

}  // extern "C"
