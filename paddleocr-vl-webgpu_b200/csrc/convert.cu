// convert.cu -- checkpoint weights on the device: BF16 -> IEEE binary16 with
// round-to-nearest, ties-to-even, rejecting what the reference rejects.  sm_100a.
//
// Arithmetic: crates/pvlc-safetensors/src/fp16.rs:171-210
// (finite_bf16_to_f16_bits, conversion id "bf16_to_ieee_f16_rne_v1"):
//   exponent 0xff (NaN, infinity)            -> rejected, non-finite;
//   unbiased exponent above 15               -> rejected, out of the f16 range;
//   exponent 0 (zero, bf16 subnormal)        -> signed zero;
//   unbiased exponent -14..15                -> f16 normal, exact (fraction << 3);
//   below -14                                -> f16 subnormal: the 8-bit
//                                               significand shifted right, RNE.
// Fast path: wherever that rule converts (every element finite and below 2^16
// in magnitude) its result is IEEE binary16 round-to-nearest-even of the value,
// checked on all 65,536 BF16 patterns, so a vector of eight such elements goes
// through the hardware conversion (cvt.rn.f16x2.f32, two elements per
// instruction; a BF16 value widens to f32 exactly by a shift).  Its range check
// is branch-free: a half-word magnitude m >= 0x4780 (2^16, infinity, NaN) is
// exactly m + 0x3880 >= 0x8000, with no carry between the two halves of a
// 32-bit word.  Only a vector holding such an element re-runs the reference's
// integer sequence below, element by element, to find the first one and its
// reason.  (A per-element integer conversion made the kernel issue-bound: 71 %
// of peak instruction issue, 52 % of peak DRAM throughput.)
//
// Rejections.  The reference's stream converter stops at the first rejected
// element in payload order and names its index (fp16.rs:212-276).  Here every
// thread converts independently; a rejected element folds the record
// ((index_base + index) << 1 | out_of_range) into one device word with
// atomicMin, so after the launch the word holds the lowest rejected index --
// the element the reference names -- and its reason.  The word is not cleared
// here: a caller converting one payload in several calls (chunks) sets it to
// ~0 once and passes each chunk's first payload index as index_base.
//
// src may equal dst (in place): each element is read once, by the thread
// that writes it, before it is written.
//
// Layout: one 16-byte vector (8 elements) per thread and step, four vectors in
// flight per thread, a grid-stride loop over 148 x 8 CTAs of 256 threads.  The
// last count % 8 elements run element-wise in the first CTA.  Pointers must be
// 16-byte aligned (checked by the entry point); every tensor of the
// PaddleOCR-VL-1.6 checkpoint is a multiple of 16 bytes, so a payload copied
// to an aligned buffer keeps every tensor aligned.
// HBM-bound streaming pass: 2 bytes read + 2 bytes written per element.

#include <cuda_runtime.h>

#include "pvlc_internal.h"

namespace pvlc {
namespace convert {

constexpr int THREADS = 256;
constexpr int UNROLL = 4;

// Bits 0..15: the f16 result.  Bit 16: non-finite source.  Bit 17: finite
// source beyond the f16 range.
__device__ __forceinline__ uint32_t bf16_to_f16(uint32_t b) {
  const uint32_t sign = b & 0x8000u, exponent = (b >> 7) & 0xffu, fraction = b & 0x7fu;
  if (exponent == 0xffu) return 0x10000u;
  if (exponent == 0u) return sign;
  const int unbiased = (int)exponent - 127;
  if (unbiased > 15) return 0x20000u;
  if (unbiased >= -14) return sign | ((uint32_t)(unbiased + 15) << 10) | (fraction << 3);
  const uint32_t significand = 0x80u | fraction;
  const int shift = -(unbiased + 17);
  if (shift <= 0) return sign | (significand << (uint32_t)(-shift));
  if (shift > 8) return sign;
  uint32_t rounded = significand >> shift;
  const uint32_t remainder = significand & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1);
  if (remainder > halfway || (remainder == halfway && (rounded & 1u))) ++rounded;
  return sign | rounded;
}

__device__ __forceinline__ void reject(unsigned long long* word, uint64_t index, uint32_t r) {
  const unsigned long long record = (index << 1) | ((r >> 17) & 1u);
  atomicMin(word, record);
}

// Two BF16 values (low, high half of w) to two f16 values, IEEE RNE.
__device__ __forceinline__ uint32_t cvt2(uint32_t w) {
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Converts one 16-byte vector; returns the converted vector and folds the
// vector's first rejected element (if any) into *word.
__device__ __forceinline__ uint4 convert_vec(const uint4 v, uint64_t first_index,
                                             unsigned long long* word) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[4];
  uint32_t flags = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    flags |= ((in[i] & 0x7fff7fffu) + 0x38803880u) & 0x80008000u;
    out[i] = cvt2(in[i]);
  }
  if (flags) {
#pragma unroll 1
    for (int e = 0; e < 8; ++e) {
      const uint32_t r = bf16_to_f16((in[e >> 1] >> ((e & 1) * 16)) & 0xffffu);
      if (r & 0x30000u) {
        reject(word, first_index + e, r);
        break;
      }
    }
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__global__ void __launch_bounds__(THREADS) bf16_to_f16_kernel(
    const uint4* src, uint4* dst, uint64_t vectors, const uint16_t* src_tail,
    uint16_t* dst_tail, uint32_t tail, uint64_t index_base, unsigned long long* rejected) {
  const uint64_t stride = (uint64_t)gridDim.x * THREADS;
  uint64_t i = (uint64_t)blockIdx.x * THREADS + threadIdx.x;
  for (; i + (UNROLL - 1) * stride < vectors; i += UNROLL * stride) {
    uint4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) v[u] = __ldcs(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      __stcs(dst + i + u * stride, convert_vec(v[u], index_base + (i + u * stride) * 8, rejected));
  }
  for (; i < vectors; i += stride)
    __stcs(dst + i, convert_vec(__ldcs(src + i), index_base + i * 8, rejected));
  if (blockIdx.x == 0 && threadIdx.x < tail) {
    const uint32_t r = bf16_to_f16(src_tail[threadIdx.x]);
    if (r & 0x30000u) reject(rejected, index_base + vectors * 8 + threadIdx.x, r);
    dst_tail[threadIdx.x] = (uint16_t)(r & 0xffffu);
  }
}

int grid_for(uint64_t vectors) {
  const uint64_t blocks = (vectors + THREADS - 1) / THREADS;
  const uint64_t cap = 148ull * 8;
  return (int)(blocks == 0 ? 1 : (blocks < cap ? blocks : cap));
}

}  // namespace convert
}  // namespace pvlc

using namespace pvlc;

extern "C" {

int pvlc_bf16_to_f16(const uint16_t* src, uint16_t* dst, uint64_t count, uint64_t index_base,
                     unsigned long long* rejected, void* stream) {
  if (!count) return PVLC_ZERO_DIMENSION;
  if (!src || !dst || !rejected) return PVLC_NULL_POINTER;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) ||
      (reinterpret_cast<uintptr_t>(rejected) & 7u))
    return PVLC_MISALIGNED_POINTER;
  if (index_base > (UINT64_MAX >> 1) || count > (UINT64_MAX >> 1) - index_base)
    return PVLC_ARITHMETIC_OVERFLOW;
  const uint64_t vectors = count / 8;
  const uint32_t tail = (uint32_t)(count % 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  convert::bf16_to_f16_kernel<<<convert::grid_for(vectors), convert::THREADS, 0, s>>>(
      reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), vectors,
      src + vectors * 8, dst + vectors * 8, tail, index_base, rejected);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // extern "C"
