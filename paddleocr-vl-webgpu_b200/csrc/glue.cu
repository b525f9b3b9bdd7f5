// glue.cu -- the elementwise work between the engine's dense layers, fused
// into single passes over the activations.  sm_100a.
//
// The arithmetic is the reference's CPU composition
// (crates/pvlc-cpu-ref/src/lib.rs:280-367: layer_norm_f32, rms_norm_f32,
// silu, gelu_pytorch_tanh, gelu_erf_f32; residual adds :142-154) with the
// engine's storage: residual streams in f32, everything a GEMM reads in fp16.
//
//   add_norm:   h += delta (fp16, optional) in f32, then LayerNorm (weight +
//               bias, two-pass mean / variance) or RMSNorm (weight) of the row
//               in f32, written as fp16.  One CTA per row: the row is read
//               once from HBM and re-read from L1 for the second and third
//               passes.
//   gelu_*:     in place on fp16, math in f32.
//   silu_mul:   [rows, 2I] gate | up -> [rows, I] = fp16(silu(gate) * up).
// All are HBM-bound streaming passes; they replace chains of four to six
// single-operation kernels (and their f32 intermediates) per norm or
// activation.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "pvlc_internal.h"

namespace pvlc {
namespace glue {

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();   // red may still hold the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NORM_THREADS / 32; ++w) t += red[w];
  return t;
}

// width is a multiple of 4; rows are 16-byte aligned.
template <bool LAYER>
__global__ void __launch_bounds__(NORM_THREADS) add_norm_kernel(
    float* __restrict__ h, const __half* __restrict__ delta, uint32_t width,
    const float* __restrict__ weight, const float* __restrict__ bias, float eps,
    __half* __restrict__ out) {
  __shared__ float red[NORM_THREADS / 32];
  const size_t row = blockIdx.x;
  float4* hr = reinterpret_cast<float4*>(h + row * width);
  const uint2* dr = delta ? reinterpret_cast<const uint2*>(delta + row * width) : nullptr;
  const uint32_t n4 = width / 4;
  float s = 0.f, ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n4; i += NORM_THREADS) {
    float4 v = hr[i];
    if (dr) {
      const uint2 d = dr[i];
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&d.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&d.y));
      v.x += a.x;
      v.y += a.y;
      v.z += b.x;
      v.w += b.y;
      hr[i] = v;
    }
    s += (v.x + v.y) + (v.z + v.w);
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  float mean = 0.f, inv;
  if (LAYER) {
    mean = block_sum(s, red) / (float)width;
    float var = 0.f;
    for (uint32_t i = threadIdx.x; i < n4; i += NORM_THREADS) {
      const float4 v = hr[i];
      const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
      var += (a * a + b * b) + (c * c + d * d);
    }
    var = block_sum(var, red) / (float)width;
    inv = 1.f / sqrtf(var + eps);
  } else {
    const float ms = block_sum(ss, red) / (float)width;
    inv = 1.f / sqrtf(ms + eps);
  }
  const float4* w4 = reinterpret_cast<const float4*>(weight);
  const float4* b4 = reinterpret_cast<const float4*>(bias);
  uint2* orow = reinterpret_cast<uint2*>(out + row * width);
  for (uint32_t i = threadIdx.x; i < n4; i += NORM_THREADS) {
    const float4 v = hr[i];
    const float4 w = __ldg(w4 + i);
    float4 y;
    if (LAYER) {
      const float4 b = __ldg(b4 + i);
      y = make_float4((v.x - mean) * inv * w.x + b.x, (v.y - mean) * inv * w.y + b.y,
                      (v.z - mean) * inv * w.z + b.z, (v.w - mean) * inv * w.w + b.w);
    } else {
      y = make_float4(v.x * inv * w.x, v.y * inv * w.y, v.z * inv * w.z, v.w * inv * w.w);
    }
    const __half2 lo = __floats2half2_rn(y.x, y.y), hi = __floats2half2_rn(y.z, y.w);
    orow[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                         *reinterpret_cast<const uint32_t*>(&hi));
  }
}

template <int KIND>   // 0: GELU tanh, 1: GELU erf
__global__ void __launch_bounds__(256) gelu_kernel(__half2* __restrict__ x, uint64_t n2) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n2;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float2 v = __half22float2(x[i]);
    float a, b;
    if (KIND == 0) {
      // crates/pvlc-cpu-ref/src/lib.rs:359-362
      a = 0.5f * v.x * (1.f + tanhf(0.7978846f * (v.x + 0.044715f * (v.x * v.x * v.x))));
      b = 0.5f * v.y * (1.f + tanhf(0.7978846f * (v.y + 0.044715f * (v.y * v.y * v.y))));
    } else {
      // crates/pvlc-cpu-ref/src/lib.rs:364-367
      a = 0.5f * v.x * (1.f + erff(v.x * 0.70710677f));
      b = 0.5f * v.y * (1.f + erff(v.y * 0.70710677f));
    }
    x[i] = __floats2half2_rn(a, b);
  }
}

// crates/pvlc-cpu-ref/src/lib.rs:354-357 (silu) and the gated product of
// :1385-1390; width (I) is even.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half2* __restrict__ gu,
                                                       uint32_t half_width, uint64_t n2,
                                                       __half2* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n2;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / half_width, c = i - r * half_width;
    const float2 g = __half22float2(gu[r * 2 * half_width + c]);
    const float2 u = __half22float2(gu[r * 2 * half_width + half_width + c]);
    out[i] = __floats2half2_rn(g.x / (1.f + expf(-g.x)) * u.x, g.y / (1.f + expf(-g.y)) * u.y);
  }
}

int grid_for(uint64_t n) {
  const uint64_t b = (n + 255) / 256;
  return (int)(b < 148ull * 32 ? b : 148ull * 32);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace glue
}  // namespace pvlc

using namespace pvlc;

extern "C" {

int pvlc_add_norm(float* residual, const pvlc_half* delta, uint32_t rows, uint32_t width,
                  const float* weight, const float* bias, float eps, pvlc_half* out,
                  void* stream) {
  if (!rows || !width) return PVLC_ZERO_DIMENSION;
  if (width % 8 || !(eps > 0.f) || !std::isfinite(eps)) return PVLC_LENGTH_MISMATCH;
  if (!residual || !weight || !out) return PVLC_NULL_POINTER;
  if (!glue::aligned16(residual) || !glue::aligned16(weight) || !glue::aligned16(out) ||
      (delta && !glue::aligned16(delta)) || (bias && !glue::aligned16(bias)))
    return PVLC_MISALIGNED_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* d = reinterpret_cast<const __half*>(delta);
  __half* o = reinterpret_cast<__half*>(out);
  if (bias)
    glue::add_norm_kernel<true><<<rows, glue::NORM_THREADS, 0, s>>>(residual, d, width, weight,
                                                                    bias, eps, o);
  else
    glue::add_norm_kernel<false><<<rows, glue::NORM_THREADS, 0, s>>>(residual, d, width, weight,
                                                                     nullptr, eps, o);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

int pvlc_gelu(pvlc_half* x, uint64_t n, int erf_form, void* stream) {
  if (!n) return PVLC_ZERO_DIMENSION;
  if (n % 2) return PVLC_LENGTH_MISMATCH;
  if (!x) return PVLC_NULL_POINTER;
  if (!glue::aligned16(x)) return PVLC_MISALIGNED_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half2* x2 = reinterpret_cast<__half2*>(x);
  if (erf_form)
    glue::gelu_kernel<1><<<glue::grid_for(n / 2), 256, 0, s>>>(x2, n / 2);
  else
    glue::gelu_kernel<0><<<glue::grid_for(n / 2), 256, 0, s>>>(x2, n / 2);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

int pvlc_silu_mul(const pvlc_half* gate_up, uint32_t rows, uint32_t width, pvlc_half* out,
                  void* stream) {
  if (!rows || !width) return PVLC_ZERO_DIMENSION;
  if (width % 2) return PVLC_LENGTH_MISMATCH;
  if (!gate_up || !out) return PVLC_NULL_POINTER;
  if (!glue::aligned16(gate_up) || !glue::aligned16(out)) return PVLC_MISALIGNED_POINTER;
  const uint64_t n2 = (uint64_t)rows * width / 2;
  glue::silu_mul_kernel<<<glue::grid_for(n2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __half2*>(gate_up), width / 2, n2, reinterpret_cast<__half2*>(out));
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // extern "C"
