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
//               in f32, written as fp16.  Widths 1024 and 1152 (the
//               decoder and vision rows) with many rows: one warp per row,
//               the row in registers (width-exact, 72-80 registers, 3 CTAs
//               of 8 rows per SM).  Otherwise one CTA per row: the row is
//               read once from HBM and re-read from L1 for the second and
//               third passes.  (A warp per row sized for rows up to 2048
//               wide needed 106 registers and was slower than the CTA
//               kernel: 296 vs 241 us for 78,400 x 1152.)
//   gelu_*:     in place on fp16, math in f32, 16-byte accesses.  The tanh form
//               is evaluated as x / (1 + e^(-2u)), the same function as
//               0.5 x (1 + tanh u) (tanh u = 1 - 2 / (1 + e^(2u))), with the
//               hardware base-2 exponential and reciprocal (relative error
//               ~1e-6 against the f32 formula, far below the fp16 rounding of
//               the result, and free of the cancellation in 1 + tanh u for
//               large negative x).
//   silu_mul:   [rows, 2I] gate | up -> [rows, I] = fp16(silu(gate) * up),
//               silu(g) = g / (1 + e^(-g)) the same way.
// All are HBM-bound streaming passes; they replace chains of four to six
// single-operation kernels (and their f32 intermediates) per norm or
// activation.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "pvlc_common.cuh"
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

// One warp per row for the engine's two row widths, 32 * VPL * 4 values (VPL =
// 9: 1152, VPL = 8: 1024), the row held in registers between the passes and
// the reductions done with shuffles alone; 8 rows per CTA, 3 CTAs per SM.
// Used from ROW_KERNEL_MIN_ROWS rows up (the encoder's 78,400-row LayerNorms:
// 162 vs 240 us, 6.7 TB/s); a decode step's few hundred rows would leave most
// SMs idle, so they keep the CTA-per-row kernel.
constexpr int ROW_WARPS = 8;
constexpr uint32_t ROW_KERNEL_MIN_ROWS = 4096;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <bool LAYER, int VPL>
__global__ void __launch_bounds__(ROW_WARPS * 32, 3) add_norm_row_kernel(
    float* __restrict__ h, const __half* __restrict__ delta, uint32_t rows,
    const float* __restrict__ weight, const float* __restrict__ bias, float eps,
    __half* __restrict__ out) {
  constexpr uint32_t width = 128u * VPL;
  const size_t row = (size_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  float4* hr = reinterpret_cast<float4*>(h + row * width);
  float4 v[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) v[k] = hr[lane + 32 * k];
  if (delta) {
    const uint2* dr = reinterpret_cast<const uint2*>(delta + row * width);
    uint2 d[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) d[k] = dr[lane + 32 * k];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&d[k].x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&d[k].y));
      v[k].x += a.x;
      v[k].y += a.y;
      v[k].z += b.x;
      v[k].w += b.y;
      hr[lane + 32 * k] = v[k];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k)
    s += LAYER ? (v[k].x + v[k].y) + (v[k].z + v[k].w)
               : (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
  float mean = 0.f, inv;
  if (LAYER) {
    mean = warp_sum(s) / (float)width;
    float var = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
      var += (a * a + b * b) + (c * c + d * d);
    }
    inv = 1.f / sqrtf(warp_sum(var) / (float)width + eps);
  } else {
    inv = 1.f / sqrtf(warp_sum(s) / (float)width + eps);
  }
  const float4* w4 = reinterpret_cast<const float4*>(weight);
  const float4* b4 = reinterpret_cast<const float4*>(bias);
  uint2* orow = reinterpret_cast<uint2*>(out + row * width);
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int i = lane + 32 * k;
    const float4 w = __ldg(w4 + i);
    float4 y;
    if (LAYER) {
      const float4 b = __ldg(b4 + i);
      y = make_float4((v[k].x - mean) * inv * w.x + b.x, (v[k].y - mean) * inv * w.y + b.y,
                      (v[k].z - mean) * inv * w.z + b.z, (v[k].w - mean) * inv * w.w + b.w);
    } else {
      y = make_float4(v[k].x * inv * w.x, v[k].y * inv * w.y, v[k].z * inv * w.z,
                      v[k].w * inv * w.w);
    }
    const __half2 lo = __floats2half2_rn(y.x, y.y), hi = __floats2half2_rn(y.z, y.w);
    orow[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                         *reinterpret_cast<const uint32_t*>(&hi));
  }
}

template <bool LAYER>
bool launch_row_kernel(float* h, const __half* d, uint32_t rows, uint32_t width, const float* w,
                       const float* b, float eps, __half* o, cudaStream_t s) {
  const uint32_t grid = (rows + ROW_WARPS - 1) / ROW_WARPS;
  if (width == 1152) {
    add_norm_row_kernel<LAYER, 9><<<grid, ROW_WARPS * 32, 0, s>>>(h, d, rows, w, b, eps, o);
    return true;
  }
  if (width == 1024) {
    add_norm_row_kernel<LAYER, 8><<<grid, ROW_WARPS * 32, 0, s>>>(h, d, rows, w, b, eps, o);
    return true;
  }
  return false;
}

// 0.5 x (1 + tanh(u)), u = sqrt(2 / pi) (x + 0.044715 x^3)
// (crates/pvlc-cpu-ref/src/lib.rs:359-362), as x / (1 + 2^(-2u log2 e)).
__device__ __forceinline__ float gelu_tanh(float x) {
  constexpr float kNeg2UL = -2.f * 0.7978846f * 1.4426950408889634f;
  const float t = x * fmaf(0.044715f * x, x, 1.f);
  return x * rcp_approx(1.f + fast_exp2(t * kNeg2UL));
}

// crates/pvlc-cpu-ref/src/lib.rs:364-367
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710677f)); }

template <int KIND>
__device__ __forceinline__ uint32_t gelu_h2(uint32_t w) {
  const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w));
  const __half2 r = KIND == 0 ? __floats2half2_rn(gelu_tanh(v.x), gelu_tanh(v.y))
                              : __floats2half2_rn(gelu_erf(v.x), gelu_erf(v.y));
  return *reinterpret_cast<const uint32_t*>(&r);
}

template <int KIND>   // 0: GELU tanh, 1: GELU erf
__global__ void __launch_bounds__(256) gelu_kernel(__half* __restrict__ x, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t n8 = n / 8;
  uint4* x8 = reinterpret_cast<uint4*>(x);
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    uint4 w = x8[i];
    w.x = gelu_h2<KIND>(w.x);
    w.y = gelu_h2<KIND>(w.y);
    w.z = gelu_h2<KIND>(w.z);
    w.w = gelu_h2<KIND>(w.w);
    x8[i] = w;
  }
  // tail: n is even, so pairs
  uint32_t* x2 = reinterpret_cast<uint32_t*>(x);
  for (uint64_t i = n8 * 4 + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n / 2;
       i += stride)
    x2[i] = gelu_h2<KIND>(x2[i]);
}

__device__ __forceinline__ uint32_t silu_mul_h2(uint32_t g2, uint32_t u2) {
  const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&g2));
  const float2 u = __half22float2(*reinterpret_cast<const __half2*>(&u2));
  const __half2 r = __floats2half2_rn(silu(g.x) * u.x, silu(g.y) * u.y);
  return *reinterpret_cast<const uint32_t*>(&r);
}

// crates/pvlc-cpu-ref/src/lib.rs:1385-1390 (gated product); VEC = 8 halves
// per access when the width is a multiple of 8, else 2.
template <int VEC>
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gu,
                                                       uint32_t width, uint64_t nv,
                                                       __half* __restrict__ out) {
  const uint32_t wv = width / VEC;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < nv;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / wv, c = (i - r * wv) * VEC;
    const __half* g = gu + r * 2 * width + c;
    if (VEC == 8) {
      const uint4 a = *reinterpret_cast<const uint4*>(g);
      const uint4 b = *reinterpret_cast<const uint4*>(g + width);
      *reinterpret_cast<uint4*>(out + r * width + c) =
          make_uint4(silu_mul_h2(a.x, b.x), silu_mul_h2(a.y, b.y), silu_mul_h2(a.z, b.z),
                     silu_mul_h2(a.w, b.w));
    } else {
      *reinterpret_cast<uint32_t*>(out + r * width + c) =
          silu_mul_h2(*reinterpret_cast<const uint32_t*>(g),
                      *reinterpret_cast<const uint32_t*>(g + width));
    }
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
  if (rows >= glue::ROW_KERNEL_MIN_ROWS &&
      (bias ? glue::launch_row_kernel<true>(residual, d, rows, width, weight, bias, eps, o, s)
            : glue::launch_row_kernel<false>(residual, d, rows, width, weight, nullptr, eps, o, s)))
    return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
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
  __half* xh = reinterpret_cast<__half*>(x);
  const uint64_t work = n / 8 > 0 ? n / 8 : n / 2;
  if (erf_form)
    glue::gelu_kernel<1><<<glue::grid_for(work), 256, 0, s>>>(xh, n);
  else
    glue::gelu_kernel<0><<<glue::grid_for(work), 256, 0, s>>>(xh, n);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

int pvlc_silu_mul(const pvlc_half* gate_up, uint32_t rows, uint32_t width, pvlc_half* out,
                  void* stream) {
  if (!rows || !width) return PVLC_ZERO_DIMENSION;
  if (width % 2) return PVLC_LENGTH_MISMATCH;
  if (!gate_up || !out) return PVLC_NULL_POINTER;
  if (!glue::aligned16(gate_up) || !glue::aligned16(out)) return PVLC_MISALIGNED_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* gu = reinterpret_cast<const __half*>(gate_up);
  __half* o = reinterpret_cast<__half*>(out);
  if (width % 8 == 0) {
    const uint64_t nv = (uint64_t)rows * width / 8;
    glue::silu_mul_kernel<8><<<glue::grid_for(nv), 256, 0, s>>>(gu, width, nv, o);
  } else {
    const uint64_t nv = (uint64_t)rows * width / 2;
    glue::silu_mul_kernel<2><<<glue::grid_for(nv), 256, 0, s>>>(gu, width, nv, o);
  }
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // extern "C"
