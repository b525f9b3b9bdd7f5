// image_patches.cu -- canonical RGB8 image -> normalised vision patches on the GPU.
//
// The reference resizes each page image on the host with Pillow's bicubic
// filter and cuts it into patches (crates/pvlc-cpu-ref/src/lib.rs:2515-2563,
// 3092-3273).  The arithmetic is integer: 22-bit fixed-point coefficients
// computed once per (input size, output size) in f64, int64 accumulation per
// output byte, rounding by the 2^21 bias and an arithmetic shift, clamp to
// [0, 255].  The coefficient tables are computed on the device by
// coeff_kernel, one thread per output index, with the reference's f64
// operations in the reference's order, each explicitly rounded (no fused
// multiply-add), so the tables equal the reference's bit for bit; nothing is
// uploaded, so a call never waits for the stream (an upload of host-computed
// tables from pageable memory made every page wait for the previous one).
// The two resample passes and the patch layout are bit-identical to the host
// computation.
//
// Pass 1 (horizontal, only when the width changes): one thread per output
//   byte (y, ox, c) of the [H, OW, 3] intermediate.
// Pass 2 (vertical + patchify): one thread per output value; it resamples
//   along y (or copies when the height is unchanged) and writes the
//   normalised value ((byte / 255 in f64, stored f32) - 0.5) / 0.5 into the
//   patch-major layout [patch_y, patch_x, channel, local_y, local_x].
// Both passes read contiguous bytes across a warp; the work is a few MB per
// page, far from any roofline that matters next to the encoder.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "pvlc_internal.h"

namespace pvlc {
namespace img {

// crates/pvlc-cpu-ref/src/lib.rs:3141-3208 (pillow_bicubic_coefficients,
// pillow_bicubic_filter with a = -0.5), one output index per thread: the
// same f64 operations in the same order, each rounded once (__d*_rn are never
// fused into a multiply-add).
__device__ double bicubic_filter_dev(double x) {
  x = fabs(x);
  if (x < 1.0) return __dadd_rn(__dmul_rn(__dmul_rn(__dsub_rn(__dmul_rn(1.5, x), 2.5), x), x), 1.0);
  if (x < 2.0)
    return __dmul_rn(__dsub_rn(__dmul_rn(__dadd_rn(__dmul_rn(__dsub_rn(x, 5.0), x), 8.0), x), 4.0),
                     -0.5);
  return 0.0;
}

__global__ void __launch_bounds__(128) coeff_kernel(uint32_t in_size, uint32_t out_size, int ksize,
                                                     int32_t* __restrict__ table) {
  const uint32_t o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out_size) return;
  const double scale = __ddiv_rn((double)in_size, (double)out_size);
  const double filter_scale = scale > 1.0 ? scale : 1.0;
  const double support = __dmul_rn(2.0, filter_scale);
  const double inv = __ddiv_rn(1.0, filter_scale);
  const double center = __dmul_rn(__dadd_rn((double)o, 0.5), scale);
  long long lo = (long long)__dadd_rn(__dsub_rn(center, support), 0.5);
  if (lo < 0) lo = 0;
  long long hi = (long long)__dadd_rn(__dadd_rn(center, support), 0.5);
  if (hi > (long long)in_size) hi = in_size;
  const int count = hi > lo ? (int)(hi - lo) : 0;
  auto weight = [&](int j) {
    return bicubic_filter_dev(
        __dmul_rn(__dadd_rn(__dsub_rn(__dadd_rn((double)j, (double)lo), center), 0.5), inv));
  };
  double sum = 0.0;
  for (int j = 0; j < count; ++j) sum = __dadd_rn(sum, weight(j));
  int32_t* row = table + (size_t)o * (2 + ksize);
  row[0] = (int32_t)lo;
  row[1] = count;
  for (int j = 0; j < ksize; ++j) {
    int32_t v = 0;
    if (j < count) {
      double w = weight(j);
      if (sum != 0.0) w = __ddiv_rn(w, sum);
      const double sc = __dmul_rn(w, (double)(1u << 22));
      v = w < 0.0 ? (int32_t)__dadd_rn(-0.5, sc) : (int32_t)__dadd_rn(0.5, sc);
    }
    row[2 + j] = v;
  }
}

int kernel_size(uint32_t in_size, uint32_t out_size) {
  const double scale = (double)in_size / (double)out_size;
  return (int)std::ceil(2.0 * (scale > 1.0 ? scale : 1.0)) * 2 + 1;
}

__device__ __forceinline__ uint8_t clip_u8(long long acc) {
  // crates/pvlc-cpu-ref/src/lib.rs:3271-3273
  long long v = acc >> 22;
  v = v < 0 ? 0 : (v > 255 ? 255 : v);
  return (uint8_t)v;
}

__global__ void __launch_bounds__(256) resample_rows_kernel(const uint8_t* __restrict__ in,
                                                             uint32_t height, uint32_t width,
                                                             uint32_t out_width,
                                                             const int32_t* __restrict__ table,
                                                             int ksize, uint8_t* __restrict__ out) {
  const size_t total = (size_t)height * out_width * 3;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % 3);
    const uint32_t ox = (uint32_t)((i / 3) % out_width);
    const uint32_t y = (uint32_t)(i / (3 * (size_t)out_width));
    const int32_t* row = table + (size_t)ox * (2 + ksize);
    const int lo = row[0], count = row[1];
    const uint8_t* src = in + ((size_t)y * width + lo) * 3 + c;
    long long acc = 1ll << 21;
    for (int j = 0; j < count; ++j) acc += (long long)src[(size_t)j * 3] * row[2 + j];
    out[i] = clip_u8(acc);
  }
}

__global__ void __launch_bounds__(256) resample_cols_patch_kernel(
    const uint8_t* __restrict__ in, uint32_t in_height, uint32_t width, uint32_t out_height,
    const int32_t* __restrict__ table, int ksize, uint32_t patch, float* __restrict__ patches) {
  const size_t total = (size_t)out_height * width * 3;
  const uint32_t grid_w = width / patch;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % 3);
    const uint32_t x = (uint32_t)((i / 3) % width);
    const uint32_t y = (uint32_t)(i / (3 * (size_t)width));
    uint8_t byte;
    if (table) {
      const int32_t* row = table + (size_t)y * (2 + ksize);
      const int lo = row[0], count = row[1];
      const uint8_t* src = in + ((size_t)lo * width + x) * 3 + c;
      long long acc = 1ll << 21;
      for (int j = 0; j < count; ++j) acc += (long long)src[(size_t)j * width * 3] * row[2 + j];
      byte = clip_u8(acc);
    } else {
      byte = in[i];
    }
    // crates/pvlc-cpu-ref/src/lib.rs:2546-2548
    const float r = (float)((double)byte / 255.0);
    const float v = (r - 0.5f) / 0.5f;
    const uint32_t py = y / patch, ly = y % patch, px = x / patch, lx = x % patch;
    const size_t p = (size_t)py * grid_w + px;
    patches[((p * 3 + c) * patch + ly) * patch + lx] = v;
  }
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

size_t workspace_layout(uint32_t height, uint32_t width, uint32_t out_height, uint32_t out_width,
                        size_t* h_off, size_t* v_off, size_t* mid_off) {
  const int kh = (int)std::ceil(2.0 * std::max(1.0, (double)width / out_width)) * 2 + 1;
  const int kv = (int)std::ceil(2.0 * std::max(1.0, (double)height / out_height)) * 2 + 1;
  size_t off = 0;
  *h_off = off;
  off += align256((size_t)out_width * (2 + kh) * sizeof(int32_t));
  *v_off = off;
  off += align256((size_t)out_height * (2 + kv) * sizeof(int32_t));
  *mid_off = off;
  off += align256((size_t)height * out_width * 3);
  return off;
}

}  // namespace img
}  // namespace pvlc

using namespace pvlc;

extern "C" {

size_t pvlc_image_patches_workspace_bytes(uint32_t height, uint32_t width, uint32_t out_height,
                                          uint32_t out_width) {
  if (!height || !width || !out_height || !out_width) return 0;
  size_t a, b, c;
  return img::workspace_layout(height, width, out_height, out_width, &a, &b, &c);
}

int pvlc_image_patches(const uint8_t* rgb, uint32_t height, uint32_t width, uint32_t out_height,
                       uint32_t out_width, uint32_t patch_size, void* workspace,
                       size_t workspace_bytes, float* patches, void* stream) {
  if (!height || !width || !out_height || !out_width || !patch_size) return PVLC_ZERO_DIMENSION;
  if (out_height % patch_size || out_width % patch_size) return PVLC_INVALID_VISION_GEOMETRY;
  if ((uint64_t)height * width * 3 > (1ull << 40) ||
      (uint64_t)out_height * out_width * 3 > (1ull << 40))
    return PVLC_ARITHMETIC_OVERFLOW;
  if (!rgb || !patches || !workspace) return PVLC_NULL_POINTER;
  size_t h_off, v_off, mid_off;
  const size_t need = img::workspace_layout(height, width, out_height, out_width, &h_off, &v_off,
                                            &mid_off);
  if (workspace_bytes < need) return PVLC_WORKSPACE_TOO_SMALL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* stage = rgb;
  if (out_width != width) {
    const int kh = img::kernel_size(width, out_width);
    int32_t* ht = reinterpret_cast<int32_t*>(ws + h_off);
    img::coeff_kernel<<<(out_width + 127) / 128, 128, 0, s>>>(width, out_width, kh, ht);
    const size_t total = (size_t)height * out_width * 3;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
    img::resample_rows_kernel<<<blocks, 256, 0, s>>>(rgb, height, width, out_width, ht, kh,
                                                      ws + mid_off);
    stage = ws + mid_off;
  }
  const int32_t* vt = nullptr;
  int kv = 0;
  if (out_height != height) {
    kv = img::kernel_size(height, out_height);
    int32_t* t = reinterpret_cast<int32_t*>(ws + v_off);
    img::coeff_kernel<<<(out_height + 127) / 128, 128, 0, s>>>(height, out_height, kv, t);
    vt = t;
  }
  const size_t total = (size_t)out_height * out_width * 3;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  img::resample_cols_patch_kernel<<<blocks, 256, 0, s>>>(stage, height, out_width, out_height,
                                                          vt, kv, patch_size, patches);
  return cudaGetLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // extern "C"
