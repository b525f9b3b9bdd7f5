// vision_varlen.cu -- vision-encoder bidirectional varlen attention with the
// 2-D RoPE fused into the Q/K tile loads (head_dim 72), sm_100a.
//
// Reference path replaced: VisionRope2dF16 followed by VisionAttentionF16
// (crates/pvlc-wgsl/src/lib.rs:2309-2454,2553-2596; call site
// crates/pvlc-runtime-web/src/web.rs:4797-4803); arithmetic
// crates/pvlc-cpu-ref/src/lib.rs:472-542 (rotation) and :2752-2878
// (segmented attention).  Unlike the reference, which loops every query over
// all packed tokens and masks, a CTA only ever visits keys of its own
// segment (sum n_i^2 work instead of T^2).
//
// Layout: q/k/v/out are token-major [T, H, 72] fp16, so one head's rows sit
// at a 2304-byte pitch; a 72-dim row (144 bytes) is staged unpadded in shared
// memory, which keeps ldmatrix conflict free (144 = 9 x 16).
// Work item = (segment, 64-query tile, head); items are ordered longest
// segment first so the longest tiles start in the first wave.
// Per warp: 16 queries; S = Q K^T with mma.m16n8k16 (dims 0..63) plus
// mma.m16n8k8 (dims 64..71), online softmax in f32 (exp2 domain),
// O += P V with mma.m16n8k16 over 9 n-tiles of 8 dims.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <algorithm>
#include <numeric>
#include <vector>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"

namespace pvlc {
namespace vision {

constexpr int HD = 72;
constexpr int PAIRS = HD / 2;      // 36
constexpr int BM = 64;             // queries per CTA
constexpr int BN = 64;             // keys per tile
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int ROW_BYTES = HD * 2;  // 144
constexpr int MAX_SEG = PVLC_VISION_MAX_SEGMENTS;

struct Sched {
  uint32_t n_segments;
  uint32_t seg_start[MAX_SEG];
  uint32_t seg_len[MAX_SEG];
  uint32_t item_prefix[MAX_SEG + 1];  // query tiles before segment s (sorted order)
};

struct Params {
  const __half* q;
  const __half* k;
  const __half* v;
  const float* rope_cos;
  const float* rope_sin;
  __half* out;
  uint32_t heads;
};

// Load rows [r0, r0+rows) of one head into shared memory (144-byte pitch),
// rotating by the per-token tables when given.  Rows past `valid` are zero.
__device__ __forceinline__ void load_rows_rotated(uint8_t* dst, const __half* src,
                                                  const float* cos_t, const float* sin_t,
                                                  uint32_t tok0, int valid, uint32_t heads,
                                                  uint32_t head, int tid) {
  // item = (row, chunk j): dims [4j, 4j+4) and partner dims [36+4j, 36+4j+4)
  for (int it = tid; it < BN * 9; it += THREADS) {
    const int r = it / 9, j = it % 9;
    uint2 lo = make_uint2(0, 0), hi = make_uint2(0, 0);
    if (r < valid) {
      const size_t t = tok0 + r;
      const __half* row = src + (t * heads + head) * HD;
      lo = *reinterpret_cast<const uint2*>(row + 4 * j);
      hi = *reinterpret_cast<const uint2*>(row + PAIRS + 4 * j);
      if (cos_t) {
        const float4 c = __ldg(reinterpret_cast<const float4*>(cos_t + t * PAIRS + 4 * j));
        const float4 s = __ldg(reinterpret_cast<const float4*>(sin_t + t * PAIRS + 4 * j));
        const __half* a = reinterpret_cast<const __half*>(&lo);
        const __half* b = reinterpret_cast<const __half*>(&hi);
        const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
        __align__(8) __half ra[4], rb[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x0 = __half2float(a[e]), x1 = __half2float(b[e]);
          ra[e] = __float2half_rn(x0 * cc[e] - x1 * ss[e]);
          rb[e] = __float2half_rn(x1 * cc[e] + x0 * ss[e]);
        }
        lo = *reinterpret_cast<uint2*>(ra);
        hi = *reinterpret_cast<uint2*>(rb);
      }
    }
    *reinterpret_cast<uint2*>(dst + r * ROW_BYTES + 8 * j) = lo;
    *reinterpret_cast<uint2*>(dst + r * ROW_BYTES + PAIRS * 2 + 8 * j) = hi;
  }
}

__device__ __forceinline__ void load_rows_plain(uint8_t* dst, const __half* src, uint32_t tok0,
                                                int valid, uint32_t heads, uint32_t head,
                                                int tid) {
  for (int it = tid; it < BN * 9; it += THREADS) {
    const int r = it / 9, j = it % 9;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < valid)
      val = *reinterpret_cast<const uint4*>(src + ((size_t)(tok0 + r) * heads + head) * HD + 8 * j);
    *reinterpret_cast<uint4*>(dst + r * ROW_BYTES + 16 * j) = val;
  }
}

__global__ void __launch_bounds__(THREADS) vision_mma_kernel(const Params p, const Sched sc) {
  __shared__ __align__(128) uint8_t sQ[BM * ROW_BYTES];
  __shared__ __align__(128) uint8_t sK[BN * ROW_BYTES];
  __shared__ __align__(128) uint8_t sV[BN * ROW_BYTES];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const uint32_t head = blockIdx.x;
  const uint32_t item = blockIdx.y;
  uint32_t s = 0;
  while (s + 1 < sc.n_segments && sc.item_prefix[s + 1] <= item) ++s;
  const uint32_t seg0 = sc.seg_start[s], seglen = sc.seg_len[s];
  const uint32_t q0 = seg0 + (item - sc.item_prefix[s]) * BM;
  const int q_valid = static_cast<int>(umin32(BM, seg0 + seglen - q0));

  load_rows_rotated(sQ, p.q, p.rope_cos, p.rope_sin, q0, q_valid, p.heads, head, tid);
  __syncthreads();

  // Q A-fragments: 16 rows x 72 dims (4 x k16 + 1 x k8)
  uint32_t qa[4][4], qa8[2];
  {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const uint32_t base = smem_u32(sQ + r * ROW_BYTES + (lane >> 4) * 16);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], base + ks * 32);
    const int r8 = warp * 16 + (lane & 15);
    ldsm_x2(qa8[0], qa8[1], smem_u32(sQ + r8 * ROW_BYTES + 128));
  }

  const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F}, l_run[2] = {0.f, 0.f};
  float o[9][4];
#pragma unroll
  for (int i = 0; i < 9; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (uint32_t kt0 = 0; kt0 < seglen; kt0 += BN) {
    const int k_valid = static_cast<int>(umin32(BN, seglen - kt0));
    __syncthreads();
    load_rows_rotated(sK, p.k, p.rope_cos, p.rope_sin, seg0 + kt0, k_valid, p.heads, head, tid);
    load_rows_plain(sV, p.v, seg0 + kt0, k_valid, p.heads, head, tid);
    __syncthreads();

    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // 16 keys per step
      // x4: m0 keys 0-7 dims d, m1 keys 0-7 dims d+8, m2 keys 8-15 dims d, m3 keys 8-15 dims d+8
      const int kr = np * 16 + (lane & 7) + (lane >> 4) * 8;
      const uint32_t kb = smem_u32(sK + kr * ROW_BYTES + ((lane >> 3) & 1) * 16);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, kb + ks * 32);
        mma_16816(sacc[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_16816(sacc[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
      uint32_t e0, e1;
      const int kr8 = np * 16 + (lane & 15);
      ldsm_x2(e0, e1, smem_u32(sK + kr8 * ROW_BYTES + 128));
      mma_1688(sacc[2 * np], qa8[0], qa8[1], e0);
      mma_1688(sacc[2 * np + 1], qa8[0], qa8[1], e1);
    }
    // online softmax (rows g and g+8 of this warp)
    float mx0 = m_run[0], mx1 = m_run[1];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = nt * 8 + 2 * c + e;
        const bool ok = key < k_valid;
        sacc[nt][e] = ok ? sacc[nt][e] * scale : -CUDART_INF_F;
        sacc[nt][2 + e] = ok ? sacc[nt][2 + e] * scale : -CUDART_INF_F;
        mx0 = fmaxf(mx0, sacc[nt][e]);
        mx1 = fmaxf(mx1, sacc[nt][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float al0 = fast_exp2(m_run[0] - mx0), al1 = fast_exp2(m_run[1] - mx1);
    m_run[0] = mx0;
    m_run[1] = mx1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sacc[nt][0] = fast_exp2(sacc[nt][0] - mx0);
      sacc[nt][1] = fast_exp2(sacc[nt][1] - mx0);
      sacc[nt][2] = fast_exp2(sacc[nt][2] - mx1);
      sacc[nt][3] = fast_exp2(sacc[nt][3] - mx1);
      rs0 += sacc[nt][0] + sacc[nt][1];
      rs1 += sacc[nt][2] + sacc[nt][3];
    }
    l_run[0] = l_run[0] * al0 + rs0;
    l_run[1] = l_run[1] * al1 + rs1;
#pragma unroll
    for (int nt = 0; nt < 9; ++nt) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_half2(sacc[2 * kk][0], sacc[2 * kk][1]);
      const uint32_t a1 = pack_half2(sacc[2 * kk][2], sacc[2 * kk][3]);
      const uint32_t a2 = pack_half2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      const uint32_t a3 = pack_half2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      // trans x4: m0 keys 0-7 dims d, m1 keys 8-15 dims d, m2 keys 0-7 dims d+8, m3 keys 8-15 dims d+8
      const int vr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const uint32_t vb = smem_u32(sV + vr * ROW_BYTES + (lane >> 4) * 16);
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, vb + dp * 32);
        mma_16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma_16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
      uint32_t b0, b1;
      const int vr8 = kk * 16 + (lane & 15);
      ldsm_x2_t(b0, b1, smem_u32(sV + vr8 * ROW_BYTES + 128));
      mma_16816(o[8], a0, a1, a2, a3, b0, b1);
    }
  }

  // normalise and store
  float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  const int r0 = warp * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int nt = 0; nt < 9; ++nt) {
    const int d = nt * 8 + 2 * c;
    if (r0 < q_valid)
      *reinterpret_cast<__half2*>(p.out + ((size_t)(q0 + r0) * p.heads + head) * HD + d) =
          __floats2half2_rn(o[nt][0] * i0, o[nt][1] * i0);
    if (r1 < q_valid)
      *reinterpret_cast<__half2*>(p.out + ((size_t)(q0 + r1) * p.heads + head) * HD + d) =
          __floats2half2_rn(o[nt][2] * i1, o[nt][3] * i1);
  }
}

}  // namespace vision

int vision_mma_launch(const VisionArgs& a, const uint32_t* cu, uint32_t segments,
                  cudaStream_t stream) {
  vision::Sched sc;
  std::vector<uint32_t> order(segments);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t x, uint32_t y) {
    return (cu[x + 1] - cu[x]) > (cu[y + 1] - cu[y]);
  });
  sc.n_segments = segments;
  uint32_t items = 0;
  for (uint32_t i = 0; i < segments; ++i) {
    const uint32_t s = order[i];
    sc.seg_start[i] = cu[s];
    sc.seg_len[i] = cu[s + 1] - cu[s];
    sc.item_prefix[i] = items;
    items += (sc.seg_len[i] + vision::BM - 1) / vision::BM;
  }
  sc.item_prefix[segments] = items;
  if (items > 65535u) return PVLC_INVALID_VISION_GEOMETRY;
  vision::Params p;
  p.q = reinterpret_cast<const __half*>(a.q);
  p.k = reinterpret_cast<const __half*>(a.k);
  p.v = reinterpret_cast<const __half*>(a.v);
  p.rope_cos = a.rope_cos;
  p.rope_sin = a.rope_sin;
  p.out = reinterpret_cast<__half*>(a.out);
  p.heads = a.heads;
  dim3 grid(a.heads, items);
  vision::vision_mma_kernel<<<grid, vision::THREADS, 0, stream>>>(p, sc);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // namespace pvlc
