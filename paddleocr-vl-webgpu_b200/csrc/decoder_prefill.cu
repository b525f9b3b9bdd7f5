// decoder_prefill.cu -- decoder causal GQA prefill (pinned Q16/KV2/D128) with
// the 3-section multimodal RoPE fused into the Q/K tile loads and the rotated
// key / raw value written into the fp16 KV cache in place, sm_100a.
//
// Reference path replaced: DecoderPrefillMropeF32 -> DecoderKvAppendRangeF32
// -> DecoderPrefillGqaF32 (crates/pvlc-wgsl/src/lib.rs:1262-1416; stage order
// crates/pvlc-runtime-core/src/lib.rs:2613-2629); arithmetic
// crates/pvlc-cpu-ref/src/lib.rs:562-672 (M-RoPE), :976-991 (KV write),
// :782-853 (causal GQA).
//
// Work item = (64-query tile, query head), heavy (late) tiles first.  A CTA
// visits key tiles 0..i only (causal tile skipping) and masks inside the
// diagonal tile.  The CTA that owns the first query head of a KV group
// writes that group's diagonal key/value tile into the cache, so every cache
// row is written exactly once.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"

namespace pvlc {
namespace prefill {

constexpr int HD = 128;
constexpr int QH = 16;
constexpr int KVH = 2;
constexpr int GROUP = QH / KVH;
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int PITCH = HD * 2 + 16;  // 272-byte rows: conflict-free ldmatrix

struct Params {
  const __half* q;
  const __half* k;
  const __half* v;
  const float* rope_cos;
  const float* rope_sin;
  uint32_t rope_rows;
  uint32_t tokens;
  __half* k_cache;
  __half* v_cache;
  __half* out;
};

// Rotate rows [t0, t0+valid) of head `head` (of `heads`) with M-RoPE into
// shared memory.  Item = (row, chunk j): dims [4j, 4j+4) and [64+4j, 64+4j+4).
__device__ __forceinline__ void load_mrope(uint8_t* dst, const __half* src, const Params& p,
                                           uint32_t t0, int valid, uint32_t heads, uint32_t head,
                                           int tid) {
  for (int it = tid; it < BN * 16; it += THREADS) {
    const int r = it >> 4, j = it & 15;
    uint2 lo = make_uint2(0, 0), hi = make_uint2(0, 0);
    if (r < valid) {
      const size_t t = t0 + r;
      const __half* row = src + (t * heads + head) * HD;
      const uint2 xa = *reinterpret_cast<const uint2*>(row + 4 * j);
      const uint2 xb = *reinterpret_cast<const uint2*>(row + 64 + 4 * j);
      const size_t tb = ((size_t)mrope_axis(4 * j) * p.rope_rows + t) * HD;
      const float4 ca = __ldg(reinterpret_cast<const float4*>(p.rope_cos + tb + 4 * j));
      const float4 sa = __ldg(reinterpret_cast<const float4*>(p.rope_sin + tb + 4 * j));
      const float4 cb = __ldg(reinterpret_cast<const float4*>(p.rope_cos + tb + 64 + 4 * j));
      const float4 sb = __ldg(reinterpret_cast<const float4*>(p.rope_sin + tb + 64 + 4 * j));
      const __half* a = reinterpret_cast<const __half*>(&xa);
      const __half* b = reinterpret_cast<const __half*>(&xb);
      const float c0[4] = {ca.x, ca.y, ca.z, ca.w}, s0[4] = {sa.x, sa.y, sa.z, sa.w};
      const float c1[4] = {cb.x, cb.y, cb.z, cb.w}, s1[4] = {sb.x, sb.y, sb.z, sb.w};
      __align__(8) __half ra[4], rb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = __half2float(a[e]), x1 = __half2float(b[e]);
        ra[e] = __float2half_rn(x0 * c0[e] + (-x1) * s0[e]);
        rb[e] = __float2half_rn(x1 * c1[e] + x0 * s1[e]);
      }
      lo = *reinterpret_cast<uint2*>(ra);
      hi = *reinterpret_cast<uint2*>(rb);
    }
    *reinterpret_cast<uint2*>(dst + r * PITCH + 8 * j) = lo;
    *reinterpret_cast<uint2*>(dst + r * PITCH + 128 + 8 * j) = hi;
  }
}

__device__ __forceinline__ void load_plain(uint8_t* dst, const __half* src, uint32_t t0, int valid,
                                           uint32_t heads, uint32_t head, int tid) {
  for (int it = tid; it < BN * 16; it += THREADS) {
    const int r = it >> 4, j = it & 15;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < valid)
      val = *reinterpret_cast<const uint4*>(src + ((size_t)(t0 + r) * heads + head) * HD + 8 * j);
    *reinterpret_cast<uint4*>(dst + r * PITCH + 16 * j) = val;
  }
}

__global__ void __launch_bounds__(THREADS) prefill_mma_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + BM * PITCH;
  uint8_t* sV = sK + BN * PITCH;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const uint32_t head = blockIdx.x;
  const uint32_t kvh = head / GROUP;
  const uint32_t n_tiles = (p.tokens + BM - 1) / BM;
  const uint32_t qt = n_tiles - 1 - blockIdx.y;  // heaviest first
  const uint32_t q0 = qt * BM;
  const int q_valid = static_cast<int>(umin32(BM, p.tokens - q0));

  load_mrope(sQ, p.q, p, q0, q_valid, QH, head, tid);
  __syncthreads();
  uint32_t qa[8][4];
  {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const uint32_t base = smem_u32(sQ + r * PITCH + (lane >> 4) * 16);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], base + ks * 32);
  }

  const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
  float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F}, l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int row0 = warp * 16 + g;  // query rows row0, row0 + 8 within the tile

  for (uint32_t kt = 0; kt <= qt; ++kt) {
    const uint32_t k0 = kt * BN;
    const int k_valid = static_cast<int>(umin32(BN, p.tokens - k0));
    __syncthreads();
    load_mrope(sK, p.k, p, k0, k_valid, KVH, kvh, tid);
    load_plain(sV, p.v, k0, k_valid, KVH, kvh, tid);
    __syncthreads();
    if (kt == qt && (head % GROUP) == 0) {
      // in-place cache write of this KV group's diagonal tile
      for (int it = tid; it < k_valid * 16; it += THREADS) {
        const int r = it >> 4, j = it & 15;
        const size_t dst = ((size_t)(k0 + r) * KVH + kvh) * HD + 8 * j;
        *reinterpret_cast<uint4*>(p.k_cache + dst) = *reinterpret_cast<uint4*>(sK + r * PITCH + 16 * j);
        *reinterpret_cast<uint4*>(p.v_cache + dst) = *reinterpret_cast<uint4*>(sV + r * PITCH + 16 * j);
      }
    }

    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const int kr = np * 16 + (lane & 7) + (lane >> 4) * 8;
      const uint32_t kb = smem_u32(sK + kr * PITCH + ((lane >> 3) & 1) * 16);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, kb + ks * 32);
        mma_16816(sacc[2 * np], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_16816(sacc[2 * np + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    const bool diag = kt == qt;
    float mx0 = m_run[0], mx1 = m_run[1];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = nt * 8 + 2 * c + e;
        const bool ok0 = key < k_valid && (!diag || key <= row0);
        const bool ok1 = key < k_valid && (!diag || key <= row0 + 8);
        sacc[nt][e] = ok0 ? sacc[nt][e] * scale : -CUDART_INF_F;
        sacc[nt][2 + e] = ok1 ? sacc[nt][2 + e] * scale : -CUDART_INF_F;
        mx0 = fmaxf(mx0, sacc[nt][e]);
        mx1 = fmaxf(mx1, sacc[nt][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    // rows past the end of the sequence see no valid key in a padded tile only
    // when the whole row is padding; keep them finite (they are never stored)
    if (mx0 == -CUDART_INF_F) mx0 = 0.f;
    if (mx1 == -CUDART_INF_F) mx1 = 0.f;
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
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_half2(sacc[2 * kk][0], sacc[2 * kk][1]);
      const uint32_t a1 = pack_half2(sacc[2 * kk][2], sacc[2 * kk][3]);
      const uint32_t a2 = pack_half2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      const uint32_t a3 = pack_half2(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      const int vr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const uint32_t vb = smem_u32(sV + vr * PITCH + (lane >> 4) * 16);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, vb + dp * 32);
        mma_16816(o[2 * dp], a0, a1, a2, a3, b0, b1);
        mma_16816(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
  }

  float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  const int r1 = row0 + 8;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * c;
    if (row0 < q_valid)
      *reinterpret_cast<__half2*>(p.out + ((size_t)(q0 + row0) * QH + head) * HD + d) =
          __floats2half2_rn(o[nt][0] * i0, o[nt][1] * i0);
    if (r1 < q_valid)
      *reinterpret_cast<__half2*>(p.out + ((size_t)(q0 + r1) * QH + head) * HD + d) =
          __floats2half2_rn(o[nt][2] * i1, o[nt][3] * i1);
  }
}

constexpr int SMEM_BYTES = (BM + 2 * BN) * PITCH;

}  // namespace prefill

int prefill_query_tile() { return prefill::BM; }

int prefill_launch(const PrefillArgs& a, cudaStream_t stream) {
  prefill::Params p;
  p.q = reinterpret_cast<const __half*>(a.q);
  p.k = reinterpret_cast<const __half*>(a.k);
  p.v = reinterpret_cast<const __half*>(a.v);
  p.rope_cos = a.rope_cos;
  p.rope_sin = a.rope_sin;
  p.rope_rows = a.rope_rows;
  p.tokens = a.tokens;
  p.k_cache = reinterpret_cast<__half*>(a.k_cache);
  p.v_cache = reinterpret_cast<__half*>(a.v_cache);
  p.out = reinterpret_cast<__half*>(a.out);
  const uint32_t n_tiles = (a.tokens + prefill::BM - 1) / prefill::BM;
  if (n_tiles > 65535u) return PVLC_INVALID_DECODER_GEOMETRY;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PVLC_CUDA_ERROR;
  if (dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(prefill::prefill_mma_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             prefill::SMEM_BYTES) != cudaSuccess)
      return PVLC_CUDA_ERROR;
    attr_set[dev] = true;
  }
  dim3 grid(prefill::QH, n_tiles);
  prefill::prefill_mma_kernel<<<grid, prefill::THREADS, prefill::SMEM_BYTES, stream>>>(p);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // namespace pvlc
