// lm_head.cu -- greedy top-1 over the LM head on the tensor cores.  sm_100a.
//
// logits = hidden[rows, K] x lm_head[vocab, K]^T with fp16 operands and f32
// accumulation (tcgen05.mma, accumulators in TMEM), reduced to each row's
// arg-max inside the kernel: the [rows, vocab] f32 logits never reach HBM.
//
// Reference: chunked_lm_head_top_k_f32 with top_k = 1 and
// compare_top_k_entries (crates/pvlc-cpu-ref/src/lib.rs:1511-1568,
// 2051-2056): a larger logit wins in f32::total_cmp order and equal logits go
// to the smaller token id; the WebGPU session's greedy step runs the same
// rule as an argmax pass over the logits buffer
// (crates/pvlc-runtime-web/src/web/decoder_stack_session.rs:308-350).
//
// Work split: one CTA per SM walks the 256-row vocabulary tiles (N tiles
// blockIdx.x, + gridDim.x, ...) with every row of hidden (up to two M tiles
// of 128).  Per K step of 64 dims the producer warp loads the N tile's
// 256 x 64 weights (32 KB, TMA, 128B swizzle) and each M tile's 128 x 64
// slice of hidden (16 KB; rows past `rows` are TMA zero fill) into a 3-stage
// ring that runs on across tiles; the MMA warp issues four M128 N256 K16
// MMAs per M tile into TMEM: with one M tile the accumulators alternate
// between columns 0 and 256 by tile, so an epilogue overlaps the next tile's
// MMAs; with two they take columns [256 m, 256 m + 256) and the next tile
// waits for the epilogue (acc_free).  Epilogue: one warpgroup
// per M tile, thread = row = TMEM lane; it reads its 256 logits and keeps the
// largest in total_cmp order (the first, i.e. smallest, index on ties), then
// folds it into the row's 64-bit key with one atomicMax:
//   key = order-preserving bits of the logit << 32 | (0xFFFFFFFF - token id),
// so the maximum key over all N tiles is the largest logit with the smallest
// id.  A second, tiny launch turns the keys into token ids.  The weights
// (vocab x K fp16) are streamed from HBM exactly once per call.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"
#include "tcgen05.cuh"

namespace pvlc {
namespace lmh {

constexpr int BN = 256;            // vocabulary rows per CTA (MMA N)
constexpr int BM = 128;            // hidden rows per M tile (MMA M)
constexpr int MAX_MT = 2;          // M tiles: up to 256 rows
constexpr int BK = 64;             // K per stage (one 128-byte swizzle row)
constexpr int STAGES = 3;
constexpr int THREADS = 10 * 32;   // 2 epilogue warpgroups, producer, MMA
constexpr uint32_t SZ_B = BN * BK * 2;                 // 32 KB
constexpr uint32_t SZ_A = BM * BK * 2;                 // 16 KB per M tile
constexpr uint32_t STAGE_BYTES = SZ_B + MAX_MT * SZ_A; // 64 KB
constexpr uint32_t OFF_BARS = STAGES * STAGE_BYTES;
constexpr int NBARS = 2 * STAGES + 4;                  // full, empty, acc_full[2], acc_free[2]
constexpr uint32_t OFF_MISC = OFF_BARS + NBARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "lm-head shared memory exceeds the sm_100 limit");
constexpr uint32_t TMEM_COLS = 512;

struct Maps {
  CUtensorMap a;   // hidden  {K, rows}, box {64, 128}
  CUtensorMap b;   // lm_head {K, vocab}, box {64, 256}
};

struct Params {
  uint32_t rows, vocab, ksteps, mtiles;
  unsigned long long* keys;
  uint32_t* flags;   // bit 3: a pipeline wait timed out
};

// f32 bits -> uint32 in f32::total_cmp order (-NaN < -inf < ... < +inf < +NaN)
__device__ __forceinline__ uint32_t total_order_bits(uint32_t u) {
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(THREADS, 1)
    lm_head_top1_kernel(const __grid_constant__ Maps maps, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BARS);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2] a tile's accumulators are complete
  uint64_t* acc_free = acc_full + 2;     // [2] the epilogue has read them
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);
  // misc[0]: TMEM base, misc[1]: abort

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ks = static_cast<int>(p.ksteps);
  const int mt = static_cast<int>(p.mtiles);
  // accumulator buffers: two (double-buffered tiles) for one M tile, one for two
  const int nacc = mt == 1 ? 2 : 1;
  // this CTA's vocabulary tiles: blockIdx.x, + gridDim.x, ...
  const uint32_t ntile = (p.vocab + BN - 1) / BN;
  const uint32_t my_tiles =
      blockIdx.x < ntile ? (ntile - 1 - blockIdx.x) / gridDim.x + 1 : 0u;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_free[a], 4 * mt);   // every epilogue warp
    }
    misc[1] = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(const_cast<uint32_t*>(misc), TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = misc[0];

  if (warp == 8) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      tc::tma_prefetch_desc(&maps.a);
      tc::tma_prefetch_desc(&maps.b);
      // hidden is produced by the kernel ahead (the final norm)
      pdl_wait();
      uint32_t g = 0;   // k steps issued so far (ring position)
      for (uint32_t tt = 0; tt < my_tiles && !misc[1]; ++tt) {
        const uint32_t n0 = (blockIdx.x + tt * gridDim.x) * BN;
        for (int s = 0; s < ks; ++s, ++g) {
          const int st = static_cast<int>(g % STAGES);
          if (misc[1] || !mbar_wait(&empty[st], ((g / STAGES) & 1) ^ 1)) { misc[1] = 1; break; }
          uint8_t* base = smem + st * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], SZ_B + mt * SZ_A);
          tc::tma_load_2d(base, &maps.b, s * BK, n0, &full[st]);
          for (int m = 0; m < mt; ++m)
            tc::tma_load_2d(base + SZ_B + m * SZ_A, &maps.a, s * BK, m * BM, &full[st]);
        }
      }
      // the last loads must land before the CTA may exit
      for (uint32_t g2 = (g > STAGES ? g - STAGES : 0); g2 < g; ++g2)
        mbar_wait(&full[g2 % STAGES], (g2 / STAGES) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = tc::idesc_f16(BM, BN, 0, 0);
    const uint32_t s0 = smem_u32(smem);
    const uint64_t db = tc::smem_desc(s0, 16, 1024, tc::kSw128);
    const uint64_t da = tc::smem_desc(s0 + SZ_B, 16, 1024, tc::kSw128);
    bool ok = true;
    uint32_t g = 0, done = 0;
    for (uint32_t tt = 0; tt < my_tiles && ok; ++tt) {
      const int a = static_cast<int>(tt % nacc);
      const uint32_t use = tt / nacc;
      if (use > 0 &&
          !__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&acc_free[a], (use - 1) & 1))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t acc = tmem + static_cast<uint32_t>(a * BN);
      for (int s = 0; s < ks; ++s, ++g) {
        const int st = static_cast<int>(g % STAGES);
        if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&full[st], (g / STAGES) & 1))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint64_t so = (uint64_t)st * (STAGE_BYTES >> 4);
        if (tc::elect_one()) {
          for (int m = 0; m < mt; ++m) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)   // 32 bytes per K16 step: +2 in the address field
              tc::mma_ss(acc + (uint32_t)(BN * m), da + so + (uint64_t)m * (SZ_A >> 4) + 2 * kk,
                         db + so + 2 * kk, idesc, (s > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(&empty[st]);
          if (s == ks - 1) tc::commit(&acc_full[a]);
        }
        __syncwarp();
      }
      if (ok) ++done;
    }
    if (!ok && lane == 0) misc[1] = 1;
    // never exit with MMAs in flight or commit arrivals still pending
    for (uint32_t g2 = (g > STAGES ? g - STAGES : 0); g2 < g; ++g2)
      mbar_wait(&empty[g2 % STAGES], (g2 / STAGES) & 1);
    if (done > 0) {
      const uint32_t last = done - 1;
      mbar_wait(&acc_full[last % nacc], (last / nacc) & 1);
    }
  } else if (warp / 4 < mt) {
    // ------------------------------------------------------- epilogue
    const int m = warp / 4;
    const int i = (warp & 3) * 32 + lane;            // row within the M tile = TMEM lane
    const uint32_t row = m * BM + i;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool good = true;
    for (uint32_t tt = 0; tt < my_tiles && good; ++tt) {
      const int a = static_cast<int>(tt % nacc);
      const uint32_t use = tt / nacc;
      const uint32_t n0 = (blockIdx.x + tt * gridDim.x) * BN;
      if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&acc_full[a], use & 1))) {
        good = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t tD = tmem + lane_off + static_cast<uint32_t>(a * BN + BN * m);
      const uint32_t valid = p.vocab - n0 < (uint32_t)BN ? p.vocab - n0 : (uint32_t)BN;
      uint32_t best = 0, best_c = 0xFFFFFFFFu;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld32(tD + c0, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const uint32_t key = total_order_bits(v[e]);
          const uint32_t c = (uint32_t)(c0 + e);
          // strictly greater: among equal logits the first (smallest) id stays
          if (c < valid && (best_c == 0xFFFFFFFFu || key > best)) {
            best = key;
            best_c = c;
          }
        }
      }
      // the accumulators may take the next tile
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[a]);
      if (row < p.rows && best_c != 0xFFFFFFFFu)
        atomicMax(p.keys + row, ((unsigned long long)best << 32) |
                                    (unsigned long long)(0xFFFFFFFFu - (n0 + best_c)));
    }
    if (!good && lane == 0) atomicOr(p.flags, kFlagTimeout);
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && misc[1]) atomicOr(p.flags, kFlagTimeout);
  if (warp == 8) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// keys -> token ids (and the winning logit)
__global__ void finish_kernel(const unsigned long long* __restrict__ keys, uint32_t rows,
                              int32_t* __restrict__ tokens, float* __restrict__ logit) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const unsigned long long k = keys[r];
  tokens[r] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
  if (logit) {
    const uint32_t o = static_cast<uint32_t>(k >> 32);
    logit[r] = __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  });
  return fn;
}

// [rows, k] fp16 row-major as a 2-D tensor {k, rows}; box {64, box_rows}, 128B swizzle
bool make_map(CUtensorMap* m, const void* base, uint32_t k, uint32_t rows, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace lmh

int lm_head_top1_launch(const LmHeadArgs& a, cudaStream_t stream) {
  if (set_smem_attribute_once(reinterpret_cast<const void*>(lmh::lm_head_top1_kernel),
                              lmh::SMEM_BYTES) != PVLC_OK)
    return PVLC_CUDA_ERROR;
  lmh::Maps maps;
  if (!lmh::make_map(&maps.a, a.hidden, a.hidden_dim, a.rows, lmh::BM) ||
      !lmh::make_map(&maps.b, a.lm_head, a.hidden_dim, a.vocab, lmh::BN))
    return PVLC_CUDA_ERROR;
  lmh::Params p;
  p.rows = a.rows;
  p.vocab = a.vocab;
  p.ksteps = a.hidden_dim / lmh::BK;
  p.mtiles = (a.rows + lmh::BM - 1) / lmh::BM;
  p.keys = reinterpret_cast<unsigned long long*>(a.workspace);
  p.flags = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.workspace) +
                                        lm_head_flags_offset(a.rows));
  // the keys start at 0 (below every real key); the fault word too
  if (cudaMemsetAsync(a.workspace, 0, lm_head_workspace_bytes(a.rows), stream) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  cudaLaunchConfig_t cfg = {};
  // persistent: one CTA per SM walks the vocabulary tiles (fewer when there are fewer tiles)
  const int sms = device_sm_count();
  if (sms <= 0) return PVLC_CUDA_ERROR;
  const uint32_t ntile = (a.vocab + lmh::BN - 1) / lmh::BN;
  cfg.gridDim = dim3(ntile < (uint32_t)sms ? ntile : (uint32_t)sms);
  cfg.blockDim = dim3(lmh::THREADS);
  cfg.dynamicSmemBytes = lmh::SMEM_BYTES;
  cfg.stream = stream;
  if (cudaLaunchKernelEx(&cfg, lmh::lm_head_top1_kernel, maps, p) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  lmh::finish_kernel<<<(a.rows + 127) / 128, 128, 0, stream>>>(p.keys, a.rows, a.tokens,
                                                                 a.logits);
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

size_t lm_head_flags_offset(uint32_t rows) { return ((size_t)rows * 8 + 255) / 256 * 256; }
size_t lm_head_workspace_bytes(uint32_t rows) { return lm_head_flags_offset(rows) + 256; }

}  // namespace pvlc

using namespace pvlc;

extern "C" {

size_t pvlc_lm_head_top1_workspace_bytes(uint32_t rows) {
  return rows == 0 || rows > PVLC_LM_HEAD_MAX_ROWS ? 0 : lm_head_workspace_bytes(rows);
}

int pvlc_lm_head_top1(const pvlc_half* hidden, uint32_t rows, const pvlc_half* lm_head,
                      uint32_t vocab, uint32_t hidden_dim, void* workspace,
                      size_t workspace_bytes, int32_t* tokens, float* logits, void* stream) {
  if (rows == 0 || vocab == 0 || hidden_dim == 0) return PVLC_ZERO_DIMENSION;
  if (rows > PVLC_LM_HEAD_MAX_ROWS || hidden_dim % 64 != 0 || hidden_dim > 8192)
    return PVLC_INVALID_DECODER_GEOMETRY;
  if (!hidden || !lm_head || !workspace || !tokens) return PVLC_NULL_POINTER;
  if (((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(lm_head) |
        reinterpret_cast<uintptr_t>(workspace)) & 15u) ||
      (reinterpret_cast<uintptr_t>(tokens) & 3u) || (reinterpret_cast<uintptr_t>(logits) & 3u))
    return PVLC_MISALIGNED_POINTER;
  if (workspace_bytes < lm_head_workspace_bytes(rows)) return PVLC_WORKSPACE_TOO_SMALL;
  LmHeadArgs a{hidden, lm_head, rows, vocab, hidden_dim, workspace, tokens, logits};
  return lm_head_top1_launch(a, static_cast<cudaStream_t>(stream));
}

int pvlc_lm_head_top1_errors(void* workspace, uint32_t rows, uint32_t* flags_out,
                             void* stream) {
  if (!workspace || !flags_out || rows == 0 || rows > PVLC_LM_HEAD_MAX_ROWS)
    return PVLC_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, static_cast<uint8_t*>(workspace) + lm_head_flags_offset(rows), 4,
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  *flags_out = v;
  return v ? PVLC_DEVICE_FAULT_FLAG : PVLC_OK;
}

}  // extern "C"
