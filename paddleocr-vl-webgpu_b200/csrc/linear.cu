// linear.cu -- the decode step's dense projections at small batch on the
// tensor cores.  sm_100a.
//
// out[r, f] = sum_k x[r, k] * w[f, k] for the decoder layer's QKV, O, gate-up
// and down projections, fp16 operands and f32 accumulation (tcgen05.mma,
// accumulators in TMEM), with rows = the decode batch (1..256).  Reference:
// the decoder-stack GEMV/GEMM passes of the WebGPU session
// (crates/pvlc-wgsl/src/lib.rs:1770-1835, scheduled by
// crates/pvlc-runtime-core/src/lib.rs:1175-1548) and their arithmetic in the
// CPU reference (matvec over the layer's weights, crates/pvlc-cpu-ref/src/lib.rs:
// 1385-1390 for the gated MLP product).
//
// At decode batch sizes every projection is a read of its weight matrix
// (1-12 MB) with a few FLOPs per byte, so the kernel is organised around
// that read:
//   * Swap-AB tiles: the MMA's M side is 128 output features (the weight
//     tile, A), its N side the batch rows padded to a multiple of 16 (B), so
//     no tensor work is spent on padding rows beyond 16.
//   * Split K: the K range of a feature tile is cut into `split` slices, one
//     CTA each, so ~150 CTAs stream the matrix at once.  The slices of one
//     tile form a thread-block cluster (co-scheduled).  Each warp stages its
//     32 features of the slice's f32 partial sums in shared memory and sends
//     every row block to the CTA that owns those rows with one bulk copy
//     into that CTA's shared memory (distributed shared memory, completion
//     counted in bytes on the owner's mbarrier; no L2 round trip and no
//     CTA-wide barrier on the way).  Owners add the slices in slice order, so
//     results do not depend on timing.
//   * Weights before the dependency: the kernel is launched with
//     programmatic dependent launch.  Its weight tiles depend on nothing the
//     kernels ahead write, so the producer issues them before
//     griddepcontrol.wait; only the activation tiles (and every store) wait.
//     The weight read overlaps the tail of the kernel ahead.
//   * Fused SiLU gate: with `silu` set, each 128-row weight tile holds 64 gate
//     rows followed by the 64 matching up rows, and the epilogue writes
//     fp16(silu(fp16(gate)) * fp16(up)) for its 64 pairs (the same roundings
//     as the unfused projection + SiLU-gate kernel), halving the output.
//
// Roles (4 warps): warp 0 lane 0 issues the TMA loads, warp 1 issues the
// MMAs (one elected lane), then all four warps read their TMEM lane quadrant
// in the epilogue.  Every mbarrier wait is bounded; a timeout sets the CTA's
// abort flag, the CTA drains its copies and MMAs, still sends (zeros) to its
// cluster peers and meets its cluster barrier, and reports
// PVLC_FAULT_LINEAR in the sticky device fault word.
//
// Measured standing (B200, inside a CUDA graph, weights larger than L2): at
// 32 rows the four projections of a decoder layer take 26.4 us against
// 24.8 us for cuBLAS + the SiLU-gate pass -- down 6.7 vs 7.7 us and gate-up
// + SiLU 7.7 vs 7.8 us, but QKV 6.0 vs 3.8 us.  A %globaltimer trace puts the
// floor of one launch at ~2.5 us after the kernel ahead ends (0.8 us until
// griddepcontrol.wait returns, 0.8 us for the activation tile from L2,
// 0.25 us of MMA, the cluster exchange) while the weights are already in
// shared memory; at 256 rows only one slice fits in shared memory and
// cuBLAS is 3x faster.  What would beat both is one persistent kernel per
// decoder layer that keeps the activations on chip between projections.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"
#include "tcgen05.cuh"

namespace pvlc {
namespace lin {

constexpr int BF = 128;             // output features per tile (MMA M)
constexpr int BK = 64;              // K per stage (one 128-byte swizzle row)
constexpr int THREADS = 128;
constexpr int MAX_STAGES = 8;
constexpr uint32_t SZ_W = BF * BK * 2;   // 16 KB weight tile per stage
constexpr uint32_t MAX_SMEM = 216 * 1024;

__device__ uint32_t g_faults;

struct Maps {
  CUtensorMap w;   // weights {K, N}, box {64, 128}
  CUtensorMap x;   // activations {K, rows}, box {64, nb}
};

struct Params {
  uint32_t rows, nb;            // batch rows; rows padded to a multiple of 16 (MMA N)
  uint32_t ksteps;              // K / 64
  uint32_t split, stages, stage_bytes, tmem_cols;
  uint32_t recv_off, rpo;       // with a split: [split][rpo][128] f32 received partials
  uint32_t data_bytes;          // stages + received partials
  uint32_t silu;
  __half* out;
  uint32_t ldo;                 // elements between output rows
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of the local shared address `addr` in CTA
// `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(addr), "r"(rank));
  return ra;
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory into another CTA's of the cluster; its
// completion counts the bytes on that CTA's mbarrier `rbar`.
__device__ __forceinline__ void bulk_s2cluster(uint32_t rdst, uint32_t src, uint32_t bytes,
                                               uint32_t rbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(rdst),
      "r"(src), "r"(bytes), "r"(rbar)
      : "memory");
}

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded wait (4x the pipeline limit: the peers' own waits come first) with
// cluster-scope acquire, for data other CTAs stored into this one.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      uint32_t ok;
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(smem_u32(bar)), "r"(parity)
          : "memory");
      if (ok) return true;
    }
    if (globaltimer() - t0 > 4 * kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// fp16(silu(fp16(g)) * fp16(u)): the roundings of a projection written as
// fp16 followed by the SiLU-gate pass
__device__ __forceinline__ float gate(float g, float u) {
  return silu(__half2float(__float2half_rn(g))) * __half2float(__float2half_rn(u));
}

__global__ void __launch_bounds__(THREADS, 1)
    linear_kernel(const __grid_constant__ Maps maps, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int st = static_cast<int>(p.stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.data_bytes);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* acc_full = empty + MAX_STAGES;
  uint64_t* recv_full = acc_full + 1;   // every slice's pushes for this CTA's rows landed
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(recv_full + 1);
  // misc[0]: TMEM base, misc[1]: abort

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t S = p.split;
  const uint32_t tile = blockIdx.x / S, slice = blockIdx.x - tile * S;
  const int k_lo = static_cast<int>(slice * p.ksteps / S);
  const int kc = static_cast<int>((slice + 1) * p.ksteps / S) - k_lo;
  const uint32_t sz_x = p.nb * 128u;

  if (tid == 0) {
    for (int s = 0; s < st; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(recv_full, 1);
    misc[1] = 0;
    fence_mbar_init();
    if (S > 1) {
      const uint32_t own = (slice + 1) * p.rows / S - slice * p.rows / S;
      mbar_arrive_expect_tx(recv_full, S * BF * own * 4u);
    }
  }
  if (warp == 0) {
    tc::tmem_alloc(const_cast<uint32_t*>(misc), p.tmem_cols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = misc[0];
  // the peers' barriers are initialised before anyone pushes into them
  if (S > 1) cluster_sync_all();
  // The kernel behind this one may start its own pre-wait work now.  Only
  // after the TMEM allocation: a dependent that allocates first while this
  // grid's CTAs wait for columns would wait on this grid in turn.
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      tc::tma_prefetch_desc(&maps.w);
      tc::tma_prefetch_desc(&maps.x);
      const int pre = kc < st ? kc : st;
      // weights first: nothing ahead of this kernel writes them
      for (int s = 0; s < pre; ++s) {
        mbar_arrive_expect_tx(&full[s], SZ_W + sz_x);
        tc::tma_load_2d(smem + s * p.stage_bytes, &maps.w, (k_lo + s) * BK, tile * BF, &full[s]);
      }
      // the activations are the kernel ahead's output
      pdl_wait();
      for (int s = 0; s < pre; ++s)
        tc::tma_load_2d(smem + s * p.stage_bytes + SZ_W, &maps.x, (k_lo + s) * BK, 0, &full[s]);
      int issued = pre;
      for (int s = pre; s < kc; ++s) {
        const int slot = s % st;
        if (misc[1] || !mbar_wait(&empty[slot], ((s / st) & 1) ^ 1)) {
          misc[1] = 1;
          break;
        }
        uint8_t* base = smem + slot * p.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], SZ_W + sz_x);
        tc::tma_load_2d(base, &maps.w, (k_lo + s) * BK, tile * BF, &full[slot]);
        tc::tma_load_2d(base + SZ_W, &maps.x, (k_lo + s) * BK, 0, &full[slot]);
        issued = s + 1;
      }
      // no copy may still be landing when the CTA exits
      for (int s = (issued > st ? issued - st : 0); s < issued; ++s)
        mbar_wait(&full[s % st], (s / st) & 1);
    } else {
      pdl_wait();   // every thread orders its stores after the kernel ahead
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    pdl_wait();
    const uint32_t idesc = tc::idesc_f16(BF, p.nb, 0, 0);
    const uint32_t s0 = smem_u32(smem);
    const uint64_t dw = tc::smem_desc(s0, 16, 1024, tc::kSw128);
    const uint64_t dx = tc::smem_desc(s0 + SZ_W, 16, 1024, tc::kSw128);
    int done = 0;
    for (int s = 0; s < kc; ++s) {
      const int slot = s % st;
      if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&full[slot], (s / st) & 1))) break;
      tc::fence_after_sync();
      const uint64_t so = (uint64_t)slot * (p.stage_bytes >> 4);
      if (tc::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)   // 32 bytes per K16 step: +2 in the address field
          tc::mma_ss(tmem, dw + so + 2 * kk, dx + so + 2 * kk, idesc, (s > 0 || kk > 0) ? 1u : 0u);
        tc::commit(&empty[slot]);
        if (s == kc - 1) tc::commit(acc_full);
      }
      __syncwarp();
      done = s + 1;
    }
    if (done < kc && lane == 0) misc[1] = 1;
    // never exit with MMAs in flight or commit arrivals still pending
    for (int s = (done > st ? done - st : 0); s < done; ++s)
      mbar_wait(&empty[s % st], (s / st) & 1);
  } else {
    pdl_wait();
  }

  // ---------------------------------------------------------- epilogue
  bool good;
  if (S == 1) {
    good = misc[1] == 0 && mbar_wait(acc_full, 0) && misc[1] == 0;
    good = __syncthreads_and(good) != 0;
  } else {
    // with a split each warp goes on alone: it stages and sends its own 32
    // features, so no CTA-wide barrier sits between the MMAs and the sends
    good = __all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(acc_full, 0) && misc[1] == 0);
  }
  tc::fence_after_sync();
  const uint32_t quad = static_cast<uint32_t>(warp & 3);
  const uint32_t tq = tmem + ((quad * 32u) << 16);
  const uint32_t fl = quad * 32u + lane;   // feature within the tile = TMEM lane
  if (good && S == 1) {
    if (!p.silu) {
      __half* o = p.out + tile * BF + fl;
      for (uint32_t c0 = 0; c0 < p.nb; c0 += 16) {
        uint32_t v[16];
        tc::tmem_ld16(tq + c0, v);
        tc::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (c0 + e < p.rows) o[(size_t)(c0 + e) * p.ldo] = __float2half_rn(__uint_as_float(v[e]));
      }
    } else {
      // up rows (lanes 64..127) hand their sums to the gate rows through
      // shared memory, 16 batch rows at a time; the stages are free now
      float* xb = reinterpret_cast<float*>(smem);   // [16][64]
      __half* o = p.out + tile * (BF / 2) + fl;
      for (uint32_t c0 = 0; c0 < p.nb; c0 += 16) {
        uint32_t v[16];
        tc::tmem_ld16(tq + c0, v);
        tc::tmem_wait_ld();
        if (quad >= 2) {
#pragma unroll
          for (int e = 0; e < 16; ++e) xb[e * 64 + fl - 64] = __uint_as_float(v[e]);
        }
        named_bar_sync(1, THREADS);
        if (quad < 2) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c0 + e < p.rows)
              o[(size_t)(c0 + e) * p.ldo] =
                  __float2half_rn(gate(__uint_as_float(v[e]), xb[e * 64 + fl]));
        }
        named_bar_sync(1, THREADS);
      }
    }
  }
  if (S > 1) {
    // This warp's 32 features of the slice's partial sums, [rows][32] f32,
    // are staged in this CTA's shared memory (the stages are free: the MMAs
    // are complete); then one bulk copy per owner moves that owner's rows
    // (owner q sums rows [q R / S, (q + 1) R / S) of the tile) into its
    // receive buffer recv[slice][warp][row - lo_q][32], completion counted in
    // bytes on the owner's recv_full.  An aborted warp sends zeros, so no
    // owner is left waiting.
    const uint32_t R = p.rows, rpo = p.rpo;
    float* stg = reinterpret_cast<float*>(smem) + quad * R * 32 + lane;
    for (uint32_t c0 = 0; c0 < R; c0 += 16) {
      uint32_t v[16];
      if (good) {
        tc::tmem_ld16(tq + c0, v);
        tc::tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0u;
      }
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c0 + e < R) stg[(c0 + e) * 32] = __uint_as_float(v[e]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const uint32_t src = smem_u32(smem) + quad * R * 128u;
      const uint32_t recv_l = smem_u32(smem + p.recv_off) + (slice * 4 + quad) * rpo * 128u;
      const uint32_t bar_l = smem_u32(recv_full);
      for (uint32_t q = 0; q < S; ++q) {
        const uint32_t lo = q * R / S, cnt = (q + 1) * R / S - lo;
        if (cnt) bulk_s2cluster(mapa(recv_l, q), src + lo * 128u, cnt * 128u, mapa(bar_l, q));
      }
      tc::bulk_commit_group();
    }
    cluster_arrive();
    // this CTA's rows: the slices' sums added in slice order
    const uint32_t lo = slice * R / S, cnt = (slice + 1) * R / S - lo;
    const bool got = mbar_wait_cluster(recv_full, 0);
    if (!got) atomicOr(&g_faults, PVLC_FAULT_LINEAR);
    if (got && good) {
      // recv[slice][warp][row][32]: this thread's feature is (quad, lane)
      const float* rb = reinterpret_cast<const float*>(smem + p.recv_off) + lane;
      const uint32_t sst = 4 * rpo * 32;   // floats per slice
      if (!p.silu) {
        const float* r0 = rb + quad * rpo * 32;
        __half* o = p.out + (size_t)lo * p.ldo + tile * BF + fl;
        for (uint32_t j = 0; j < cnt; ++j) {
          float a = r0[j * 32];
          for (uint32_t sl = 1; sl < S; ++sl) a += r0[sl * sst + j * 32];
          o[(size_t)j * p.ldo] = __float2half_rn(a);
        }
      } else if (quad < 2) {
        const float* rg = rb + quad * rpo * 32;         // gate rows: warps 0-1
        const float* ru = rb + (quad + 2) * rpo * 32;   // their up rows: warps 2-3
        __half* o = p.out + (size_t)lo * p.ldo + tile * (BF / 2) + fl;
        for (uint32_t j = 0; j < cnt; ++j) {
          float a = rg[j * 32], b = ru[j * 32];
          for (uint32_t sl = 1; sl < S; ++sl) {
            a += rg[sl * sst + j * 32];
            b += ru[sl * sst + j * 32];
          }
          o[(size_t)j * p.ldo] = __float2half_rn(gate(a, b));
        }
      }
    }
    // the staged partials have been read out; no CTA leaves while a peer may
    // still copy into its shared memory
    if (lane == 0) tc::bulk_wait_read_all();
    cluster_wait();
  }

  tc::fence_before_sync();
  __syncthreads();
  if (lane == 0 && !good) atomicOr(&g_faults, PVLC_FAULT_LINEAR);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, p.tmem_cols);
  }
}

}  // namespace lin

namespace lin {

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

// [rows, k] fp16 with row pitch ld elements as a 2-D tensor {k, rows};
// box {64, box_rows}, 128B swizzle; rows past the end read as zeros
bool make_map(CUtensorMap* m, const void* base, uint32_t k, uint32_t rows, uint32_t ld,
              uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t padded_rows(uint32_t rows) { return (rows + 15u) / 16u * 16u; }

uint32_t stage_bytes(uint32_t rows) { return SZ_W + padded_rows(rows) * 128u; }

}  // namespace lin

int linear_fault_word(uint32_t* out, cudaStream_t s) {
  uint32_t v = 0;
  const uint32_t zero = 0;
  if (cudaMemcpyFromSymbolAsync(&v, lin::g_faults, 4, 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaMemcpyToSymbolAsync(lin::g_faults, &zero, 4, 0, cudaMemcpyHostToDevice, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  *out = v;
  return PVLC_OK;
}

namespace lin {

// Shared memory of one CTA: the stages (or, with a split, at least the
// [rows][128] f32 partials staged in their place), the received partials
// of its rows, barriers.  False when it does not fit.
bool plan(uint32_t rows, uint32_t k, uint32_t S, uint32_t* stages_out, uint32_t* stage_area_out,
          uint32_t* rpo_out, uint32_t* smem_out) {
  const uint32_t ks = k / BK;
  const uint32_t kc_max = (ks + S - 1) / S;
  const uint32_t sb = stage_bytes(rows);
  // with a split each CTA receives every slice's partials of its rows
  const uint32_t rpo = S > 1 ? (rows + S - 1) / S : 0;
  const uint32_t recv = S * rpo * BF * 4;
  uint32_t stages = kc_max < (uint32_t)MAX_STAGES ? kc_max : MAX_STAGES;
  while (stages > 1 && stages * sb + recv > MAX_SMEM) --stages;
  const uint32_t staged = S > 1 ? (rows * BF * 4 + 1023) / 1024 * 1024 : 0;
  const uint32_t stage_area = stages * sb > staged ? stages * sb : staged;
  const uint32_t data = stage_area + recv;
  if (data > MAX_SMEM) return false;
  *stages_out = stages;
  *stage_area_out = stage_area;
  *rpo_out = rpo;
  *smem_out = data + (2 * MAX_STAGES + 2) * 8 + 16 + 1024;
  return true;
}

}  // namespace lin

bool linear_split_fits(uint32_t rows, uint32_t k, uint32_t split) {
  uint32_t a, b, c, d;
  return lin::plan(rows, k, split, &a, &b, &c, &d);
}

// The K split: the largest power of two (at most 16 and at most K / 64)
// that keeps tiles x split within 1.5 waves of one CTA per SM, so the
// matrix is read by about every SM and each CTA's slice stays a few stages.
uint32_t linear_auto_split(uint32_t rows, uint32_t n, uint32_t k, int sms) {
  const uint32_t tiles = n / lin::BF, ks = k / lin::BK;
  uint32_t s = 1;
  while (s * 2 <= 16 && s * 2 <= ks && tiles * s * 2 * 2 <= 3u * (uint32_t)sms) s *= 2;
  while (s > 1 && !linear_split_fits(rows, k, s)) s /= 2;
  return s;
}

int linear_launch(const LinearArgs& a, cudaStream_t stream) {
  const uint32_t S = a.split;
  const uint32_t tiles = a.n / lin::BF, ks = a.k / lin::BK;
  uint32_t stages, stage_area, rpo, smem;
  if (!lin::plan(a.rows, a.k, S, &stages, &stage_area, &rpo, &smem)) return PVLC_CUDA_ERROR;
  const uint32_t sb = lin::stage_bytes(a.rows);
  const uint32_t nb = lin::padded_rows(a.rows);
  const uint32_t data = smem - (2 * lin::MAX_STAGES + 2) * 8 - 16 - 1024;
  if (set_smem_attribute_once(reinterpret_cast<const void*>(lin::linear_kernel),
                              lin::MAX_SMEM + 4096) != PVLC_OK)
    return PVLC_CUDA_ERROR;
  if (S > 8 && cudaFuncSetAttribute(lin::linear_kernel,
                                    cudaFuncAttributeNonPortableClusterSizeAllowed,
                                    1) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  lin::Maps maps;
  if (!lin::make_map(&maps.w, a.w, a.k, a.n, a.k, lin::BF) ||
      !lin::make_map(&maps.x, a.x, a.k, a.rows, a.ldx, nb))
    return PVLC_CUDA_ERROR;
  lin::Params p;
  p.rows = a.rows;
  p.nb = nb;
  p.ksteps = ks;
  p.split = S;
  p.stages = stages;
  p.stage_bytes = sb;
  p.recv_off = stage_area;
  p.rpo = rpo;
  p.data_bytes = data;
  uint32_t cols = 32;
  while (cols < nb) cols *= 2;
  p.tmem_cols = cols;
  p.silu = a.gate ? 1u : 0u;
  p.out = reinterpret_cast<__half*>(a.out);
  p.ldo = a.ldo;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * S);
  cfg.blockDim = dim3(lin::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = S > 1 ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, lin::linear_kernel, maps, p) != cudaSuccess) {
    cudaGetLastError();   // a refused launch (e.g. no room for the cluster) is not sticky
    return PVLC_CUDA_ERROR;
  }
  return PVLC_OK;
}

}  // namespace pvlc

using namespace pvlc;

extern "C" {

int pvlc_linear(const pvlc_half* x, uint32_t rows, uint32_t ldx, const pvlc_half* w, uint32_t n,
                uint32_t k, uint32_t gate, uint32_t split, pvlc_half* out, uint32_t ldo,
                void* stream) {
  if (rows == 0 || n == 0 || k == 0) return PVLC_ZERO_DIMENSION;
  if (rows > PVLC_LINEAR_MAX_ROWS || n % 128 || k % 64 || k > PVLC_LINEAR_MAX_K ||
      n > PVLC_LINEAR_MAX_N || ldx < k || ldx % 8 || ldo % 8 || ldo < (gate ? n / 2 : n) ||
      gate > 1)
    return PVLC_INVALID_DECODER_GEOMETRY;
  if (!x || !w || !out) return PVLC_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return PVLC_MISALIGNED_POINTER;
  if (split == 0) {
    const int sms = device_sm_count();
    if (sms <= 0) return PVLC_CUDA_ERROR;
    split = linear_auto_split(rows, n, k, sms);
  }
  if ((split & (split - 1)) || split > 16 || split > k / 64 || !linear_split_fits(rows, k, split))
    return PVLC_INVALID_DECODER_GEOMETRY;
  LinearArgs a{x, rows, ldx, w, n, k, gate, split, out, ldo};
  return linear_launch(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
