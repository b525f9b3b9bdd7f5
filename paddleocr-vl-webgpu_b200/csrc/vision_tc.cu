// vision_tc.cu -- vision-encoder bidirectional varlen attention on the
// Blackwell tensor cores (tcgen05 + TMEM + TMA), head_dim 72, with the 2-D
// RoPE.  sm_100a.
//
// Reference path replaced: VisionRope2dF16 followed by VisionAttentionF16
// (crates/pvlc-wgsl/src/lib.rs:2309-2454,2553-2596; call site
// crates/pvlc-runtime-web/src/web.rs:4797-4803); arithmetic
// crates/pvlc-cpu-ref/src/lib.rs:472-542 (rotation) and :2752-2878
// (segmented attention).  A CTA only visits keys of its own segment.
//
// Two launches, like the reference's two passes:
//   vision_rope_kernel   rotates Q and K once into a scratch buffer
//                        (HBM-bound elementwise pass).  Rotating inside the
//                        attention kernel would repeat the rotation of every
//                        K tile once per query tile pair of its segment.
//   vision_tc_kernel     attention over the rotated Q and K.
//
// Attention: one CTA = one (segment, 256-query pair of tiles, head) work
// item, one CTA per SM.  head_dim 72 never gets padded in HBM: TMA zero-fills
// the columns past dim 72 as out-of-bounds.
//   Q, K (MMA K dimension): a 64-dim block (128-byte rows, 128B swizzle) and
//     a 16-dim block (32-byte rows, 32B swizzle) -> 4 + 1 MMAs of K = 16.
//   V (MMA N dimension): two 64-dim blocks of 128-byte rows (the second one
//     holds dims 64..71 and zeros) -> one N = 80 MMA per K step.
//
//   warp 8       TMA producer: both Q tiles once, then K/V tiles of 128 keys
//                through a 3-stage ring
//   warp 9       MMA issuer (the whole warp walks the schedule, one elected
//                lane issues), ping-pong over the two tiles:
//                PV(t0, j), QK(t0, j+1), PV(t1, j), QK(t1, j+1), ... so the
//                tensor pipe works on one tile while the other's softmax runs
//   warps 10-11  write the row-sum column of every staged V tile
//   warps 0-3,   softmax for Q tile 0 / Q tile 1: thread i owns query row i =
//   warps 4-7    TMEM lane i; per K tile reads S from TMEM, online softmax in
//                f32 (exp2 domain, packed f32x2 math), writes P (fp16) over
//                S; the running max only moves (and O is rescaled in TMEM)
//                when a row max grows by more than 8 in log2 units, so P
//                stays <= 256 and the rescale is rare
// TMEM (512 columns): S/P of tile t at [128t, 128t+128), O of tile t at
// [256+128t, 256+128t+80).
// setmaxnreg moves registers from the control warpgroup to the two softmax
// warpgroups.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <numeric>
#include <vector>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"
#include "tcgen05.cuh"

namespace pvlc {
namespace vtc {

// Sticky fault word of this device's vision launches (see prefill_tc.cu).
__device__ uint32_t g_faults;

constexpr int HD = 72;
constexpr int PAIRS = 36;
constexpr int QUADS = PAIRS / 4;  // rotation pairs in groups of four (16 bytes of table)
constexpr int BM = 128;           // rows per Q tile
// Q tiles per CTA (one softmax warpgroup each) and keys per K/V tile: two
// tiles of 128 keys (TMEM: 2 x (128 S + 80 O) columns).  Three tiles of 80
// keys (3 x (80 S + 80 O) = 480 columns, 512 threads) also pass the parity
// tests but measured slower on configs[1] (174 vs 165 us): the per-step
// costs (S load, row max, hand-offs, MMA issue) are paid per 80 keys instead
// of per 128.
#ifndef PVLC_VISION_QT
#define PVLC_VISION_QT 2
#endif
constexpr int QT = PVLC_VISION_QT;
static_assert(QT == 2 || QT == 3, "2 or 3 Q tiles per CTA");
constexpr int BN = QT == 3 ? 80 : 128;
constexpr int THREADS = (QT + 1) * 128;  // QT softmax warpgroups + producer/MMA/row-sum
constexpr int CTRL_WARP = 4 * QT;        // first warp of the control warpgroup
// Register split (setmaxnreg) against the registers of the launch: the
// launch gives each thread 65536 / THREADS rounded down to the allocation
// unit of 8 (168 for 384 threads, 128 for 512).
constexpr uint32_t REGS_LAUNCH = QT == 3 ? 128 : 168;
constexpr uint32_t REGS_SOFTMAX = QT == 3 ? 144 : 208, REGS_CTRL = QT == 3 ? 80 : 88;
static_assert(128 * (QT * REGS_SOFTMAX + REGS_CTRL) <= THREADS * REGS_LAUNCH, "register split");
static_assert(THREADS * REGS_LAUNCH <= 65536, "launch registers");
constexpr int MAX_SEG = PVLC_VISION_MAX_SEGMENTS;

// shared memory map (offsets from a 1024-aligned base)
constexpr uint32_t SZ_QW = BM * 128;    // Q: 128 rows x 64 dims fp16, 128B swizzle
constexpr uint32_t SZ_QN = BM * 32;     // Q: 128 rows x 16 dims fp16, 32B swizzle
constexpr uint32_t Q_BYTES = SZ_QW + SZ_QN;
constexpr uint32_t OFF_Q = 0;           // tile t at OFF_Q + t * Q_BYTES: wide block, narrow block
constexpr uint32_t OFF_STAGE = QT * Q_BYTES;
// stage: K dims 0..63 (BN rows x 128 B), V dims 0..63, V dims 64..127 (both BN
// x 128 B), K dims 64..79 (BN x 32 B); every 128B-swizzled block 1 KB aligned
constexpr uint32_t ST_K0 = 0, ST_V0 = BN * 128, ST_V1 = 2 * BN * 128, ST_K1 = 3 * BN * 128;
constexpr uint32_t LOAD_BYTES = ST_K1 + BN * 32;   // bytes the four TMA boxes of a stage bring
constexpr uint32_t STAGE_BYTES = (LOAD_BYTES + 1023) / 1024 * 1024;
constexpr int STAGES = QT == 3 ? 4 : 3;
constexpr uint32_t OFF_BARS = OFF_STAGE + STAGES * STAGE_BYTES;
// q_full, kv_full[STAGES], v_ready[STAGES], kv_empty[STAGES], s_full[QT], p_ready[QT], o_done[QT]
constexpr int NBARS = 1 + 3 * STAGES + 3 * QT;
// TMEM columns: S/P of tile t at S_COL(t), O (80 columns) at O_COL(t)
constexpr uint32_t O_COLS = 80;
__host__ __device__ constexpr uint32_t S_COL(int t) { return (uint32_t)t * BN; }
__host__ __device__ constexpr uint32_t O_COL(int t) { return (uint32_t)QT * BN + (uint32_t)t * O_COLS; }
static_assert(O_COL(QT) <= 512, "TMEM columns");
static_assert(BN % 16 == 0 && BN % 8 == 0 && ST_V0 % 1024 == 0 && ST_K1 % 1024 == 0,
              "tile shapes");
constexpr uint32_t OFF_MISC = OFF_BARS + NBARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 64 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "vision shared memory exceeds the sm_100 limit");
static_assert(STAGE_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0, "swizzle atoms need 1 KB alignment");
constexpr uint32_t TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;             // log2 units
// V's dims 72..79 are padding (TMA zero fill).  Dim 72 is set to 1.0 in every
// staged V tile, so the PV MMA accumulates the softmax row sum of the exact
// fp16 P into O column 72 -- rescaled together with O -- and the softmax
// needs no per-element sum.
constexpr int SUM_COL = 72;
// Pairs c (of each 16-pair chunk of a score row) whose exponentials run on the
// FMA / integer pipes (exp2_h2_poly) instead of MUFU: the MUFU / conversion
// pipe retires a quarter warp per cycle, so moving part of the work off it
// shortens the exponential phase.
#ifndef PVLC_VISION_EXP_POLY_MASK
#define PVLC_VISION_EXP_POLY_MASK 0x4924u
#endif
constexpr uint32_t EXP_POLY_MASK = PVLC_VISION_EXP_POLY_MASK;

struct Sched {
  uint32_t n_segments;
  uint32_t seg_start[MAX_SEG];
  uint32_t seg_len[MAX_SEG];
  uint32_t item_prefix[MAX_SEG + 1];
};

struct Maps {
  CUtensorMap q0, q1, k0, k1, v0;
};

struct Params {
  __half* out;
  uint32_t heads;
};

__device__ __forceinline__ uint64_t u2_pack(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

// ------------------------------------------------------------ 2-D RoPE pass
// One thread per (token, head, quad of 4 rotation pairs): pair p rotates
// dims (p, p + 36) of the head by table entry p of the token
// (crates/pvlc-cpu-ref/src/lib.rs:472-542): x' = x cos - y sin,
// y' = y cos + x sin in f32, rounded to fp16.  q and k share the table loads.
// Consecutive threads touch consecutive 8-byte pieces of a row and
// consecutive 16-byte table quads, so every access is coalesced (measured
// faster than one thread per 144-byte row, whose 16-byte accesses stride by
// a row).
__global__ void __launch_bounds__(256)
    vision_rope_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                       const float* __restrict__ cs, const float* __restrict__ sn,
                       __half* __restrict__ q_rot, __half* __restrict__ k_rot, uint32_t heads,
                       uint32_t in_stride, uint64_t quads) {
  // the attention launch may start its prologue (barriers, TMEM) now; it
  // waits for this kernel before loading the rotated q and k
  pdl_launch_dependents();
  const uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= quads) return;
  const uint64_t row = g / QUADS;               // token * heads + head
  const uint32_t quad = (uint32_t)(g - row * QUADS);
  const uint64_t token = row / heads;
  const float4 c = __ldg(reinterpret_cast<const float4*>(cs + token * PAIRS) + quad);
  const float4 s = __ldg(reinterpret_cast<const float4*>(sn + token * PAIRS) + quad);
  // inputs at a token stride of in_stride elements; the rotated copies packed
  const size_t lo = row * HD + 4 * quad, hi = lo + PAIRS;
  const size_t ilo = token * in_stride + (row - token * heads) * HD + 4 * quad, ihi = ilo + PAIRS;
  auto rot = [&](const __half* src, __half* dst) {
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(src + ilo));
    const uint2 b = __ldg(reinterpret_cast<const uint2*>(src + ihi));
    const float2 a0 = __half22float2(*reinterpret_cast<const __half2*>(&a.x));
    const float2 a1 = __half22float2(*reinterpret_cast<const __half2*>(&a.y));
    const float2 b0 = __half22float2(*reinterpret_cast<const __half2*>(&b.x));
    const float2 b1 = __half22float2(*reinterpret_cast<const __half2*>(&b.y));
    *reinterpret_cast<uint2*>(dst + lo) =
        make_uint2(pack_half2(a0.x * c.x - b0.x * s.x, a0.y * c.y - b0.y * s.y),
                   pack_half2(a1.x * c.z - b1.x * s.z, a1.y * c.w - b1.y * s.w));
    *reinterpret_cast<uint2*>(dst + hi) =
        make_uint2(pack_half2(b0.x * c.x + a0.x * s.x, b0.y * c.y + a0.y * s.y),
                   pack_half2(b1.x * c.z + a1.x * s.z, b1.y * c.w + a1.y * s.w));
  };
  rot(q, q_rot);
  rot(k, k_rot);
}

// --------------------------------------------------------------- attention
__global__ void __launch_bounds__(THREADS, 1)
    vision_tc_kernel(const __grid_constant__ Maps maps, const Params p, const Sched sc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BARS);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                   // [STAGES]
  uint64_t* v_ready = kv_full + STAGES;           // [STAGES] K/V landed, row-sum column written
  uint64_t* kv_empty = v_ready + STAGES;          // [STAGES]
  uint64_t* s_full = kv_empty + STAGES;           // [QT]
  uint64_t* p_ready = s_full + QT;                // [QT]
  uint64_t* o_done = p_ready + QT;                // [QT]
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);
  // misc[0]: TMEM base, misc[1]: abort

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t head = blockIdx.x;
  const uint32_t item = blockIdx.y;
  uint32_t sg = 0;
  while (sg + 1 < sc.n_segments && sc.item_prefix[sg + 1] <= item) ++sg;
  const uint32_t seg0 = sc.seg_start[sg], seglen = sc.seg_len[sg];
  const uint32_t q0 = seg0 + (item - sc.item_prefix[sg]) * (QT * BM);
  const uint32_t seg_end = seg0 + seglen;
  // Q tiles of this item that hold rows of the segment
  const int ntile = static_cast<int>(umin32(QT, (seg_end - q0 + BM - 1) / BM));
  const int nk = static_cast<int>((seglen + BN - 1) / BN);

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&v_ready[s], 2);     // the two row-sum warps
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_done[t], 1);
    }
    misc[1] = 0;
    fence_mbar_init();
  }
  if (warp == CTRL_WARP) {
    tc::tmem_alloc(const_cast<uint32_t*>(misc), TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = misc[0];

  // Registers follow the work (softmax rows hold 128 scores each); each
  // warpgroup changes its budget at the head of its own branch.
  const int wg = warp >> 2;
  if (wg == CTRL_WARP / 4) {
    tc::regs_dec<REGS_CTRL>();
    if (warp == CTRL_WARP && lane == 0) {
      // ---------------------------------------------------- TMA producer
      tc::tma_prefetch_desc(&maps.q0);
      tc::tma_prefetch_desc(&maps.k0);
      tc::tma_prefetch_desc(&maps.v0);
      // q and k come from the rotation pass (the preceding launch, when rotated)
      pdl_wait();
      mbar_arrive_expect_tx(q_full, ntile * Q_BYTES);
      for (int t = 0; t < ntile; ++t) {
        tc::tma_load_3d(smem + OFF_Q + t * Q_BYTES, &maps.q0, 0, head, q0 + t * BM, q_full);
        tc::tma_load_3d(smem + OFF_Q + t * Q_BYTES + SZ_QW, &maps.q1, 64, head, q0 + t * BM, q_full);
      }
      int issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int s = j % STAGES;
        const uint32_t use = j / STAGES;
        if (misc[1] || !mbar_wait(&kv_empty[s], (use & 1) ^ 1)) { misc[1] = 1; break; }
        uint8_t* st = smem + OFF_STAGE + s * STAGE_BYTES;
        const int z = seg0 + j * BN;
        mbar_arrive_expect_tx(&kv_full[s], LOAD_BYTES);
        tc::tma_load_3d(st + ST_K0, &maps.k0, 0, head, z, &kv_full[s]);
        tc::tma_load_3d(st + ST_K1, &maps.k1, 64, head, z, &kv_full[s]);
        tc::tma_load_3d(st + ST_V0, &maps.v0, 0, head, z, &kv_full[s]);
        tc::tma_load_3d(st + ST_V1, &maps.v0, 64, head, z, &kv_full[s]);
        issued = j + 1;
      }
      // the last loads must land before the CTA may exit
      for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % STAGES], (j / STAGES) & 1);
    } else if (warp == CTRL_WARP + 1) {
      // ---------------------------------------------------- MMA issuer
      // The whole warp walks the schedule, so descriptors and loop state stay
      // warp-uniform; one elected lane issues each group of tcgen05.mma and
      // the commit that tracks it.  Descriptors are built once; each K step
      // only adds a constant to the start-address field (address >> 4 in the
      // low bits).
      constexpr uint32_t idesc_qk = tc::idesc_f16(128, BN, 0, 0);
      constexpr uint32_t idesc_pv = tc::idesc_f16(128, O_COLS, 0, 1);
      // Descriptors of tile t / stage s are the tile-0 / stage-0 descriptors
      // plus the byte offset >> 4 in the start-address field (which never
      // carries out of its 14 bits inside 227 KB of shared memory).
      const uint32_t sq = smem_u32(smem + OFF_Q);
      const uint32_t st0 = smem_u32(smem + OFF_STAGE);
      const uint64_t dq_w = tc::smem_desc(sq, 16, 1024, tc::kSw128);
      const uint64_t dq_n = tc::smem_desc(sq + SZ_QW, 16, 256, tc::kSw32);
      const uint64_t dk_w = tc::smem_desc(st0 + ST_K0, 16, 1024, tc::kSw128);
      const uint64_t dk_n = tc::smem_desc(st0 + ST_K1, 16, 256, tc::kSw32);
      // MN-major V: 64-column swizzle atoms ST_V1 - ST_V0 apart (LBO), 8-key groups 1 KB apart
      const uint64_t dv = tc::smem_desc(st0 + ST_V0, ST_V1 - ST_V0, 1024, tc::kSw128);
      auto qk = [&](int t, int s) {
        const uint32_t tS = tmem + S_COL(t);
        const uint64_t qo = (uint64_t)t * (Q_BYTES >> 4), so = (uint64_t)s * (STAGE_BYTES >> 4);
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)   // 32 bytes (16 dims) per K step -> +2 in the address field
            tc::mma_ss(tS, dq_w + qo + 2 * ks, dk_w + so + 2 * ks, idesc_qk, ks > 0);
          tc::mma_ss(tS, dq_n + qo, dk_n + so, idesc_qk, 1);
          tc::commit(&s_full[t]);
        }
        __syncwarp();
      };
      auto pv = [&](int t, int s, bool first, bool release) {
        const uint32_t tS = tmem + S_COL(t), tO = tmem + O_COL(t);
        const uint64_t so = (uint64_t)s * (STAGE_BYTES >> 4);
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)   // 16 keys = two 1 KB groups per K step -> +128
            tc::mma_ts(tO, tS + ks * 8, dv + so + 128 * ks, idesc_pv, (!first || ks > 0) ? 1u : 0u);
          tc::commit(&o_done[t]);
          if (release) tc::commit(&kv_empty[s]);   // the stage is free once every tile's PV is done
        }
        __syncwarp();
      };
      constexpr uint32_t kAll = 0xffffffffu;
      bool ok = __all_sync(kAll, mbar_wait(q_full, 0) && mbar_wait(&v_ready[0], 0));
      int done = 0;   // K tiles whose PV was issued for every Q tile
      if (ok) {
        tc::fence_after_sync();
        for (int t = 0; t < ntile; ++t) qk(t, 0);
        for (int j = 0; j < nk && ok && !__any_sync(kAll, misc[1] != 0); ++j) {
          const bool more = j + 1 < nk;
          const int s = j % STAGES, s1 = (j + 1) % STAGES;
          for (int t = 0; t < ntile; ++t) {
            if (!__all_sync(kAll, mbar_wait(&p_ready[t], j & 1))) { ok = false; break; }
            // the next QK needs the next K/V tile; checked before the PV
            // issue so that PV and QK reach the tensor pipe back to back
            if (more && t == 0 &&
                !__all_sync(kAll, mbar_wait(&v_ready[s1], ((j + 1) / STAGES) & 1))) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            pv(t, s, j == 0, t == ntile - 1);
            if (more) qk(t, s1);
          }
          if (ok) done = j + 1;
        }
      }
      if (!ok && lane == 0) misc[1] = 1;
      // never exit with MMAs in flight or commit arrivals still pending
      if (done > 0) {
        for (int t = 0; t < ntile; ++t) mbar_wait(&o_done[t], (done - 1) & 1);
        for (int j = (done > STAGES ? done - STAGES : 0); j < done; ++j)
          mbar_wait(&kv_empty[j % STAGES], (j / STAGES) & 1);
      }
    } else if (warp >= CTRL_WARP + 2) {
      // ---------------------------------------------------- row-sum column
      // V row r, dims 72..79 (chunk 1 of the second 64-dim block) = {1, 0 x 7}
      const int u = tid - 32 * (CTRL_WARP + 2);   // 0..63: rows u, u + 64, ...
      for (int j = 0; j < nk; ++j) {
        const int s = j % STAGES;
        if (misc[1] || !mbar_wait(&kv_full[s], (j / STAGES) & 1)) { misc[1] = 1; break; }
        uint8_t* v1 = smem + OFF_STAGE + s * STAGE_BYTES + ST_V1;
        for (int r = u; r < BN; r += 64)
          *reinterpret_cast<uint4*>(v1 + r * 128 + ((1 ^ (r & 7)) << 4)) =
              make_uint4(0x3C00u, 0u, 0u, 0u);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&v_ready[s]);
      }
    }
  } else {
    tc::regs_inc<REGS_SOFTMAX>();
    // ------------------------------------------------------ softmax
    const int t = wg;                              // Q tile of this warpgroup
    const int i = tid - 128 * t;                   // query row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + S_COL(t);
    const uint32_t tO = tmem + lane_base + O_COL(t);
    const uint32_t row = q0 + t * BM + i;          // token of this query row
    if (t < ntile) {
      const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
      const uint64_t scale2 = f2_pack(scale, scale);
      float m_run = -CUDART_INF_F;   // running max (the row sum lives in O[:, 72])
      bool good = true;
      for (int j = 0; j < nk && good; ++j) {
        // warp-uniform control flow around the collective tcgen05.ld / .st
        if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&s_full[t], j & 1))) {
          good = false;
          break;
        }
        tc::fence_after_sync();
        const int kv = static_cast<int>(umin32(BN, seglen - j * BN));
        uint32_t sv[BN];
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 32) {
          if (c0 + 32 <= BN) tc::tmem_ld32(tS + c0, sv + c0);
          else tc::tmem_ld16(tS + c0, sv + c0);
        }
        tc::tmem_wait_ld();
        if (kv < BN) {   // last tile of the segment: keys past its end score -inf
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= kv) sv[c] = __float_as_uint(-CUDART_INF_F);
        }
        // row max over four independent chains
        float m4[4] = {__uint_as_float(sv[0]), __uint_as_float(sv[1]), __uint_as_float(sv[2]),
                       __uint_as_float(sv[3])};
#pragma unroll
        for (int c = 4; c + 8 <= BN; c += 8) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            m4[e] = fmax3(m4[e], __uint_as_float(sv[c + 2 * e]), __uint_as_float(sv[c + 2 * e + 1]));
        }
        static_assert(BN % 8 == 0, "the max tail is the last four columns");
        m4[0] = fmax3(m4[0], __uint_as_float(sv[BN - 4]), __uint_as_float(sv[BN - 3]));
        m4[1] = fmax3(m4[1], __uint_as_float(sv[BN - 2]), __uint_as_float(sv[BN - 1]));
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale;
        // move the running max only when it grew past the threshold
        const bool need = mx > m_run + RESCALE_THRESHOLD;
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2(m_run - mx);   // 0 on the first tile
          m_run = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[t], (j - 1) & 1))) { good = false; break; }
          tc::fence_after_sync();
#pragma unroll
          for (int cc = 0; cc < 80; cc += 16) {
            uint32_t ov[16];
            tc::tmem_ld16(tO + cc, ov);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tc::tmem_st16(tO + cc, ov);
          }
        }
        // P = 2^(x - m) as fp16 pairs, split between two pipes: the pairs of
        // EXP_POLY_MASK by the polynomial on the FMA / integer pipes, the
        // others by scaling in f32, rounding the exponent to fp16 and one
        // MUFU operation per two values
        const uint64_t negm2 = f2_pack(-m_run, -m_run);
        const uint64_t negmh2 = f2_pack(6.5f - m_run, 6.5f - m_run);   // exp2_h2_poly takes x + 6.5
        // chunks of up to 16 pairs (32 keys); P of keys 2c, 2c+1 lands in column c
#pragma unroll
        for (int ch = 0; ch < (BN + 31) / 32; ++ch) {
          constexpr int kPairs = BN / 2;
          const int np = kPairs - 16 * ch < 16 ? kPairs - 16 * ch : 16;
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c >= np) break;
            const int k = 32 * ch + 2 * c;
            if ((EXP_POLY_MASK >> c) & 1u) {
              pk[c] = exp2_h2_poly(f2_fma(u2_pack(sv[k], sv[k + 1]), scale2, negmh2));
            } else {
              const float2 x = f2_unpack(f2_fma(u2_pack(sv[k], sv[k + 1]), scale2, negm2));
              pk[c] = ex2_h2(pack_half2(x.x, x.y));
            }
          }
          if (np == 16) tc::tmem_st16(tS + 16 * ch, pk);
          else tc::tmem_st8(tS + 16 * ch, pk);
        }
        static_assert(BN % 32 == 0 || BN % 32 == 16, "a P chunk is 16 or 8 columns");
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[t]);
      }
      if (!good) misc[1] = 1;
      // epilogue: O / l -> fp16 rows
      if (__all_sync(0xffffffffu, good && mbar_wait(&o_done[t], (nk - 1) & 1))) {
        tc::fence_after_sync();
        const bool store = row < seg_end;
        __half* orow = p.out + ((size_t)row * p.heads + head) * HD;
        // the whole O row (80 columns; column 72 holds the row sum) in one round trip
        uint32_t ov[80];
        tc::tmem_ld32(tO, ov);
        tc::tmem_ld32(tO + 32, ov + 32);
        tc::tmem_ld16(tO + 64, ov + 64);
        tc::tmem_wait_ld();
        const float inv = 1.f / __uint_as_float(ov[SUM_COL]);
#pragma unroll
        for (int c8 = 0; c8 < HD; c8 += 8) {   // columns 72..79: row sum and padding
          uint4 v;
          v.x = pack_half2(__uint_as_float(ov[c8 + 0]) * inv, __uint_as_float(ov[c8 + 1]) * inv);
          v.y = pack_half2(__uint_as_float(ov[c8 + 2]) * inv, __uint_as_float(ov[c8 + 3]) * inv);
          v.z = pack_half2(__uint_as_float(ov[c8 + 4]) * inv, __uint_as_float(ov[c8 + 5]) * inv);
          v.w = pack_half2(__uint_as_float(ov[c8 + 6]) * inv, __uint_as_float(ov[c8 + 7]) * inv);
          if (store) *reinterpret_cast<uint4*>(orow + c8) = v;
        }
      } else {
        misc[1] = 1;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && misc[1]) atomicOr(&g_faults, PVLC_FAULT_VISION);
  if (warp == CTRL_WARP) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// [tokens, heads, 72] fp16 rows `stride` elements apart, viewed as a 3-D tensor
// {72, heads, tokens}; box {inner, 1, rows} rows of one head.
bool make_map(CUtensorMap* m, const void* base, uint32_t tokens, uint32_t heads, uint32_t stride,
              uint32_t inner, uint32_t rows, CUtensorMapSwizzle sw) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {HD, heads, tokens};
  const cuuint64_t strides[2] = {HD * 2, (cuuint64_t)stride * 2};
  const cuuint32_t box[3] = {inner, 1, rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace vtc

int vision_fault_word(uint32_t* out, cudaStream_t s) {
  uint32_t v = 0;
  const uint32_t zero = 0;
  if (cudaMemcpyFromSymbolAsync(&v, vtc::g_faults, 4, 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaMemcpyToSymbolAsync(vtc::g_faults, &zero, 4, 0, cudaMemcpyHostToDevice, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  *out = v;
  return PVLC_OK;
}

int vision_query_tile() { return vtc::QT * vtc::BM; }
int vision_block_threads() { return vtc::THREADS; }

size_t vision_workspace_bytes(uint32_t tokens, uint32_t heads) {
  return 2ull * tokens * heads * vtc::HD * sizeof(__half);
}

int vision_launch(const VisionArgs& a, const uint32_t* cu, uint32_t segments, void* workspace,
                  cudaStream_t stream) {
  if (set_smem_attribute_once(reinterpret_cast<const void*>(vtc::vision_tc_kernel), vtc::SMEM_BYTES) != PVLC_OK)
    return PVLC_CUDA_ERROR;
  // rotated q and k (the scratch) or the inputs themselves when there is no RoPE
  const void* qa = a.q;
  const void* ka = a.k;
  uint32_t qk_stride = a.qkv_stride;   // the rotated copies are packed
  if (a.rope_cos != nullptr) {
    __half* q_rot = static_cast<__half*>(workspace);
    __half* k_rot = q_rot + (size_t)a.tokens * a.heads * vtc::HD;
    const uint64_t quads = (uint64_t)a.tokens * a.heads * vtc::QUADS;
    const uint64_t blocks = (quads + 255) / 256;
    if (blocks > 0x7fffffffull) return PVLC_ARITHMETIC_OVERFLOW;
    vtc::vision_rope_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
        reinterpret_cast<const __half*>(a.q), reinterpret_cast<const __half*>(a.k), a.rope_cos,
        a.rope_sin, q_rot, k_rot, a.heads, a.qkv_stride, quads);
    if (cudaPeekAtLastError() != cudaSuccess) return PVLC_CUDA_ERROR;
    qa = q_rot;
    ka = k_rot;
    qk_stride = a.heads * vtc::HD;
  }
  vtc::Maps maps;
  using vtc::BM;
  using vtc::BN;
  const bool ok =
      vtc::make_map(&maps.q0, qa, a.tokens, a.heads, qk_stride, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B) &&
      vtc::make_map(&maps.q1, qa, a.tokens, a.heads, qk_stride, 16, BM, CU_TENSOR_MAP_SWIZZLE_32B) &&
      vtc::make_map(&maps.k0, ka, a.tokens, a.heads, qk_stride, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B) &&
      vtc::make_map(&maps.k1, ka, a.tokens, a.heads, qk_stride, 16, BN, CU_TENSOR_MAP_SWIZZLE_32B) &&
      vtc::make_map(&maps.v0, a.v, a.tokens, a.heads, a.qkv_stride, 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok) return PVLC_CUDA_ERROR;
  vtc::Sched sc;
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
    items += (sc.seg_len[i] + vtc::QT * vtc::BM - 1) / (vtc::QT * vtc::BM);
  }
  sc.item_prefix[segments] = items;
  if (items > 65535u) return PVLC_INVALID_VISION_GEOMETRY;
  vtc::Params p;
  p.out = reinterpret_cast<__half*>(a.out);
  p.heads = a.heads;
  // programmatic dependent launch: the attention CTAs' prologue overlaps the
  // tail of the rotation pass; their q/k loads wait for it (pdl_wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads, items);
  cfg.blockDim = dim3(vtc::THREADS);
  cfg.dynamicSmemBytes = vtc::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.rope_cos != nullptr ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, vtc::vision_tc_kernel, maps, p, sc) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // namespace pvlc
