// decode_splitkv.cu -- batched single-token GQA decode (pinned Q16/KV2/D128)
// against per-sequence fp16 KV caches, for B200 (sm_100a).
//
// Reference path replaced (one launch per layer step for the whole batch):
//   DecoderMropeF32 -> DecoderKvAppendF32 -> DecoderGqaSplitPartialF32 ->
//   DecoderGqaSplitMergeF32
//   (crates/pvlc-runtime-native/src/decoder_kv_session.rs:548-768;
//    arithmetic crates/pvlc-cpu-ref/src/lib.rs:858-927,1420-1450).
//
// Design (HBM-bound: ~8 FLOP per byte of KV):
//   * Stream-K split: the batch's KV rows, cut into 32-row tiles, are laid
//     end to end and split over one CTA per SM in proportion to work: each
//     tile counts one unit and each sequence end (its merge, partial record
//     and combine) END_WEIGHT units, so every SM does about the same work
//     whatever the per-sequence lengths are.  A CTA's range may cover the
//     tail of one sequence and the head of the next.
//   * A copy warp streams 512-byte cache rows (both KV heads) into a 5-stage
//     shared-memory ring with 16-byte cp.async copies (one coalesced row per
//     warp instruction) whose completion arrives on per-stage mbarriers; rows
//     land at a 528-byte pitch so ldmatrix is conflict free.  (Per-row 1-D
//     bulk copies were issue-bound at ~2 TB/s: 64 small TMA operations per
//     32 KB tile.)
//   * Eight consumer warps (2 tile-parity groups x 2 KV heads x 2 row halves)
//     run the 8 query heads of a KV group as the N=8 side of mma.m16n8k16:
//     S^T = K Q^T (keys on M), online softmax over keys in f32 (exp2 domain),
//     P^T transposed in registers with movmatrix, O^T += V^T P^T.
//   * A sequence warp does the per-sequence work ahead of the stream: for
//     each sequence of the CTA's range it writes the decode-M-RoPE-rotated q
//     into a double-buffered shared-memory slot and performs the KV append
//     (the rotated new key and the new value into cache row
//     cache_tokens[b]) before the copy warp reaches that row.  A sequence
//     change costs the consumers one shared-memory read of their Q fragments
//     and the copy warp nothing.
//   * The ring is never zeroed: rows past a sequence end are masked to
//     P = 0 and the consumer zeroes their V bytes before the PV product.
//   * Per-sequence partials (unnormalised O, running max, running sum): each
//     consumer warp hands its (O, m, l) to a merge warp through shared memory
//     and moves on to the next sequence, so a sequence end inside the range
//     does not stall the stream; the merge warp combines the 8 warps and
//     writes the output or, for a sequence split over several CTAs, this
//     CTA's partial record.  The range's last sequence, with nothing left to
//     overlap, is merged by all 256 consumer threads.  The last CTA to finish
//     a split sequence (atomic ticket, no spinning) combines every CTA's
//     record in CTA (= token) order and resets the ticket for the next launch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <mutex>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"

namespace pvlc {
namespace decode {

constexpr int HD = 128;
constexpr int KVH = 2;
constexpr int QH = 16;
constexpr int GROUP = 8;
constexpr int TILE = 32;          // cache rows per pipeline stage
constexpr int STAGES = 5;
constexpr int ROW_BYTES = KVH * HD * 2;   // 512
constexpr int ROW_PITCH = ROW_BYTES + 16; // 528: conflict-free ldmatrix rows
constexpr int STAGE_BYTES = TILE * ROW_PITCH;
constexpr int CONSUMER_WARPS = 8;
constexpr int PRODUCER_WARPS = 2;             // copy warp, sequence warp
constexpr int THREADS = (CONSUMER_WARPS + PRODUCER_WARPS + 1) * 32;   // + the merge warp
constexpr int CONSUMER_THREADS = CONSUMER_WARPS * 32;
constexpr int MAX_BATCH = 2048;
constexpr int PART_FLOATS = QH * HD + 2 * QH;   // O[16][128], m[16], l[16]
// Work allowance of a sequence end in the stream-K split, in tiles: the CTA
// that holds a sequence's last tile also merges its consumer warps, writes a
// partial record, takes the combine ticket and may combine every CTA's
// record.  Swept on B200 at 64 sequences x 18 layers (0..16): 4 is best
// (+4 % over an even tile split; larger values overshoot).
#ifndef PVLC_DECODE_END_WEIGHT
#define PVLC_DECODE_END_WEIGHT 4
#endif
constexpr uint32_t END_WEIGHT = PVLC_DECODE_END_WEIGHT;
#ifndef PVLC_DECODE_MIN_TILES_PER_CTA
#define PVLC_DECODE_MIN_TILES_PER_CTA 4
#endif
constexpr uint64_t MIN_TILES_PER_CTA = PVLC_DECODE_MIN_TILES_PER_CTA;
// Tiles of a CTA's range prefetched into L2 before the programmatic-launch wait.
// Swept on B200 at 64 sequences x 18 layers (0, 2, 3, 5, 10, 16 tiles): 0 is
// best (0.729 of the copy peak; 5 tiles 0.721, 16 tiles 0.686) -- the early
// CTAs' prefetches compete with the previous launch's last streaming CTAs.
#ifndef PVLC_DECODE_PREFETCH_TILES
#define PVLC_DECODE_PREFETCH_TILES 0
#endif
constexpr uint64_t PREFETCH_TILES = PVLC_DECODE_PREFETCH_TILES;
// A sequence piece of at most this many tiles has its append written before
// the next sequence's q (the consumers reach its last tile soon); longer
// pieces get the next q first.  Swept on B200 (2, 4, 6, 8, 12): 6 keeps the
// 64-sequence gain and 32 sequences of ~1250 rows at their earlier time (2:
// +8 % there).
#ifndef PVLC_DECODE_APPEND_FIRST_TILES
#define PVLC_DECODE_APPEND_FIRST_TILES 6
#endif
constexpr uint64_t APPEND_FIRST_TILES = PVLC_DECODE_APPEND_FIRST_TILES;

// shared memory map (bytes)
constexpr int SM_K = 0;
constexpr int SM_V = SM_K + STAGES * STAGE_BYTES;
// per-sequence (O, m, l) of the consumer warps, handed to the merge warp
constexpr int SM_MERGE_ACC = SM_V + STAGES * STAGE_BYTES;          // [8 warps][8 heads][128]
constexpr int SM_MERGE_M = SM_MERGE_ACC + CONSUMER_WARPS * GROUP * HD * 4;
constexpr int SM_MERGE_L = SM_MERGE_M + CONSUMER_WARPS * GROUP * 4;
constexpr int SM_TILE_OFF = SM_MERGE_L + CONSUMER_WARPS * GROUP * 4;  // [MAX_BATCH+1]
constexpr int SM_COST_OFF = SM_TILE_OFF + ((MAX_BATCH + 1) * 4 + 15) / 16 * 16;  // [MAX_BATCH+1]
// rotated q of the current / next sequence: [2 slots][16 heads][Q_PITCH halves]
constexpr int Q_PITCH = HD + 8;          // 272-byte rows: conflict-free fragment reads
constexpr int SM_Q = SM_COST_OFF + ((MAX_BATCH + 1) * 4 + 15) / 16 * 16;
constexpr int SM_BARS = SM_Q + 2 * QH * Q_PITCH * 2;
// full[STAGES], empty[STAGES], q_full[2], q_empty[2], merge_full, merge_empty,
// app_stage[APP_SLOTS]
// Append handshakes in flight: every claimed append stage waits for the
// sequence warp before it can be consumed, so at most STAGES are open at once.
constexpr int APP_SLOTS = 8;
static_assert(APP_SLOTS > STAGES, "append handshake slots must outnumber the ring stages");
constexpr int SM_MISC = SM_BARS + (2 * STAGES + 6 + APP_SLOTS) * 8;
constexpr int SMEM_BYTES = SM_MISC + 64;

static_assert(SMEM_BYTES <= 227 * 1024, "decode shared memory exceeds the sm_100 limit");

struct Params {
  const __half* q;
  const __half* k_new;
  const __half* v_new;
  const float* rope_cos;
  const float* rope_sin;
  const uint32_t* rope_row;
  __half* const* k_cache;
  __half* const* v_cache;
  const uint32_t* cache_tokens;
  uint32_t q_stride;     // elements between sequences' q rows (16 x 128 when packed)
  uint32_t kv_stride;    // elements between sequences' k_new / v_new rows (2 x 128)
  uint32_t rope_rows;
  uint32_t capacity;
  uint32_t max_cache_tokens;
  uint32_t batch;
  uint32_t* flags;
  uint32_t* tickets;
  float* partials;
  __half* out;
};

// Number of 32-row tiles of sequence b after the append, 0 when the sequence
// is invalid (and then flagged by block 0).
__device__ __forceinline__ uint32_t seq_tiles(const Params& p, uint32_t b, bool report) {
  const uint32_t ct = __ldg(p.cache_tokens + b);
  uint32_t bad = 0;
  if (ct > p.max_cache_tokens || ct >= p.capacity) bad |= kFlagCacheRow;
  const uint32_t rr = p.rope_row ? __ldg(p.rope_row + b) : ct;
  if (rr >= p.rope_rows) bad |= kFlagRopeRow;
  const uintptr_t kp = reinterpret_cast<uintptr_t>(p.k_cache[b]);
  const uintptr_t vp = reinterpret_cast<uintptr_t>(p.v_cache[b]);
  if ((kp | vp) & 15u) bad |= kFlagMisaligned;
  if (bad) {
    if (report) atomicOr(p.flags, bad);
    return 0;
  }
  return (ct + 1 + TILE - 1) / TILE;
}

// max{i : floor(i*C/G) <= y}: the CTA whose cost range holds cost position y
// (the position of a tile: the CTA that streams that tile).
__device__ __forceinline__ uint32_t owner_cta(uint64_t y, uint64_t G, uint64_t C) {
  return static_cast<uint32_t>(((y + 1) * G + C - 1) / C - 1);
}

// M-RoPE of 8 consecutive dims d0..d0+7 of a 128-wide head (d0 a multiple of
// 8, so they share one table plane: the section edges 16 and 40 are multiples
// of 8).  x holds the dims, y their partners (d + 64 below 64, d - 64 above):
// d < 64 becomes x cos - y sin, d >= 64 becomes x cos + y sin
// (crates/pvlc-cpu-ref/src/lib.rs:645-668).
__device__ __forceinline__ uint4 mrope8(uint4 x, uint4 y, uint32_t d0, const Params& p,
                                        uint32_t rrow) {
  const size_t tb = ((size_t)mrope_axis(d0) * p.rope_rows + rrow) * HD + d0;
  const float4* cp = reinterpret_cast<const float4*>(p.rope_cos + tb);
  const float4* sp = reinterpret_cast<const float4*>(p.rope_sin + tb);
  const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
  const bool lower = d0 < 64;
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&xw[e]));
    float2 bp = __half22float2(*reinterpret_cast<const __half2*>(&yw[e]));
    if (lower) bp = make_float2(-bp.x, -bp.y);
    o[e] = pack_half2(a.x * cs[2 * e] + bp.x * sn[2 * e], a.y * cs[2 * e + 1] + bp.y * sn[2 * e + 1]);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Final combine of a sequence split over CTAs first..last (CTA = token order):
// out = sum_i 2^(m_i - M) O_i / sum_i 2^(m_i - M) l_i over the partial records
// of query head hq, dims d0 .. d0 + 8 NCH - 1.  With eight records or fewer
// and eight dims a thread (the consumers' combine, on the launch's critical
// path) every m, l and O is loaded in one round of independent loads.
// Otherwise the records are read in groups of eight with independent loads:
// two dependent L2 rounds per group (the maxima, then m, l and O together)
// instead of a round per record and pass.  Either way the sums run record by
// record in CTA order.
template <int NCH>
__device__ __forceinline__ void combine_split(const Params& p, uint32_t b, uint32_t first,
                                              uint32_t last, int hq, int d0) {
  const float* base = p.partials + (size_t)b * PART_FLOATS;
  if (NCH == 1 && last - first < 8) {
    // up to eight records (the common case): m, l and O of every record in
    // one round of independent loads, then the same sums in CTA order
    float mv[8], lv[8];
    float4 u[8], w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (first + e <= last) {
        const float* r = base + (size_t)(first + e) * PART_FLOATS;
        mv[e] = __ldcg(r + QH * HD + hq);
        lv[e] = __ldcg(r + QH * HD + QH + hq);
        u[e] = __ldcg(reinterpret_cast<const float4*>(r + hq * HD + d0));
        w[e] = __ldcg(reinterpret_cast<const float4*>(r + hq * HD + d0 + 4));
      }
    }
    float Mc = -CUDART_INF_F;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (first + e <= last) Mc = fmaxf(Mc, mv[e]);
    float Lc = 0.f, A[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (first + e <= last) {
        const float f = mv[e] == -CUDART_INF_F ? 0.f : fast_exp2(mv[e] - Mc);
        Lc += lv[e] * f;
        A[0] += u[e].x * f; A[1] += u[e].y * f; A[2] += u[e].z * f; A[3] += u[e].w * f;
        A[4] += w[e].x * f; A[5] += w[e].y * f; A[6] += w[e].z * f; A[7] += w[e].w * f;
      }
    }
    const float inv = 1.f / Lc;
    __align__(16) __half o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(A[e] * inv);
    *reinterpret_cast<uint4*>(p.out + ((size_t)b * QH + hq) * HD + d0) =
        *reinterpret_cast<uint4*>(o);
    return;
  }
  float Mc = -CUDART_INF_F;
  for (uint32_t i0 = first; i0 <= last; i0 += 8) {
    float mv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      mv[e] = i0 + e <= last ? __ldcg(base + (size_t)(i0 + e) * PART_FLOATS + QH * HD + hq)
                             : -CUDART_INF_F;
#pragma unroll
    for (int e = 0; e < 8; ++e) Mc = fmaxf(Mc, mv[e]);
  }
  float Lc = 0.f;
  float A[NCH][8];
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int e = 0; e < 8; ++e) A[ch][e] = 0.f;
  for (uint32_t i0 = first; i0 <= last; i0 += 8) {
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      f[e] = 0.f;
      if (i0 + e <= last) {
        const float* r = base + (size_t)(i0 + e) * PART_FLOATS;
        const float mi = __ldcg(r + QH * HD + hq);
        f[e] = mi == -CUDART_INF_F ? 0.f : fast_exp2(mi - Mc);
        Lc += __ldcg(r + QH * HD + QH + hq) * f[e];
      }
    }
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (i0 + e <= last) {
          const float* r = base + (size_t)(i0 + e) * PART_FLOATS + hq * HD + d0 + 8 * ch;
          const float4 u = __ldcg(reinterpret_cast<const float4*>(r));
          const float4 w = __ldcg(reinterpret_cast<const float4*>(r + 4));
          A[ch][0] += u.x * f[e]; A[ch][1] += u.y * f[e]; A[ch][2] += u.z * f[e]; A[ch][3] += u.w * f[e];
          A[ch][4] += w.x * f[e]; A[ch][5] += w.y * f[e]; A[ch][6] += w.z * f[e]; A[ch][7] += w.w * f[e];
        }
      }
    }
  }
  const float inv = 1.f / Lc;
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    __align__(16) __half o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(A[ch][e] * inv);
    *reinterpret_cast<uint4*>(p.out + ((size_t)b * QH + hq) * HD + d0 + 8 * ch) =
        *reinterpret_cast<uint4*>(o);
  }
}

__global__ void __launch_bounds__(THREADS, 1) decode_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t* tile_off = reinterpret_cast<uint32_t*>(smem + SM_TILE_OFF);
  uint32_t* cost_off = reinterpret_cast<uint32_t*>(smem + SM_COST_OFF);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + SM_BARS);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* q_full = empty_bar + STAGES;   // [2] the rotated q of a sequence is in its slot
  uint64_t* q_empty = q_full + 2;          // [2] every consumer warp has read the slot
  uint64_t* merge_full = q_empty + 2;      // every consumer warp wrote its (O, m, l)
  uint64_t* merge_empty = merge_full + 1;  // the merge warp has read the merge buffer
  uint64_t* app_stage = merge_empty + 1;   // [APP_SLOTS] a sequence's append tile has its ring stage
  __half* qs = reinterpret_cast<__half*>(smem + SM_Q);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + SM_MISC);
  // misc[0]: abort flag, misc[1]: "this CTA combines" flag, misc[2..3]: the
  // combine's CTA range, misc[4]: the sequence warp's opening loads are issued,
  // misc[8..15]: the ring stage of the append tile of sequence n, at 8 + n % APP_SLOTS

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t B = p.batch;
  // Programmatic dependent launch: this grid may start while the kernel ahead
  // of it on the stream still runs (its CTAs take an SM as soon as one of that
  // grid's CTAs leaves it), and lets the next launch do the same.  Until
  // pdl_wait it reads only cache_tokens, rope_row and the two cache-pointer
  // arrays -- which the kernel ahead does not produce (a documented
  // condition of the call) -- to build the schedule, and it prefetches into
  // L2 the first cache tiles of its range and its first sequence's q, table
  // and new rows: prefetches only warm the cache, so they are harmless even
  // if that data is still being written.  Everything else waits.
  pdl_launch_dependents();

  // ---- schedule: per-sequence tile counts (every thread), then an in-place
  // exclusive prefix sum over them (warp 0)
  for (uint32_t bb = tid; bb < B; bb += THREADS) tile_off[bb + 1] = seq_tiles(p, bb, false);
  if (tid == 0) {
    tile_off[0] = 0;
    cost_off[0] = 0;
    misc[0] = 0;
    misc[1] = 0;
    misc[4] = 0;
    for (int s = 0; s < STAGES; ++s) {
      // the copy warp's lanes twice: once when their copies land, once more
      // from the lanes that fill the tile's last row -- the copy warp's own,
      // or, for the tile holding a sequence's appended row, the sequence
      // warp's, which write that row straight into the stage
      mbar_init(&full_bar[s], 64);
      mbar_init(&empty_bar[s], 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 32);     // the sequence warp's lanes
      mbar_init(&q_empty[s], CONSUMER_WARPS);
    }
    for (int s = 0; s < APP_SLOTS; ++s) mbar_init(&app_stage[s], 1);   // the copy warp's lane 0
    mbar_init(merge_full, CONSUMER_WARPS);
    mbar_init(merge_empty, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    // prefix sums of the tile counts and of the split costs (tiles + the
    // allowance of the sequence's end), one pass
    const uint32_t per = (B + 31) / 32;
    const uint32_t b0 = min(B, lane * per), b1 = min(B, b0 + per);
    uint32_t s = 0, sc = 0;
    for (uint32_t bb = b0; bb < b1; ++bb) {
      const uint32_t n = tile_off[bb + 1];
      s += n;
      sc += n ? n + END_WEIGHT : 0u;
    }
    uint32_t incl = s, inclc = sc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      const uint32_t yc = __shfl_up_sync(0xffffffffu, inclc, o);
      if (lane >= o) {
        incl += y;
        inclc += yc;
      }
    }
    uint32_t run = incl - s, runc = inclc - sc;
    for (uint32_t bb = b0; bb < b1; ++bb) {
      const uint32_t n = tile_off[bb + 1];
      run += n;
      runc += n ? n + END_WEIGHT : 0u;
      tile_off[bb + 1] = run;
      cost_off[bb + 1] = runc;
    }
  }
  __syncthreads();

  const uint64_t NT = tile_off[B];
  // Stream-K split of the cost line: sequence b covers [cost_off[b],
  // cost_off[b+1]) = its tiles, then END_WEIGHT units for its end-merge.  CTA
  // c takes the tiles whose cost positions fall in [c C / G, (c+1) C / G):
  // contiguous, monotone tile ranges that give the CTAs holding sequence ends
  // fewer tiles.  A range inside one allowance is empty.
  const uint64_t C = cost_off[B];
  // a small batch (few tiles) uses fewer CTAs, each streaming at least
  // MIN_TILES_PER_CTA tiles: a one-tile CTA is all latency, and every split
  // adds a partial record to the sequence's combine
  const uint64_t G = umax64(1, umin64(gridDim.x, (NT + MIN_TILES_PER_CTA - 1) / MIN_TILES_PER_CTA));
  auto tile_at = [&](uint64_t y) -> uint64_t {   // first tile at cost position >= y
    if (y >= C) return NT;
    uint32_t lo = 0, hi = B;  // invariant: cost_off[lo] <= y < cost_off[hi]
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (cost_off[mid] <= y) lo = mid; else hi = mid;
    }
    const uint64_t u = y - cost_off[lo];
    const uint64_t n = tile_off[lo + 1] - tile_off[lo];
    return u < n ? tile_off[lo] + u : tile_off[lo + 1];
  };
  // first sequence touching t: last b with tile_off[b] <= t < tile_off[b+1]
  auto seq_of = [&](uint64_t t) -> uint32_t {
    uint32_t lo = 0, hi = B;  // invariant: tile_off[lo] <= t < tile_off[hi]
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (tile_off[mid] <= t) lo = mid; else hi = mid;
    }
    return lo;
  };
  const bool active = NT > 0 && blockIdx.x < G;
  const uint64_t t0 = active ? tile_at(blockIdx.x * C / G) : 0;
  const uint64_t t1 = active ? tile_at((blockIdx.x + 1) * C / G) : 0;
  if (t0 < t1 && warp == CONSUMER_WARPS + 1) {
    // sequence warp: the first sequence's q row (32 lines), table rows (3
    // planes x cos/sin x 4 lines) and new K/V rows (2 x 4 lines) toward L2;
    // they are on the consumers' critical path at the start
    const uint32_t b = seq_of(t0);
    const uint32_t ct0 = __ldg(p.cache_tokens + b);
    const uint32_t rr0 = p.rope_row ? __ldg(p.rope_row + b) : ct0;
    prefetch_l2(reinterpret_cast<const uint8_t*>(p.q + (size_t)b * p.q_stride) + lane * 128);
    if (lane < 24 && rr0 < p.rope_rows) {
      const float* tab = (lane & 4) ? p.rope_sin : p.rope_cos;
      prefetch_l2(reinterpret_cast<const uint8_t*>(tab + ((size_t)(lane >> 3) * p.rope_rows + rr0) * HD) +
                  (lane & 3) * 128);
    } else if (lane >= 24) {
      const __half* nr = (lane & 4) ? p.v_new : p.k_new;
      prefetch_l2(reinterpret_cast<const uint8_t*>(nr + (size_t)b * p.kv_stride) + (lane & 3) * 128);
    }
  } else if (t0 < t1 && warp == CONSUMER_WARPS && lane == 0) {
    // copy warp: the range's first PREFETCH_TILES tiles (K and V rows) toward L2 with
    // one bulk prefetch per tile and plane
    uint32_t b = seq_of(t0);
    for (uint64_t gt = t0; gt < t1 && gt < t0 + PREFETCH_TILES; ++gt) {
      while (gt >= tile_off[b + 1]) ++b;
      const uint32_t L = __ldg(p.cache_tokens + b) + 1;
      const uint32_t row0 = static_cast<uint32_t>(gt - tile_off[b]) * TILE;
      const uint32_t n = umin32(TILE, L - row0);
      const size_t off = (size_t)row0 * ROW_BYTES;
      prefetch_l2_bulk(reinterpret_cast<const uint8_t*>(p.k_cache[b]) + off, n * ROW_BYTES);
      prefetch_l2_bulk(reinterpret_cast<const uint8_t*>(p.v_cache[b]) + off, n * ROW_BYTES);
    }
  }
  pdl_wait();

  // Block 0 flags the sequences that were rejected and zero-fills their outputs.
  if (blockIdx.x == 0) {
    for (uint32_t b = warp; b < B; b += THREADS / 32) {
      if (tile_off[b] == tile_off[b + 1]) {
        if (lane == 0) seq_tiles(p, b, true);
        uint2* o = reinterpret_cast<uint2*>(p.out + (size_t)b * QH * HD);
        for (int i = lane; i < QH * HD / 4; i += 32) o[i] = make_uint2(0, 0);
      }
    }
  }
  if (t0 >= t1) return;

  if (warp >= CONSUMER_WARPS) {
    // ======================= producer warps =======================
    // Warp 8, the copy warp, streams the tiles: each warp instruction moves
    // one whole 512-byte cache row (16 bytes per lane, fully coalesced) into
    // the padded staging row, and every lane arrives on the stage's full
    // barrier once its own copies have landed.  It never stalls on anything
    // but free ring stages, so the ring stays full across sequence changes.
    // Warp 9, the sequence warp, does the per-sequence work ahead of the
    // stream: for each sequence of the CTA's range, in order, it writes the
    // decode-M-RoPE-rotated q into a double-buffered shared-memory slot and
    // announces the slot to the consumers (q_full); then, when the range
    // holds the sequence's appended row (the last row of its last tile), it
    // writes the rotated new key and the new value straight into that tile's
    // ring stage -- which the copy warp claims, fills with the tile's other
    // rows and names (app_stage) without waiting -- completes the stage's
    // full barrier, and stores the row in cache row cache_tokens[b] (the KV
    // append) for the steps to come.  So neither the stream nor the consumers
    // wait for the append to reach memory and come back, and the copy warp
    // never waits for the sequence warp: it may run ahead of it by as many
    // sequences as the ring has stages.
    bool aborted = false;
    uint32_t b = seq_of(t0);
    if (warp == CONSUMER_WARPS) {
      // Give the sequence warp's few opening loads (the first sequence's q,
      // tables and new row) a head start on this launch's DRAM burst: they
      // are on the consumers' critical path, the stream is not yet (bounded
      // wait).
      {
        const uint64_t w0 = globaltimer();
        while (misc[4] == 0 && globaltimer() - w0 < 20000ull) {
        }
      }
      uint32_t nseq = 0;
      uint8_t* kc = reinterpret_cast<uint8_t*>(p.k_cache[b]);
      uint8_t* vc = reinterpret_cast<uint8_t*>(p.v_cache[b]);
      uint32_t L = __ldg(p.cache_tokens + b) + 1;
      for (uint64_t it = 0; it < t1 - t0; ++it) {
        const uint64_t gt = t0 + it;
        if (gt >= tile_off[b + 1]) {
          ++nseq;
          while (gt >= tile_off[b + 1]) ++b;
          kc = reinterpret_cast<uint8_t*>(p.k_cache[b]);
          vc = reinterpret_cast<uint8_t*>(p.v_cache[b]);
          L = __ldg(p.cache_tokens + b) + 1;
        }
        const uint32_t row0 = static_cast<uint32_t>(gt - tile_off[b]) * TILE;
        const uint32_t n = umin32(TILE, L - row0);
        const int stage = static_cast<int>(it % STAGES);
        const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
        if (misc[0] || !mbar_wait(&empty_bar[stage], ph ^ 1u)) {
          aborted = true;
          break;
        }
        // the tile that holds the appended row L - 1: the sequence warp
        // writes that row into this stage
        const bool append = row0 + n == L;
        if (append) {
          __syncwarp();
          if (lane == 0) {
            misc[8 + nseq % APP_SLOTS] = static_cast<uint32_t>(stage);
            mbar_arrive(&app_stage[nseq % APP_SLOTS]);
          }
        }
        const uint32_t ks = smem_u32(smem + SM_K + stage * STAGE_BYTES) + lane * 16;
        const uint32_t vs = smem_u32(smem + SM_V + stage * STAGE_BYTES) + lane * 16;
        const uint32_t nc = append ? n - 1 : n;
        for (uint32_t r = 0; r < nc; ++r) {
          const size_t src = (size_t)(row0 + r) * ROW_BYTES + lane * 16;
          cp_async_16(ks + r * ROW_PITCH, kc + src);
          cp_async_16(vs + r * ROW_PITCH, vc + src);
        }
        cp_async_arrive_noinc(&full_bar[stage]);
        if (!append) mbar_arrive(&full_bar[stage]);
      }
    } else if (warp == CONSUMER_WARPS + 1) {
      // sequence warp: lane l rotates query head l/2, dims 32(l%2)..+31 and
      // their partners 64 above
      // the opening prefetches (before the wait) are issued: release the copy warp
      __syncwarp();
      if (lane == 0) {
        asm volatile("" ::: "memory");
        misc[4] = 1;
      }
      // Sequence n of the range takes q slot n % 2; its rotated q is written
      // one sequence ahead of its append, so the consumers find the next
      // sequence's q ready when they reach it (the append of sequence n
      // waits for the copy warp to reach that sequence's last tile).  When
      // the range holds at most two tiles of sequence n, its append comes
      // first: the consumers reach that tile almost at once.
      auto next_seq = [&](uint32_t bb) -> uint32_t {   // the range's sequence after bb, or B
        const uint64_t s1 = umin64(t1, tile_off[bb + 1]);
        if (s1 >= t1) return B;
        ++bb;
        while (tile_off[bb + 1] <= s1) ++bb;   // skip sequences with no tiles
        return bb;
      };
      auto produce_q = [&](uint32_t n, uint32_t bb) -> bool {
        const uint32_t slot = n & 1u, round = n >> 1;
        if (misc[0] || !mbar_wait(&q_empty[slot], (round & 1u) ^ 1u)) return false;
        const uint32_t ct = __ldg(p.cache_tokens + bb);
        const uint32_t rrow = p.rope_row ? __ldg(p.rope_row + bb) : ct;
        const int h = lane >> 1;
        const __half* qrow = p.q + (size_t)bb * p.q_stride + (size_t)h * HD;
        __half* qdst = qs + (slot * QH + h) * Q_PITCH;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t d = 32 * (lane & 1) + 8 * u;
          const uint4 lo = __ldg(reinterpret_cast<const uint4*>(qrow + d));
          const uint4 hi = __ldg(reinterpret_cast<const uint4*>(qrow + d + 64));
          *reinterpret_cast<uint4*>(qdst + d) = mrope8(lo, hi, d, p, rrow);
          *reinterpret_cast<uint4*>(qdst + d + 64) = mrope8(hi, lo, d + 64, p, rrow);
        }
        mbar_arrive(&q_full[slot]);
        return true;
      };
      auto append = [&](uint32_t n, uint32_t bb) -> bool {
        const uint32_t ct = __ldg(p.cache_tokens + bb);
        const uint64_t append_tile = tile_off[bb] + ct / TILE;
        if (append_tile < t0 || append_tile >= t1) return true;
        const uint32_t rrow = p.rope_row ? __ldg(p.rope_row + bb) : ct;
        // appended row: lane l holds bytes 16l..16l+15 = head l/16, dims
        // 8(l%16)..+7; the M-RoPE partners (d +- 64) sit in lane l ^ 8
        const uint4 kx = __ldg(reinterpret_cast<const uint4*>(p.k_new + (size_t)bb * p.kv_stride) + lane);
        const uint4 vx = __ldg(reinterpret_cast<const uint4*>(p.v_new + (size_t)bb * p.kv_stride) + lane);
        uint4 ky;
        ky.x = __shfl_xor_sync(0xffffffffu, kx.x, 8);
        ky.y = __shfl_xor_sync(0xffffffffu, kx.y, 8);
        ky.z = __shfl_xor_sync(0xffffffffu, kx.z, 8);
        ky.w = __shfl_xor_sync(0xffffffffu, kx.w, 8);
        const uint4 kr = mrope8(kx, ky, (lane & 15) * 8, p, rrow);
        // into the append tile's ring stage, once the copy warp has claimed it.
        // The copy warp may run up to STAGES sequences ahead, so the
        // handshake has APP_SLOTS slots by sequence number; every sequence
        // but possibly the range's last has its append here, so a slot's
        // phases advance once per APP_SLOTS sequences
        if (misc[0] || !mbar_wait(&app_stage[n % APP_SLOTS], (n / APP_SLOTS) & 1u)) return false;
        const uint32_t stage = misc[8 + n % APP_SLOTS];
        const uint32_t r = ct % TILE;
        *reinterpret_cast<uint4*>(smem + SM_K + stage * STAGE_BYTES + r * ROW_PITCH + lane * 16) = kr;
        *reinterpret_cast<uint4*>(smem + SM_V + stage * STAGE_BYTES + r * ROW_PITCH + lane * 16) = vx;
        mbar_arrive(&full_bar[stage]);
        // and into the cache for the steps to come (a later launch reads it)
        const size_t off = (size_t)ct * ROW_BYTES + lane * 16;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.k_cache[bb]) + off) = kr;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.v_cache[bb]) + off) = vx;
        return true;
      };
      uint32_t nseq = 0;
      aborted = !produce_q(0, b);
      while (!aborted) {
        const uint32_t bn = next_seq(b);
        // tiles of sequence b in the range: a short piece's append goes first
        const uint64_t pc = umin64(t1, tile_off[b + 1]) - umax64(t0, tile_off[b]);
        if (pc <= APPEND_FIRST_TILES) {
          if (!append(nseq, b) || (bn < B && !produce_q(nseq + 1, bn))) aborted = true;
        } else {
          if ((bn < B && !produce_q(nseq + 1, bn)) || !append(nseq, b)) aborted = true;
        }
        if (aborted || bn >= B) break;
        ++nseq;
        b = bn;
      }
    } else {
      // merge warp: per sequence of the range except the last, in order,
      // combines the eight consumer warps' (O, m, l) from the buffer they
      // filled and writes the output (whole sequence) or this CTA's partial
      // record; for a split sequence the last CTA to finish (atomic ticket, no
      // spinning) combines every CTA's record in CTA (= token) order and
      // resets the ticket.  The consumers hand over and move on, so a sequence
      // end inside the range does not stall the stream; the range's last
      // sequence, after which nothing is left to overlap, is merged by all
      // consumer threads.  Lane l owns query head l/2, dims 64(l%2)..+63.
      const int hq = lane >> 1, dbase = (lane & 1) * 64;
      const int kg = hq >> 3, hig = hq & 7;
      float* merge_acc = reinterpret_cast<float*>(smem + SM_MERGE_ACC);
      float* merge_m = reinterpret_cast<float*>(smem + SM_MERGE_M);
      float* merge_l = reinterpret_cast<float*>(smem + SM_MERGE_L);
      uint32_t j = 0;
      while (true) {
        const uint64_t s0 = umax64(t0, tile_off[b]);
        const uint64_t s1 = umin64(t1, tile_off[b + 1]);
        if (s1 >= t1) break;   // the range's last sequence: merged by the consumers
        if (misc[0] || !mbar_wait(merge_full, j & 1u)) {
          aborted = true;
          break;
        }
        const float* mm = merge_m;
        const float* ml = merge_l;
        const float* ma = merge_acc;
        // the four warps of KV group kg: (grp, half) in {0,1}^2 -> warp 4*grp + 2*kg + half
        float M = -CUDART_INF_F;
#pragma unroll
        for (int i = 0; i < 4; ++i) M = fmaxf(M, mm[(2 * kg + (i & 1) + 4 * (i >> 1)) * GROUP + hig]);
        float f[4], Lsum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int w = 2 * kg + (i & 1) + 4 * (i >> 1);
          const float mi = mm[w * GROUP + hig];
          f[i] = mi == -CUDART_INF_F ? 0.f : fast_exp2(mi - M);
          Lsum += ml[w * GROUP + hig] * f[i];
        }
        const bool whole = (s0 == tile_off[b]) && (s1 == tile_off[b + 1]);
        const uint32_t slot = blockIdx.x + b;
        float* rec = p.partials + (size_t)slot * PART_FLOATS;
        const float inv = 1.f / Lsum;
#pragma unroll 2
        for (int ch = 0; ch < 8; ++ch) {
          const int d0 = dbase + 8 * ch;
          float A[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int w = 2 * kg + (i & 1) + 4 * (i >> 1);
            const float4 u = *reinterpret_cast<const float4*>(ma + (w * GROUP + hig) * HD + d0);
            const float4 x = *reinterpret_cast<const float4*>(ma + (w * GROUP + hig) * HD + d0 + 4);
            A[0] += u.x * f[i]; A[1] += u.y * f[i]; A[2] += u.z * f[i]; A[3] += u.w * f[i];
            A[4] += x.x * f[i]; A[5] += x.y * f[i]; A[6] += x.z * f[i]; A[7] += x.w * f[i];
          }
          if (whole) {
            __align__(16) __half o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(A[e] * inv);
            *reinterpret_cast<uint4*>(p.out + ((size_t)b * QH + hq) * HD + d0) =
                *reinterpret_cast<uint4*>(o);
          } else {
            *reinterpret_cast<float4*>(rec + hq * HD + d0) = make_float4(A[0], A[1], A[2], A[3]);
            *reinterpret_cast<float4*>(rec + hq * HD + d0 + 4) = make_float4(A[4], A[5], A[6], A[7]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(merge_empty);   // the buffer has been read
        if (!whole) {
          if ((lane & 1) == 0) {
            rec[QH * HD + hq] = M;
            rec[QH * HD + QH + hq] = Lsum;
          }
          __threadfence();
          __syncwarp();
          uint32_t first = 0, last = 0, mine = 0;
          if (lane == 0) {
            first = owner_cta(cost_off[b], G, C);
            last = owner_cta(cost_off[b] + (tile_off[b + 1] - tile_off[b]) - 1, G, C);
            const uint32_t prev = atomicAdd(p.tickets + b, 1u);
            mine = prev == last - first;
            if (mine) {
              __threadfence();
              p.tickets[b] = 0;  // ready for the next launch
            }
          }
          mine = __shfl_sync(0xffffffffu, mine, 0);
          first = __shfl_sync(0xffffffffu, first, 0);
          last = __shfl_sync(0xffffffffu, last, 0);
          if (mine) combine_split<8>(p, b, first, last, hq, dbase);
        }
        ++j;
        ++b;
        while (tile_off[b + 1] <= s1) ++b;   // skip sequences with no tiles
      }
    }
    if (aborted) {
      if (lane == 0) atomicOr(p.flags, kFlagTimeout);
      misc[0] = 1;
    }
    // never leave the CTA with copies in flight
    cp_async_wait_all();
    return;
  }

  // ======================= consumer warps =======================
  const int grp = warp >> 2;          // tile parity handled by this warp
  const int kvh = (warp >> 1) & 1;    // KV head
  const int half = warp & 1;          // rows [16*half, 16*half+16) of a tile
  const int g = lane >> 2;            // fragment row group
  const int c = lane & 3;             // fragment column pair
  const float qk_scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));  // log2(e)/sqrt(d)

  float* merge_acc = reinterpret_cast<float*>(smem + SM_MERGE_ACC);
  float* merge_m = reinterpret_cast<float*>(smem + SM_MERGE_M);
  float* merge_l = reinterpret_cast<float*>(smem + SM_MERGE_L);

  uint32_t b = seq_of(t0);
  uint32_t nseq = 0;   // sequences of this CTA so far (q slot parity, in producer order)
  while (true) {
    const uint64_t s0 = umax64(t0, tile_off[b]);
    const uint64_t s1 = umin64(t1, tile_off[b + 1]);
    const uint32_t L = __ldg(p.cache_tokens + b) + 1;

    // ---- rotated Q^T fragments (B operand: k = dim, n = head) for this KV
    // group, from the shared-memory slot the producers filled for sequence b
    uint32_t qf[8][2];
    {
      const int slot = static_cast<int>(nseq & 1u);
      // On an abort (or a timed-out wait) every consumer warp still walks the
      // same merges and named barriers below: the tile loop does nothing once
      // misc[0] is set, so no warp can leave another waiting at a barrier.
      const bool go = __all_sync(0xffffffffu, misc[0] == 0);
      if (go && !__all_sync(0xffffffffu, mbar_wait(&q_full[slot], (nseq >> 1) & 1u))) {
        if (lane == 0) atomicOr(p.flags, kFlagTimeout);
        misc[0] = 1;
      }
      const __half* qrow = qs + (slot * QH + kvh * GROUP + g) * Q_PITCH;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          qf[ks][hh] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + hh * 8 + 2 * c);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[slot]);
      ++nseq;
    }

    float m_run[2] = {-CUDART_INF_F, -CUDART_INF_F};
    float l_run[2] = {0.f, 0.f};
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    for (uint64_t gt = s0 + (((s0 - t0) ^ grp) & 1); gt < s1; gt += 2) {
      const uint64_t it = gt - t0;
      const int stage = static_cast<int>(it % STAGES);
      const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
      // warp-uniform exits: the tile body below is warp-collective
      if (!__all_sync(0xffffffffu, misc[0] == 0)) break;
      if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[stage], ph))) {
        if (lane == 0) atomicOr(p.flags, kFlagTimeout);
        misc[0] = 1;
        break;
      }
      const uint32_t row0 = static_cast<uint32_t>(gt - tile_off[b]) * TILE;
      const int n_valid = static_cast<int>(umin32(TILE, L - row0)) - half * 16;
      uint8_t* kst = smem + SM_K + stage * STAGE_BYTES;
      uint8_t* vst = smem + SM_V + stage * STAGE_BYTES;
      if (n_valid > 0) {
        if (n_valid < 16) {
          // past the sequence end the staged rows hold whatever the ring last
          // carried (or nothing yet): zero this warp's V rows there, since
          // P = 0 meets them in the PV product and 0 * NaN would poison O
          for (int r = n_valid; r < 16; ++r)
            *reinterpret_cast<uint2*>(vst + (half * 16 + r) * ROW_PITCH + kvh * HD * 2 + lane * 8) =
                make_uint2(0u, 0u);
          __syncwarp();
        }

        // ---- S^T[16 keys x 8 heads] = K[16 x 128] * Q^T[128 x 8]
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        {
          // ldmatrix.x4 lanes: matrix j = lane/8: rows (keys) +8*(j&1), dims +8*(j>>1)
          const int mrow = half * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const uint32_t kaddr = smem_u32(kst + mrow * ROW_PITCH + kvh * HD * 2 + (lane >> 4) * 16);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(a0, a1, a2, a3, kaddr + ks * 32);
            mma_16816(s, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
          }
        }
        // s[0]: key g head 2c, s[1]: key g head 2c+1, s[2]/s[3]: key g+8
        const bool v0 = g < n_valid, v1 = g + 8 < n_valid;
        float x0 = v0 ? s[0] * qk_scale : -CUDART_INF_F;
        float x1 = v0 ? s[1] * qk_scale : -CUDART_INF_F;
        float x2 = v1 ? s[2] * qk_scale : -CUDART_INF_F;
        float x3 = v1 ? s[3] * qk_scale : -CUDART_INF_F;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
        const float al0 = fast_exp2(m_run[0] - mn0), al1 = fast_exp2(m_run[1] - mn1);
        m_run[0] = mn0;
        m_run[1] = mn1;
        const float p0 = fast_exp2(x0 - mn0), p1 = fast_exp2(x1 - mn1);
        const float p2 = fast_exp2(x2 - mn0), p3 = fast_exp2(x3 - mn1);
        l_run[0] = l_run[0] * al0 + (p0 + p2);
        l_run[1] = l_run[1] * al1 + (p1 + p3);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          acc[mt][0] *= al0;
          acc[mt][1] *= al1;
          acc[mt][2] *= al0;
          acc[mt][3] *= al1;
        }
        // P^T as the B operand (k = key, n = head): transpose the two 8x8 blocks
        const uint32_t pb0 = movmatrix_t(pack_half2(p0, p1));
        const uint32_t pb1 = movmatrix_t(pack_half2(p2, p3));

        // ---- O^T[128 x 8] += V^T[128 x 16 keys] * P^T[16 keys x 8 heads]
        {
          // ldmatrix.x4.trans lanes: matrix j: keys +8*(j>>1), dims +8*(j&1)
          const int vrow = half * 16 + (lane & 7) + (lane >> 4) * 8;
          const uint32_t vaddr =
              smem_u32(vst + vrow * ROW_PITCH + kvh * HD * 2 + ((lane >> 3) & 1) * 16);
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(a0, a1, a2, a3, vaddr + mt * 32);
            mma_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
    }

    // ---- hand this warp's (O, m, l) for the sequence over: to the merge warp,
    // or, for the range's last sequence, to the merge below by all consumers
    {
      const uint32_t e = nseq - 1;   // this sequence's index in the CTA's range
      if (!__all_sync(0xffffffffu, mbar_wait(merge_empty, (e & 1u) ^ 1u))) {
        if (lane == 0) atomicOr(p.flags, kFlagTimeout);
        misc[0] = 1;
      }
      float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
      }
      if (g == 0) {
        merge_m[warp * GROUP + 2 * c] = m_run[0];
        merge_m[warp * GROUP + 2 * c + 1] = m_run[1];
        merge_l[warp * GROUP + 2 * c] = l0;
        merge_l[warp * GROUP + 2 * c + 1] = l1;
      }
      float* ma = merge_acc + warp * GROUP * HD;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        ma[(2 * c) * HD + mt * 16 + g] = acc[mt][0];
        ma[(2 * c + 1) * HD + mt * 16 + g] = acc[mt][1];
        ma[(2 * c) * HD + mt * 16 + g + 8] = acc[mt][2];
        ma[(2 * c + 1) * HD + mt * 16 + g + 8] = acc[mt][3];
      }
      __syncwarp();
      if (s1 < t1 && lane == 0) mbar_arrive(merge_full);
    }
    if (s1 >= t1) {
      named_bar_sync(1, CONSUMER_THREADS);
      const bool whole = (s0 == tile_off[b]) && (s1 == tile_off[b + 1]);
      const uint32_t slot = blockIdx.x + b;
      // thread -> (query head, 8 dims)
      const int hq = tid >> 4;               // 0..15
      const int d0 = (tid & 15) * 8;
      const int kg = hq >> 3, hig = hq & 7;
      // the four warps of KV group kg: (grp, half) in {0,1}^2 -> warp 4*grp + 2*kg + half
      float M = -CUDART_INF_F;
#pragma unroll
      for (int i = 0; i < 4; ++i) M = fmaxf(M, merge_m[(2 * kg + (i & 1) + 4 * (i >> 1)) * GROUP + hig]);
      float f[4], Lsum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int w = 2 * kg + (i & 1) + 4 * (i >> 1);
        const float mi = merge_m[w * GROUP + hig];
        f[i] = mi == -CUDART_INF_F ? 0.f : fast_exp2(mi - M);
        Lsum += merge_l[w * GROUP + hig] * f[i];
      }
      float A[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) A[e] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int w = 2 * kg + (i & 1) + 4 * (i >> 1);
        const float4 u = *reinterpret_cast<const float4*>(merge_acc + (w * GROUP + hig) * HD + d0);
        const float4 x = *reinterpret_cast<const float4*>(merge_acc + (w * GROUP + hig) * HD + d0 + 4);
        A[0] += u.x * f[i]; A[1] += u.y * f[i]; A[2] += u.z * f[i]; A[3] += u.w * f[i];
        A[4] += x.x * f[i]; A[5] += x.y * f[i]; A[6] += x.z * f[i]; A[7] += x.w * f[i];
      }
      if (whole) {
        const float inv = 1.f / Lsum;
        __align__(16) __half o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(A[e] * inv);
        *reinterpret_cast<uint4*>(p.out + ((size_t)b * QH + hq) * HD + d0) =
            *reinterpret_cast<uint4*>(o);
      } else {
        float* rec = p.partials + (size_t)slot * PART_FLOATS;
        *reinterpret_cast<float4*>(rec + hq * HD + d0) = make_float4(A[0], A[1], A[2], A[3]);
        *reinterpret_cast<float4*>(rec + hq * HD + d0 + 4) = make_float4(A[4], A[5], A[6], A[7]);
        if ((tid & 15) == 0) {
          rec[QH * HD + hq] = M;
          rec[QH * HD + QH + hq] = Lsum;
        }
        __threadfence();
      }
      named_bar_sync(1, CONSUMER_THREADS);
      if (!whole) {
        if (tid == 0) {
          const uint32_t first = owner_cta(cost_off[b], G, C);
          const uint32_t last = owner_cta(cost_off[b] + (tile_off[b + 1] - tile_off[b]) - 1, G, C);
          const uint32_t prev = atomicAdd(p.tickets + b, 1u);
          const bool mine = prev == last - first;
          if (mine) {
            __threadfence();
            p.tickets[b] = 0;  // ready for the next launch
          }
          misc[1] = mine ? 1u : 0u;
          misc[2] = first;
          misc[3] = last;
        }
        named_bar_sync(1, CONSUMER_THREADS);
        // combine every CTA's record of sequence b in CTA (= token) order
        if (misc[1]) combine_split<1>(p, b, misc[2], misc[3], hq, d0);
        named_bar_sync(1, CONSUMER_THREADS);
      }
      break;
    }
    ++b;
    while (tile_off[b + 1] <= s1) ++b;  // skip sequences with no tiles
  }
}

}  // namespace decode

// ----------------------------------------------------------------- launcher
int decode_block_threads() { return decode::THREADS; }

size_t decode_workspace_bytes(uint32_t batch, int num_sms) {
  const size_t header = 256;
  const size_t tickets = ((size_t)batch * 4 + 255) / 256 * 256;
  const size_t parts = ((size_t)num_sms + batch) * decode::PART_FLOATS * sizeof(float);
  return header + tickets + parts;
}

int decode_launch(const DecodeArgs& a, cudaStream_t stream) {
  if (set_smem_attribute_once(reinterpret_cast<const void*>(decode::decode_kernel), decode::SMEM_BYTES) != PVLC_OK)
    return PVLC_CUDA_ERROR;
  decode::Params p;
  p.q = reinterpret_cast<const __half*>(a.q);
  p.k_new = reinterpret_cast<const __half*>(a.k_new);
  p.v_new = reinterpret_cast<const __half*>(a.v_new);
  p.rope_cos = a.rope_cos;
  p.rope_sin = a.rope_sin;
  p.rope_row = a.rope_row;
  p.k_cache = reinterpret_cast<__half* const*>(a.k_cache);
  p.v_cache = reinterpret_cast<__half* const*>(a.v_cache);
  p.cache_tokens = a.cache_tokens;
  p.q_stride = a.q_stride;
  p.kv_stride = a.kv_stride;
  p.rope_rows = a.rope_rows;
  p.capacity = a.capacity;
  p.max_cache_tokens = a.max_cache_tokens;
  p.batch = a.batch;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a.workspace);
  p.flags = reinterpret_cast<uint32_t*>(ws);
  p.tickets = reinterpret_cast<uint32_t*>(ws + 256);
  p.partials = reinterpret_cast<float*>(ws + 256 + ((size_t)a.batch * 4 + 255) / 256 * 256);
  p.out = reinterpret_cast<__half*>(a.out);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_ctas);
  cfg.blockDim = dim3(decode::THREADS);
  cfg.dynamicSmemBytes = decode::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, decode::decode_kernel, p) != cudaSuccess) return PVLC_CUDA_ERROR;
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

// ------------------------------------------------ allocation-free decode
// Some callers can hand us input and output buffers but cannot allocate device
// memory themselves: a host whose device memory is planned once up front by a
// static arena, or a foreign-language binding with no handle on a CUDA
// allocator.  For them the split-KV scratch (fault flags, combine tickets and
// per-CTA partial records) lives in this fixed file-scope device array instead
// of a caller workspace.  Every GPU that loads this library holds the array
// (PVLC_DECODE_NOALLOC_SCRATCH_BYTES) until the process exits.
namespace {

__device__ __align__(256) uint8_t g_decode_noalloc_scratch[PVLC_DECODE_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device.  In host code
// `g_decode_noalloc_scratch` names a host-side stand-in, never the device
// memory, so the address is asked for on every call, with the device current:
// a host-only lookup that stays right if the context is ever re-created
// (cudaDeviceReset reloads the module, possibly elsewhere).
int noalloc_scratch(void** out) {
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_decode_noalloc_scratch) != cudaSuccess || ptr == nullptr)
    return PVLC_CUDA_ERROR;
  *out = ptr;
  return PVLC_OK;
}

bool aligned16_ptr(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace pvlc

extern "C" int pvlc_attn_decode_noalloc(const pvlc_half* q, const pvlc_half* k_new,
                                        const pvlc_half* v_new, const float* rope_cos,
                                        const float* rope_sin, uint32_t rope_rows,
                                        const uint32_t* rope_row, pvlc_half* const* k_cache,
                                        pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                                        uint32_t cache_capacity, uint32_t max_cache_tokens,
                                        uint32_t batch, pvlc_half* out, void* stream) {
  using namespace pvlc;
  // same host-side checks and precedence as pvlc_attn_decode
  if (batch == 0 || cache_capacity == 0 || rope_rows == 0) return PVLC_ZERO_DIMENSION;
  if (batch > PVLC_DECODE_MAX_BATCH) return PVLC_INVALID_DECODER_GEOMETRY;
  if (max_cache_tokens >= cache_capacity) return PVLC_CAPACITY_EXHAUSTED;
  if ((uint64_t)cache_capacity * 512ull > (1ull << 40)) return PVLC_ARITHMETIC_OVERFLOW;
  if (!q || !k_new || !v_new || !rope_cos || !rope_sin || !k_cache || !v_cache || !cache_tokens ||
      !out)
    return PVLC_NULL_POINTER;
  if (!aligned16_ptr(q) || !aligned16_ptr(k_new) || !aligned16_ptr(v_new) || !aligned16_ptr(out) ||
      !aligned16_ptr(rope_cos) || !aligned16_ptr(rope_sin))
    return PVLC_MISALIGNED_POINTER;
  // the fixed scratch bounds the batch
  if (batch > PVLC_DECODE_NOALLOC_MAX_BATCH) return PVLC_WORKSPACE_TOO_SMALL;
  const int sms = device_sm_count();
  if (sms <= 0) return PVLC_CUDA_ERROR;
  const size_t need = decode_workspace_bytes(batch, sms);
  if (need > PVLC_DECODE_NOALLOC_SCRATCH_BYTES) return PVLC_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != PVLC_OK) return st;
  // The array keeps the previous call's contents: the fault flags and the
  // combine tickets must start at zero (the partial records need not).
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t zero_bytes = 256 + ((size_t)batch * 4 + 255) / 256 * 256;
  if (cudaMemsetAsync(scratch, 0, zero_bytes, s) != cudaSuccess) return PVLC_CUDA_ERROR;
  DecodeArgs a{q,       k_new,    v_new,   rope_cos,     rope_sin,       rope_rows,
               rope_row, k_cache, v_cache, cache_tokens, cache_capacity, max_cache_tokens,
               batch,   scratch,  out,     sms,          16u * 128u,     2u * 128u};
  return decode_launch(a, s);
}
