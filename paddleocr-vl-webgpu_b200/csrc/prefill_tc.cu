// prefill_tc.cu -- decoder causal GQA prefill (pinned Q16/KV2/D128) on the
// Blackwell tensor cores (tcgen05 + TMEM + TMA), with the 3-section
// multimodal RoPE applied to every key exactly once and the fp16 KV cache
// written in place.  sm_100a.
//
// Reference path replaced: DecoderPrefillMropeF32 -> DecoderKvAppendRangeF32
// -> DecoderPrefillGqaF32 (crates/pvlc-wgsl/src/lib.rs:1262-1416; stage order
// crates/pvlc-runtime-core/src/lib.rs:2613-2629); arithmetic
// crates/pvlc-cpu-ref/src/lib.rs:562-672 (M-RoPE), :976-991 (KV write),
// :782-853 (causal GQA).
//
// Two launches on the caller's stream:
//   1. kv_rope_kernel: M-RoPE of K fused with the KV-cache write -- each key
//      row is rotated once and stored (with its raw value row) in the cache.
//   2. prefill_attn_kernel: attention whose keys are TMA-loaded from that
//      cache (already rotated) and whose Q M-RoPE is fused into the Q tile.
// Rotating keys inside the attention CTAs instead would repeat the rotation
// of every key tile in every query block that reads it (measured: 60 of
// 100 us at T = 1564), while the cache row has to be written anyway.
//
// GQA packing: a Q tile is 16 tokens x the 8 query heads of one KV group =
// 128 MMA rows (row r = token r/8, head r%8), loaded by one 3-D TMA box, so a
// K/V tile of 128 keys serves all 8 heads.  A CTA (one KV head) runs two
// streams with their own S and O in TMEM, which ping-pong on the MMA warp:
//   split: one Q tile whose causal key range (K tiles 0 .. the diagonal) is
//          dealt to the streams as even and odd K tiles, the two streams'
//          (O, m, l) merged inside the CTA at the end -- the chain of
//          dependent K tiles is at most ceil(13 / 2) = 7 at T = 1564;
//   pair:  two Q tiles, one per stream, sharing every K/V tile (the second
//          tile's K tiles a prefix of the first's).
// A single prompt splits its heaviest tiles and pairs the lightest (light
// tile n - 1 - i with i) only while that keeps one wave within the heaviest
// split CTA's time; a batched launch (up to 256 prompts packed back to back,
// the prompt table a grid constant) pairs each prompt's adjacent tiles.
// Causal masking inside tiles that cross the diagonal.
// head_dim 128 = two 64-dim blocks of 128-byte rows (128B swizzle); QK = 8 x
// K16 steps (M128 N128), PV = 8 x K16 steps (M128 N128, V MN-major across
// both blocks), P from TMEM.
//
//   warps 0-3, 4-7  softmax for stream 0 / 1: thread i owns row i = TMEM lane
//                   i; both rotate their half of the Q tile's dims once
//                   (M-RoPE), then per K tile of the stream the online
//                   softmax (f32, exp2 domain) and P (fp16) over S; at the
//                   end each writes output columns 64t..64t+63 from both
//                   streams' O
//   warp 8          TMA producer: the Q tile(s), then K/V tiles (3 stages
//                   split, 2 paired)
//   warp 9          MMA issuer (the whole warp walks the schedule, one
//                   elected lane issues)
// TMEM (512 columns): S/P of stream t at [128t, 128t+128), O at [256+128t, +128).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <mutex>

#include "pvlc_common.cuh"
#include "pvlc_internal.h"
#include "tcgen05.cuh"

namespace pvlc {
namespace ptc {

// Sticky fault word of this device's prefill launches: a CTA whose bounded
// wait ran out (misc[1]) ORs in its kernel's bit when it ends.  Read and
// cleared by pvlc_attn_fault_flags.
__device__ uint32_t g_faults;

constexpr int HD = 128;
constexpr int QH = 16;
constexpr int KVH = 2;
constexpr int GROUP = 8;
constexpr int TOK = 16;          // tokens per Q tile (x 8 heads = 128 rows)
constexpr int QT = 1;            // Q tiles per CTA
constexpr int STREAMS = 2;       // K-tile streams per CTA (even / odd K tiles)
constexpr int BN = 128;          // keys per K/V tile
constexpr int THREADS = 12 * 32;
// launch: 384 threads x 168 registers; softmax warpgroups take 200, control 104
constexpr uint32_t REGS_SOFTMAX = 200, REGS_CTRL = 104;
static_assert(256 * REGS_SOFTMAX + 128 * REGS_CTRL <= 384 * 168, "register split");

constexpr uint32_t SZ_W = 128 * 128;          // 128 rows x 64 dims fp16, 128B swizzle
constexpr uint32_t Q_BYTES = 2 * SZ_W;        // two 64-dim blocks
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_STAGE = QT * Q_BYTES;
constexpr uint32_t ST_K = 0, ST_V = 2 * SZ_W;
constexpr uint32_t STAGE_BYTES = 4 * SZ_W;
constexpr int STAGES = 3;
constexpr uint32_t OFF_BARS = OFF_STAGE + STAGES * STAGE_BYTES;
// pair CTAs: Q buffer 1 then PAIR_STAGES stages inside the same region
constexpr int PAIR_STAGES = 2;
constexpr uint32_t OFF_STAGE_PAIR = 2 * Q_BYTES;
static_assert(OFF_STAGE_PAIR + PAIR_STAGES * STAGE_BYTES <= OFF_BARS, "pair layout overflows");
// q_full, q_ready, kv_full[3], kv_empty[3], s_full[2], p_ready[2], o_done[2], ml_ready
constexpr int NBARS = 15;
constexpr uint32_t OFF_MISC = OFF_BARS + NBARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 64 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "prefill shared memory exceeds the sm_100 limit");
constexpr uint32_t TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;
// Pairs c (of each 16-pair chunk of a score row) whose exponentials run on the
// FMA / integer pipes (exp2_h2_poly) instead of MUFU.
#ifndef PVLC_PREFILL_EXP_POLY_MASK
#define PVLC_PREFILL_EXP_POLY_MASK 0x4924u
#endif
constexpr uint32_t EXP_POLY_MASK = PVLC_PREFILL_EXP_POLY_MASK;
// 1: batched launches run the persistent kernel (prefill_persist_kernel)
#ifndef PVLC_PREFILL_PERSIST
#define PVLC_PREFILL_PERSIST 1
#endif


struct Maps {
  // q, v: the packed input rows; k: the KV caches (rotated keys) as
  // {128, 2, capacity, prompts}; o: the packed output rows (batched kernel's
  // epilogue, Q-tile boxes)
  CUtensorMap q, k, v, o;
};

struct Params {
  uint32_t n_split;       // single prompt: split CTAs per KV head (the heaviest Q tiles)
  uint32_t n_light;       // single prompt: lightest Q tiles, paired two per CTA
  uint64_t cache_stride;  // elements from one prompt's cache to the next
  __half* k_cache;        // prompt b's [capacity, 2, 128] caches at + b * cache_stride
  __half* v_cache;
  __half* out;            // packed [rows, 16, 128]
};

// The prompts of one launch, packed back to back in q / k / v / out: one for
// a single call, up to MAXB for a batched call (then each CTA takes two
// adjacent Q tiles of one prompt, the prompt's heaviest first).  Passed by
// value as a grid constant, so a launch copies nothing from the host.
template <int MAXB>
struct Prompts {
  uint32_t count;
  uint32_t ranks_max;              // largest CTA count of a prompt (persistent item slots)
  uint32_t cta_prefix[MAXB + 1];   // CTAs (per KV head) of the prompts before b
  uint32_t row0[MAXB + 1];         // first packed row of prompt b; row0[count] = rows
  uint32_t rope_rows[MAXB];
  const float* rope_cos[MAXB];     // [3, rope_rows[b], 128]
  const float* rope_sin[MAXB];
};

// index b with v[b] <= x < v[b + 1] among v[0 .. n] (v ascending, v[0] <= x < v[n])
__device__ __forceinline__ uint32_t find_segment(const uint32_t* v, uint32_t n, uint32_t x) {
  uint32_t lo = 0, hi = n;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (v[mid] <= x) lo = mid; else hi = mid;
  }
  return lo;
}

// ------------------------------------------------------------------------
// 1. M-RoPE of the keys fused with the KV-cache write.  Thread = (token, KV
// head, chunk c): dims 8c..8c+7 and their partners 64+8c..64+8c+7.  Dim d of
// a 128-wide head takes table plane 0/1/2 for (d mod 64) in [0,16)/[16,40)/
// [40,64); d < 64 becomes x[d] cos[d] - x[d+64] sin[d] and d+64 becomes
// x[d+64] cos[d+64] + x[d] sin[d+64] (crates/pvlc-cpu-ref/src/lib.rs:645-668).
template <int MAXB>
__global__ void __launch_bounds__(256) kv_rope_kernel(const __half* __restrict__ k,
                                                      const __half* __restrict__ v,
                                                      const __grid_constant__ Prompts<MAXB> pr,
                                                      const Params p) {
  // the attention launch may start its prologue (barriers, TMEM, Q load and
  // rotation) now; it waits for this kernel before reading the cache
  pdl_launch_dependents();
  const uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t c = gid & 7, head = (gid >> 3) & 1, row = gid >> 4;   // packed row
  if (row >= pr.row0[pr.count]) return;
  const uint32_t pi = MAXB == 1 ? 0u : find_segment(pr.row0, pr.count, row);
  const uint32_t token = row - pr.row0[pi];
  const size_t in = ((size_t)row * KVH + head) * HD;
  const size_t cr = (size_t)pi * p.cache_stride + ((size_t)token * KVH + head) * HD;
  const size_t tb = ((size_t)mrope_axis(8 * c) * pr.rope_rows[pi] + token) * HD + 8 * c;
  const float4* cs = reinterpret_cast<const float4*>(pr.rope_cos[pi] + tb);
  const float4* sn = reinterpret_cast<const float4*>(pr.rope_sin[pi] + tb);
  const float4 cl0 = __ldg(cs), cl1 = __ldg(cs + 1), ch0 = __ldg(cs + 16), ch1 = __ldg(cs + 17);
  const float4 sl0 = __ldg(sn), sl1 = __ldg(sn + 1), sh0 = __ldg(sn + 16), sh1 = __ldg(sn + 17);
  const uint4 a = *reinterpret_cast<const uint4*>(k + in + 8 * c);
  const uint4 b = *reinterpret_cast<const uint4*>(k + in + 64 + 8 * c);
  const float cl[8] = {cl0.x, cl0.y, cl0.z, cl0.w, cl1.x, cl1.y, cl1.z, cl1.w};
  const float chh[8] = {ch0.x, ch0.y, ch0.z, ch0.w, ch1.x, ch1.y, ch1.z, ch1.w};
  const float sl[8] = {sl0.x, sl0.y, sl0.z, sl0.w, sl1.x, sl1.y, sl1.z, sl1.w};
  const float shh[8] = {sh0.x, sh0.y, sh0.z, sh0.w, sh1.x, sh1.y, sh1.z, sh1.w};
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
  uint32_t ra[4], rb[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&aw[e]));
    const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&bw[e]));
    ra[e] = pack_half2(x.x * cl[2 * e] + (-y.x) * sl[2 * e], x.y * cl[2 * e + 1] + (-y.y) * sl[2 * e + 1]);
    rb[e] = pack_half2(y.x * chh[2 * e] + x.x * shh[2 * e], y.y * chh[2 * e + 1] + x.y * shh[2 * e + 1]);
  }
  *reinterpret_cast<uint4*>(p.k_cache + cr + 8 * c) = make_uint4(ra[0], ra[1], ra[2], ra[3]);
  *reinterpret_cast<uint4*>(p.k_cache + cr + 64 + 8 * c) = make_uint4(rb[0], rb[1], rb[2], rb[3]);
  *reinterpret_cast<uint4*>(p.v_cache + cr + 8 * c) =
      *reinterpret_cast<const uint4*>(v + in + 8 * c);
  *reinterpret_cast<uint4*>(p.v_cache + cr + 64 + 8 * c) =
      *reinterpret_cast<const uint4*>(v + in + 64 + 8 * c);
}

// ------------------------------------------------------------------------
// 2. Attention.
__device__ __forceinline__ uint8_t* chunk_addr(uint8_t* blk, int r, int c) {
  return blk + r * 128 + ((c ^ (r & 7)) << 4);
}

// M-RoPE table entries of one Q row's chunks c0..c0+3 (dims 8c..8c+7 and
// their partners 64 above): [chunk][cos lo 2, cos hi 2, sin lo 2, sin hi 2].
// Loaded before the Q tile lands, so the table latency overlaps the TMA load.
template <int NC = 4>
struct RowTables {
  float4 v[NC][8];
};

template <int NC>
__device__ __forceinline__ void mrope_tables(RowTables<NC>& t, const float* rope_cos,
                                             const float* rope_sin, uint32_t rope_rows,
                                             uint32_t token, int c0) {
#pragma unroll
  for (int u = 0; u < NC; ++u) {
    const int c = c0 + u;
    const uint32_t axis = mrope_axis(8 * c);   // section edges are multiples of 8
    const size_t tb = ((size_t)axis * rope_rows + token) * HD + 8 * c;
    const float4* cs = reinterpret_cast<const float4*>(rope_cos + tb);
    const float4* sn = reinterpret_cast<const float4*>(rope_sin + tb);
    t.v[u][0] = __ldg(cs);
    t.v[u][1] = __ldg(cs + 1);
    t.v[u][2] = __ldg(cs + 16);
    t.v[u][3] = __ldg(cs + 17);
    t.v[u][4] = __ldg(sn);
    t.v[u][5] = __ldg(sn + 1);
    t.v[u][6] = __ldg(sn + 16);
    t.v[u][7] = __ldg(sn + 17);
  }
}

// M-RoPE of chunk c of one 128-dim Q row r held in two 128B-swizzled 64-dim
// blocks, in place: dims 8c..8c+7 and their partners 64 above, with that
// chunk's table entries tv = {cos lo 2, cos hi 2, sin lo 2, sin hi 2}.
__device__ __forceinline__ void rope_chunk(uint8_t* b0, uint8_t* b1, int r, int c,
                                           const float4* tv) {
  const float4 cl0 = tv[0], cl1 = tv[1], ch0 = tv[2], ch1 = tv[3];
  const float4 sl0 = tv[4], sl1 = tv[5], sh0 = tv[6], sh1 = tv[7];
  uint4* pa = reinterpret_cast<uint4*>(chunk_addr(b0, r, c));
  uint4* pb = reinterpret_cast<uint4*>(chunk_addr(b1, r, c));
  const uint4 a = *pa, b = *pb;
  const float cl[8] = {cl0.x, cl0.y, cl0.z, cl0.w, cl1.x, cl1.y, cl1.z, cl1.w};
  const float chh[8] = {ch0.x, ch0.y, ch0.z, ch0.w, ch1.x, ch1.y, ch1.z, ch1.w};
  const float sl[8] = {sl0.x, sl0.y, sl0.z, sl0.w, sl1.x, sl1.y, sl1.z, sl1.w};
  const float shh[8] = {sh0.x, sh0.y, sh0.z, sh0.w, sh1.x, sh1.y, sh1.z, sh1.w};
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
  uint32_t ra[4], rb[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&aw[e]));
    const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&bw[e]));
    ra[e] = pack_half2(x.x * cl[2 * e] + (-y.x) * sl[2 * e], x.y * cl[2 * e + 1] + (-y.y) * sl[2 * e + 1]);
    rb[e] = pack_half2(y.x * chh[2 * e] + x.x * shh[2 * e], y.y * chh[2 * e + 1] + x.y * shh[2 * e + 1]);
  }
  *pa = make_uint4(ra[0], ra[1], ra[2], ra[3]);
  *pb = make_uint4(rb[0], rb[1], rb[2], rb[3]);
}

// M-RoPE of one Q row, chunks c0..c0+NC-1, in place.
template <int NC>
__device__ __forceinline__ void mrope_row(uint8_t* b0, uint8_t* b1, int r, const RowTables<NC>& t,
                                          int c0) {
#pragma unroll
  for (int u = 0; u < NC; ++u) rope_chunk(b0, b1, r, c0 + u, t.v[u]);
}

__device__ __forceinline__ uint64_t u2_pack(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

// One online-softmax step of stream tile row i (TMEM lane i) over K tile j:
// S from TMEM columns [tS, tS + 128), causal mask past `token` (also removing
// cache rows past the prompt), lazy running max (O rescaled in TMEM, after
// waiting for the previous PV through o_done at parity o_prev_parity, only
// when a row max grows by more than RESCALE_THRESHOLD), then P = 2^(x - m)
// as fp16 written over S (P of keys 2c, 2c + 1 in column c) and the row sum
// of that fp16 P added to l_run.  Returns false when a wait timed out.
__device__ __forceinline__ bool softmax_step(uint32_t tS, uint32_t tO, int j, uint32_t token,
                                         uint32_t warp_tok_lo, bool has_prev,
                                         uint64_t* o_done, uint32_t o_prev_parity,
                                         float scale, uint64_t scale2, float& m_run,
                                         float& l_run) {
  tc::fence_after_sync();
  uint32_t sv[128];
  tc::tmem_ld32(tS + 0, sv);
  tc::tmem_ld32(tS + 32, sv + 32);
  tc::tmem_ld32(tS + 64, sv + 64);
  tc::tmem_ld32(tS + 96, sv + 96);
  tc::tmem_wait_ld();
  // causal mask where this tile reaches past the warp's first token;
  // it also removes cache rows past the prompt (unwritten, any bits)
  if (j * BN + BN - 1 > warp_tok_lo) {
#pragma unroll
    for (int c = 0; c < 128; ++c)
      if (j * BN + c > token) sv[c] = __float_as_uint(-CUDART_INF_F);
  }
  // row max over four independent chains
  float m4[4] = {__uint_as_float(sv[0]), __uint_as_float(sv[1]), __uint_as_float(sv[2]),
                 __uint_as_float(sv[3])};
#pragma unroll
  for (int c = 4; c < 124; c += 8) {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      m4[e] = fmax3(m4[e], __uint_as_float(sv[c + 2 * e]), __uint_as_float(sv[c + 2 * e + 1]));
  }
  m4[0] = fmax3(m4[0], __uint_as_float(sv[124]), __uint_as_float(sv[125]));
  m4[1] = fmax3(m4[1], __uint_as_float(sv[126]), __uint_as_float(sv[127]));
  const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale;
  const bool need = mx > m_run + RESCALE_THRESHOLD;
  float alpha = 1.f;
  if (need) {
    alpha = fast_exp2(m_run - mx);
    m_run = mx;
    l_run *= alpha;
  }
  if (has_prev && __any_sync(0xffffffffu, need)) {
    if (!__all_sync(0xffffffffu, mbar_wait(o_done, o_prev_parity))) return false;
    tc::fence_after_sync();
#pragma unroll
    for (int cc = 0; cc < 128; cc += 16) {
      uint32_t ov[16];
      tc::tmem_ld16(tO + cc, ov);
      tc::tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
      tc::tmem_st16(tO + cc, ov);
    }
  }
  // a row whose keys in this stream are all masked keeps m = -inf: its
  // P is 0 (guard the subtraction)
  const float mm = m_run == -CUDART_INF_F ? 0.f : m_run;
  // P = 2^(x - m) as fp16 pairs, split between two pipes as in the
  // vision kernel: the pairs of EXP_POLY_MASK by the polynomial on the
  // FMA / integer pipes, the others by one f32 -> f16x2 rounding and one
  // MUFU operation per two values.  The row sum adds the fp16 P the PV
  // product consumes, in f32 (one mixed-precision add per value), over four
  // accumulator chains.
  const uint64_t negm2 = f2_pack(-mm, -mm);
  const uint64_t negmh2 = f2_pack(6.5f - mm, 6.5f - mm);   // exp2_h2_poly takes x + 6.5
  float acc[4] = {0.f, 0.f, 0.f, 0.f};   // four row-sum chains
  // One 32-key chunk per trip of a rolled loop, S reloaded from TMEM (P of
  // chunk c lands in columns 16c..16c+15, below every chunk still to be
  // read): a quarter of the code of the unrolled form, which missed in
  // the instruction cache.
  const bool diag = j * BN + BN - 1 > warp_tok_lo;
#pragma unroll 1
  for (int ch = 0; ch < 4; ++ch) {
    uint32_t sc[32];
    tc::tmem_ld32(tS + 32 * ch, sc);
    tc::tmem_wait_ld();
    if (diag) {
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (j * BN + 32 * ch + c > token) sc[c] = __float_as_uint(-CUDART_INF_F);
    }
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint64_t s2 = f2_pack(__uint_as_float(sc[2 * c]), __uint_as_float(sc[2 * c + 1]));
      if ((EXP_POLY_MASK >> c) & 1u) {
        pk[c] = exp2_h2_poly(f2_fma(s2, scale2, negmh2));
      } else {
        const float2 x = f2_unpack(f2_fma(s2, scale2, negm2));
        pk[c] = ex2_h2(pack_half2(x.x, x.y));
      }
      add_f16x2_to_f32(pk[c], acc[2 * (c & 1)], acc[2 * (c & 1) + 1]);
    }
    tc::tmem_st16(tS + 16 * ch, pk);
  }
  tc::tmem_wait_st();
  l_run += (acc[0] + acc[2]) + (acc[1] + acc[3]);
  return true;
}

template <int MAXB>
__global__ void __launch_bounds__(THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ Maps maps, const Params p,
                        const __grid_constant__ Prompts<MAXB> pr) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BARS);
  uint64_t* q_full = bars + 0;
  uint64_t* q_ready = bars + 1;
  uint64_t* kv_full = bars + 2;    // [3]
  uint64_t* kv_empty = bars + 5;   // [3]
  uint64_t* s_full = bars + 8;     // [2] per stream
  uint64_t* p_ready = bars + 10;   // [2]
  uint64_t* o_done = bars + 12;    // [2]
  uint64_t* ml_ready = bars + 14;  // both streams' (m, l) are in the exchange area
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t g = blockIdx.x;                      // KV head
  // prompt of this CTA and its rank among the prompt's CTAs (heaviest first)
  const uint32_t pi = MAXB == 1 ? 0u : find_segment(pr.cta_prefix, pr.count, blockIdx.y);
  const uint32_t rank = blockIdx.y - pr.cta_prefix[pi];
  const uint32_t row0 = pr.row0[pi];
  const uint32_t tokens = pr.row0[pi + 1] - row0;
  const uint32_t n_qt = (tokens + TOK - 1) / TOK;
  // Two kinds of CTA:
  //  split: one Q tile; stream t takes its K tiles t, t + 2, ... and the two
  //         streams' (O, m, l) merge at the end (the long causal ranges);
  //  pair:  two Q tiles, one per stream, sharing every K/V tile.
  // Single prompt: the heaviest tiles split, the lightest paired two per CTA
  // (light tile n_light - 1 - i with i) so that the grid is one wave.
  // Batched: CTA r of a prompt pairs its adjacent tiles n_qt - 1 - 2r and
  // n_qt - 2 - 2r (nearly equal K ranges, so both streams stay busy and the
  // CTA's fixed costs cover two tiles of work); an odd prompt's last CTA
  // takes tile 0 alone, split.
  bool pair;
  uint32_t qa, qb = 0;       // pair: stream 0 / stream 1 tile (qb's K tiles a prefix of qa's)
  if (MAXB == 1) {
    pair = blockIdx.y >= p.n_split;
    qa = pair ? p.n_light - 1 - (blockIdx.y - p.n_split) : n_qt - 1 - rank;
    qb = pair ? blockIdx.y - p.n_split : 0u;
  } else {
    qa = n_qt - 1 - 2 * rank;
    pair = qa >= 1;
    qb = pair ? qa - 1 : 0u;
  }
  uint32_t tile0[STREAMS];   // first token of each stream's Q tile
  int nks[STREAMS];          // K tiles of each stream
  int ntiles;                // K/V tiles the CTA loads
  if (!pair) {
    const uint32_t qt = qa;
    const uint32_t last_tok = umin32(qt * TOK + TOK, tokens) - 1;
    const int nk = static_cast<int>(last_tok / BN) + 1;    // K tiles 0 .. the diagonal
    tile0[0] = tile0[1] = qt * TOK;
    nks[0] = (nk + 1) / 2;
    nks[1] = nk / 2;
    ntiles = nk;
  } else {
    tile0[0] = qa * TOK;
    tile0[1] = qb * TOK;
    nks[0] = static_cast<int>((umin32(qa * TOK + TOK, tokens) - 1) / BN) + 1;
    nks[1] = static_cast<int>((umin32(qb * TOK + TOK, tokens) - 1) / BN) + 1;
    ntiles = nks[0];
  }
  // shared memory: Q buffer 0, then (split) 3 K/V stages or (pair) Q buffer 1
  // and 2 K/V stages
  const int nst = pair ? PAIR_STAGES : STAGES;
  const uint32_t off_stage = pair ? OFF_STAGE_PAIR : OFF_STAGE;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 8);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < STREAMS; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(ml_ready, 8);
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

  const int wg = warp >> 2;
  if (wg == 2) {
    tc::regs_dec<REGS_CTRL>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------- TMA producer
      tc::tma_prefetch_desc(&maps.q);
      tc::tma_prefetch_desc(&maps.k);
      tc::tma_prefetch_desc(&maps.v);
      const int nq = pair ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * Q_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
        if (t < nq)
          for (int b = 0; b < 2; ++b)
            tc::tma_load_3d(smem + OFF_Q + t * Q_BYTES + b * SZ_W, &maps.q, 64 * b, GROUP * g,
                            row0 + tile0[t], q_full);
      // keys are read from the cache that kv_rope_kernel (the preceding launch) writes
      pdl_wait();
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % nst;
        if (misc[1] || !mbar_wait(&kv_empty[s], ((j / nst) & 1) ^ 1)) { misc[1] = 1; break; }
        uint8_t* st = smem + off_stage + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&kv_full[s], STAGE_BYTES);
        for (int b = 0; b < 2; ++b) {
          tc::tma_load_4d(st + ST_K + b * SZ_W, &maps.k, 64 * b, g, j * BN, pi, &kv_full[s]);
          // values past the prompt (the next prompt's rows, or zero fill past
          // the packed rows) meet P = 0
          tc::tma_load_3d(st + ST_V + b * SZ_W, &maps.v, 64 * b, g, row0 + j * BN, &kv_full[s]);
        }
        issued = j + 1;
      }
      for (int j = (issued > nst ? issued - nst : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % nst], (j / nst) & 1);
    } else if (warp == 9) {
      // ---------------------------------------------------- MMA issuer
      // split: tile j lives in stage j % 3, stream t = j % 2; per step the PV
      // of the stream's current tile, then the QK of its next tile (two
      // ahead).  pair: tile j lives in stage j % 2 and serves both streams;
      // per step and stream the PV of tile j, then the QK of tile j + 1.
      constexpr uint32_t idesc_qk = tc::idesc_f16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = tc::idesc_f16(128, 128, 0, 1);
      const uint32_t sq = smem_u32(smem + OFF_Q), st0 = smem_u32(smem + off_stage);
      const uint64_t dq = tc::smem_desc(sq, 16, 1024, tc::kSw128);
      const uint64_t dk = tc::smem_desc(st0 + ST_K, 16, 1024, tc::kSw128);
      // MN-major V: the two 64-dim blocks are SZ_W apart (LBO), 8-key groups 1 KB apart
      const uint64_t dv = tc::smem_desc(st0 + ST_V, SZ_W, 1024, tc::kSw128);
      auto qk = [&](int t, int s) {
        const uint32_t tS = tmem + 128u * t;
        const uint64_t so = (uint64_t)s * (STAGE_BYTES >> 4);
        const uint64_t qo = pair ? (uint64_t)t * (Q_BYTES >> 4) : 0;
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {   // block ks/4, 32 bytes per K step within a block
            const uint64_t off = (uint64_t)(ks >> 2) * (SZ_W >> 4) + 2 * (ks & 3);
            tc::mma_ss(tS, dq + qo + off, dk + so + off, idesc_qk, ks > 0);
          }
          tc::commit(&s_full[t]);
        }
        __syncwarp();
      };
      auto pv = [&](int t, int s, bool first, bool release) {
        const uint32_t tS = tmem + 128u * t, tO = tmem + 256u + 128u * t;
        const uint64_t so = (uint64_t)s * (STAGE_BYTES >> 4);
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)     // 16 keys = two 1 KB groups per K step
            tc::mma_ts(tO, tS + ks * 8, dv + so + 128 * ks, idesc_pv, (!first || ks > 0) ? 1u : 0u);
          tc::commit(&o_done[t]);
          if (release) tc::commit(&kv_empty[s]);   // every stream reading the stage is done
        }
        __syncwarp();
      };
      constexpr uint32_t kAll = 0xffffffffu;
      auto kv_ready = [&](int j) { return mbar_wait(&kv_full[j % nst], (j / nst) & 1); };
      bool ok = __all_sync(kAll, mbar_wait(q_ready, 0) && kv_ready(0));
      int done = 0;   // K tiles whose last PV was issued
      if (ok && !pair) {
        tc::fence_after_sync();
        qk(0, 0);
        if (ntiles > 1) {
          ok = __all_sync(kAll, kv_ready(1));
          if (ok) {
            tc::fence_after_sync();
            qk(1, 1);
          }
        }
        for (int j = 0; j < ntiles && ok && !__any_sync(kAll, misc[1] != 0); ++j) {
          const int t = j & 1, i = j >> 1;   // stream, its step
          if (!__all_sync(kAll, mbar_wait(&p_ready[t], i & 1))) { ok = false; break; }
          const bool more = j + 2 < ntiles;
          if (more && !__all_sync(kAll, kv_ready(j + 2))) { ok = false; break; }
          tc::fence_after_sync();
          pv(t, j % STAGES, i == 0, true);
          if (more) qk(t, (j + 2) % STAGES);
          done = j + 1;
        }
      } else if (ok) {
        tc::fence_after_sync();
        qk(0, 0);
        qk(1, 0);
        for (int j = 0; j < ntiles && ok && !__any_sync(kAll, misc[1] != 0); ++j) {
          const int s = j % PAIR_STAGES, s1 = (j + 1) % PAIR_STAGES;
          if (j + 1 < ntiles && !__all_sync(kAll, kv_ready(j + 1))) { ok = false; break; }
#pragma unroll
          for (int t = 0; t < STREAMS; ++t) {
            if (j >= nks[t]) continue;
            if (!__all_sync(kAll, mbar_wait(&p_ready[t], j & 1))) { ok = false; break; }
            tc::fence_after_sync();
            // stream 1's tiles are a prefix of stream 0's: the last reader of
            // tile j is stream 1 while it still has tiles
            pv(t, s, j == 0, t == 1 || j >= nks[1]);
            if (j + 1 < nks[t]) qk(t, s1);
          }
          if (ok) done = j + 1;
        }
      }
      if (!ok && lane == 0) misc[1] = 1;
      // never exit with MMAs in flight or commit arrivals still pending
#pragma unroll
      for (int t = 0; t < STREAMS; ++t) {
        const int issued_t = pair ? (done < nks[t] ? done : nks[t]) : (done + 1 - t) / 2;
        if (issued_t > 0) mbar_wait(&o_done[t], (issued_t - 1) & 1);
      }
      for (int j = (done > nst ? done - nst : 0); j < done; ++j)
        mbar_wait(&kv_empty[j % nst], (j / nst) & 1);
    }
  } else {
    tc::regs_inc<REGS_SOFTMAX>();
    // ------------------------------------------------------ softmax
    const int t = wg;                                // stream of this warpgroup
    const int i = (warp & 3) * 32 + lane;            // row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + 128u * t;
    const uint32_t my_tile0 = t ? tile0[1] : tile0[0];
    const int my_nk = t ? nks[1] : nks[0];
    const uint32_t token = my_tile0 + (i >> 3);
    // Q rotation: split -- the two warpgroups rotate disjoint halves of the
    // shared tile's dims; pair -- each rotates its own tile.  The table
    // entries are fetched while the Q tiles are still in flight.
    uint8_t* qb0 = smem + OFF_Q + (pair ? t * Q_BYTES : 0);
    bool ok = true;
    {
      RowTables<4> rt;
      const int c0 = pair ? 0 : 4 * t;
      const float* rcos = pr.rope_cos[pi];
      const float* rsin = pr.rope_sin[pi];
      const uint32_t rrows = pr.rope_rows[pi];
      if (token < tokens) mrope_tables(rt, rcos, rsin, rrows, token, c0);
      ok = mbar_wait(q_full, 0);
      if (ok && token < tokens) {
        mrope_row(qb0, qb0 + SZ_W, i, rt, c0);
        if (pair) {
          mrope_tables(rt, rcos, rsin, rrows, token, 4);
          mrope_row(qb0, qb0 + SZ_W, i, rt, 4);
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_ready);
    if (!ok) misc[1] = 1;

    const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
    const uint64_t scale2 = f2_pack(scale, scale);
    float m_run = -CUDART_INF_F, l_run = 0.f;
    bool good = __all_sync(0xffffffffu, ok);
    // rows 32w'..32w'+31 of this warp hold tokens +4w' .. +4w'+3
    const uint32_t warp_tok_lo = my_tile0 + ((warp & 3) * 32 >> 3);
    const uint32_t tO = tmem + lane_base + 256u + 128u * t;
    // K tile of step `step`: step (pair) or 2 step + t (split)
    const int j0 = pair ? 0 : t, jstride = pair ? 1 : 2;
    for (int step = 0; step < my_nk && good; ++step) {
      const int j = j0 + jstride * step;
      if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&s_full[t], step & 1))) {
        good = false;
        break;
      }
      if (!softmax_step(tS, tO, j, token, warp_tok_lo, step > 0, &o_done[t], (step - 1) & 1,
                        scale, scale2, m_run, l_run)) {
        good = false;
        break;
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t]);
    }
    if (!good) misc[1] = 1;
    const bool fin = __all_sync(0xffffffffu,
                                good && (my_nk == 0 || mbar_wait(&o_done[t], (my_nk - 1) & 1)));
    const bool store = token < tokens;
    const bool two = nks[1] > 0;                     // stream 1 had work
    __half* orow = p.out + ((size_t)(row0 + token) * QH + GROUP * g + (i & 7)) * HD;
    if (pair) {
      // epilogue of a paired tile: this stream's O / l -> all 128 columns
      if (fin) {
        tc::fence_after_sync();
        const float inv = 1.f / l_run;
#pragma unroll
        for (int cc = 0; cc < 128; cc += 16) {
          uint32_t ov[16];
          tc::tmem_ld16(tO + cc, ov);
          tc::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(ov[8 * h + 0]) * inv, __uint_as_float(ov[8 * h + 1]) * inv);
            w.y = pack_half2(__uint_as_float(ov[8 * h + 2]) * inv, __uint_as_float(ov[8 * h + 3]) * inv);
            w.z = pack_half2(__uint_as_float(ov[8 * h + 4]) * inv, __uint_as_float(ov[8 * h + 5]) * inv);
            w.w = pack_half2(__uint_as_float(ov[8 * h + 6]) * inv, __uint_as_float(ov[8 * h + 7]) * inv);
            if (store) *reinterpret_cast<uint4*>(orow + cc + 8 * h) = w;
          }
        }
      } else {
        misc[1] = 1;
      }
    } else {
      // epilogue of a split tile: each warpgroup waits for its own stream's
      // last PV (its own o_done phases, which it tracks exactly) and posts
      // (m, l) in its stream's S columns, which no MMA touches after that PV;
      // ml_ready completing means both streams are done.  Then this
      // warpgroup writes output columns 64t..64t+63 =
      //   (O0 2^(m0-M) + O1 2^(m1-M)) / (l0 2^(m0-M) + l1 2^(m1-M))
      if (fin) {
        tc::fence_after_sync();
        uint32_t ml[16] = {};
        ml[0] = __float_as_uint(m_run);
        ml[1] = __float_as_uint(l_run);
        tc::tmem_st16(tS, ml);
        tc::tmem_wait_st();
        tc::fence_before_sync();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(ml_ready);
      if (__all_sync(0xffffffffu, fin && mbar_wait(ml_ready, 0))) {
        tc::fence_after_sync();
        uint32_t x0[16], x1[16];
        tc::tmem_ld16(tmem + lane_base, x0);           // stream 0's (m, l)
        tc::tmem_ld16(tmem + lane_base + 128u, x1);    // stream 1's (m, l)
        tc::tmem_wait_ld();
        const float m0 = __uint_as_float(x0[0]), l0 = __uint_as_float(x0[1]);
        const float m1 = two ? __uint_as_float(x1[0]) : -CUDART_INF_F;
        const float l1 = two ? __uint_as_float(x1[1]) : 0.f;
        const float M = fmaxf(m0, m1);
        const float f0 = m0 == -CUDART_INF_F ? 0.f : fast_exp2(m0 - M);
        const float f1 = m1 == -CUDART_INF_F ? 0.f : fast_exp2(m1 - M);
        const float inv = 1.f / (l0 * f0 + l1 * f1);
        const float a0 = f0 * inv, a1 = f1 * inv;
        const uint32_t tO0 = tmem + lane_base + 256u, tO1 = tmem + lane_base + 384u;
#pragma unroll
        for (int cc = 64 * t; cc < 64 * t + 64; cc += 16) {
          uint32_t o0[16], o1[16];
          tc::tmem_ld16(tO0 + cc, o0);
          if (two) tc::tmem_ld16(tO1 + cc, o1);
          tc::tmem_wait_ld();
          float v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            v[e] = __uint_as_float(o0[e]) * a0 + (two ? __uint_as_float(o1[e]) * a1 : 0.f);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 w;
            w.x = pack_half2(v[8 * h + 0], v[8 * h + 1]);
            w.y = pack_half2(v[8 * h + 2], v[8 * h + 3]);
            w.z = pack_half2(v[8 * h + 4], v[8 * h + 5]);
            w.w = pack_half2(v[8 * h + 6], v[8 * h + 7]);
            if (store) *reinterpret_cast<uint4*>(orow + cc + 8 * h) = w;
          }
        }
      } else {
        misc[1] = 1;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && misc[1]) atomicOr(&g_faults, PVLC_FAULT_PREFILL);
  if (warp == 8) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

inline uint32_t umin_host(uint32_t a, uint32_t b) { return a < b ? a : b; }

// ------------------------------------------------------------------------
// 3. Persistent attention for a batched launch.  One CTA per SM walks the
// work items (a prompt's adjacent Q tiles n-1-2r and n-2-2r, one per stream,
// sharing every K/V tile; an odd prompt's tile 0 alone on stream 0) in a
// static round-robin over an order that lists every prompt's heaviest items
// first.  Four warpgroups: the softmax of stream 0 and of stream 1; control
// (TMA producer warp, MMA warp); and a boundary warpgroup that takes the
// per-item work off the softmax warpgroups' chain: it applies M-RoPE to the
// next item's Q tiles as soon as they land, and writes each item's output
// (O from TMEM, divided by the row sums the softmax warpgroups leave in
// shared memory) while the softmax warpgroups already work on the next item.
// Barrier phases run on across items: the producer loads item n+1's Q tiles
// once the last QK of item n has completed for each stream (q_free); the
// first PV of item n+1 waits until the boundary warpgroup has read item n's
// O (o_free).  (With the rotation and the epilogue in the softmax
// warpgroups, removing either of them from the kernel had cut the batched
// launch by ~17 %.)
//
// Items: index x of [0, prompts * ranks_max * 2): prompt b = x / (2 ranks_max),
// rank r = (x / 2) mod ranks_max (the prompt's heaviest first), KV head
// g = x mod 2; a rank past the prompt's CTA count is empty and skipped.
// Prompt-major, so the CTAs working at one time share a few prompts' keys and
// values in L2: a rank-major order (every prompt's heaviest items first)
// spread them over the whole launch and measured 13 % slower (3.14 against
// 2.77 ms for 256 x 1238 tokens).
// output staging: one 64-dim half of a Q-tile-shaped output box (128 rows x
// 128 B, 128B-swizzled), written by the boundary warpgroup, stored by TMA
constexpr uint32_t OFF_STG_P = OFF_STAGE_PAIR + PAIR_STAGES * STAGE_BYTES;
constexpr uint32_t OFF_BARS_P = OFF_STG_P + SZ_W;
// q_full, q_ready, kv_full[2], kv_empty[2], s_full[2], p_ready[2], o_done[2], q_free[2],
// o_last, o_free, l_ready[2][2]
constexpr int NBARS_P = 20;
constexpr uint32_t OFF_L_P = OFF_BARS_P + NBARS_P * 8;       // row sums [2][2][128] f32
constexpr uint32_t OFF_MISC_P = OFF_L_P + 2 * STREAMS * 128 * 4;
constexpr uint32_t SMEM_BYTES_P = OFF_MISC_P + 64 + 1024;
// launch 512 x 128 registers, then per warpgroup: softmax 144, control 88,
// boundary 136 (set by setmaxnreg .inc / .dec from the launch count; the
// launch checks that the compiled kernel uses exactly LAUNCH_REGS_P)
constexpr int THREADS_P = 16 * 32;
constexpr uint32_t LAUNCH_REGS_P = 128;   // 65536 / THREADS_P
constexpr uint32_t REGS_SOFTMAX_P = 144, REGS_CTRL_P = 88, REGS_BOUND_P = 136;
static_assert(256 * REGS_SOFTMAX_P + 128 * (REGS_CTRL_P + REGS_BOUND_P) <= THREADS_P * LAUNCH_REGS_P,
              "persistent register split");
static_assert(LAUNCH_REGS_P * THREADS_P <= 65536, "persistent launch registers");
static_assert(SMEM_BYTES_P <= 227 * 1024, "persistent prefill shared memory exceeds the limit");

struct Item {
  uint32_t pi, g, row0, tokens;
  uint32_t tile0[STREAMS];
  int nks[STREAMS];   // K tiles of each stream (0: stream idle)
  bool valid;
};

template <int MAXB>
__device__ __forceinline__ Item item_at(uint32_t x, const Prompts<MAXB>& pr) {
  Item it;
  const uint32_t R = pr.ranks_max;
  it.pi = x / (2 * R);
  const uint32_t rem = x - it.pi * 2 * R;
  const uint32_t r = rem >> 1;
  it.g = rem & 1;
  it.row0 = pr.row0[it.pi];
  it.tokens = pr.row0[it.pi + 1] - it.row0;
  const uint32_t n_qt = (it.tokens + TOK - 1) / TOK;
  it.valid = r < pr.cta_prefix[it.pi + 1] - pr.cta_prefix[it.pi];
  it.tile0[0] = it.tile0[1] = 0;
  it.nks[0] = it.nks[1] = 0;
  if (!it.valid) return it;
  const uint32_t qa = n_qt - 1 - 2 * r;
  it.tile0[0] = qa * TOK;
  it.nks[0] = static_cast<int>((umin32(qa * TOK + TOK, it.tokens) - 1) / BN) + 1;
  if (qa >= 1) {
    const uint32_t qb = qa - 1;
    it.tile0[1] = qb * TOK;
    it.nks[1] = static_cast<int>((umin32(qb * TOK + TOK, it.tokens) - 1) / BN) + 1;
  }
  return it;
}

template <int MAXB>
__global__ void __launch_bounds__(THREADS_P, 1)
    prefill_persist_kernel(const __grid_constant__ Maps maps, const Params p,
                           const __grid_constant__ Prompts<MAXB> pr, uint32_t n_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BARS_P);
  uint64_t* q_full = bars + 0;
  uint64_t* q_ready = bars + 1;
  uint64_t* kv_full = bars + 2;    // [2]
  uint64_t* kv_empty = bars + 4;   // [2]
  uint64_t* s_full = bars + 6;     // [2] per stream
  uint64_t* p_ready = bars + 8;    // [2]
  uint64_t* o_done = bars + 10;    // [2]
  uint64_t* q_free = bars + 12;    // [2] the item's last QK of the stream is complete
  uint64_t* o_last = bars + 14;    // every PV of the item is complete
  uint64_t* o_free = bars + 15;    // the boundary warpgroup has read the item's O
  // [stream][parity of the stream's active-item count]: that item's row sums are in l_sm
  uint64_t* l_ready = bars + 16;
  float* l_sm = reinterpret_cast<float*>(smem + OFF_L_P);   // [stream][parity][row]
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC_P);
  // misc[0]: TMEM base, misc[1]: abort

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t first_x = blockIdx.x, step_x = gridDim.x;
  // the next valid item index at or after x (n_items when none)
  auto next_item = [&](uint32_t x) -> uint32_t {
    while (x < n_items && !item_at<MAXB>(x, pr).valid) x += step_x;
    return x < n_items ? x : n_items;
  };

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < STREAMS; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_done[t], 1);
      mbar_init(&q_free[t], 1);
      mbar_init(&l_ready[2 * t], 4);
      mbar_init(&l_ready[2 * t + 1], 4);
    }
    mbar_init(o_last, 1);
    mbar_init(o_free, 4);
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

  const int wg = warp >> 2;
  if (wg == 2) {
    tc::regs_to<LAUNCH_REGS_P, REGS_CTRL_P>();
    if (warp == 8 && lane == 0) {
      // ---------------------------------------------------- TMA producer
      tc::tma_prefetch_desc(&maps.q);
      tc::tma_prefetch_desc(&maps.k);
      tc::tma_prefetch_desc(&maps.v);
      bool waited = false;     // pdl_wait done (keys come from the preceding kv_rope_kernel)
      uint32_t G = 0;          // K/V tiles loaded so far (ring position)
      uint32_t n = 0;          // items so far
      for (uint32_t x = next_item(first_x); x < n_items && !misc[1];
           x = next_item(x + step_x), ++n) {
        const Item it = item_at<MAXB>(x, pr);
        if (n > 0 && (!mbar_wait(&q_free[0], (n - 1) & 1) || !mbar_wait(&q_free[1], (n - 1) & 1))) {
          misc[1] = 1;
          break;
        }
        const int nq = it.nks[1] > 0 ? 2 : 1;
        mbar_arrive_expect_tx(q_full, nq * Q_BYTES);
        for (int t = 0; t < nq; ++t)
          for (int b = 0; b < 2; ++b)
            tc::tma_load_3d(smem + OFF_Q + t * Q_BYTES + b * SZ_W, &maps.q, 64 * b,
                            GROUP * it.g, it.row0 + it.tile0[t], q_full);
        if (!waited) {
          pdl_wait();
          waited = true;
        }
        for (int j = 0; j < it.nks[0]; ++j, ++G) {
          const int s = G % PAIR_STAGES;
          if (misc[1] || !mbar_wait(&kv_empty[s], ((G / PAIR_STAGES) & 1) ^ 1)) {
            misc[1] = 1;
            break;
          }
          uint8_t* st = smem + OFF_STAGE_PAIR + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&kv_full[s], STAGE_BYTES);
          for (int b = 0; b < 2; ++b) {
            tc::tma_load_4d(st + ST_K + b * SZ_W, &maps.k, 64 * b, it.g, j * BN, it.pi,
                            &kv_full[s]);
            tc::tma_load_3d(st + ST_V + b * SZ_W, &maps.v, 64 * b, it.g, it.row0 + j * BN,
                            &kv_full[s]);
          }
        }
      }
      // the last loads must land before the CTA may exit
      for (uint32_t g2 = (G > PAIR_STAGES ? G - PAIR_STAGES : 0); g2 < G; ++g2)
        mbar_wait(&kv_full[g2 % PAIR_STAGES], (g2 / PAIR_STAGES) & 1);
      if (n > 0) mbar_wait(q_full, (n - 1) & 1);
    } else if (warp == 9) {
      // ---------------------------------------------------- MMA issuer
      // per item: both streams' first QK, then per K tile j and stream the PV of
      // tile j and the QK of tile j + 1; q_free[t] is committed right after the
      // stream's last QK of the item (its Q buffer may then be refilled), o_last
      // after the item's last PV; the item's first PV waits until the boundary
      // warpgroup has read the previous item's O (o_free)
      constexpr uint32_t idesc_qk = tc::idesc_f16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = tc::idesc_f16(128, 128, 0, 1);
      const uint32_t sq = smem_u32(smem + OFF_Q), st0 = smem_u32(smem + OFF_STAGE_PAIR);
      const uint64_t dq = tc::smem_desc(sq, 16, 1024, tc::kSw128);
      const uint64_t dk = tc::smem_desc(st0 + ST_K, 16, 1024, tc::kSw128);
      const uint64_t dv = tc::smem_desc(st0 + ST_V, SZ_W, 1024, tc::kSw128);
      auto qk = [&](int t, int s) {
        const uint32_t tS = tmem + 128u * t;
        const uint64_t so = (uint64_t)s * (STAGE_BYTES >> 4);
        const uint64_t qo = (uint64_t)t * (Q_BYTES >> 4);
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t off = (uint64_t)(ks >> 2) * (SZ_W >> 4) + 2 * (ks & 3);
            tc::mma_ss(tS, dq + qo + off, dk + so + off, idesc_qk, ks > 0);
          }
          tc::commit(&s_full[t]);
        }
        __syncwarp();
      };
      auto pv = [&](int t, int s, bool first, bool release) {
        const uint32_t tS = tmem + 128u * t, tO = tmem + 256u + 128u * t;
        const uint64_t so = (uint64_t)s * (STAGE_BYTES >> 4);
        if (tc::elect_one()) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            tc::mma_ts(tO, tS + ks * 8, dv + so + 128 * ks, idesc_pv, (!first || ks > 0) ? 1u : 0u);
          tc::commit(&o_done[t]);
          if (release) tc::commit(&kv_empty[s]);
        }
        __syncwarp();
      };
      auto commit_to = [&](uint64_t* bar) {
        if (tc::elect_one()) tc::commit(bar);
        __syncwarp();
      };
      constexpr uint32_t kAll = 0xffffffffu;
      uint32_t G = 0;                        // K/V tiles consumed so far
      uint32_t steps[STREAMS] = {0, 0};      // P hand-offs (= PVs issued) per stream so far
      uint32_t n = 0;
      bool ok = true;
      for (uint32_t x = next_item(first_x); x < n_items && ok; x = next_item(x + step_x), ++n) {
        const Item it = item_at<MAXB>(x, pr);
        const int nk = it.nks[0];
        ok = __all_sync(kAll, misc[1] == 0 && mbar_wait(q_ready, n & 1) &&
                                  mbar_wait(&kv_full[G % PAIR_STAGES], (G / PAIR_STAGES) & 1));
        if (!ok) break;
        tc::fence_after_sync();
        const int s0 = G % PAIR_STAGES;
        qk(0, s0);
        if (nk == 1) commit_to(&q_free[0]);
        if (it.nks[1] > 0) {
          qk(1, s0);
          if (it.nks[1] == 1) commit_to(&q_free[1]);
        } else {
          commit_to(&q_free[1]);   // stream 1 idle in this item
        }
        for (int j = 0; j < nk && ok; ++j) {
          const int s = (G + j) % PAIR_STAGES, s1 = (G + j + 1) % PAIR_STAGES;
          const uint32_t gn = G + j + 1;
          if (j + 1 < nk &&
              !__all_sync(kAll, misc[1] == 0 &&
                                    mbar_wait(&kv_full[s1], (gn / PAIR_STAGES) & 1))) {
            ok = false;
            break;
          }
#pragma unroll
          for (int t = 0; t < STREAMS; ++t) {
            if (j >= it.nks[t]) continue;
            if (!__all_sync(kAll, mbar_wait(&p_ready[t], steps[t] & 1))) { ok = false; break; }
            if (j == 0 && t == 0 && n > 0 &&
                !__all_sync(kAll, mbar_wait(o_free, (n - 1) & 1))) {
              ok = false;
              break;
            }
            ++steps[t];
            tc::fence_after_sync();
            // stream 1's tiles are a prefix of stream 0's: the last reader of
            // tile j is stream 1 while it still has tiles
            pv(t, s, j == 0, t == 1 || j >= it.nks[1]);
            if (j + 1 < it.nks[t]) {
              qk(t, s1);
              if (j + 2 == it.nks[t]) commit_to(&q_free[t]);
            }
          }
        }
        if (ok) {
          commit_to(o_last);
          G += nk;
        }
      }
      if (!ok && lane == 0) misc[1] = 1;
      // never exit with MMAs in flight or commit arrivals still pending
#pragma unroll
      for (int t = 0; t < STREAMS; ++t)
        if (steps[t] > 0) mbar_wait(&o_done[t], (steps[t] - 1) & 1);
      if (n > 0) {
        mbar_wait(&q_free[0], (n - 1) & 1);
        mbar_wait(&q_free[1], (n - 1) & 1);
        if (ok) mbar_wait(o_last, (n - 1) & 1);
      }
    }
  } else if (wg == 3) {
    tc::regs_to<LAUNCH_REGS_P, REGS_BOUND_P>();
    // ------------------------------------------------------ boundary
    const int i = (warp & 3) * 32 + lane;            // row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    // M-RoPE by (token, chunk): thread i takes token slot i / 8 and chunk
    // i % 8 (dims 8c..8c+7 and their partners 64 above) of both streams'
    // tiles, so one set of table entries serves the 8 heads' rows of the
    // token; the entries are loaded before waiting for the tiles to land.
    auto rotate = [&](const Item& it, uint32_t ph) -> bool {
      const int u = i >> 3, c = i & 7;
      const uint32_t axis = mrope_axis(8 * c);   // section edges are multiples of 8
      const uint32_t rr = pr.rope_rows[it.pi];
      float4 tv[STREAMS][8];
      bool mine[STREAMS];
#pragma unroll
      for (int t = 0; t < STREAMS; ++t) {
        const uint32_t token = it.tile0[t] + u;
        mine[t] = it.nks[t] > 0 && token < it.tokens;
        if (mine[t]) {
          const size_t tb = ((size_t)axis * rr + token) * HD + 8 * c;
          const float4* cs = reinterpret_cast<const float4*>(pr.rope_cos[it.pi] + tb);
          const float4* sn = reinterpret_cast<const float4*>(pr.rope_sin[it.pi] + tb);
          tv[t][0] = __ldg(cs);
          tv[t][1] = __ldg(cs + 1);
          tv[t][2] = __ldg(cs + 16);
          tv[t][3] = __ldg(cs + 17);
          tv[t][4] = __ldg(sn);
          tv[t][5] = __ldg(sn + 1);
          tv[t][6] = __ldg(sn + 16);
          tv[t][7] = __ldg(sn + 17);
        }
      }
      const bool landed = mbar_wait(q_full, ph);
      if (landed) {
#pragma unroll
        for (int t = 0; t < STREAMS; ++t) {
          if (!mine[t]) continue;
          uint8_t* qb = smem + OFF_Q + t * Q_BYTES;
#pragma unroll
          for (int h = 0; h < GROUP; ++h) rope_chunk(qb, qb + SZ_W, u * GROUP + h, c, tv[t]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
      return landed;
    };
    if (i == 0) tc::tma_prefetch_desc(&maps.o);
    uint32_t n = 0;
    uint32_t na[STREAMS] = {0, 0};   // active items per stream so far (l_ready slots)
    uint32_t x = next_item(first_x);
    // The four warps meet on named barrier 1 around every staging-buffer
    // use, and a bar.sync has no time limit: so every outcome that can end
    // the loop (a bounded wait, the abort flag) is agreed on by all four
    // warps through named barrier 2 (bar.red.and) first, and they leave
    // together.
    auto agree = [&](bool ok) { return named_bar_and(2, 128, ok); };
    bool good = x >= n_items || agree(rotate(item_at<MAXB>(x, pr), 0));
    for (; x < n_items && good; ++n) {
      const Item it = item_at<MAXB>(x, pr);
      const uint32_t xn = next_item(x + step_x);
      // the next item's Q first: its first QKs then run during this epilogue
      if (xn < n_items && !agree(rotate(item_at<MAXB>(xn, pr), (n + 1) & 1))) {
        good = false;
        break;
      }
      if (!agree(misc[1] == 0 && mbar_wait(o_last, n & 1))) {
        good = false;
        break;
      }
      tc::fence_after_sync();
      // O of each active stream in two 64-column halves; the accumulators are
      // released (o_free) once the last half is in registers.  A full Q tile
      // goes out through the staging buffer and one TMA store per half
      // (coalesced: each token's 8 heads are 2 KB of contiguous output); the
      // last tile of a prompt, whose box would reach into the next prompt's
      // rows, is stored row by row.  Row sums are counted per active item of
      // a stream: the warpgroup of a stream that is idle in an item passes it
      // without waiting for anything, so it may run one active item ahead.
      const int last_t = it.nks[1] > 0 ? 1 : 0;
      uint8_t* stg = smem + OFF_STG_P;
#pragma unroll 1
      for (int t = 0; t <= last_t && good; ++t) {
        const uint32_t slot = 2 * t + (na[t] & 1);
        if (!agree(mbar_wait(&l_ready[slot], (na[t] >> 1) & 1))) {
          good = false;
          break;
        }
        ++na[t];
        const uint32_t token = it.tile0[t] + (i >> 3);
        const bool full = it.tile0[t] + TOK <= it.tokens;
        const bool store = token < it.tokens;
        const float inv = 1.f / l_sm[slot * 128 + i];
        __half* orow = p.out + ((size_t)(it.row0 + token) * QH + GROUP * it.g + (i & 7)) * HD;
        const uint32_t tO = tmem + lane_base + 256u + 128u * t;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint32_t ov[32];
            tc::tmem_ld32(tO + 64 * half + 32 * q, ov);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[16 * q + e] =
                  pack_half2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
          }
          if (t == last_t && half == 1) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
          }
          if (full) {
            // the previous store has read the staging buffer
            if (i == 0) tc::bulk_wait_read_all();
            named_bar_sync(1, 128);
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(chunk_addr(stg, i, c)) =
                  make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_proxy_async_smem();
            named_bar_sync(1, 128);
            if (i == 0) {
              tc::tma_store_3d(&maps.o, stg, 64 * half, GROUP * it.g, it.row0 + it.tile0[t]);
              tc::bulk_commit_group();
            }
          } else if (store) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(orow + 64 * half + 8 * c) =
                  make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          }
        }
      }
      if (!good) break;
      x = xn;
    }
    if (i == 0) tc::bulk_wait_all();   // no store may still read the staging buffer at exit
    if (!good) misc[1] = 1;
  } else {
    tc::regs_to<LAUNCH_REGS_P, REGS_SOFTMAX_P>();
    // ------------------------------------------------------ softmax
    const int t = wg;                                // stream of this warpgroup
    const int i = (warp & 3) * 32 + lane;            // row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + 128u * t;
    const uint32_t tO = tmem + lane_base + 256u + 128u * t;
    const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
    const uint64_t scale2 = f2_pack(scale, scale);
    uint32_t step_g = 0;     // this stream's steps so far (s_full / p_ready / o_done phases)
    uint32_t na = 0;         // this stream's active items so far (l_ready slots)
    bool good = true;
    for (uint32_t x = next_item(first_x); x < n_items && good; x = next_item(x + step_x)) {
      const Item it = item_at<MAXB>(x, pr);
      const int my_nk = it.nks[t];
      if (my_nk == 0) continue;
      const uint32_t token = it.tile0[t] + (i >> 3);
      const uint32_t warp_tok_lo = it.tile0[t] + ((warp & 3) * 32 >> 3);
      float m_run = -CUDART_INF_F, l_run = 0.f;
      for (int step = 0; step < my_nk && good; ++step, ++step_g) {
        if (!__all_sync(0xffffffffu, misc[1] == 0 && mbar_wait(&s_full[t], step_g & 1))) {
          good = false;
          break;
        }
        if (!softmax_step(tS, tO, step, token, warp_tok_lo, step > 0, &o_done[t],
                          (step_g - 1) & 1, scale, scale2, m_run, l_run)) {
          good = false;
          break;
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[t]);
      }
      if (!good) break;
      // the row sums for the boundary warpgroup's epilogue
      const uint32_t slot = 2 * t + (na & 1);
      l_sm[slot * 128 + i] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_ready[slot]);
      ++na;
    }
    if (!good) misc[1] = 1;
  }

  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0 && misc[1]) atomicOr(&g_faults, PVLC_FAULT_PREFILL_BATCH);
  if (warp == 8) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, TMEM_COLS);
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

// [rows, heads, 128] fp16 as a 3-D tensor {128, heads, rows}; box
// {64 dims, box_heads, box_rows}, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, uint32_t rows, uint32_t heads,
              uint32_t box_heads, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {HD, heads, rows};
  const cuuint64_t strides[2] = {HD * 2, (cuuint64_t)heads * HD * 2};
  const cuuint32_t box[3] = {64, box_heads, box_rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The caches of `prompts` prompts, prompt b's [capacity, 2, 128] fp16 at
// base + b * prompt_stride elements, as a 4-D tensor {128, 2, capacity,
// prompts}; box {64 dims, 1 head, 128 keys, 1 prompt}, 128B swizzle.
bool make_cache_map(CUtensorMap* m, const void* base, uint32_t capacity, uint32_t prompts,
                    uint64_t prompt_stride) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[4] = {HD, KVH, capacity, prompts};
  const cuuint64_t strides[3] = {HD * 2, (cuuint64_t)KVH * HD * 2, prompt_stride * 2};
  const cuuint32_t box[4] = {64, 1, BN, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// kv_rope_kernel then the attention: prefill_attn_kernel (grid_y CTAs per KV
// head) or, when `persist_items` is nonzero, prefill_persist_kernel over that
// many item slots with one CTA per SM (programmatic dependent launch either way).
template <int MAXB>
int launch(const void* q, const void* k, const void* v, uint32_t rows, const Prompts<MAXB>& pr,
           Params p, uint32_t capacity, uint32_t grid_y, cudaStream_t stream,
           uint32_t persist_items = 0) {
  if (persist_items) {
    if (set_smem_attribute_once(reinterpret_cast<const void*>(prefill_persist_kernel<MAXB>),
                                SMEM_BYTES_P) != PVLC_OK)
      return PVLC_CUDA_ERROR;
    // the warpgroups' setmaxnreg counts assume this launch register count
    static const int launch_regs = [] {
      cudaFuncAttributes fa;
      return cudaFuncGetAttributes(&fa, prefill_persist_kernel<MAXB>) == cudaSuccess ? fa.numRegs
                                                                                    : -1;
    }();
    if (launch_regs != static_cast<int>(LAUNCH_REGS_P)) return PVLC_CUDA_ERROR;
  } else if (set_smem_attribute_once(reinterpret_cast<const void*>(prefill_attn_kernel<MAXB>),
                                     SMEM_BYTES) != PVLC_OK) {
    return PVLC_CUDA_ERROR;
  }
  if (grid_y == 0 || grid_y > 65535u) return PVLC_INVALID_DECODER_GEOMETRY;
  Maps maps;
  // keys come from the caches (rotated by kv_rope_kernel): rows past a
  // prompt are masked, rows past the capacity are TMA zero fill; values come
  // from the packed input rows
  if (!make_map(&maps.q, q, rows, QH, GROUP, TOK) ||
      (persist_items && !make_map(&maps.o, p.out, rows, QH, GROUP, TOK)) ||
      !make_cache_map(&maps.k, p.k_cache, capacity, pr.count, p.cache_stride) ||
      !make_map(&maps.v, v, rows, KVH, 1, BN))
    return PVLC_CUDA_ERROR;
  const uint64_t rope_threads = (uint64_t)rows * KVH * 8;
  kv_rope_kernel<MAXB><<<(unsigned)((rope_threads + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __half*>(k), reinterpret_cast<const __half*>(v), pr, p);
  if (cudaPeekAtLastError() != cudaSuccess) return PVLC_CUDA_ERROR;
  // programmatic dependent launch: the attention CTAs' prologue overlaps
  // kv_rope_kernel; only their cache reads wait for it (pdl_wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(KVH, grid_y);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (persist_items) {
    const int sms = device_sm_count();
    if (sms <= 0) return PVLC_CUDA_ERROR;
    const uint32_t ctas = umin_host(static_cast<uint32_t>(sms), 2 * grid_y);
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(THREADS_P);
    cfg.dynamicSmemBytes = SMEM_BYTES_P;
    if (cudaLaunchKernelEx(&cfg, prefill_persist_kernel<MAXB>, maps, p, pr, persist_items) !=
        cudaSuccess)
      return PVLC_CUDA_ERROR;
  } else if (cudaLaunchKernelEx(&cfg, prefill_attn_kernel<MAXB>, maps, p, pr) != cudaSuccess) {
    return PVLC_CUDA_ERROR;
  }
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // namespace ptc

int prefill_fault_word(uint32_t* out, cudaStream_t s) {
  uint32_t v = 0;
  const uint32_t zero = 0;
  if (cudaMemcpyFromSymbolAsync(&v, ptc::g_faults, 4, 0, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaMemcpyToSymbolAsync(ptc::g_faults, &zero, 4, 0, cudaMemcpyHostToDevice, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  *out = v;
  return PVLC_OK;
}

int prefill_query_tile() { return ptc::QT * ptc::TOK; }

// Q tiles per KV head, split into the heaviest (one CTA each, K range split
// between the two streams) and the lightest (paired two per CTA).  Pairing
// is used only where it makes the CTAs of both KV heads one wave of `sms`
// AND each pair's heavier tile, whose K tiles one stream walks alone, ends no
// later than the heaviest split CTA (ceil(nk_max / 2) steps); otherwise every
// Q tile is a split CTA and the grid runs in several waves, heaviest first.
// (Pairing a long tile with a 1-tile one at T = 4100 ran its 32 K tiles on
// one stream: 109 us per call against ~86 us for the split waves.)
void prefill_schedule(uint32_t tokens, int sms, uint32_t* n_split, uint32_t* n_light) {
  const uint32_t n_qt = (tokens + ptc::TOK - 1) / ptc::TOK;
  const uint32_t per_head = sms > 0 ? (uint32_t)sms / ptc::KVH : n_qt;
  uint32_t light = 0;
  if (n_qt > per_head && 2 * (n_qt - per_head) <= n_qt) {
    const uint32_t l1 = 2 * (n_qt - per_head);
    const uint32_t nk_pair = ((l1 - 1) * ptc::TOK + ptc::TOK - 1) / ptc::BN + 1;
    const uint32_t nk_max = (tokens - 1) / ptc::BN + 1;
    if (nk_pair <= (nk_max + 1) / 2) light = l1;
  }
  *n_light = light;
  *n_split = n_qt - light;
}
int prefill_block_threads() { return ptc::THREADS; }

int prefill_launch(const PrefillArgs& a, cudaStream_t stream) {
  ptc::Prompts<1> pr{};
  pr.count = 1;
  pr.row0[0] = 0;
  pr.row0[1] = a.tokens;
  pr.cta_prefix[0] = 0;
  pr.rope_rows[0] = a.rope_rows;
  pr.rope_cos[0] = a.rope_cos;
  pr.rope_sin[0] = a.rope_sin;
  ptc::Params p{};
  p.cache_stride = (uint64_t)a.capacity * ptc::KVH * ptc::HD;
  p.k_cache = reinterpret_cast<__half*>(a.k_cache);
  p.v_cache = reinterpret_cast<__half*>(a.v_cache);
  p.out = reinterpret_cast<__half*>(a.out);
  // one wave: pair the lightest Q tiles so that the CTAs fit the SMs
  const int sms = device_sm_count();
  if (sms <= 0) return PVLC_CUDA_ERROR;
  prefill_schedule(a.tokens, sms, &p.n_split, &p.n_light);
  pr.cta_prefix[1] = p.n_split + p.n_light / 2;
  return ptc::launch<1>(a.q, a.k, a.v, a.tokens, pr, p, a.capacity, p.n_split + p.n_light / 2,
                        stream);
}

int prefill_batch_launch(const PrefillBatchArgs& a, cudaStream_t stream) {
  static_assert(PVLC_PREFILL_MAX_PROMPTS <= 1024, "prompt table size");
  ptc::Prompts<PVLC_PREFILL_MAX_PROMPTS> pr{};
  pr.count = a.prompts;
  uint32_t ctas = 0;
  for (uint32_t b = 0; b < a.prompts; ++b) {
    const uint32_t t = a.offsets[b + 1] - a.offsets[b];
    pr.row0[b] = a.offsets[b];
    pr.cta_prefix[b] = ctas;
    ctas += ((t + ptc::TOK - 1) / ptc::TOK + 1) / 2;   // adjacent Q tiles paired
    pr.rope_rows[b] = a.rope_rows[b];
    pr.rope_cos[b] = a.rope_cos[b];
    pr.rope_sin[b] = a.rope_sin[b];
  }
  pr.row0[a.prompts] = a.offsets[a.prompts];
  pr.cta_prefix[a.prompts] = ctas;
  ptc::Params p{};
  p.cache_stride = a.cache_stride;
  p.k_cache = reinterpret_cast<__half*>(a.k_cache);
  p.v_cache = reinterpret_cast<__half*>(a.v_cache);
  p.out = reinterpret_cast<__half*>(a.out);
#if PVLC_PREFILL_PERSIST
  // item slots of the persistent kernel: ranks (CTA count of the longest prompt) x
  // prompts x KV heads
  uint32_t ranks = 0;
  for (uint32_t b = 0; b < a.prompts; ++b)
    ranks = ranks > pr.cta_prefix[b + 1] - pr.cta_prefix[b] ? ranks
                                                            : pr.cta_prefix[b + 1] - pr.cta_prefix[b];
  const uint32_t items = ranks * a.prompts * ptc::KVH;
  pr.ranks_max = ranks;
  return ptc::launch<PVLC_PREFILL_MAX_PROMPTS>(a.q, a.k, a.v, a.offsets[a.prompts], pr, p,
                                               a.capacity, ctas, stream, items);
#else
  return ptc::launch<PVLC_PREFILL_MAX_PROMPTS>(a.q, a.k, a.v, a.offsets[a.prompts], pr, p,
                                               a.capacity, ctas, stream);
#endif
}

}  // namespace pvlc
