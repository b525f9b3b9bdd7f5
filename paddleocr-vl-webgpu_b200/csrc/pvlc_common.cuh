// pvlc_common.cuh -- device helpers shared by the attention kernels (sm_100a).
//
// Inline-PTX wrappers for mbarriers, bulk async copies, ldmatrix, mma.sync,
// movmatrix, plus bounded waits: every spin on an mbarrier gives up after a
// fixed wall-clock budget (%globaltimer), records a flag and lets the kernel
// drain and return instead of hanging the GPU.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace pvlc {

// Wall-clock limit of any single wait inside a kernel (nanoseconds).
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// Fault flags written into a workspace word (bit positions are ABI).
constexpr uint32_t kFlagCacheRow = 1u << 0;
constexpr uint32_t kFlagRopeRow = 1u << 1;
constexpr uint32_t kFlagMisaligned = 1u << 2;
constexpr uint32_t kFlagTimeout = 1u << 3;

__device__ __forceinline__ uint32_t umin32(uint32_t a, uint32_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity` to complete.  Returns false when the
// wall-clock budget ran out (the caller records kFlagTimeout and bails out).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) return false;
  }
}

// Prefetch the 128-byte line holding `p` into L2 (no register result).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Bulk L2 prefetch of `bytes` (a multiple of 16) from a 16-byte aligned global
// address: one instruction for a whole contiguous range.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ------------------------------------------------------ bulk async copies
// 1-D bulk copy global -> shared, completion signalled on `bar` (tx bytes).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte global -> shared copy through L2 only (LDGSTS .cg).
__device__ __forceinline__ void cp_async_16(uint32_t smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_dst), "l"(gmem_src)
               : "memory");
}

// Arrive on `bar` once all of this thread's earlier cp.async copies have
// landed; the arrival counts against the barrier's expected count.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ------------------------------------------------------------ tensor core
__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                          uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x1(uint32_t& r0, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(r0) : "r"(addr));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
__device__ __forceinline__ void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 f32) += A(16x8 f16, row) * B(8x8 f16, col)
__device__ __forceinline__ void mma_1688(float* d, uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// Transpose an 8x8 b16 fragment held across the warp (ldmatrix layout).
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// SiLU of the decoder MLP gate, g / (1 + e^(-g))
// (crates/pvlc-cpu-ref/src/lib.rs:354-357), with the hardware base-2
// exponential and reciprocal; shared by the SiLU-gate glue kernel and the
// fused gate epilogue of the decode-step projections.
__device__ __forceinline__ float silu(float g) {
  return g * rcp_approx(1.f + fast_exp2(g * -1.4426950408889634f));
}

// Packed f32x2 arithmetic (one instruction for two lanes of a pair).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// acc_lo += low half of h2, acc_hi += high half: each fp16 half widened
// exactly and added in f32 with one rounding (the sm_100 mixed-precision add,
// one instruction per value), so the sums equal widen-then-add bit for bit.
__device__ __forceinline__ void add_f16x2_to_f32(uint32_t h2, float& acc_lo, float& acc_hi) {
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "add.rn.f32.f16 %0, lo, %0;\n\t"
      "add.rn.f32.f16 %1, hi, %1;\n\t}"
      : "+f"(acc_lo), "+f"(acc_hi)
      : "r"(h2));
}

// Packed half-precision 2^x (one MUFU operation for two values).
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// 2^x for a pair of f32 exponents, returned as fp16x2 bits, computed on the
// FMA and integer pipes only (no MUFU, no f32 -> f16 conversion), so that a
// kernel can split its exponentials between this and ex2_h2.  The argument is
// xs = x + 6.5 (callers fold the 6.5 into their shift): the fp16 bits of
// 2^(x + 7) are built first, where x + 7 >= -14 stays in the normal fp16
// range, and one f16x2 multiply by 2^-7 brings them down, rounding into the
// subnormal range where 2^x < 2^-14 (gradual underflow, as ex2_h2 gives).
//   j = round-to-nearest(xs) = floor(x + 7), via the 1.5 * 2^23 rounding constant;
//   g = xs - j in [-0.5, 0.5];
//   2^(g + 0.5) by a degree-3 minimax polynomial (relative error 7.5e-5 on
//   [-0.5, 0.5], Remez exchange), evaluated scaled by 1024 with
//   2^23 + 15 * 1024 - 1024 added, so the last fused multiply-add rounds the
//   10-bit fp16 mantissa (plus the exponent bias 15 << 10) into the low bits
//   of its f32 result; a carry out of the mantissa bumps the exponent, as it
//   should.  The fp16 exponent j is then added as an integer (j << 10).
// Results are within one fp16 ulp of 2^x for x >= -21 (subnormal ulps below
// 2^-14); x <= -22 gives exactly 0.  Valid for x <= 8 (2^(x + 7) <= 2^15).
__device__ __forceinline__ uint32_t exp2_h2_poly(uint64_t xs2) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr float kA3 = 79.89711f, kA2 = 351.33844f, kA1 = 1003.94916f, kA0 = 8404392.f;
  constexpr uint32_t kPow2m7x2 = 0x20002000u;   // fp16x2 {2^-7, 2^-7}
  float2 xh = f2_unpack(xs2);
  xh.x = fmaxf(xh.x, -15.5f);
  xh.y = fmaxf(xh.y, -15.5f);
  const uint64_t x2 = f2_pack(xh.x, xh.y);
  const uint64_t t2 = f2_add(x2, f2_pack(kRound, kRound));
  const uint64_t j2 = f2_add(t2, f2_pack(-kRound, -kRound));
  const uint64_t g2 = f2_fma(j2, f2_pack(-1.f, -1.f), x2);
  uint64_t q2 = f2_fma(f2_pack(kA3, kA3), g2, f2_pack(kA2, kA2));
  q2 = f2_fma(q2, g2, f2_pack(kA1, kA1));
  q2 = f2_fma(q2, g2, f2_pack(kA0, kA0));
  uint32_t t0, t1, q0, q1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(t0), "=r"(t1) : "l"(t2));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(q0), "=r"(q1) : "l"(q2));
  // low 16 bits: (j << 10) + (15 << 10) + mantissa; the high halves are dropped
  const uint32_t up = __byte_perm(t0 * 1024u + q0, t1 * 1024u + q1, 0x5410);
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(up), "r"(kPow2m7x2));
  return r;
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the preceding kernel of its
// stream still runs, once every CTA of that kernel has called
// pdl_launch_dependents (or exited); it must call pdl_wait before it reads
// anything the preceding kernel writes, which returns once that kernel has
// completed and its memory is visible.  Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `threads` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ANDs a predicate over its `threads` threads: every
// thread gets the same answer, so warps that go on to meet on other named
// barriers all take the same branch after it.
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// Select the M-RoPE axis plane for head dimension d of a 128-wide head:
// sections [16, 24, 24] repeated on both halves
// (crates/pvlc-cpu-ref/src/lib.rs:613-643, crates/pvlc-wgsl/src/lib.rs:1218-1220).
__device__ __forceinline__ uint32_t mrope_axis(uint32_t d) {
  const uint32_t local = d & 63u;
  return local < 16u ? 0u : (local < 40u ? 1u : 2u);
}

}  // namespace pvlc
