// blake3.cu -- BLAKE3 digests of device buffers (sm_100a): the section
// checksums of the reference's .pvlc model packs (crates/pvlc-pack/src/lib.rs:
// every directory entry carries blake3(section bytes), checked by
// PackReader::open), computed where the weights already sit, in HBM.
//
// BLAKE3 as published (Aumasson, Neves, O'Connor, Wilcox-O'Hearn): 1024-byte
// chunks of 64-byte blocks, each block compressed by 7 rounds of the G mixing
// function over a 16-word state (the chaining value, the first four IV words,
// the 64-bit counter, the block length and the domain flags), the message
// words permuted between rounds; chunk chaining values are merged pairwise by
// parent compressions (flag PARENT) in a binary tree whose left subtrees are
// complete (2^k chunks), and the last compression carries flag ROOT.  Plain
// hash mode: the key is the IV (the SHA-256 initial hash values).
//
// Work split: one thread per chunk (16 dependent compressions, the block's
// 64 bytes read as four 16-byte loads), then one launch per tree level, one
// thread per parent.  Pairing adjacent nodes level by level, an odd last node
// carried up unchanged, builds exactly the tree above (the left subtree of
// any node is the largest power of two of chunks that leaves at least one
// for the right).  The compression is integer-ALU bound: ~12 32-bit
// operations per input byte.
#include <cuda_runtime.h>
#include <stdint.h>

#include "pvlc_internal.h"

namespace pvlc {
namespace b3 {

constexpr uint32_t CHUNK = 1024, BLOCK = 64;
constexpr uint32_t CHUNK_START = 1, CHUNK_END = 2, PARENT = 4, ROOT = 8;

__host__ __device__ constexpr uint32_t iv(int i) {
  return i == 0 ? 0x6A09E667u : i == 1 ? 0xBB67AE85u : i == 2 ? 0x3C6EF372u : i == 3 ? 0xA54FF53Au
       : i == 4 ? 0x510E527Fu : i == 5 ? 0x9B05688Cu : i == 6 ? 0x1F83D9ABu : 0x5BE0CD19u;
}

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

// x + y as a multiply-add by a run-time 1 (`one`, a kernel argument the
// compiler cannot fold), which issues to the FMA pipe instead of the integer
// ALU that the XORs, rotates and three-input adds saturate.
__device__ __forceinline__ uint32_t add_fma(uint32_t x, uint32_t y, uint32_t one) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(one), "r"(y));
  return r;
}

// Which additions go to the FMA pipe: 0 none, 1 the two-operand ones, 2 all
// (the three-operand a + b + m as two multiply-adds).  Measured on 1 GiB:
// 1596, 1561 and 1682 GB/s; ncu of form 0 shows the integer ALU pipe 97 % busy
// and the FMA pipe 10 %.
#ifndef PVLC_BLAKE3_FMA_ADDS
#define PVLC_BLAKE3_FMA_ADDS 2
#endif

__device__ __forceinline__ void g(uint32_t* s, int a, int b, int c, int d, uint32_t mx,
                                  uint32_t my, uint32_t one) {
#if PVLC_BLAKE3_FMA_ADDS >= 2
  s[a] = add_fma(s[b], add_fma(s[a], mx, one), one);
#else
  s[a] = s[a] + s[b] + mx;
#endif
  s[d] = rotr(s[d] ^ s[a], 16);
#if PVLC_BLAKE3_FMA_ADDS >= 1
  s[c] = add_fma(s[d], s[c], one);
#else
  s[c] = s[c] + s[d];
#endif
  s[b] = rotr(s[b] ^ s[c], 12);
#if PVLC_BLAKE3_FMA_ADDS >= 2
  s[a] = add_fma(s[b], add_fma(s[a], my, one), one);
#else
  s[a] = s[a] + s[b] + my;
#endif
  s[d] = rotr(s[d] ^ s[a], 8);
#if PVLC_BLAKE3_FMA_ADDS >= 1
  s[c] = add_fma(s[d], s[c], one);
#else
  s[c] = s[c] + s[d];
#endif
  s[b] = rotr(s[b] ^ s[c], 7);
}

// Message word order of round r: the schedule permutation applied r times.
__device__ __forceinline__ constexpr int sched(int r, int i) {
  constexpr int P[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};
  int w = i;
  for (int k = 0; k < r; ++k) w = P[w];
  return w;
}

// out[0..7] = the compression's chaining-value half (state words 0..7 after the
// feed-forward); the root output is its first 32 bytes.
__device__ __forceinline__ void compress(const uint32_t* cv, const uint32_t* m, uint64_t counter,
                                         uint32_t block_len, uint32_t flags, uint32_t* out,
                                         uint32_t one) {
  uint32_t s[16] = {cv[0], cv[1], cv[2], cv[3], cv[4], cv[5], cv[6], cv[7],
                    iv(0), iv(1), iv(2), iv(3), static_cast<uint32_t>(counter),
                    static_cast<uint32_t>(counter >> 32), block_len, flags};
#pragma unroll
  for (int r = 0; r < 7; ++r) {
    g(s, 0, 4, 8, 12, m[sched(r, 0)], m[sched(r, 1)], one);
    g(s, 1, 5, 9, 13, m[sched(r, 2)], m[sched(r, 3)], one);
    g(s, 2, 6, 10, 14, m[sched(r, 4)], m[sched(r, 5)], one);
    g(s, 3, 7, 11, 15, m[sched(r, 6)], m[sched(r, 7)], one);
    g(s, 0, 5, 10, 15, m[sched(r, 8)], m[sched(r, 9)], one);
    g(s, 1, 6, 11, 12, m[sched(r, 10)], m[sched(r, 11)], one);
    g(s, 2, 7, 8, 13, m[sched(r, 12)], m[sched(r, 13)], one);
    g(s, 3, 4, 9, 14, m[sched(r, 14)], m[sched(r, 15)], one);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = s[i] ^ s[i + 8];
}

// One thread per chunk: its chaining value (or, for a one-chunk input, the
// root output) into cvs[chunk].  Full blocks are read with 16-byte loads when
// the buffer is 16-byte aligned, the partial last block byte by byte.
__global__ void __launch_bounds__(128) chunk_kernel(const uint8_t* __restrict__ data,
                                                    uint64_t bytes, uint64_t chunks,
                                                    uint32_t* __restrict__ cvs, int aligned,
                                                    uint32_t one) {
  const uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (c >= chunks) return;
  const uint64_t off = c * CHUNK;
  const uint32_t len = static_cast<uint32_t>(bytes - off < CHUNK ? bytes - off : CHUNK);
  const uint32_t nblocks = len == 0 ? 1u : (len + BLOCK - 1) / BLOCK;
  uint32_t cv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) cv[i] = iv(i);
  for (uint32_t b = 0; b < nblocks; ++b) {
    const uint32_t blen = len - b * BLOCK < BLOCK ? len - b * BLOCK : BLOCK;
    uint32_t m[16];
    const uint8_t* p = data + off + b * BLOCK;
    if (blen == BLOCK && aligned) {
      const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 v = __ldg(q + k);
        m[4 * k] = v.x;
        m[4 * k + 1] = v.y;
        m[4 * k + 2] = v.z;
        m[4 * k + 3] = v.w;
      }
    } else {   // partial (zero-padded) block or unaligned buffer: byte by byte
#pragma unroll
      for (int w = 0; w < 16; ++w) {
        uint32_t v = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (static_cast<uint32_t>(4 * w + q) < blen)
            v |= static_cast<uint32_t>(__ldg(p + 4 * w + q)) << (8 * q);
        m[w] = v;
      }
    }
    uint32_t flags = 0;
    if (b == 0) flags |= CHUNK_START;
    if (b + 1 == nblocks) flags |= CHUNK_END | (chunks == 1 ? ROOT : 0u);
    compress(cv, m, c, blen, flags, cv, one);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) cvs[c * 8 + i] = cv[i];
}

// One tree level: node i of the next level is parent(in[2i], in[2i + 1]), or
// in[2i] itself for an odd last node; the level of two nodes makes the root.
__global__ void __launch_bounds__(128) parent_kernel(const uint32_t* __restrict__ in, uint64_t n,
                                                     uint32_t* __restrict__ out, uint32_t one) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const uint64_t m = (n + 1) / 2;
  if (i >= m) return;
  if (2 * i + 1 >= n) {
#pragma unroll
    for (int k = 0; k < 8; ++k) out[i * 8 + k] = in[2 * i * 8 + k];
    return;
  }
  uint32_t key[8], blk[16], cv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) key[k] = iv(k);
#pragma unroll
  for (int k = 0; k < 16; ++k) blk[k] = in[2 * i * 8 + k];
  compress(key, blk, 0, BLOCK, PARENT | (n == 2 ? ROOT : 0u), cv, one);
#pragma unroll
  for (int k = 0; k < 8; ++k) out[i * 8 + k] = cv[k];
}

}  // namespace b3

size_t blake3_workspace_bytes(uint64_t bytes) {
  const uint64_t chunks = bytes == 0 ? 1 : (bytes + b3::CHUNK - 1) / b3::CHUNK;
  // two node arrays of 32 bytes a chunk (levels ping-pong between them)
  return static_cast<size_t>(2 * chunks * 32);
}

int blake3_launch(const void* data, uint64_t bytes, void* workspace, uint8_t* digest,
                  cudaStream_t s) {
  const uint64_t chunks = bytes == 0 ? 1 : (bytes + b3::CHUNK - 1) / b3::CHUNK;
  uint32_t* a = static_cast<uint32_t*>(workspace);
  uint32_t* b = a + chunks * 8;
  const int aligned = (reinterpret_cast<uintptr_t>(data) & 15u) == 0;
  const uint64_t g0 = (chunks + 127) / 128;
  if (g0 > 0x7fffffffull) return PVLC_ARITHMETIC_OVERFLOW;
  b3::chunk_kernel<<<(unsigned)g0, 128, 0, s>>>(static_cast<const uint8_t*>(data), bytes, chunks,
                                                a, aligned, 1u);
  uint64_t n = chunks;
  while (n > 1) {
    const uint64_t m = (n + 1) / 2;
    b3::parent_kernel<<<(unsigned)((m + 127) / 128), 128, 0, s>>>(a, n, b, 1u);
    uint32_t* t = a;
    a = b;
    b = t;
    n = m;
  }
  // the root's first 32 bytes, little-endian words
  if (cudaMemcpyAsync(digest, a, 32, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  return cudaPeekAtLastError() == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR;
}

}  // namespace pvlc

using namespace pvlc;

extern "C" {

size_t pvlc_blake3_workspace_bytes(uint64_t bytes) { return blake3_workspace_bytes(bytes); }

int pvlc_blake3(const void* data, uint64_t bytes, void* workspace, size_t workspace_bytes,
                uint8_t* digest, void* stream) {
  if (!workspace || !digest || (bytes > 0 && !data)) return PVLC_NULL_POINTER;
  if (bytes > (1ull << 46)) return PVLC_ARITHMETIC_OVERFLOW;
  if (workspace_bytes < blake3_workspace_bytes(bytes)) return PVLC_WORKSPACE_TOO_SMALL;
  if (reinterpret_cast<uintptr_t>(workspace) & 15u) return PVLC_MISALIGNED_POINTER;
  return blake3_launch(data, bytes, workspace, digest, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
