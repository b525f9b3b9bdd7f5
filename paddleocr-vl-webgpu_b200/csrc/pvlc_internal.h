// pvlc_internal.h -- launchers shared between the C ABI layer (pvlc_abi.cu)
// and the kernel translation units.  Not installed; not part of the ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/pvlc_cuda_attn.h"

namespace pvlc {

struct DecodeArgs {
  const pvlc_half* q;
  const pvlc_half* k_new;
  const pvlc_half* v_new;
  const float* rope_cos;
  const float* rope_sin;
  uint32_t rope_rows;
  const uint32_t* rope_row;
  pvlc_half* const* k_cache;
  pvlc_half* const* v_cache;
  const uint32_t* cache_tokens;
  uint32_t capacity;
  uint32_t max_cache_tokens;
  uint32_t batch;
  void* workspace;
  pvlc_half* out;
  int num_ctas;
  uint32_t q_stride;    // elements between consecutive sequences' q rows
  uint32_t kv_stride;   // elements between consecutive sequences' k_new / v_new rows
};
size_t decode_workspace_bytes(uint32_t batch, int num_sms);
int decode_block_threads();
int decode_launch(const DecodeArgs& a, cudaStream_t stream);

struct VisionArgs {
  const pvlc_half* q;
  const pvlc_half* k;
  const pvlc_half* v;
  const float* rope_cos;
  const float* rope_sin;
  uint32_t tokens;
  uint32_t heads;
  pvlc_half* out;
  uint32_t qkv_stride;   // elements between consecutive tokens' q / k / v rows (heads x 72 packed)
};
// Read and clear the calling device's sticky fault word of the vision /
// prefill kernels (PVLC_FAULT_* bits); synchronizes `s`.
int vision_fault_word(uint32_t* out, cudaStream_t s);
int prefill_fault_word(uint32_t* out, cudaStream_t s);
// BLAKE3 of a device buffer (blake3.cu): scratch of blake3_workspace_bytes,
// the 32-byte digest written to device memory.
size_t blake3_workspace_bytes(uint64_t bytes);
int blake3_launch(const void* data, uint64_t bytes, void* workspace, uint8_t* digest,
                  cudaStream_t s);
int vision_query_tile();
int vision_block_threads();
// Scratch for the rotated q and k (2 x tokens x heads x 72 fp16).
size_t vision_workspace_bytes(uint32_t tokens, uint32_t heads);
// workspace: vision_workspace_bytes of device memory when rope tables are
// given (unused otherwise).
int vision_launch(const VisionArgs& a, const uint32_t* cu_seqlens, uint32_t segments,
                  void* workspace, cudaStream_t stream);

struct PrefillArgs {
  const pvlc_half* q;
  const pvlc_half* k;
  const pvlc_half* v;
  const float* rope_cos;
  const float* rope_sin;
  uint32_t rope_rows;
  uint32_t tokens;
  uint32_t capacity;
  pvlc_half* k_cache;
  pvlc_half* v_cache;
  pvlc_half* out;
};
struct PrefillBatchArgs {
  const pvlc_half* q;          // packed [rows, 16, 128]
  const pvlc_half* k;          // packed [rows, 2, 128]
  const pvlc_half* v;
  const uint32_t* offsets;     // host [prompts + 1]
  uint32_t prompts;
  const float* const* rope_cos;  // host [prompts] device pointers
  const float* const* rope_sin;
  const uint32_t* rope_rows;     // host [prompts]
  pvlc_half* k_cache;            // prompt b's cache at + b * cache_stride elements
  pvlc_half* v_cache;
  uint64_t cache_stride;
  uint32_t capacity;
  pvlc_half* out;                // packed [rows, 16, 128]
};
int prefill_batch_launch(const PrefillBatchArgs& a, cudaStream_t stream);
int prefill_query_tile();
void prefill_schedule(uint32_t tokens, int sms, uint32_t* n_split, uint32_t* n_light);
int prefill_block_threads();
int prefill_launch(const PrefillArgs& a, cudaStream_t stream);

// Greedy top-1 over the LM head (lm_head.cu).
struct LmHeadArgs {
  const pvlc_half* hidden;    // [rows, hidden_dim]
  const pvlc_half* lm_head;   // [vocab, hidden_dim]
  uint32_t rows, vocab, hidden_dim;
  void* workspace;            // lm_head_workspace_bytes(rows)
  int32_t* tokens;            // [rows]
  float* logits;              // [rows] winning logit, or null
};
size_t lm_head_workspace_bytes(uint32_t rows);
size_t lm_head_flags_offset(uint32_t rows);
int lm_head_top1_launch(const LmHeadArgs& a, cudaStream_t stream);

// Decode-step projections (linear.cu).
struct LinearArgs {
  const pvlc_half* x;    // [rows, k], row pitch ldx
  uint32_t rows, ldx;
  const pvlc_half* w;    // [n, k] contiguous
  uint32_t n, k;
  uint32_t gate;         // 1: fused SiLU gate, out has n / 2 columns
  uint32_t split;        // K slices per feature tile (power of two <= 16)
  pvlc_half* out;
  uint32_t ldo;
};
uint32_t linear_auto_split(uint32_t rows, uint32_t n, uint32_t k, int sms);
bool linear_split_fits(uint32_t rows, uint32_t k, uint32_t split);
int linear_launch(const LinearArgs& a, cudaStream_t stream);
int linear_fault_word(uint32_t* out, cudaStream_t s);

int device_sm_count();
// The current device's SM count, or the B200's 148 when no GPU is visible.
int sms_or_default_count();
// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, smem_bytes) once per
// kernel, device and context (thread-safe); a PVLC_* status.
int set_smem_attribute_once(const void* kernel, int smem_bytes);

}  // namespace pvlc
