// pvlc_abi.cu -- the extern "C" boundary declared in include/pvlc_cuda_attn.h.
//
// Host-side half of the reference's attention operator contract: every entry
// point validates its geometry with the same rules and error precedence as
// crates/pvlc-runtime-core (zero dimensions first, then head-dim support,
// then sequence boundaries / pinned geometry, then lengths) and returns before
// any device effect when they fail.  The plan functions expose the launch
// geometry without touching a GPU.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/pvlc_cuda_attn.h"
#include "pvlc_internal.h"

namespace pvlc {

// The current CUDA context (the driver's cuCtxGetCurrent, looked up once
// through the runtime), or nullptr when it cannot be read.
static void* current_context() {
  using GetCurrent = int (*)(void**);
  static GetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetCurrent>(ptr);
  });
  void* ctx = nullptr;
  if (!fn || fn(&ctx) != 0) return nullptr;
  return ctx;
}

int set_smem_attribute_once(const void* kernel, int smem_bytes) {
  // One entry per (kernel, device) holding the context the attribute was set
  // in: an attribute belongs to its context, so the context that follows a
  // cudaDeviceReset gets it again.  The mutex covers concurrent first calls
  // from several threads.
  struct Entry { const void* kernel; int dev; void* ctx; };
  static std::mutex mu;
  static Entry done[256];
  static int n_done = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PVLC_CUDA_ERROR;
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(mu);
  Entry* e = nullptr;
  for (int i = 0; i < n_done; ++i)
    if (done[i].kernel == kernel && done[i].dev == dev) e = &done[i];
  if (e && ctx && e->ctx == ctx) return PVLC_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
      cudaSuccess)
    return PVLC_CUDA_ERROR;
  if (!e && n_done < 256) e = &done[n_done++];
  if (e) *e = Entry{kernel, dev, ctx};
  return PVLC_OK;
}

int device_sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

constexpr int kDefaultSms = 148;  // B200; used by plans when no GPU is visible

int sms_or_default_count() {
  int dev_count = 0;
  if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) {
    cudaGetLastError();
    return kDefaultSms;
  }
  const int n = device_sm_count();
  return n > 0 ? n : kDefaultSms;
}

namespace {

int sms_or_default() { return sms_or_default_count(); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The library's own stream-ordered memory pool of the current device, for the
// scratch of the entry points that take none from the caller.  Memory freed
// into it stays reserved (release threshold: unlimited), so back-to-back
// calls reuse it instead of returning it to the driver at every synchronize;
// the process's default pool is left untouched.
cudaMemPool_t scratch_pool() {
  static cudaMemPool_t pools[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) return nullptr;
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = pool;
  }
  return pools[dev];
}

// crates/pvlc-runtime-core/src/lib.rs:443-478 (+ validate_sequence_boundaries
// crates/pvlc-cpu-ref/src/lib.rs:3393-3405)
int check_vision(const uint32_t* cu, uint32_t segments, uint32_t tokens, uint32_t heads,
                 uint32_t head_dim) {
  if (tokens == 0 || heads == 0 || head_dim == 0) return PVLC_ZERO_DIMENSION;
  if (head_dim > PVLC_VISION_MAX_HEAD_DIM) return PVLC_UNSUPPORTED_HEAD_DIMENSION;
  if (head_dim != PVLC_VISION_MAX_HEAD_DIM) return PVLC_UNSUPPORTED_HEAD_DIMENSION;
  if (cu == nullptr) return PVLC_NULL_POINTER;
  if (segments == 0 || cu[0] != 0 || cu[segments] != tokens) return PVLC_INVALID_SEQUENCE_BOUNDARIES;
  for (uint32_t i = 0; i < segments; ++i)
    if (cu[i] >= cu[i + 1]) return PVLC_INVALID_SEQUENCE_BOUNDARIES;
  if (segments > PVLC_VISION_MAX_SEGMENTS || heads > 64) return PVLC_INVALID_VISION_GEOMETRY;
  const uint64_t elems = (uint64_t)tokens * heads * head_dim;
  if (elems > (1ull << 40)) return PVLC_ARITHMETIC_OVERFLOW;
  return PVLC_OK;
}

// crates/pvlc-runtime-core/src/lib.rs:2500-2653 (pinned decoder geometry)
int check_prefill(uint32_t tokens, uint32_t capacity, uint32_t rope_rows) {
  if (tokens == 0 || capacity == 0 || rope_rows == 0) return PVLC_ZERO_DIMENSION;
  if (tokens > capacity) return PVLC_CAPACITY_EXHAUSTED;
  if (tokens > rope_rows) return PVLC_INVALID_DECODER_GEOMETRY;
  const uint64_t n_tiles = (tokens + 15) / 16;   // one CTA per 16-token Q tile and KV head
  if (n_tiles > 65535) return PVLC_INVALID_DECODER_GEOMETRY;
  return PVLC_OK;
}

// crates/pvlc-runtime-core/src/lib.rs:1091-1159 (plan_decoder_kv_session_geometry)
int check_session(uint32_t qh, uint32_t kvh, uint32_t hd, uint32_t prefix, uint32_t capacity) {
  if (qh == 0 || kvh == 0 || hd == 0 || prefix == 0 || capacity == 0) return PVLC_ZERO_DIMENSION;
  if (hd > PVLC_DECODER_HEAD_DIM) return PVLC_UNSUPPORTED_HEAD_DIMENSION;
  const uint64_t cache_elems = (uint64_t)capacity * kvh * hd;
  if (cache_elems - 1 > 0xffffffffull) return PVLC_ARITHMETIC_OVERFLOW;
  if (qh % kvh || qh != PVLC_DECODER_QUERY_HEADS || kvh != PVLC_DECODER_KV_HEADS ||
      hd != PVLC_DECODER_HEAD_DIM)
    return PVLC_INVALID_DECODER_GEOMETRY;
  if (prefix >= capacity) return PVLC_INVALID_DECODER_GEOMETRY;
  return PVLC_OK;
}

int check_decode(uint32_t batch, uint32_t capacity, uint32_t max_cache_tokens, uint32_t rope_rows) {
  if (batch == 0 || capacity == 0 || rope_rows == 0) return PVLC_ZERO_DIMENSION;
  if (batch > PVLC_DECODE_MAX_BATCH) return PVLC_INVALID_DECODER_GEOMETRY;
  if (max_cache_tokens >= capacity) return PVLC_CAPACITY_EXHAUSTED;
  if ((uint64_t)capacity * 512ull > (1ull << 40)) return PVLC_ARITHMETIC_OVERFLOW;
  return PVLC_OK;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? PVLC_OK : PVLC_CUDA_ERROR; }

}  // namespace
}  // namespace pvlc

using namespace pvlc;

extern "C" {

const char* pvlc_attn_status_string(int status) {
  switch (status) {
    case PVLC_OK: return "ok";
    case PVLC_ZERO_DIMENSION: return "ZeroDimension";
    case PVLC_LENGTH_MISMATCH: return "LengthMismatch";
    case PVLC_ARITHMETIC_OVERFLOW: return "ArithmeticOverflow";
    case PVLC_INVALID_ROTARY_DIMENSION: return "InvalidRotaryDimension";
    case PVLC_INVALID_ROPE_BASE: return "InvalidRopeBase";
    case PVLC_UNSUPPORTED_HEAD_DIMENSION: return "UnsupportedHeadDimension";
    case PVLC_INVALID_DECODER_GEOMETRY: return "InvalidDecoderGeometry";
    case PVLC_INVALID_VISION_GEOMETRY: return "InvalidVisionGeometry";
    case PVLC_INVALID_SEQUENCE_BOUNDARIES: return "InvalidSequenceBoundaries";
    case PVLC_NON_FINITE_INPUT: return "NonFiniteInput";
    case PVLC_NULL_POINTER: return "NullPointer";
    case PVLC_MISALIGNED_POINTER: return "MisalignedPointer";
    case PVLC_WORKSPACE_TOO_SMALL: return "WorkspaceTooSmall";
    case PVLC_CAPACITY_EXHAUSTED: return "CapacityExhausted";
    case PVLC_CUDA_ERROR: return "CudaError";
    case PVLC_DEVICE_UNSUPPORTED: return "DeviceUnsupported";
    case PVLC_DEVICE_FAULT_FLAG: return "DeviceFaultFlag";
    default: return "Unknown";
  }
}

int pvlc_attn_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return PVLC_DEVICE_UNSUPPORTED;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  return (major == 10 && minor == 0) ? PVLC_OK : PVLC_DEVICE_UNSUPPORTED;
}

// ------------------------------------------------------------------ vision
int pvlc_plan_vision_varlen(const uint32_t* cu, uint32_t segments, uint32_t tokens, uint32_t heads,
                            uint32_t head_dim, pvlc_plan* plan) {
  const int st = check_vision(cu, segments, tokens, heads, head_dim);
  if (st) return st;
  if (!plan) return PVLC_NULL_POINTER;
  memset(plan, 0, sizeof(*plan));
  const uint32_t bm = (uint32_t)vision_query_tile();
  uint32_t items = 0;
  double sumsq = 0;
  for (uint32_t i = 0; i < segments; ++i) {
    const uint32_t n = cu[i + 1] - cu[i];
    items += (n + bm - 1) / bm;
    sumsq += (double)n * n;
  }
  plan->grid[0] = heads;
  plan->grid[1] = items;
  plan->grid[2] = 1;
  plan->block[0] = (uint32_t)vision_block_threads();
  plan->block[1] = plan->block[2] = 1;
  plan->work_items = items * heads;
  plan->output_elements = (uint64_t)tokens * heads * head_dim;
  plan->output_bytes = plan->output_elements * 2;
  plan->workspace_bytes = vision_workspace_bytes(tokens, heads);   // rotated q, k (with tables)
  plan->flops = 4.0 * head_dim * heads * sumsq;
  plan->hbm_bytes = 4.0 * plan->output_bytes + (double)tokens * head_dim * 4.0;  // q,k,v,o + tables
  return PVLC_OK;
}

size_t pvlc_attn_vision_workspace_bytes(uint32_t tokens, uint32_t heads, uint32_t head_dim) {
  if (head_dim != 72) return 0;
  return vision_workspace_bytes(tokens, heads);
}

static int vision_checks(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                         const uint32_t* cu, uint32_t segments, uint32_t tokens, uint32_t heads,
                         uint32_t head_dim, const float* rope_cos, const float* rope_sin,
                         const pvlc_half* out) {
  const int st = check_vision(cu, segments, tokens, heads, head_dim);
  if (st) return st;
  if (!q || !k || !v || !out) return PVLC_NULL_POINTER;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return PVLC_NULL_POINTER;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (rope_cos && (!aligned16(rope_cos) || !aligned16(rope_sin))))
    return PVLC_MISALIGNED_POINTER;
  return PVLC_OK;
}

int pvlc_attn_vision_varlen_ws(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                               const uint32_t* cu, uint32_t segments, uint32_t tokens,
                               uint32_t heads, uint32_t head_dim, const float* rope_cos,
                               const float* rope_sin, void* workspace, size_t workspace_bytes,
                               pvlc_half* out, void* stream) {
  const int st = vision_checks(q, k, v, cu, segments, tokens, heads, head_dim, rope_cos, rope_sin,
                               out);
  if (st) return st;
  if (rope_cos) {
    if (!workspace) return PVLC_NULL_POINTER;
    if (!aligned16(workspace)) return PVLC_MISALIGNED_POINTER;
    if (workspace_bytes < vision_workspace_bytes(tokens, heads)) return PVLC_WORKSPACE_TOO_SMALL;
  }
  VisionArgs a{q, k, v, rope_cos, rope_sin, tokens, heads, out, heads * head_dim};
  return vision_launch(a, cu, segments, workspace, static_cast<cudaStream_t>(stream));
}

int pvlc_attn_vision_varlen_strided_ws(const pvlc_half* q, const pvlc_half* k,
                                       const pvlc_half* v, uint32_t qkv_row_stride,
                                       const uint32_t* cu, uint32_t segments, uint32_t tokens,
                                       uint32_t heads, uint32_t head_dim, const float* rope_cos,
                                       const float* rope_sin, void* workspace,
                                       size_t workspace_bytes, pvlc_half* out, void* stream) {
  const int st = vision_checks(q, k, v, cu, segments, tokens, heads, head_dim, rope_cos, rope_sin,
                               out);
  if (st) return st;
  if (qkv_row_stride < heads * head_dim || qkv_row_stride % 8 != 0) return PVLC_LENGTH_MISMATCH;
  if (rope_cos) {
    if (!workspace) return PVLC_NULL_POINTER;
    if (!aligned16(workspace)) return PVLC_MISALIGNED_POINTER;
    if (workspace_bytes < vision_workspace_bytes(tokens, heads)) return PVLC_WORKSPACE_TOO_SMALL;
  }
  VisionArgs a{q, k, v, rope_cos, rope_sin, tokens, heads, out, qkv_row_stride};
  return vision_launch(a, cu, segments, workspace, static_cast<cudaStream_t>(stream));
}

int pvlc_attn_vision_varlen(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                            const uint32_t* cu, uint32_t segments, uint32_t tokens, uint32_t heads,
                            uint32_t head_dim, const float* rope_cos, const float* rope_sin,
                            pvlc_half* out, void* stream) {
  const int st = vision_checks(q, k, v, cu, segments, tokens, heads, head_dim, rope_cos, rope_sin,
                               out);
  if (st) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* ws = nullptr;
  if (rope_cos) {
    // stream-ordered scratch for the rotated q and k, released after the launch
    cudaMemPool_t pool = scratch_pool();
    if (!pool ||
        cudaMallocFromPoolAsync(&ws, vision_workspace_bytes(tokens, heads), pool, s) != cudaSuccess) {
      cudaGetLastError();
      return PVLC_CUDA_ERROR;
    }
  }
  VisionArgs a{q, k, v, rope_cos, rope_sin, tokens, heads, out, heads * head_dim};
  const int rc = vision_launch(a, cu, segments, ws, s);
  if (ws && cudaFreeAsync(ws, s) != cudaSuccess && rc == PVLC_OK) return PVLC_CUDA_ERROR;
  return rc;
}

// ------------------------------------------------------------------ prefill
int pvlc_plan_decoder_prefill(uint32_t tokens, uint32_t capacity, uint32_t rope_rows,
                              pvlc_plan* plan) {
  const int st = check_prefill(tokens, capacity, rope_rows);
  if (st) return st;
  if (!plan) return PVLC_NULL_POINTER;
  memset(plan, 0, sizeof(*plan));
  const uint32_t bm = (uint32_t)prefill_query_tile();
  // one CTA per (KV group, 16-token Q tile), the lightest tiles paired two per
  // CTA so that the grid is one wave
  uint32_t n_split = 0, n_light = 0;
  prefill_schedule(tokens, sms_or_default(), &n_split, &n_light);
  plan->grid[0] = PVLC_DECODER_KV_HEADS;
  plan->grid[1] = n_split + n_light / 2;
  plan->grid[2] = 1;
  plan->block[0] = (uint32_t)prefill_block_threads();
  plan->block[1] = plan->block[2] = 1;
  plan->work_items = PVLC_DECODER_KV_HEADS * ((tokens + bm - 1) / bm);
  plan->output_elements = (uint64_t)tokens * 16 * 128;
  plan->output_bytes = plan->output_elements * 2;
  plan->flops = 4.0 * 128 * 16 * (double)tokens * (tokens + 1) / 2.0;
  // q + o (16 heads) + k, v in + k, v cache out (2 heads), fp16
  plan->hbm_bytes = (double)tokens * (2 * 16 * 128 * 2 + 4 * 2 * 128 * 2);
  return PVLC_OK;
}

int pvlc_attn_decoder_prefill(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                              const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                              uint32_t tokens, uint32_t capacity, pvlc_half* k_cache,
                              pvlc_half* v_cache, pvlc_half* out, void* stream) {
  const int st = check_prefill(tokens, capacity, rope_rows);
  if (st) return st;
  if (!q || !k || !v || !rope_cos || !rope_sin || !k_cache || !v_cache || !out)
    return PVLC_NULL_POINTER;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(rope_cos) ||
      !aligned16(rope_sin) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return PVLC_MISALIGNED_POINTER;
  PrefillArgs a{q, k, v, rope_cos, rope_sin, rope_rows, tokens, capacity, k_cache, v_cache, out};
  return prefill_launch(a, static_cast<cudaStream_t>(stream));
}

int pvlc_attn_decoder_prefill_batch(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                                    const uint32_t* offsets, uint32_t prompts,
                                    const float* const* rope_cos, const float* const* rope_sin,
                                    const uint32_t* rope_rows, pvlc_half* k_cache,
                                    pvlc_half* v_cache, uint64_t cache_stride, uint32_t capacity,
                                    pvlc_half* out, void* stream) {
  if (prompts == 0) return PVLC_ZERO_DIMENSION;
  if (prompts > PVLC_PREFILL_MAX_PROMPTS) return PVLC_INVALID_DECODER_GEOMETRY;
  if (!offsets || !rope_cos || !rope_sin || !rope_rows) return PVLC_NULL_POINTER;
  if (offsets[0] != 0) return PVLC_INVALID_SEQUENCE_BOUNDARIES;
  uint64_t tiles = 0;
  for (uint32_t b = 0; b < prompts; ++b) {
    if (offsets[b + 1] <= offsets[b]) return PVLC_INVALID_SEQUENCE_BOUNDARIES;
    const uint32_t t = offsets[b + 1] - offsets[b];
    const int st = check_prefill(t, capacity, rope_rows[b]);
    if (st) return st;
    tiles += (t + 15) / 16;
  }
  if (tiles > 65535u) return PVLC_INVALID_DECODER_GEOMETRY;
  if ((uint64_t)offsets[prompts] * 16 * 128 * 2 > (1ull << 40)) return PVLC_ARITHMETIC_OVERFLOW;
  if (cache_stride < (uint64_t)capacity * 256 || cache_stride % 8) return PVLC_LENGTH_MISMATCH;
  if (!q || !k || !v || !k_cache || !v_cache || !out) return PVLC_NULL_POINTER;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(k_cache) ||
      !aligned16(v_cache) || !aligned16(out))
    return PVLC_MISALIGNED_POINTER;
  for (uint32_t b = 0; b < prompts; ++b) {
    if (!rope_cos[b] || !rope_sin[b]) return PVLC_NULL_POINTER;
    if (!aligned16(rope_cos[b]) || !aligned16(rope_sin[b])) return PVLC_MISALIGNED_POINTER;
  }
  PrefillBatchArgs a{q,        k,       v,       offsets, prompts,      rope_cos, rope_sin,
                     rope_rows, k_cache, v_cache, cache_stride, capacity, out};
  return prefill_batch_launch(a, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------ decode
int pvlc_plan_decoder_kv_session(uint32_t qh, uint32_t kvh, uint32_t hd, uint32_t prefix,
                                 uint32_t capacity, pvlc_plan* plan) {
  const int st = check_session(qh, kvh, hd, prefix, capacity);
  if (st) return st;
  if (!plan) return PVLC_NULL_POINTER;
  uint32_t ct = prefix;
  return pvlc_plan_decode(&ct, 1, capacity, plan);
}

int pvlc_plan_decode(const uint32_t* cache_tokens, uint32_t batch, uint32_t capacity,
                     pvlc_plan* plan) {
  if (!cache_tokens) return PVLC_NULL_POINTER;
  uint32_t mx = 0;
  for (uint32_t b = 0; b < batch; ++b) mx = cache_tokens[b] > mx ? cache_tokens[b] : mx;
  const int st = check_decode(batch, capacity, mx, 1);
  if (st) return st;
  if (!plan) return PVLC_NULL_POINTER;
  memset(plan, 0, sizeof(*plan));
  const int sms = sms_or_default();
  uint64_t tiles = 0;
  double kv_rows = 0;
  for (uint32_t b = 0; b < batch; ++b) {
    tiles += (cache_tokens[b] + 1 + 31) / 32;
    kv_rows += cache_tokens[b] + 1.0;
  }
  plan->grid[0] = (uint32_t)(tiles < (uint64_t)sms ? tiles : (uint64_t)sms);
  plan->grid[1] = plan->grid[2] = 1;
  plan->block[0] = (uint32_t)decode_block_threads();
  plan->block[1] = plan->block[2] = 1;
  plan->work_items = (uint32_t)tiles;
  plan->output_elements = (uint64_t)batch * 16 * 128;
  plan->output_bytes = plan->output_elements * 2;
  plan->workspace_bytes = decode_workspace_bytes(batch, sms);
  plan->flops = 4.0 * 16 * 128 * kv_rows;
  // K and V rows (2 heads x 128 fp16 each) + q + out + the appended row
  plan->hbm_bytes = kv_rows * 1024.0 + batch * (4096.0 + 4096.0 + 1024.0);
  return PVLC_OK;
}

size_t pvlc_attn_decode_workspace_bytes(uint32_t batch) {
  return decode_workspace_bytes(batch, sms_or_default());
}

int pvlc_attn_decode_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (!workspace) return PVLC_NULL_POINTER;
  return cuda_status(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)));
}

int pvlc_attn_decode_strided(const pvlc_half* q, uint32_t q_row_stride, const pvlc_half* k_new,
                             const pvlc_half* v_new, uint32_t kv_row_stride,
                             const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                             const uint32_t* rope_row, pvlc_half* const* k_cache,
                             pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                             uint32_t capacity, uint32_t max_cache_tokens, uint32_t batch,
                             void* workspace, size_t workspace_bytes, pvlc_half* out,
                             void* stream) {
  const int st = check_decode(batch, capacity, max_cache_tokens, rope_rows);
  if (st) return st;
  if (q_row_stride < 16u * 128u || kv_row_stride < 2u * 128u || q_row_stride % 8 ||
      kv_row_stride % 8)
    return PVLC_LENGTH_MISMATCH;
  if (!q || !k_new || !v_new || !rope_cos || !rope_sin || !k_cache || !v_cache ||
      !cache_tokens || !workspace || !out)
    return PVLC_NULL_POINTER;
  if (!aligned16(q) || !aligned16(k_new) || !aligned16(v_new) || !aligned16(out) ||
      !aligned16(workspace) || !aligned16(rope_cos) || !aligned16(rope_sin))
    return PVLC_MISALIGNED_POINTER;
  const int sms = device_sm_count();
  if (sms <= 0) return PVLC_CUDA_ERROR;
  if (workspace_bytes < decode_workspace_bytes(batch, sms)) return PVLC_WORKSPACE_TOO_SMALL;
  DecodeArgs a{q,       k_new,    v_new,           rope_cos,     rope_sin,  rope_rows,
               rope_row, k_cache, v_cache,         cache_tokens, capacity,  max_cache_tokens,
               batch,   workspace, out,            sms,          q_row_stride, kv_row_stride};
  return decode_launch(a, static_cast<cudaStream_t>(stream));
}

int pvlc_attn_decode(const pvlc_half* q, const pvlc_half* k_new, const pvlc_half* v_new,
                     const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                     const uint32_t* rope_row, pvlc_half* const* k_cache,
                     pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                     uint32_t capacity, uint32_t max_cache_tokens, uint32_t batch,
                     void* workspace, size_t workspace_bytes, pvlc_half* out, void* stream) {
  return pvlc_attn_decode_strided(q, 16u * 128u, k_new, v_new, 2u * 128u, rope_cos, rope_sin,
                                  rope_rows, rope_row, k_cache, v_cache, cache_tokens, capacity,
                                  max_cache_tokens, batch, workspace, workspace_bytes, out,
                                  stream);
}

int pvlc_attn_fault_flags(uint32_t* flags_out, void* stream) {
  if (!flags_out) return PVLC_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t a = 0, b = 0;
  int st = vision_fault_word(&a, s);
  if (st != PVLC_OK) return st;
  st = prefill_fault_word(&b, s);
  if (st != PVLC_OK) return st;
  uint32_t c = 0;
  st = linear_fault_word(&c, s);
  if (st != PVLC_OK) return st;
  *flags_out = a | b | c;
  return (a | b | c) ? PVLC_DEVICE_FAULT_FLAG : PVLC_OK;
}

int pvlc_attn_decode_errors(void* workspace, uint32_t* flags_out, void* stream) {
  if (!workspace || !flags_out) return PVLC_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t flags = 0;
  if (cudaMemcpyAsync(&flags, workspace, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return PVLC_CUDA_ERROR;
  if (cudaStreamSynchronize(s) != cudaSuccess) return PVLC_CUDA_ERROR;
  if (cudaMemsetAsync(workspace, 0, 4, s) != cudaSuccess) return PVLC_CUDA_ERROR;
  *flags_out = flags;
  return flags ? PVLC_DEVICE_FAULT_FLAG : PVLC_OK;
}

}  // extern "C"
