/*
 * pvlc_cuda_attn.h -- C ABI of the B200 (sm_100a) attention backend for the
 * PaddleOCR-VL engine.
 *
 * This library replaces the attention subset of the reference engine's
 * operator contract (crate pvlc-runtime-core, KernelId / KernelInvocation /
 * descriptor -> plan) and the WGSL kernels that implement it (crate
 * pvlc-wgsl).  Every entry point:
 *   - validates its arguments on the host first and returns a nonzero status
 *     with no device effect when they are invalid (the reference's
 *     "preflight, no effect" rule, crates/pvlc-runtime-core/src/lib.rs:5335-5395);
 *   - takes caller-owned device pointers and performs no allocation;
 *   - enqueues work asynchronously on the caller's stream (`stream` is a
 *     cudaStream_t passed as void*; NULL means the legacy default stream);
 *   - is thread-safe as long as concurrent calls use distinct output buffers
 *     and workspaces.
 * Plain C types only, so a Rust `extern "C"` block, cgo or ctypes can bind it.
 *
 * Tensor layout is token-major throughout, as in the reference
 * (crates/pvlc-cpu-ref/src/lib.rs:3424-3432): element (token, head, dim) of a
 * [tokens, heads, head_dim] tensor sits at (token*heads + head)*head_dim + dim.
 * The decoder KV cache of one layer is [capacity, 2, 128]
 * (crates/pvlc-runtime-core/src/lib.rs:883-888).  pvlc_half is IEEE binary16.
 */
#ifndef PVLC_CUDA_ATTN_H
#define PVLC_CUDA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t pvlc_half;

/* Status codes.  1..15 mirror InvocationErrorCode in declaration order
 * (crates/pvlc-runtime-core/src/lib.rs:5335-5351); 64+ are CUDA-side. */
enum pvlc_status {
  PVLC_OK = 0,
  PVLC_ZERO_DIMENSION = 1,
  PVLC_LENGTH_MISMATCH = 2,
  PVLC_ARITHMETIC_OVERFLOW = 3,
  PVLC_INVALID_ROTARY_DIMENSION = 5,
  PVLC_INVALID_ROPE_BASE = 6,
  PVLC_UNSUPPORTED_HEAD_DIMENSION = 7,
  PVLC_INVALID_DECODER_GEOMETRY = 8,
  PVLC_INVALID_VISION_GEOMETRY = 9,
  PVLC_INVALID_SEQUENCE_BOUNDARIES = 11,
  PVLC_NON_FINITE_INPUT = 15,
  PVLC_NULL_POINTER = 64,
  PVLC_MISALIGNED_POINTER = 65,
  PVLC_WORKSPACE_TOO_SMALL = 66,
  PVLC_CAPACITY_EXHAUSTED = 67,
  PVLC_CUDA_ERROR = 68,
  PVLC_DEVICE_UNSUPPORTED = 69,
  PVLC_DEVICE_FAULT_FLAG = 70
};

/* Pinned geometry (crates/pvlc-cpu-ref/src/lib.rs:544-553,
 * crates/pvlc-runtime-core/src/lib.rs:179-180). */
#define PVLC_DECODER_QUERY_HEADS 16u
#define PVLC_DECODER_KV_HEADS 2u
#define PVLC_DECODER_HEAD_DIM 128u
#define PVLC_VISION_MAX_HEAD_DIM 72u
#define PVLC_VISION_MAX_SEGMENTS 256u
#define PVLC_DECODE_MAX_BATCH 2048u

/* Human-readable name of a status code (static storage). */
const char* pvlc_attn_status_string(int status);

/* Library / device identification: returns PVLC_OK when the current device is
 * an sm_100 part this library was built for. */
int pvlc_attn_device_check(void);

/* ----------------------------------------------------------------------------
 * Path 1: vision-encoder bidirectional varlen attention with fused 2-D RoPE.
 *
 * Replaces KernelId::VisionRope2dF16 followed by KernelId::VisionAttentionF16
 * (crates/pvlc-runtime-core/src/lib.rs:65-79, invocation :248-256 plan
 * :443-478; WGSL crates/pvlc-wgsl/src/lib.rs:2309-2454,2553-2596; call site
 * crates/pvlc-runtime-web/src/web.rs:4797-4803).
 *
 * q, k, v, out: device [tokens, heads, head_dim] fp16.
 * cu_seqlens_host: HOST array of segments+1 packed-image boundaries (starts at
 *   0, strictly increasing, ends at tokens; validate_sequence_boundaries,
 *   crates/pvlc-cpu-ref/src/lib.rs:3393-3405).  Copied into the launch, so it
 *   may be reused as soon as the call returns.
 * rope_cos, rope_sin: device [tokens, head_dim/2] f32 tables (the reference's
 *   visionRope2dTables, web/engine/multimodal_ocr.mjs:98-155), or both NULL
 *   for no rotation.  Pair p of a head rotates dims (p, p + head_dim/2).
 * Attention never crosses a segment boundary; scale is 1/sqrt(head_dim).
 * head_dim must be 72 (the pinned vision head); heads <= 64.
 * Like the reference's two passes, the rotated q and k go through a device
 * scratch of pvlc_attn_vision_workspace_bytes: pvlc_attn_vision_varlen takes
 * it from the stream-ordered allocator (cudaMallocAsync / cudaFreeAsync on
 * `stream`), pvlc_attn_vision_varlen_ws from the caller (any 16-byte aligned
 * buffer of at least that size; ignored, and may be NULL, without tables).
 */
int pvlc_attn_vision_varlen(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                            const uint32_t* cu_seqlens_host, uint32_t segments,
                            uint32_t tokens, uint32_t heads, uint32_t head_dim,
                            const float* rope_cos, const float* rope_sin, pvlc_half* out,
                            void* stream);
/* Scratch bytes of a vision call (0 when head_dim is not 72). */
size_t pvlc_attn_vision_workspace_bytes(uint32_t tokens, uint32_t heads, uint32_t head_dim);
int pvlc_attn_vision_varlen_ws(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                               const uint32_t* cu_seqlens_host, uint32_t segments,
                               uint32_t tokens, uint32_t heads, uint32_t head_dim,
                               const float* rope_cos, const float* rope_sin, void* workspace,
                               size_t workspace_bytes, pvlc_half* out, void* stream);
/* pvlc_attn_vision_varlen_ws with q, k and v rows qkv_row_stride elements apart
 * (token t's q row at q + t * qkv_row_stride, each row heads x head_dim
 * contiguous); out stays packed.  It has no counterpart in the reference.  It
 * lets the three vision projections come out of one GEMM: with a [tokens,
 * 3 x 1152] output, q = base, k = base + 1152, v = base + 2304,
 * qkv_row_stride = 3456.  The stride must be a multiple of 8 and at least
 * heads x head_dim, otherwise PVLC_LENGTH_MISMATCH. */
int pvlc_attn_vision_varlen_strided_ws(const pvlc_half* q, const pvlc_half* k,
                                       const pvlc_half* v, uint32_t qkv_row_stride,
                                       const uint32_t* cu_seqlens_host, uint32_t segments,
                                       uint32_t tokens, uint32_t heads, uint32_t head_dim,
                                       const float* rope_cos, const float* rope_sin,
                                       void* workspace, size_t workspace_bytes, pvlc_half* out,
                                       void* stream);

/* ----------------------------------------------------------------------------
 * Path 2: decoder causal GQA prefill with fused 3-section M-RoPE and in-place
 * fp16 KV-cache write, for one layer of the pinned decoder (Q16/KV2/D128).
 *
 * Replaces KernelId::DecoderPrefillMropeF32 -> DecoderKvAppendRangeF32 ->
 * DecoderPrefillGqaF32 (crates/pvlc-runtime-core/src/lib.rs:51-55, stage
 * order :2613-2629, plan :2592-2596,2637-2642; WGSL
 * crates/pvlc-wgsl/src/lib.rs:1262-1416).
 *
 * q: device [tokens, 16, 128] fp16 (before RoPE); k, v: device [tokens, 2, 128]
 * fp16 (k before RoPE).  rope_cos/rope_sin: device [3, rope_rows, 128] f32
 * axis-major tables (ropeTables, web/engine/multimodal_ocr.mjs:937-986); rows
 * [0, tokens) are used, dim d takes axis 0/1/2 for (d mod 64) in [0,16) /
 * [16,40) / [40,64).  k_cache, v_cache: device [cache_capacity, 2, 128] fp16;
 * rows [0, tokens) receive the rotated key and the raw value.  out: device
 * [tokens, 16, 128] fp16.  Requires tokens <= cache_capacity, tokens <= rope_rows.
 */
int pvlc_attn_decoder_prefill(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                              const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                              uint32_t tokens, uint32_t cache_capacity, pvlc_half* k_cache,
                              pvlc_half* v_cache, pvlc_half* out, void* stream);

/* Batched variant of pvlc_attn_decoder_prefill (no counterpart in the
 * reference): `prompts` prompts packed back to back in one launch pair, so a
 * serving engine makes one call per layer instead of one per prompt, and the
 * Q tiles of all prompts share the GPU (each prompt's tiles heaviest first).
 *   q: [rows, 16, 128], k, v: [rows, 2, 128], out: [rows, 16, 128] fp16,
 *     prompt b at rows offsets[b] .. offsets[b + 1] (host array, offsets[0] = 0,
 *     every prompt at least one token, rows = offsets[prompts]).
 *   rope_cos[b], rope_sin[b]: host arrays of device pointers to prompt b's
 *     [3, rope_rows[b], 128] f32 tables (rope_rows: host array).
 *   k_cache, v_cache: prompt b's [cache_capacity, 2, 128] fp16 caches at
 *     + b * cache_stride elements (cache_stride >= cache_capacity * 256, a
 *     multiple of 8).
 * Each prompt is held to pvlc_attn_decoder_prefill's checks, with the same
 * codes; 1 <= prompts <= PVLC_PREFILL_MAX_PROMPTS and at most 65535 Q tiles
 * of 16 tokens in all, else PVLC_INVALID_DECODER_GEOMETRY.  Each CTA takes two
 * adjacent 16-token Q tiles of one prompt, so the outputs equal
 * pvlc_attn_decoder_prefill's per prompt within the fp16 output rounding (the
 * key order of the online softmax differs); the caches are bit-identical. */
#define PVLC_PREFILL_MAX_PROMPTS 256u
int pvlc_attn_decoder_prefill_batch(const pvlc_half* q, const pvlc_half* k, const pvlc_half* v,
                                    const uint32_t* offsets, uint32_t prompts,
                                    const float* const* rope_cos, const float* const* rope_sin,
                                    const uint32_t* rope_rows, pvlc_half* k_cache,
                                    pvlc_half* v_cache, uint64_t cache_stride,
                                    uint32_t cache_capacity, pvlc_half* out, void* stream);

/* ----------------------------------------------------------------------------
 * Path 3: batched single-token GQA decode against per-sequence fp16 KV caches
 * (split-KV flash decoding with an in-kernel combine), with the decode M-RoPE
 * and the KV append fused.
 *
 * Replaces, per sequence, KernelId::DecoderMropeF32 -> DecoderKvAppendF32 ->
 * DecoderGqaSplitPartialF32 -> DecoderGqaSplitMergeF32
 * (crates/pvlc-runtime-core/src/lib.rs:39-47; split plan :2861-2979; session
 * step crates/pvlc-runtime-native/src/decoder_kv_session.rs:548-768).
 *
 * q: device [batch, 16, 128] fp16 (before RoPE); k_new, v_new: device
 *   [batch, 2, 128] fp16 (k before RoPE).
 * rope_cos/rope_sin: device [3, rope_rows, 128] f32; sequence b rotates with
 *   row rope_row[b] (device array), or row cache_tokens[b] when rope_row is NULL.
 * k_cache, v_cache: device arrays of `batch` device pointers, each to a
 *   [cache_capacity, 2, 128] fp16 cache (16-byte aligned).
 * cache_tokens: device [batch] rows already in each cache (before the append).
 *   The rotated k_new and v_new are written at row cache_tokens[b] and the
 *   attention runs over cache_tokens[b] + 1 rows.  The caller advances
 *   cache_tokens after the call.
 * max_cache_tokens: host upper bound of cache_tokens[b]; must be < cache_capacity.
 *   A sequence whose device value exceeds it (or rope row out of range) is
 *   skipped and flagged; read flags with pvlc_attn_decode_errors.
 * workspace: device scratch of pvlc_attn_decode_workspace_bytes(batch) bytes,
 *   zeroed once with pvlc_attn_decode_workspace_init before first use; it
 *   is reusable across calls on the same stream without re-initialisation.
 * out: device [batch, 16, 128] fp16.
 * Ordering: the kernel is launched with programmatic dependent launch, so it
 *   may start while the kernel ahead of it on `stream` is still finishing; it
 *   waits for that kernel before touching q, k_new, v_new, the tables, the
 *   caches, the workspace or out, but it reads cache_tokens, rope_row and the
 *   two pointer arrays (to plan its split) before that wait.  Those four may
 *   be written by any earlier stream operation, but not by a kernel launched
 *   directly ahead of this call that itself allows programmatic dependent
 *   launch (triggers early); the same holds for the two variants below.
 */
size_t pvlc_attn_decode_workspace_bytes(uint32_t batch);
int pvlc_attn_decode_workspace_init(void* workspace, size_t workspace_bytes, void* stream);
int pvlc_attn_decode(const pvlc_half* q, const pvlc_half* k_new, const pvlc_half* v_new,
                     const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                     const uint32_t* rope_row, pvlc_half* const* k_cache,
                     pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                     uint32_t cache_capacity, uint32_t max_cache_tokens, uint32_t batch,
                     void* workspace, size_t workspace_bytes, pvlc_half* out, void* stream);
/* pvlc_attn_decode with row strides: sequence b's q row starts at
 * q + b * q_row_stride and its k_new / v_new rows at k_new / v_new +
 * b * kv_row_stride (elements; each row itself contiguous).  It has no
 * counterpart in the reference.  It lets the three projections come out of
 * one GEMM: with a [batch, 2560] output, q = base, k_new = base + 2048,
 * v_new = base + 2304, q_row_stride = kv_row_stride = 2560.  Strides must be
 * multiples of 8 and at least 2048 (q) / 256 (k_new, v_new); otherwise
 * PVLC_LENGTH_MISMATCH.  pvlc_attn_decode is this call with strides 2048 and
 * 256. */
int pvlc_attn_decode_strided(const pvlc_half* q, uint32_t q_row_stride, const pvlc_half* k_new,
                             const pvlc_half* v_new, uint32_t kv_row_stride,
                             const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                             const uint32_t* rope_row, pvlc_half* const* k_cache,
                             pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                             uint32_t cache_capacity, uint32_t max_cache_tokens, uint32_t batch,
                             void* workspace, size_t workspace_bytes, pvlc_half* out,
                             void* stream);
/* Synchronously reads and clears the device-side fault flags of a decode
 * workspace (bit 0: cache row out of range, bit 1: rope row out of range,
 * bit 2: misaligned cache pointer, bit 3: pipeline wait timed out).  Returns
 * PVLC_OK when no flag was set, PVLC_DEVICE_FAULT_FLAG otherwise. */
int pvlc_attn_decode_errors(void* workspace, uint32_t* flags_out, void* stream);

/* Sticky fault word of the vision, prefill and projection (pvlc_linear)
 * kernels on the calling thread's current device.  It has no counterpart in the reference (its WebGPU
 * dispatches cannot time out inside a shader).  A launch whose bounded
 * pipeline wait ran out stops early -- its output is then incomplete -- and
 * sets its kernel's bit; the bits of every such launch on the device since
 * the last read accumulate (calls on several streams share the word).
 * pvlc_attn_fault_flags synchronizes `stream`, then reads and clears the word;
 * it returns PVLC_OK when no bit was set, PVLC_DEVICE_FAULT_FLAG otherwise. */
#define PVLC_FAULT_VISION 1u
#define PVLC_FAULT_PREFILL 2u
#define PVLC_FAULT_PREFILL_BATCH 4u
#define PVLC_FAULT_LINEAR 8u
int pvlc_attn_fault_flags(uint32_t* flags_out, void* stream);

/* Allocation-free variant of pvlc_attn_decode.  It has no counterpart in the
 * reference.  It serves callers that can pass input and output buffers but
 * cannot allocate device memory -- a host whose device memory is planned once
 * by a static arena, or a foreign-language binding with no handle on a CUDA
 * allocator -- so it takes no workspace: its scratch is a fixed file-scope
 * device array of PVLC_DECODE_NOALLOC_SCRATCH_BYTES that every GPU loading
 * this library holds until the process exits.  Same arguments and results as
 * pvlc_attn_decode otherwise.
 *   - batch may not exceed PVLC_DECODE_NOALLOC_MAX_BATCH; a larger batch (or a
 *     device whose SM count needs more scratch) returns
 *     PVLC_WORKSPACE_TOO_SMALL before any device effect.
 *   - Every call looks up the array's device address on the current device
 *     (a host-only query); the first call on a device may also load the
 *     library's device code there, so make that first call before any stream
 *     capture.
 *   - The call makes no cudaMalloc/cudaFree or other allocation; it clears the
 *     array's flag and ticket words on `stream` before the kernel.
 *   - All calls share the one array: calls that may overlap on the GPU (other
 *     streams, other threads) race and must be serialised by the caller.
 *   - Device-side fault flags of this variant are not readable; use
 *     pvlc_attn_decode when they are needed. */
#define PVLC_DECODE_NOALLOC_MAX_BATCH 256u
#define PVLC_DECODE_NOALLOC_SCRATCH_BYTES (4u << 20)
int pvlc_attn_decode_noalloc(const pvlc_half* q, const pvlc_half* k_new, const pvlc_half* v_new,
                             const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                             const uint32_t* rope_row, pvlc_half* const* k_cache,
                             pvlc_half* const* v_cache, const uint32_t* cache_tokens,
                             uint32_t cache_capacity, uint32_t max_cache_tokens, uint32_t batch,
                             pvlc_half* out, void* stream);

/* ----------------------------------------------------------------------------
 * Vision preprocessing on the device (engine glue beside the attention path).
 *
 * Replaces the reference's host-side canonical_rgb8_to_patches
 * (crates/pvlc-cpu-ref/src/lib.rs:2515-2563) after smart_resize has chosen
 * the output size (:2442-2513): Pillow bicubic resample of an [H, W, 3] RGB8
 * image to [out_height, out_width, 3] (22-bit fixed-point coefficients, int64
 * accumulation, :3092-3273) and the normalised patch-major f32 values
 * [(out_height/p)*(out_width/p), 3*p*p], bit-identical to the host path.
 * The coefficient tables are computed into `workspace` by a kernel on
 * `stream` (bit-identical to the reference's f64 computation); the call
 * copies nothing from the host.
 */
size_t pvlc_image_patches_workspace_bytes(uint32_t height, uint32_t width, uint32_t out_height,
                                          uint32_t out_width);
int pvlc_image_patches(const uint8_t* rgb, uint32_t height, uint32_t width, uint32_t out_height,
                       uint32_t out_width, uint32_t patch_size, void* workspace,
                       size_t workspace_bytes, float* patches, void* stream);

/* ----------------------------------------------------------------------------
 * Engine glue: the elementwise work between the dense layers, each one pass.
 *
 * Replaces the reference's LayerNorm / RMSNorm / SiLU / GELU kernels of the
 * vision and decoder layers (WGSL catalog crates/pvlc-wgsl/src/lib.rs:438-499;
 * arithmetic crates/pvlc-cpu-ref/src/lib.rs:280-367) with the engine's storage:
 * residual streams f32, GEMM operands fp16, math in f32.
 *
 * pvlc_add_norm: per row of [rows, width] (width a multiple of 8):
 *   residual += delta (fp16, when delta is not NULL), then
 *   out = LayerNorm(residual) * weight + bias   (bias not NULL; eps as given), or
 *   out = RMSNorm(residual) * weight            (bias NULL), as fp16.
 * pvlc_gelu: in place on n fp16 values (n even): tanh form (erf_form = 0,
 *   gelu_pytorch_tanh) or erf form (erf_form = 1).
 * pvlc_silu_mul: gate_up [rows, 2*width] (gate | up) -> out [rows, width] =
 *   silu(gate) * up, fp16.
 * All pointers 16-byte aligned device pointers; work on `stream`.
 */
int pvlc_add_norm(float* residual, const pvlc_half* delta, uint32_t rows, uint32_t width,
                  const float* weight, const float* bias, float eps, pvlc_half* out,
                  void* stream);
int pvlc_gelu(pvlc_half* x, uint64_t n, int erf_form, void* stream);
int pvlc_silu_mul(const pvlc_half* gate_up, uint32_t rows, uint32_t width, pvlc_half* out,
                  void* stream);

/* ----------------------------------------------------------------------------
 * Greedy top-1 over the LM head (decoder-stack glue beside the attention path).
 *
 * Replaces the logits GEMM and the argmax of the reference's greedy step:
 * chunked_lm_head_top_k_f32 with top_k = 1 and compare_top_k_entries
 * (crates/pvlc-cpu-ref/src/lib.rs:1511-1568, 2051-2056), run in the WebGPU
 * session as an LM-head pass and an argmax pass
 * (crates/pvlc-runtime-web/src/web/decoder_stack_session.rs:308-350).
 *
 * tokens[r] = the id v maximising logit(r, v) = sum_d hidden[r, d] *
 * lm_head[v, d] (fp16 operands, f32 accumulation), larger logits first in
 * f32::total_cmp order and equal logits to the smaller id; logits[r] (when
 * not NULL) receives that logit.  The [rows, vocab] logits are never written.
 * hidden: device [rows, hidden_dim] fp16 (the final-norm output), rows <=
 * PVLC_LM_HEAD_MAX_ROWS; lm_head: device [vocab, hidden_dim] fp16; hidden_dim
 * a multiple of 64 (1024 in the pinned decoder).  workspace: device scratch of
 * pvlc_lm_head_top1_workspace_bytes(rows) bytes, 16-byte aligned; the call
 * clears it on `stream` first.  pvlc_lm_head_top1_errors reads the fault word
 * (bit 3: a pipeline wait timed out) and waits for the stream.
 */
#define PVLC_LM_HEAD_MAX_ROWS 256u
size_t pvlc_lm_head_top1_workspace_bytes(uint32_t rows);
int pvlc_lm_head_top1(const pvlc_half* hidden, uint32_t rows, const pvlc_half* lm_head,
                      uint32_t vocab, uint32_t hidden_dim, void* workspace,
                      size_t workspace_bytes, int32_t* tokens, float* logits, void* stream);
int pvlc_lm_head_top1_errors(void* workspace, uint32_t rows, uint32_t* flags_out, void* stream);

/* ----------------------------------------------------------------------------
 * Decode-step projections (decoder-stack glue beside the attention path).
 *
 * Replaces the decoder layer's GEMV/GEMM passes at decode batch sizes -- the
 * QKV, O, gate-up and down projections of the WebGPU session
 * (crates/pvlc-wgsl/src/lib.rs:1770-1835, crates/pvlc-runtime-core/src/lib.rs:
 * 1175-1548) -- and the gated MLP product (crates/pvlc-cpu-ref/src/lib.rs:
 * 1385-1390) fused into the gate-up projection.
 *
 * gate = 0: out[r, f] = fp16(sum_k x[r, k] * w[f, k]) for r < rows, f < n.
 * gate = 1: w's rows come in blocks of 128: 64 gate rows, then the 64 up rows
 *   of the same output columns (row 128 b + j gates column 64 b + j, row
 *   128 b + 64 + j is its up row); out[r, c] = fp16(silu(fp16(g)) * fp16(u))
 *   for c < n / 2, with g, u the two projections of column c.
 * fp16 operands, f32 accumulation.  x: device [rows, k] with row pitch ldx
 * elements; w: device [n, k] contiguous; out: device with row pitch ldo.
 * rows 1..PVLC_LINEAR_MAX_ROWS, n a multiple of 128, k a multiple of 64, ldx
 * and ldo multiples of 8, pointers 16-byte aligned.  split: the K slices per
 * 128-feature tile (1, 2, 4, 8 or 16, at most k / 64), 0 for the library's
 * choice; the slices of a tile run as one thread-block cluster and their
 * partial sums are added in slice order, so results are reproducible.  No
 * device memory is allocated and no scratch is needed.
 * The call is launched with programmatic dependent launch: the weight tiles
 * are read before the kernel waits for the work ahead of it on `stream`, so
 * `w` must not be written by that work; x and out are ordered as usual.  A pipeline timeout sets PVLC_FAULT_LINEAR in the sticky fault word
 * (pvlc_attn_fault_flags).
 */
#define PVLC_LINEAR_MAX_ROWS 256u
#define PVLC_LINEAR_MAX_K 16384u
#define PVLC_LINEAR_MAX_N 65536u
int pvlc_linear(const pvlc_half* x, uint32_t rows, uint32_t ldx, const pvlc_half* w, uint32_t n,
                uint32_t k, uint32_t gate, uint32_t split, pvlc_half* out, uint32_t ldo,
                void* stream);

/* ---- model packs: BLAKE3 section digests on the device ----------------- */
/* BLAKE3 (plain hash mode, 32-byte output) of `bytes` bytes of device memory
 * at `data`: the checksum every .pvlc pack directory entry carries for its
 * section (crates/pvlc-pack/src/lib.rs: PackBuilder::build hashes each
 * section with blake3::hash, PackReader::open recomputes and compares), so a
 * pack uploaded to HBM is verified where it sits.  `digest` is 32 bytes of
 * device memory; `workspace` (16-byte aligned) holds
 * pvlc_blake3_workspace_bytes(bytes) of scratch.  Enqueued on `stream`. */
size_t pvlc_blake3_workspace_bytes(uint64_t bytes);
int pvlc_blake3(const void* data, uint64_t bytes, void* workspace, size_t workspace_bytes,
                uint8_t* digest, void* stream);

/* ----------------------------------------------------------------------------
 * Checkpoint import on the device: BF16 -> IEEE binary16, round to nearest,
 * ties to even.
 *
 * Replaces the payload half of the reference's checkpoint converter
 * (crates/pvlc-safetensors/src/fp16.rs:171-210 finite_bf16_to_f16_bits,
 * :212-276 stream_bf16_payload_to_f16; conversion id
 * "bf16_to_ieee_f16_rne_v1"): the engine uploads the BF16 payload and converts
 * it in HBM instead of writing an FP16 file on the host.
 *
 * Converts `count` elements of `src` into `dst` (both 16-byte aligned device
 * pointers; src == dst converts in place).  A NaN / infinity source, or a finite one beyond the f16 range,
 * is rejected as the reference rejects it: `*rejected` (an 8-byte aligned
 * device word) is lowered with atomicMin to
 *     (index_base + i) << 1 | out_of_range
 * for the rejected element i (out_of_range = 0: non-finite, 1: finite but out
 * of range), so after the launch it holds the lowest rejected payload index --
 * the element the reference's stream converter names -- and its reason.  The
 * call does not reset the word: set it to ~0 (no rejection) before the first
 * call of a payload, and pass each chunk's first payload index as index_base
 * when a payload is converted in several calls.  The contents of dst are
 * unspecified for a payload with a rejection.
 */
int pvlc_bf16_to_f16(const uint16_t* src, uint16_t* dst, uint64_t count, uint64_t index_base,
                     unsigned long long* rejected, void* stream);

/* ----------------------------------------------------------------------------
 * Plans: the host-side half of the contract, callable without a GPU.
 * They run the same validation as the launch entry points and report the
 * launch geometry the library will use.
 */
typedef struct pvlc_plan {
  uint32_t grid[3];
  uint32_t block[3];
  uint32_t shared_bytes;
  uint32_t work_items;       /* tiles or (sequence, chunk) units */
  uint64_t output_elements;
  uint64_t output_bytes;
  uint64_t workspace_bytes;
  double flops;              /* algorithmic FLOPs (unpadded) */
  double hbm_bytes;          /* algorithmic bytes */
} pvlc_plan;

/* Mirrors KernelInvocation::VisionAttentionF32::plan
 * (crates/pvlc-runtime-core/src/lib.rs:443-478). */
int pvlc_plan_vision_varlen(const uint32_t* cu_seqlens_host, uint32_t segments, uint32_t tokens,
                            uint32_t heads, uint32_t head_dim, pvlc_plan* plan);
/* Mirrors the prefill geometry checks of plan_decoder_stack_prefill_geometry
 * (crates/pvlc-runtime-core/src/lib.rs:2500-2653). */
int pvlc_plan_decoder_prefill(uint32_t tokens, uint32_t cache_capacity, uint32_t rope_rows,
                              pvlc_plan* plan);
/* Mirrors DecoderKvSessionDescriptor / plan_decoder_kv_session_geometry and
 * plan_cache_transition (crates/pvlc-runtime-core/src/lib.rs:980-1159):
 * pinned Q16/KV2/D128, prefix_tokens < cache_capacity. */
int pvlc_plan_decoder_kv_session(uint32_t query_heads, uint32_t kv_heads, uint32_t head_dim,
                                 uint32_t prefix_tokens, uint32_t cache_capacity,
                                 pvlc_plan* plan);
/* Batched decode launch plan for a batch whose cache rows (before append)
 * are cache_tokens_host[0..batch). */
int pvlc_plan_decode(const uint32_t* cache_tokens_host, uint32_t batch, uint32_t cache_capacity,
                     pvlc_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* PVLC_CUDA_ATTN_H */
