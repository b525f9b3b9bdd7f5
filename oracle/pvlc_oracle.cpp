// pvlc_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C++17 restatement of the attention-path arithmetic of the reference's
// `pvlc-cpu-ref` crate (plain f32 Rust, "the kernel oracle") and of the JS
// RoPE-table helpers that feed the reference's GPU path.  It is the checker
// for the CUDA kernels in this repository and the timed CPU baseline; the
// product library never links or calls it.
//
// Operation order follows the reference function by function (cited per
// function below, paths relative to the reference project root), so the f32
// results are bitwise equal to the Rust code when the platform libm agrees:
//   * sums accumulate left to right in f32, exactly as the Rust loops do;
//   * `x * s` products are NOT contracted into FMAs (built with
//     -ffp-contract=off, matching rustc, which never contracts);
//   * exp / sin / cos / pow call the C library (`expf`, `sinf`, `cosf`,
//     `powf`), which is what Rust's f32 methods lower to.
// Parallelism (OpenMP) is only across independent (token, head) outputs, so
// every output element is produced by the same scalar sequence of operations
// whatever the thread count.
//
// Parity pinning: tests/test_oracle_kat.py checks these functions against the
// reference's literal blake3 digests and literal examples.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <limits>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// Status codes mirror `CpuRefErrorCode` (crates/pvlc-cpu-ref/src/lib.rs:15-29).
enum {
  ORC_OK = 0,
  ORC_DIMENSION_MISMATCH = 1,
  ORC_ALL_MASKED = 3,
  ORC_INVALID_ROTARY_DIMENSION = 4,
  ORC_INVALID_ROPE_BASE = 5,
  ORC_NON_FINITE_INPUT = 7,
  ORC_INVALID_IMAGE_GEOMETRY = 8,
  ORC_INVALID_SEQUENCE_BOUNDARIES = 11,
  ORC_INVALID_TILE_SIZE = 12,
};

int pvlc_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void pvlc_oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"

namespace {

inline size_t attention_index(size_t token, size_t head, size_t dim, size_t heads,
                              size_t head_dim) {
  // crates/pvlc-cpu-ref/src/lib.rs:3424-3432
  return (token * heads + head) * head_dim + dim;
}

bool all_finite(const float* v, size_t n) {
  // crates/pvlc-cpu-ref/src/lib.rs:3459-3467
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(v[i])) return false;
  return true;
}

inline float fmax_rust(float a, float b) {
  // Rust f32::max: IEEE maxNum (ignores a NaN operand).
  return std::fmax(a, b);
}

int validate_sequence_boundaries(size_t tokens, const uint32_t* cu, size_t n) {
  // crates/pvlc-cpu-ref/src/lib.rs:3393-3405
  if (n < 2 || cu[0] != 0 || cu[n - 1] != tokens) return ORC_INVALID_SEQUENCE_BOUNDARIES;
  for (size_t i = 0; i + 1 < n; ++i)
    if (cu[i] >= cu[i + 1]) return ORC_INVALID_SEQUENCE_BOUNDARIES;
  return ORC_OK;
}

// Scaled dot product in dimension order, then `* scale`
// (crates/pvlc-cpu-ref/src/lib.rs:3407-3422 attention_dot; callers multiply by
// scale after the dot).
inline float dot_rows(const float* a, const float* b, size_t n) {
  float s = 0.0f;
  for (size_t d = 0; d < n; ++d) s += a[d] * b[d];
  return s;
}

// The same dot as dot_rows (left to right over dims, then `* scale`) for one
// query row against n keys at once.  Keys are stored transposed,
// kt[d * ld + key], so that 64 keys' independent sums advance side by side in
// vector lanes; every score still sees exactly dot_rows' sequence of roundings.
inline void scaled_scores(const float* q, const float* kt, size_t ld, size_t n, size_t hd,
                          float scale, float* out) {
  constexpr size_t B = 64;
  for (size_t k0 = 0; k0 < n; k0 += B) {
    float acc[B];
    for (size_t j = 0; j < B; ++j) acc[j] = 0.0f;
    if (n - k0 >= B) {
      for (size_t d = 0; d < hd; ++d) {
        const float qd = q[d];
        const float* row = kt + d * ld + k0;
        for (size_t j = 0; j < B; ++j) acc[j] += qd * row[j];
      }
      for (size_t j = 0; j < B; ++j) out[k0 + j] = acc[j] * scale;
    } else {
      const size_t nb = n - k0;
      for (size_t d = 0; d < hd; ++d) {
        const float qd = q[d];
        const float* row = kt + d * ld + k0;
        for (size_t j = 0; j < nb; ++j) acc[j] += qd * row[j];
      }
      for (size_t j = 0; j < nb; ++j) out[k0 + j] = acc[j] * scale;
    }
  }
}

// Keys [n][stride] (dims contiguous from `first`) into the transposed form
// scaled_scores reads: kt[d * n + key].  Called outside parallel regions; the
// copy itself is split across threads by key blocks.
inline void transpose_keys(const float* first, size_t stride, size_t n, size_t hd, float* kt) {
  const long long blocks = (long long)((n + 255) / 256);
#pragma omp parallel for schedule(static) if (n >= 2048)
  for (long long b = 0; b < blocks; ++b) {
    const size_t t1 = std::min(n, (size_t)(b + 1) * 256);
    for (size_t t = (size_t)b * 256; t < t1; ++t)
      for (size_t d = 0; d < hd; ++d) kt[d * n + t] = first[t * stride + d];
  }
}

// out[d] = sum over keys k in ascending order of p[k] * v[k][d], each sum from
// 0.0 -- the reference's per-dimension weighted-value loop; the dims advance
// side by side, the order of every sum is unchanged.
inline void weighted_values(const float* p, const float* v, size_t stride, size_t n, size_t hd,
                            float* out) {
  for (size_t d = 0; d < hd; ++d) out[d] = 0.0f;
  for (size_t k = 0; k < n; ++k) {
    const float pk = p[k];
    const float* row = v + k * stride;
    for (size_t d = 0; d < hd; ++d) out[d] += pk * row[d];
  }
}

// One softmax row as the reference computes it: max fold from -inf, exp of
// (x - max) summed left to right, then divide each by the sum.
// crates/pvlc-cpu-ref/src/lib.rs:369-422 (softmax_rows_f32, unmasked) and the
// identical inline sequence in causal_gqa_f32 / decode_gqa_f32 (:824-836, :897-909).
inline void softmax_row(float* p, size_t n) {
  float maximum = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < n; ++i) maximum = fmax_rust(maximum, p[i]);
  float denominator = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    p[i] = std::exp(p[i] - maximum);
    denominator += p[i];
  }
  for (size_t i = 0; i < n; ++i) p[i] /= denominator;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// Vision 2-D RoPE, direct form.
// crates/pvlc-cpu-ref/src/lib.rs:472-542 (vision_rope_2d_f32): pair p < hd/4
// rotates by the row (height) position, the rest by the column (width)
// position; frequency index p mod (hd/4); angle = pos * base^(-2 f / (hd/2))
// in f32; partner of dim p is p + hd/2.
// pos_hw holds [tokens][2] = (height, width).
int pvlc_oracle_vision_rope_2d(const float* query, const float* key, uint32_t tokens,
                               uint32_t heads, uint32_t head_dim, const uint32_t* pos_hw,
                               float base, float* q_out, float* k_out) {
  if (tokens == 0 || heads == 0) return ORC_DIMENSION_MISMATCH;
  if (head_dim == 0 || head_dim % 4 != 0) return ORC_INVALID_ROTARY_DIMENSION;
  if (!std::isfinite(base) || base <= 0.0f) return ORC_INVALID_ROPE_BASE;
  const size_t n = (size_t)tokens * heads * head_dim;
  if (!all_finite(query, n) || !all_finite(key, n)) return ORC_NON_FINITE_INPUT;
  std::memcpy(q_out, query, n * sizeof(float));
  std::memcpy(k_out, key, n * sizeof(float));
  const size_t pair_count = head_dim / 2;
  const size_t frequency_count = pair_count / 2;
#pragma omp parallel for schedule(static)
  for (long long t = 0; t < (long long)tokens; ++t) {
    const uint32_t height = pos_hw[2 * t], width = pos_hw[2 * t + 1];
    for (size_t h = 0; h < heads; ++h) {
      const size_t head_start = ((size_t)t * heads + h) * head_dim;
      for (size_t pair = 0; pair < pair_count; ++pair) {
        const size_t axis_position = pair < frequency_count ? height : width;
        const size_t frequency_index = pair % frequency_count;
        const float exponent = -(2.0f * (float)frequency_index / (float)pair_count);
        const float angle = (float)axis_position * std::pow(base, exponent);
        const float sine = std::sin(angle), cosine = std::cos(angle);
        const size_t i0 = head_start + pair, i1 = i0 + pair_count;
        const float q0 = query[i0], q1 = query[i1];
        q_out[i0] = q0 * cosine - q1 * sine;
        q_out[i1] = q1 * cosine + q0 * sine;
        const float k0 = key[i0], k1 = key[i1];
        k_out[i0] = k0 * cosine - k1 * sine;
        k_out[i1] = k1 * cosine + k0 * sine;
      }
    }
  }
  return ORC_OK;
}

// Vision RoPE tables as the reference's JS host builds them (f64 math, stored
// f32): web/engine/multimodal_ocr.mjs:98-155 (visionRope2dTables).  grids is
// [n_grids][3] = (t, h, w) in patches; tables are [tokens][hd/2].
int pvlc_oracle_vision_rope_tables(const uint32_t* grids, uint32_t n_grids, uint32_t head_dim,
                                   double theta, float* cos_out, float* sin_out) {
  if (n_grids == 0 || head_dim == 0 || head_dim % 4 != 0 || !(theta > 0.0))
    return ORC_INVALID_ROTARY_DIMENSION;
  const uint32_t pair_count = head_dim / 2, frequency_count = pair_count / 2;
  size_t token = 0;
  for (uint32_t g = 0; g < n_grids; ++g) {
    const uint32_t T = grids[3 * g], H = grids[3 * g + 1], W = grids[3 * g + 2];
    if (T == 0 || H == 0 || W == 0) return ORC_INVALID_IMAGE_GEOMETRY;
    for (uint32_t time = 0; time < T; ++time)
      for (uint32_t y = 0; y < H; ++y)
        for (uint32_t x = 0; x < W; ++x) {
          const size_t base = token * pair_count;
          for (uint32_t pair = 0; pair < pair_count; ++pair) {
            const double position = pair < frequency_count ? (double)y : (double)x;
            const uint32_t frequency = pair % frequency_count;
            const double inverse_frequency =
                std::pow(theta, -(2.0 * (double)frequency) / (double)pair_count);
            const double angle = position * inverse_frequency;
            cos_out[base + pair] = (float)std::cos(angle);
            sin_out[base + pair] = (float)std::sin(angle);
          }
          ++token;
        }
  }
  return ORC_OK;
}

// Table-driven vision RoPE, the arithmetic of the reference's vision_rope_2d
// GPU kernel (crates/pvlc-wgsl/src/lib.rs:1691-1730): pair p of each head uses
// table entry [token][p].
int pvlc_oracle_vision_rope_apply_tables(const float* query, const float* key, uint32_t tokens,
                                         uint32_t heads, uint32_t head_dim, const float* cos_t,
                                         const float* sin_t, float* q_out, float* k_out) {
  if (tokens == 0 || heads == 0) return ORC_DIMENSION_MISMATCH;
  if (head_dim == 0 || head_dim % 4 != 0) return ORC_INVALID_ROTARY_DIMENSION;
  const size_t n = (size_t)tokens * heads * head_dim;
  std::memcpy(q_out, query, n * sizeof(float));
  std::memcpy(k_out, key, n * sizeof(float));
  const size_t pc = head_dim / 2;
#pragma omp parallel for schedule(static)
  for (long long t = 0; t < (long long)tokens; ++t)
    for (size_t h = 0; h < heads; ++h)
      for (size_t p = 0; p < pc; ++p) {
        const size_t i0 = ((size_t)t * heads + h) * head_dim + p, i1 = i0 + pc;
        const float c = cos_t[(size_t)t * pc + p], s = sin_t[(size_t)t * pc + p];
        const float q0 = query[i0], q1 = query[i1], k0 = key[i0], k1 = key[i1];
        q_out[i0] = q0 * c - q1 * s;
        q_out[i1] = q1 * c + q0 * s;
        k_out[i0] = k0 * c - k1 * s;
        k_out[i1] = k1 * c + k0 * s;
      }
  return ORC_OK;
}

// ---------------------------------------------------------------------------
// Segmented (block-diagonal) bidirectional attention, materialized form.
// crates/pvlc-cpu-ref/src/lib.rs:2752-2802 (materialized_segmented_attention_f32)
// with validate_attention_inputs :3275-3302.  Per (segment, head, query row):
// scores = dot * scale over the segment's keys, softmax_rows_f32, then the
// weighted value sum in key order for each dimension.
int pvlc_oracle_segmented_attention(const float* query, const float* key, const float* value,
                                    uint32_t tokens, uint32_t heads, uint32_t head_dim,
                                    const uint32_t* cu_seqlens, uint32_t n_cu, float* out) {
  if (tokens == 0 || heads == 0 || head_dim == 0) return ORC_DIMENSION_MISMATCH;
  const size_t n = (size_t)tokens * heads * head_dim;
  if (!all_finite(query, n) || !all_finite(key, n) || !all_finite(value, n))
    return ORC_NON_FINITE_INPUT;
  int st = validate_sequence_boundaries(tokens, cu_seqlens, n_cu);
  if (st) return st;
  const float scale = 1.0f / std::sqrt((float)head_dim);
  const size_t stride = (size_t)heads * head_dim;
  for (uint32_t seg = 0; seg + 1 < n_cu; ++seg) {
    const size_t start = cu_seqlens[seg], end = cu_seqlens[seg + 1], len = end - start;
    std::vector<float> kt((size_t)heads * head_dim * len);
    for (long long h = 0; h < (long long)heads; ++h)
      transpose_keys(key + attention_index(start, h, 0, heads, head_dim), stride, len, head_dim,
                     kt.data() + (size_t)h * head_dim * len);
#pragma omp parallel
    {
      std::vector<float> row(len);
#pragma omp for collapse(2) schedule(static)
      for (long long h = 0; h < (long long)heads; ++h)
        for (long long qo = 0; qo < (long long)len; ++qo) {
          const size_t qt = start + qo;
          const float* qrow = query + attention_index(qt, h, 0, heads, head_dim);
          scaled_scores(qrow, kt.data() + (size_t)h * head_dim * len, len, len, head_dim, scale,
                        row.data());
          softmax_row(row.data(), len);
          weighted_values(row.data(), value + attention_index(start, h, 0, heads, head_dim),
                          stride, len, head_dim,
                          out + attention_index(qt, h, 0, heads, head_dim));
        }
    }
  }
  return ORC_OK;
}

// Streaming (online-softmax) segmented attention.
// crates/pvlc-cpu-ref/src/lib.rs:2805-2878 (streaming_segmented_attention_f32):
// for each key, m' = max(m, s); d = d*exp(m-m') + exp(s-m');
// acc = acc*exp(m-m') + v*exp(s-m'); key blocks of `key_tile` visited forward
// (order 0) or with blocks in reverse order (order 1); out = acc / d.
int pvlc_oracle_streaming_segmented_attention(const float* query, const float* key,
                                              const float* value, uint32_t tokens,
                                              uint32_t heads, uint32_t head_dim,
                                              const uint32_t* cu_seqlens, uint32_t n_cu,
                                              uint32_t key_tile, int order, float* out) {
  if (key_tile == 0) return ORC_INVALID_TILE_SIZE;
  if (tokens == 0 || heads == 0 || head_dim == 0) return ORC_DIMENSION_MISMATCH;
  const size_t n = (size_t)tokens * heads * head_dim;
  if (!all_finite(query, n) || !all_finite(key, n) || !all_finite(value, n))
    return ORC_NON_FINITE_INPUT;
  int st = validate_sequence_boundaries(tokens, cu_seqlens, n_cu);
  if (st) return st;
  const float scale = 1.0f / std::sqrt((float)head_dim);
  for (uint32_t seg = 0; seg + 1 < n_cu; ++seg) {
    const size_t s0 = cu_seqlens[seg], s1 = cu_seqlens[seg + 1];
#pragma omp parallel
    {
      std::vector<float> wv(head_dim);
#pragma omp for collapse(2) schedule(static)
      for (long long qt = (long long)s0; qt < (long long)s1; ++qt)
        for (long long h = 0; h < (long long)heads; ++h) {
          std::fill(wv.begin(), wv.end(), 0.0f);
          float maximum = -std::numeric_limits<float>::infinity();
          float denominator = 0.0f;
          const float* qrow = query + attention_index(qt, h, 0, heads, head_dim);
          auto process_key = [&](size_t kt) {
            const float score =
                dot_rows(qrow, key + attention_index(kt, h, 0, heads, head_dim), head_dim) * scale;
            const float next_maximum = fmax_rust(maximum, score);
            const float previous_scale = std::exp(maximum - next_maximum);
            const float score_scale = std::exp(score - next_maximum);
            denominator = denominator * previous_scale + score_scale;
            const float* vrow = value + attention_index(kt, h, 0, heads, head_dim);
            for (size_t d = 0; d < head_dim; ++d) wv[d] = wv[d] * previous_scale + vrow[d] * score_scale;
            maximum = next_maximum;
          };
          if (order == 0) {
            for (size_t b0 = s0; b0 < s1;) {
              const size_t b1 = std::min(b0 + key_tile, s1);
              for (size_t kt = b0; kt < b1; ++kt) process_key(kt);
              b0 = b1;
            }
          } else {
            for (size_t b1 = s1; b1 > s0;) {
              const size_t b0 = (b1 - s0 > key_tile) ? b1 - key_tile : s0;
              for (size_t kt = b0; kt < b1; ++kt) process_key(kt);
              b1 = b0;
            }
          }
          float* orow = out + attention_index(qt, h, 0, heads, head_dim);
          for (size_t d = 0; d < head_dim; ++d) orow[d] = wv[d] / denominator;
        }
    }
  }
  return ORC_OK;
}

// ---------------------------------------------------------------------------
// Decoder multimodal RoPE.
// crates/pvlc-cpu-ref/src/lib.rs:562-672 (apply_multimodal_rope_f32): the
// per-token cos/sin row is assembled from axis planes [3][tokens][hd] in chunk
// order sections (s0,s1,s2,s0,s1,s2), chunk c reading axis c mod 3 at the
// same dim offset; then out[d] = x[d]*cos[d] + partner*sin[d] with partner
// -x[d+hd/2] for d < hd/2 and x[d-hd/2] otherwise.
int pvlc_oracle_apply_multimodal_rope(const float* query, const float* key, uint32_t tokens,
                                      uint32_t query_heads, uint32_t kv_heads,
                                      uint32_t head_dim, const float* raw_cos,
                                      const float* raw_sin, const uint32_t* sections,
                                      float* q_out, float* k_out) {
  if (tokens == 0 || query_heads == 0 || kv_heads == 0 || head_dim == 0)
    return ORC_DIMENSION_MISMATCH;
  if (query_heads % kv_heads) return ORC_DIMENSION_MISMATCH;
  if (sections[0] == 0 || sections[1] == 0 || sections[2] == 0) return ORC_DIMENSION_MISMATCH;
  if ((sections[0] + sections[1] + sections[2]) * 2 != head_dim) return ORC_DIMENSION_MISMATCH;
  const size_t qn = (size_t)tokens * query_heads * head_dim;
  const size_t kn = (size_t)tokens * kv_heads * head_dim;
  const size_t rn = (size_t)3 * tokens * head_dim;
  if (!all_finite(query, qn) || !all_finite(key, kn) || !all_finite(raw_cos, rn) ||
      !all_finite(raw_sin, rn))
    return ORC_NON_FINITE_INPUT;
  const uint32_t rep[6] = {sections[0], sections[1], sections[2],
                           sections[0], sections[1], sections[2]};
  const size_t half = head_dim / 2;
#pragma omp parallel
  {
    std::vector<float> sc(head_dim), ss(head_dim);
#pragma omp for schedule(static)
    for (long long t = 0; t < (long long)tokens; ++t) {
      size_t off = 0;
      for (int c = 0; c < 6; ++c) {
        const size_t axis = c % 3;
        const size_t base = axis * tokens * head_dim + (size_t)t * head_dim + off;
        for (uint32_t i = 0; i < rep[c]; ++i) {
          sc[off + i] = raw_cos[base + i];
          ss[off + i] = raw_sin[base + i];
        }
        off += rep[c];
      }
      auto rotate = [&](const float* in, float* o, uint32_t heads) {
        for (size_t h = 0; h < heads; ++h) {
          const size_t rs = attention_index(t, h, 0, heads, head_dim);
          for (size_t d = 0; d < head_dim; ++d) {
            const float src = d < half ? -in[rs + d + half] : in[rs + d - half];
            o[rs + d] = in[rs + d] * sc[d] + src * ss[d];
          }
        }
      };
      rotate(query, q_out, query_heads);
      rotate(key, k_out, kv_heads);
    }
  }
  return ORC_OK;
}

// M-RoPE cos/sin tables, axis-major [3][capacity][hd], as the reference's JS
// host builds them: web/engine/multimodal_ocr.mjs:937-986 (ropeTables).
// inverse frequencies in f64, angle = position * inv_freq[d mod hd/2] in f64,
// cos/sin in f64 stored as f32; rows >= prompt_tokens use (row + rope_delta).
// positions is [3][prompt_tokens] (int64).
int pvlc_oracle_rope_tables(const int64_t* positions, uint32_t prompt_tokens, int64_t rope_delta,
                            uint32_t capacity, double theta, uint32_t head_dim, float* cos_out,
                            float* sin_out) {
  if (prompt_tokens == 0 || capacity < prompt_tokens || !(theta > 0.0) || head_dim % 2)
    return ORC_DIMENSION_MISMATCH;
  const uint32_t half = head_dim / 2;
  std::vector<double> inv(half);
  for (uint32_t i = 0; i < half; ++i) inv[i] = std::pow(theta, -(2.0 * (double)i) / (double)head_dim);
  for (uint32_t axis = 0; axis < 3; ++axis)
    for (uint32_t t = 0; t < capacity; ++t) {
      const double position = t < prompt_tokens ? (double)positions[(size_t)axis * prompt_tokens + t]
                                                : (double)((int64_t)t + rope_delta);
      for (uint32_t d = 0; d < head_dim; ++d) {
        const uint32_t hf = d >= half ? d - half : d;
        const double angle = position * inv[hf];
        const size_t idx = ((size_t)axis * capacity + t) * head_dim + d;
        cos_out[idx] = (float)std::cos(angle);
        sin_out[idx] = (float)std::sin(angle);
      }
    }
  return ORC_OK;
}

// ---------------------------------------------------------------------------
// Causal GQA prefill.  crates/pvlc-cpu-ref/src/lib.rs:782-853 (causal_gqa_f32):
// q-head h reads kv-head h / (Q/KV); score = dot * scale; max fold; exp and
// sum; divide; weighted V per dimension in key order.
int pvlc_oracle_causal_gqa(const float* query, const float* key, const float* value,
                           uint32_t tokens, uint32_t query_heads, uint32_t kv_heads,
                           uint32_t head_dim, float* out) {
  if (tokens == 0 || query_heads == 0 || kv_heads == 0 || head_dim == 0)
    return ORC_DIMENSION_MISMATCH;
  if (query_heads % kv_heads) return ORC_DIMENSION_MISMATCH;
  const size_t qn = (size_t)tokens * query_heads * head_dim;
  const size_t kn = (size_t)tokens * kv_heads * head_dim;
  if (!all_finite(query, qn) || !all_finite(key, kn) || !all_finite(value, kn))
    return ORC_NON_FINITE_INPUT;
  const size_t group = query_heads / kv_heads;
  const float scale = 1.0f / std::sqrt((float)head_dim);
  const size_t kstride = (size_t)kv_heads * head_dim;
  std::vector<float> kt((size_t)kv_heads * head_dim * tokens);
  for (size_t g = 0; g < kv_heads; ++g)
    transpose_keys(key + g * head_dim, kstride, tokens, head_dim,
                   kt.data() + g * head_dim * tokens);
#pragma omp parallel
  {
    std::vector<float> p(tokens);
#pragma omp for collapse(2) schedule(dynamic, 16)
    for (long long qt = 0; qt < (long long)tokens; ++qt)
      for (long long h = 0; h < (long long)query_heads; ++h) {
        const size_t kvh = h / group;
        const float* qrow = query + attention_index(qt, h, 0, query_heads, head_dim);
        const size_t n = qt + 1;
        scaled_scores(qrow, kt.data() + kvh * head_dim * tokens, tokens, n, head_dim, scale,
                      p.data());
        softmax_row(p.data(), n);
        weighted_values(p.data(), value + kvh * head_dim, kstride, n, head_dim,
                        out + attention_index(qt, h, 0, query_heads, head_dim));
      }
  }
  return ORC_OK;
}

// Single-token decode GQA over a full cache.
// crates/pvlc-cpu-ref/src/lib.rs:858-927 (decode_gqa_f32).
int pvlc_oracle_decode_gqa(const float* query, const float* key, const float* value,
                           uint32_t cache_tokens, uint32_t query_heads, uint32_t kv_heads,
                           uint32_t head_dim, float* out) {
  if (cache_tokens == 0 || query_heads == 0 || kv_heads == 0 || head_dim == 0)
    return ORC_DIMENSION_MISMATCH;
  if (query_heads % kv_heads) return ORC_DIMENSION_MISMATCH;
  const size_t kn = (size_t)cache_tokens * kv_heads * head_dim;
  if (!all_finite(query, (size_t)query_heads * head_dim) || !all_finite(key, kn) ||
      !all_finite(value, kn))
    return ORC_NON_FINITE_INPUT;
  const size_t group = query_heads / kv_heads;
  const float scale = 1.0f / std::sqrt((float)head_dim);
  const size_t kstride = (size_t)kv_heads * head_dim;
  std::vector<float> kt((size_t)kv_heads * head_dim * cache_tokens);
  for (size_t g = 0; g < kv_heads; ++g)
    transpose_keys(key + g * head_dim, kstride, cache_tokens, head_dim,
                   kt.data() + g * head_dim * cache_tokens);
#pragma omp parallel
  {
    std::vector<float> p(cache_tokens);
#pragma omp for schedule(static)
    for (long long h = 0; h < (long long)query_heads; ++h) {
      const size_t kvh = h / group;
      const float* qrow = query + (size_t)h * head_dim;
      scaled_scores(qrow, kt.data() + kvh * head_dim * cache_tokens, cache_tokens, cache_tokens,
                    head_dim, scale, p.data());
      softmax_row(p.data(), cache_tokens);
      weighted_values(p.data(), value + kvh * head_dim, kstride, cache_tokens, head_dim,
                      out + (size_t)h * head_dim);
    }
  }
  return ORC_OK;
}

// One decoder decode-attention step as the reference composes it
// (crates/pvlc-cpu-ref/src/lib.rs:1648-1680 decoder_layer_decode_f32, with the
// append of :1420-1450 and the single-row M-RoPE of the decode path): rotate
// the raw query/key with table row `rope_row` of [3][rope_rows][hd] (section
// layout `sections`), append the rotated key and raw value at row
// `prefix_tokens` of the cache, then decode_gqa over prefix_tokens + 1 rows.
// The caches are [capacity][kv_heads][hd] f32 and are updated in place.
int pvlc_oracle_decode_step(const float* query, const float* key_new, const float* value_new,
                            const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                            uint32_t rope_row, const uint32_t* sections, float* key_cache,
                            float* value_cache, uint32_t prefix_tokens, uint32_t capacity,
                            uint32_t query_heads, uint32_t kv_heads, uint32_t head_dim,
                            float* out) {
  if (prefix_tokens >= capacity || rope_row >= rope_rows) return ORC_DIMENSION_MISMATCH;
  // Assemble the one-token tables the way apply_multimodal_rope_f32 indexes
  // them (axis planes of a 1-token table).
  std::vector<float> c1(3 * head_dim), s1(3 * head_dim);
  for (uint32_t a = 0; a < 3; ++a)
    for (uint32_t d = 0; d < head_dim; ++d) {
      c1[a * head_dim + d] = rope_cos[((size_t)a * rope_rows + rope_row) * head_dim + d];
      s1[a * head_dim + d] = rope_sin[((size_t)a * rope_rows + rope_row) * head_dim + d];
    }
  std::vector<float> qr((size_t)query_heads * head_dim), kr((size_t)kv_heads * head_dim);
  int st = pvlc_oracle_apply_multimodal_rope(query, key_new, 1, query_heads, kv_heads, head_dim,
                                             c1.data(), s1.data(), sections, qr.data(), kr.data());
  if (st) return st;
  const size_t w = (size_t)kv_heads * head_dim;
  std::memcpy(key_cache + (size_t)prefix_tokens * w, kr.data(), w * sizeof(float));
  std::memcpy(value_cache + (size_t)prefix_tokens * w, value_new, w * sizeof(float));
  return pvlc_oracle_decode_gqa(qr.data(), key_cache, value_cache, prefix_tokens + 1, query_heads,
                                kv_heads, head_dim, out);
}

// Decoder prefill attention as composed by the reference
// (crates/pvlc-cpu-ref/src/lib.rs:1592-1627 decoder_layer_prefill_f32, closure
// :1607-1625): apply_multimodal_rope_f32 with tables sliced to the prompt
// rows, write_decoder_prefill_kv_f32 (:976-991) of the rotated key and raw
// value into cache rows [0, tokens), then causal_gqa_f32 on rotated q/k.
// Tables are [3][rope_rows][hd]; rows [0, tokens) are used.
int pvlc_oracle_decoder_prefill(const float* query, const float* key, const float* value,
                                const float* rope_cos, const float* rope_sin, uint32_t rope_rows,
                                const uint32_t* sections, uint32_t tokens, uint32_t query_heads,
                                uint32_t kv_heads, uint32_t head_dim, float* key_cache,
                                float* value_cache, uint32_t capacity, float* out) {
  if (tokens == 0 || tokens > capacity || tokens > rope_rows) return ORC_DIMENSION_MISMATCH;
  std::vector<float> cs((size_t)3 * tokens * head_dim), ss(cs.size());
  for (uint32_t a = 0; a < 3; ++a) {
    std::memcpy(cs.data() + (size_t)a * tokens * head_dim, rope_cos + (size_t)a * rope_rows * head_dim,
                (size_t)tokens * head_dim * sizeof(float));
    std::memcpy(ss.data() + (size_t)a * tokens * head_dim, rope_sin + (size_t)a * rope_rows * head_dim,
                (size_t)tokens * head_dim * sizeof(float));
  }
  std::vector<float> qr((size_t)tokens * query_heads * head_dim), kr((size_t)tokens * kv_heads * head_dim);
  int st = pvlc_oracle_apply_multimodal_rope(query, key, tokens, query_heads, kv_heads, head_dim,
                                             cs.data(), ss.data(), sections, qr.data(), kr.data());
  if (st) return st;
  const size_t kvn = (size_t)tokens * kv_heads * head_dim;
  std::memcpy(key_cache, kr.data(), kvn * sizeof(float));
  std::memcpy(value_cache, value, kvn * sizeof(float));
  return pvlc_oracle_causal_gqa(qr.data(), kr.data(), value, tokens, query_heads, kv_heads, head_dim,
                                out);
}

// ---------------------------------------------------------------------------
// M-RoPE position ids.  crates/pvlc-cpu-ref/src/multimodal.rs:28-78
// (mrope_position_ids, no attention mask) with image_positions :249-321,
// append_text_positions :323-340, append_image_positions :342-365,
// checked_rope_delta :367-373.  grids_thw are pre-merge patch grids.
// positions_out is [3][n_ids]; returns ORC_INVALID_SEQUENCE_BOUNDARIES on a
// malformed prompt.
int pvlc_oracle_mrope_position_ids(const uint32_t* input_ids, uint32_t n_ids,
                                   const uint32_t* grids_thw, uint32_t n_grids,
                                   uint32_t image_token_id, uint32_t vision_start_token_id,
                                   uint32_t spatial_merge_size, int64_t* positions_out,
                                   int64_t* rope_delta_out) {
  if (n_ids == 0 || image_token_id == vision_start_token_id) return ORC_INVALID_SEQUENCE_BOUNDARIES;
  if (spatial_merge_size == 0) return ORC_INVALID_IMAGE_GEOMETRY;
  struct Grid { int64_t t, h, w, tokens; };
  std::vector<Grid> grids;
  for (uint32_t g = 0; g < n_grids; ++g) {
    const uint32_t t = grids_thw[3 * g], h = grids_thw[3 * g + 1], w = grids_thw[3 * g + 2];
    if (t == 0 || h == 0 || w == 0 || h % spatial_merge_size || w % spatial_merge_size)
      return ORC_INVALID_IMAGE_GEOMETRY;
    const int64_t hm = h / spatial_merge_size, wm = w / spatial_merge_size;
    grids.push_back({(int64_t)t, hm, wm, (int64_t)t * hm * wm});
  }
  std::vector<int64_t> ax[3];
  auto finish = [&](int64_t max_pos) {
    for (int a = 0; a < 3; ++a)
      std::memcpy(positions_out + (size_t)a * n_ids, ax[a].data(), n_ids * sizeof(int64_t));
    *rope_delta_out = max_pos + 1 - (int64_t)n_ids;
    return ORC_OK;
  };
  if (grids.empty()) {
    for (uint32_t i = 0; i < n_ids; ++i)
      if (input_ids[i] == image_token_id || input_ids[i] == vision_start_token_id)
        return ORC_INVALID_SEQUENCE_BOUNDARIES;
    for (int a = 0; a < 3; ++a)
      for (uint32_t i = 0; i < n_ids; ++i) ax[a].push_back(i);
    return finish((int64_t)n_ids - 1);
  }
  size_t cursor = 0, grid_index = 0;
  int64_t next_position = 0;
  auto append_text = [&](size_t length, int64_t start) {
    for (size_t o = 0; o < length; ++o)
      for (int a = 0; a < 3; ++a) ax[a].push_back(start + (int64_t)o);
  };
  while (true) {
    size_t vs = cursor;
    while (vs < n_ids && input_ids[vs] != vision_start_token_id) ++vs;
    if (vs >= n_ids) break;
    for (size_t i = cursor; i < vs; ++i)
      if (input_ids[i] == image_token_id) return ORC_INVALID_SEQUENCE_BOUNDARIES;
    if (grid_index >= grids.size()) return ORC_INVALID_SEQUENCE_BOUNDARIES;
    const Grid g = grids[grid_index];
    const size_t image_start = vs + 1, image_end = image_start + (size_t)g.tokens;
    if (image_end > n_ids) return ORC_INVALID_SEQUENCE_BOUNDARIES;
    for (size_t i = image_start; i < image_end; ++i)
      if (input_ids[i] != image_token_id) return ORC_INVALID_SEQUENCE_BOUNDARIES;
    if (image_end < n_ids && input_ids[image_end] == image_token_id)
      return ORC_INVALID_SEQUENCE_BOUNDARIES;
    const size_t text_length = image_start - cursor;
    append_text(text_length, next_position);
    const int64_t visual_start = next_position + (int64_t)text_length;
    for (int64_t tt = 0; tt < g.t; ++tt)
      for (int64_t y = 0; y < g.h; ++y)
        for (int64_t x = 0; x < g.w; ++x) {
          ax[0].push_back(visual_start);
          ax[1].push_back(visual_start + y);
          ax[2].push_back(visual_start + x);
        }
    next_position = visual_start + std::max(g.h - 1, g.w - 1) + 1;
    cursor = image_end;
    ++grid_index;
  }
  if (grid_index != grids.size()) return ORC_INVALID_SEQUENCE_BOUNDARIES;
  for (size_t i = cursor; i < n_ids; ++i)
    if (input_ids[i] == image_token_id || input_ids[i] == vision_start_token_id)
      return ORC_INVALID_SEQUENCE_BOUNDARIES;
  append_text(n_ids - cursor, next_position);
  int64_t mx = ax[0][0];
  for (int a = 0; a < 3; ++a)
    for (int64_t v : ax[a]) mx = std::max(mx, v);
  return finish(mx);
}

// Decode-time M-RoPE position, crates/pvlc-cpu-ref/src/multimodal.rs:80-113:
// cache_position + rope_delta on all three axes (must be >= 0).
int pvlc_oracle_decode_mrope_position(uint32_t cache_position, int64_t rope_delta,
                                      int64_t* position_out) {
  const int64_t p = (int64_t)cache_position + rope_delta;
  if (p < 0) return ORC_INVALID_SEQUENCE_BOUNDARIES;
  *position_out = p;
  return ORC_OK;
}

}  // extern "C"
