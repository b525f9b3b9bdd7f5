// pvlc_model_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Model-level composition of the reference's CPU oracle (`pvlc-cpu-ref`), on
// top of the attention functions of pvlc_oracle.cpp: the f32 primitives
// (linear, RMSNorm, LayerNorm, SiLU, GELU), the decoder layer, the vision
// encoder layer with its 2-D RoPE, the projector, the LM head and greedy
// top-1 generation, composed into one PaddleOCR-VL request.  It is the checker
// for the GPU engine's end-to-end greedy tokens; the product never links it.
//
// Operation order follows the reference function by function (citations per
// function, paths relative to the reference project root), under the same
// rules as pvlc_oracle.cpp: left-to-right f32 sums, no FMA contraction
// (-ffp-contract=off), libm exp/tanh/erf.
//
// fp16 storage (the `fp16_storage` flag of pvlc_oracle_generate): the GPU
// engine keeps weights and every intermediate tensor in fp16 except the
// residual streams and the logits (f32).  With the flag set, this oracle rounds
// to fp16 (round to nearest even) at exactly those storage points, so the
// remaining GPU/CPU difference is only summation order.  With the flag clear
// it is the plain f32 reference composition.

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
// pvlc_oracle.cpp
int pvlc_oracle_vision_rope_tables(const uint32_t* grids, uint32_t n_grids, uint32_t head_dim,
                                   double theta, float* cos_out, float* sin_out);
int pvlc_oracle_vision_rope_apply_tables(const float* query, const float* key, uint32_t tokens,
                                         uint32_t heads, uint32_t head_dim, const float* cos_t,
                                         const float* sin_t, float* q_out, float* k_out);
int pvlc_oracle_segmented_attention(const float* query, const float* key, const float* value,
                                    uint32_t tokens, uint32_t heads, uint32_t head_dim,
                                    const uint32_t* cu_seqlens, uint32_t n_cu, float* out);
int pvlc_oracle_apply_multimodal_rope(const float* query, const float* key, uint32_t tokens,
                                      uint32_t query_heads, uint32_t kv_heads,
                                      uint32_t head_dim, const float* raw_cos,
                                      const float* raw_sin, const uint32_t* sections,
                                      float* q_out, float* k_out);
int pvlc_oracle_rope_tables(const int64_t* positions, uint32_t prompt_tokens, int64_t rope_delta,
                            uint32_t capacity, double theta, uint32_t head_dim, float* cos_out,
                            float* sin_out);
int pvlc_oracle_causal_gqa(const float* query, const float* key, const float* value,
                           uint32_t tokens, uint32_t query_heads, uint32_t kv_heads,
                           uint32_t head_dim, float* out);
int pvlc_oracle_decode_gqa(const float* query, const float* key, const float* value,
                           uint32_t cache_tokens, uint32_t query_heads, uint32_t kv_heads,
                           uint32_t head_dim, float* out);
int pvlc_oracle_mrope_position_ids(const uint32_t* input_ids, uint32_t n_ids,
                                   const uint32_t* grids_thw, uint32_t n_grids,
                                   uint32_t image_token_id, uint32_t vision_start_token_id,
                                   uint32_t spatial_merge_size, int64_t* positions_out,
                                   int64_t* rope_delta_out);

// Model geometry of pvlc_oracle_generate (doubles first: no padding questions
// for the ctypes mirror).
typedef struct {
  double vision_theta, decoder_theta;
  float vision_eps, projector_eps, decoder_eps, reserved;
  uint32_t vision_layers, vision_hidden, vision_heads, vision_head_dim, vision_intermediate;
  uint32_t patch_input, pos_side, merge;
  uint32_t decoder_layers, decoder_hidden, query_heads, kv_heads, head_dim,
      decoder_intermediate;
  uint32_t vocab, eos_token_id, image_token_id, vision_start_token_id;
  uint32_t sections[3], reserved2;
} pvlc_oracle_model_dims;
}

namespace {

enum { OK = 0, DIMENSION_MISMATCH = 1, NON_FINITE_INPUT = 7 };

using Vec = std::vector<float>;

inline float f16_round(float x) { return (float)(_Float16)x; }

// Elementwise passes below are split across threads only by element, so each
// element sees the same single operation whatever the thread count.
void store(Vec& v, bool f16) {
  if (!f16) return;
  const long long n = (long long)v.size();
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) v[i] = f16_round(v[i]);
}

inline float widen_half(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}

Vec widen(const uint16_t* p, size_t n) {
  Vec out(n);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) out[i] = widen_half(p[i]);
  return out;
}

// crates/pvlc-cpu-ref/src/lib.rs:88-140 (patch_projection_f32, linear_f32) and
// :1294-1303 (linear_no_bias_f32, a zero bias): the accumulator starts at the
// bias and adds input * weight in input order; weights are output-major
// [out][in].
void linear(const float* in, size_t rows, size_t iw, const float* w, const float* bias, size_t ow,
            float* out) {
  // Every output is the same scalar sequence (start at the bias, then
  // `acc += x[d] * w[o][d]` for d ascending); only independent outputs are
  // computed side by side.  Few rows (a decode step, the LM head): 8 outputs
  // per thread step, weights read in place.  Many rows: the weights are first
  // transposed to [in][out] so a block of 4 rows x 64 outputs advances in
  // vector lanes.
  if (rows < 8) {
    const long long groups = (long long)((ow + 7) / 8);
#pragma omp parallel for schedule(static)
    for (long long gi = 0; gi < groups; ++gi) {
      const size_t o0 = (size_t)gi * 8, no = std::min<size_t>(8, ow - o0);
      for (size_t r = 0; r < rows; ++r) {
        const float* x = in + r * iw;
        float acc[8];
        for (size_t j = 0; j < no; ++j) acc[j] = bias ? bias[o0 + j] : 0.0f;
        if (no == 8) {
          for (size_t d = 0; d < iw; ++d) {
            const float xd = x[d];
            for (size_t j = 0; j < 8; ++j) acc[j] += xd * w[(o0 + j) * iw + d];
          }
        } else {
          for (size_t d = 0; d < iw; ++d)
            for (size_t j = 0; j < no; ++j) acc[j] += x[d] * w[(o0 + j) * iw + d];
        }
        for (size_t j = 0; j < no; ++j) out[r * ow + o0 + j] = acc[j];
      }
    }
    return;
  }
  std::vector<float> wt(iw * ow);
#pragma omp parallel for schedule(static)
  for (long long o = 0; o < (long long)ow; ++o)
    for (size_t d = 0; d < iw; ++d) wt[d * ow + (size_t)o] = w[(size_t)o * iw + d];
  constexpr size_t RB = 4, OB = 64;
  const long long rblocks = (long long)((rows + RB - 1) / RB);
  const long long oblocks = (long long)((ow + OB - 1) / OB);
#pragma omp parallel for collapse(2) schedule(static)
  for (long long rb = 0; rb < rblocks; ++rb)
    for (long long ob = 0; ob < oblocks; ++ob) {
      const size_t r0 = (size_t)rb * RB, nr = std::min(RB, rows - r0);
      const size_t o0 = (size_t)ob * OB, no = std::min(OB, ow - o0);
      float acc[RB][OB];
      for (size_t r = 0; r < RB; ++r)
        for (size_t j = 0; j < OB; ++j) acc[r][j] = (bias && j < no) ? bias[o0 + j] : 0.0f;
      if (nr == RB && no == OB) {
        for (size_t d = 0; d < iw; ++d) {
          const float* wr = &wt[d * ow + o0];
          for (size_t r = 0; r < RB; ++r) {
            const float xd = in[(r0 + r) * iw + d];
            for (size_t j = 0; j < OB; ++j) acc[r][j] += xd * wr[j];
          }
        }
      } else {
        for (size_t d = 0; d < iw; ++d) {
          const float* wr = &wt[d * ow + o0];
          for (size_t r = 0; r < nr; ++r) {
            const float xd = in[(r0 + r) * iw + d];
            for (size_t j = 0; j < no; ++j) acc[r][j] += xd * wr[j];
          }
        }
      }
      for (size_t r = 0; r < nr; ++r)
        for (size_t j = 0; j < no; ++j) out[(r0 + r) * ow + o0 + j] = acc[r][j];
    }
}

Vec linear_v(const Vec& in, size_t rows, size_t iw, const float* w, const float* bias, size_t ow,
             bool f16) {
  Vec out(rows * ow);
  linear(in.data(), rows, iw, w, bias, ow, out.data());
  store(out, f16);
  return out;
}

// crates/pvlc-cpu-ref/src/lib.rs:321-352 (rms_norm_f32)
void rms_norm(const float* in, size_t rows, size_t width, const float* weight, float eps,
              float* out) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const float* s = in + r * width;
    float ms = 0.0f;
    for (size_t i = 0; i < width; ++i) ms += s[i] * s[i];
    ms /= (float)width;
    const float inv = 1.0f / std::sqrt(ms + eps);
    for (size_t c = 0; c < width; ++c) out[r * width + c] = s[c] * inv * weight[c];
  }
}

// crates/pvlc-cpu-ref/src/lib.rs:280-319 (layer_norm_f32)
void layer_norm(const float* in, size_t rows, size_t width, const float* weight,
                const float* bias, float eps, float* out) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const float* s = in + r * width;
    float mean = 0.0f;
    for (size_t i = 0; i < width; ++i) mean += s[i];
    mean /= (float)width;
    float var = 0.0f;
    for (size_t i = 0; i < width; ++i) {
      const float c = s[i] - mean;
      var += c * c;
    }
    var /= (float)width;
    const float inv = 1.0f / std::sqrt(var + eps);
    for (size_t c = 0; c < width; ++c)
      out[r * width + c] = (s[c] - mean) * inv * weight[c] + bias[c];
  }
}

// crates/pvlc-cpu-ref/src/lib.rs:354-367
inline float silu(float v) { return v / (1.0f + std::exp(-v)); }
inline float gelu_tanh(float v) {
  const float cube = v * v * v;   // f32::powi(3)
  return 0.5f * v * (1.0f + std::tanh(0.7978846f * (v + 0.044715f * cube)));
}
inline float gelu_erf(float v) { return 0.5f * v * (1.0f + std::erf(v * 0.70710677f)); }

void add_into(Vec& acc, const Vec& x) {
  // crates/pvlc-cpu-ref/src/lib.rs:142-154 (add_vectors_f32)
  const long long n = (long long)acc.size();
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) acc[i] = acc[i] + x[i];
}

void apply(Vec& v, float (*f)(float)) {
  const long long n = (long long)v.size();
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) v[i] = f(v[i]);
}

void silu_gate(const Vec& gate, const Vec& up, Vec& act) {
  const long long n = (long long)act.size();
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; ++i) act[i] = silu(gate[i]) * up[i];
}

// Bilinear source coordinate, crates/pvlc-cpu-ref/src/lib.rs:265-278.
void bilinear_axis(size_t source, size_t target, size_t index, size_t* lo, size_t* hi,
                   float* frac) {
  const float coord =
      target == 1 ? 0.0f : (float)index * (float)(source - 1) / (float)(target - 1);
  size_t l = (size_t)std::floor(coord);
  l = std::min(l, source - 1);
  *lo = l;
  *hi = std::min(l + 1, source - 1);
  *frac = coord - (float)l;
}

// crates/pvlc-cpu-ref/src/lib.rs:156-217 (add_interpolated_position_embedding_f32)
void add_position_embedding(Vec& x, size_t hidden, const Vec& table, size_t side,
                            const uint32_t* grids, size_t n_grids) {
  size_t offset = 0;
  for (size_t g = 0; g < n_grids; ++g) {
    const size_t t = grids[3 * g], h = grids[3 * g + 1], w = grids[3 * g + 2];
    for (size_t tt = 0; tt < t; ++tt)
      for (size_t y = 0; y < h; ++y) {
        size_t y0, y1;
        float yf;
        bilinear_axis(side, h, y, &y0, &y1, &yf);
        for (size_t xx = 0; xx < w; ++xx) {
          size_t x0, x1;
          float xf;
          bilinear_axis(side, w, xx, &x0, &x1, &xf);
          float* dst = x.data() + (offset + tt * h * w + y * w + xx) * hidden;
          const float* tl = table.data() + (y0 * side + x0) * hidden;
          const float* tr = table.data() + (y0 * side + x1) * hidden;
          const float* bl = table.data() + (y1 * side + x0) * hidden;
          const float* br = table.data() + (y1 * side + x1) * hidden;
          for (size_t c = 0; c < hidden; ++c) {
            const float top = tl[c] + (tr[c] - tl[c]) * xf;
            const float bottom = bl[c] + (br[c] - bl[c]) * xf;
            dst[c] += top + (bottom - top) * yf;
          }
        }
      }
    offset += t * h * w;
  }
}

// crates/pvlc-cpu-ref/src/lib.rs:219-263 (projector_merge_2x2_f32)
Vec merge_2x2(const Vec& x, size_t hidden, const uint32_t* grids, size_t n_grids) {
  Vec out;
  out.reserve(x.size());
  size_t offset = 0;
  for (size_t g = 0; g < n_grids; ++g) {
    const size_t t = grids[3 * g], h = grids[3 * g + 1], w = grids[3 * g + 2];
    for (size_t tt = 0; tt < t; ++tt)
      for (size_t my = 0; my < h / 2; ++my)
        for (size_t mx = 0; mx < w / 2; ++mx)
          for (size_t py = 0; py < 2; ++py)
            for (size_t px = 0; px < 2; ++px) {
              const size_t src = offset + tt * h * w + (my * 2 + py) * w + (mx * 2 + px);
              out.insert(out.end(), x.begin() + src * hidden, x.begin() + (src + 1) * hidden);
            }
    offset += t * h * w;
  }
  return out;
}

// Top-1 under compare_top_k_entries (crates/pvlc-cpu-ref/src/lib.rs:2051-2056):
// the larger value in IEEE total order, ties to the smaller index.
inline int32_t total_key(float v) {
  int32_t b;
  std::memcpy(&b, &v, 4);
  return b ^ ((b >> 31) & 0x7fffffff);
}

void top2(const float* logits, size_t n, uint32_t* i1, float* v1, uint32_t* i2, float* v2) {
  size_t b1 = 0, b2 = n > 1 ? 1 : 0;
  if (n > 1 && total_key(logits[1]) > total_key(logits[0])) std::swap(b1, b2);
  for (size_t i = 2; i < n; ++i) {
    const int32_t k = total_key(logits[i]);
    if (k > total_key(logits[b1])) {
      b2 = b1;
      b1 = i;
    } else if (k > total_key(logits[b2])) {
      b2 = i;
    }
  }
  *i1 = (uint32_t)b1;
  *v1 = logits[b1];
  *i2 = (uint32_t)b2;
  *v2 = logits[b2];
}

// --------------------------------------------------------------- decoder layer
struct DecoderWeights {
  const float *input_norm, *q, *k, *v, *o, *post_norm, *gate, *up, *down;
};

struct DecoderGeom {
  size_t hidden, inter, qh, kvh, hd;
  float eps;
  const uint32_t* sections;
};

// Trace slots, in the order of the reference's DecoderLayerPrefillTrace
// (crates/pvlc-cpu-ref/src/lib.rs:1047-1066) minus the cache copies.
enum {
  T_NORM1, T_QUERY, T_KEY, T_VALUE, T_MROPE_Q, T_MROPE_K, T_CONTEXT, T_ATTN_OUT, T_ATTN_RES,
  T_NORM2, T_GATE, T_UP, T_ACT, T_DOWN, T_OUTPUT, T_COUNT
};

void trace_put(float* const* trace, int slot, const Vec& v) {
  if (trace && trace[slot]) std::memcpy(trace[slot], v.data(), v.size() * sizeof(float));
}

// One prefill layer: crates/pvlc-cpu-ref/src/lib.rs:1305-1418
// (decoder_layer_trace_from_validated_operands) with the attention closure of
// decoder_layer_prefill_f32 (:1592-1627): M-RoPE, cache write of the rotated
// key and raw value, causal GQA.  `h` is the residual stream (updated in
// place); cos/sin are axis planes [3][tokens][hd]; the cache receives rows
// [0, tokens) when given.
int decoder_layer_prefill(Vec& h, size_t T, const DecoderGeom& g, const float* cos,
                          const float* sin, const DecoderWeights& w, bool f16,
                          float* const* trace, float* k_cache, float* v_cache) {
  const size_t D = g.hidden, QW = g.qh * g.hd, KW = g.kvh * g.hd;
  Vec n1(T * D);
  rms_norm(h.data(), T, D, w.input_norm, g.eps, n1.data());
  store(n1, f16);
  Vec q = linear_v(n1, T, D, w.q, nullptr, QW, f16);
  Vec k = linear_v(n1, T, D, w.k, nullptr, KW, f16);
  Vec v = linear_v(n1, T, D, w.v, nullptr, KW, f16);
  Vec mq(T * QW), mk(T * KW);
  int st = pvlc_oracle_apply_multimodal_rope(q.data(), k.data(), (uint32_t)T, (uint32_t)g.qh,
                                             (uint32_t)g.kvh, (uint32_t)g.hd, cos, sin,
                                             g.sections, mq.data(), mk.data());
  if (st) return st;
  store(mq, f16);
  store(mk, f16);
  if (k_cache) std::memcpy(k_cache, mk.data(), mk.size() * sizeof(float));
  if (v_cache) std::memcpy(v_cache, v.data(), v.size() * sizeof(float));
  Vec ctx(T * QW);
  st = pvlc_oracle_causal_gqa(mq.data(), mk.data(), v.data(), (uint32_t)T, (uint32_t)g.qh,
                              (uint32_t)g.kvh, (uint32_t)g.hd, ctx.data());
  if (st) return st;
  store(ctx, f16);
  Vec ao = linear_v(ctx, T, QW, w.o, nullptr, D, f16);
  trace_put(trace, T_NORM1, n1);
  trace_put(trace, T_QUERY, q);
  trace_put(trace, T_KEY, k);
  trace_put(trace, T_VALUE, v);
  trace_put(trace, T_MROPE_Q, mq);
  trace_put(trace, T_MROPE_K, mk);
  trace_put(trace, T_CONTEXT, ctx);
  trace_put(trace, T_ATTN_OUT, ao);
  add_into(h, ao);
  trace_put(trace, T_ATTN_RES, h);
  Vec n2(T * D);
  rms_norm(h.data(), T, D, w.post_norm, g.eps, n2.data());
  store(n2, f16);
  Vec gate = linear_v(n2, T, D, w.gate, nullptr, g.inter, f16);
  Vec up = linear_v(n2, T, D, w.up, nullptr, g.inter, f16);
  Vec act(T * g.inter);
  silu_gate(gate, up, act);
  store(act, f16);
  Vec down = linear_v(act, T, g.inter, w.down, nullptr, D, f16);
  add_into(h, down);
  trace_put(trace, T_NORM2, n2);
  trace_put(trace, T_GATE, gate);
  trace_put(trace, T_UP, up);
  trace_put(trace, T_ACT, act);
  trace_put(trace, T_DOWN, down);
  trace_put(trace, T_OUTPUT, h);
  return OK;
}

// One decode layer: crates/pvlc-cpu-ref/src/lib.rs:1648-1680
// (decoder_layer_decode_f32): the same composition for one token whose M-RoPE
// rows are row `row` of the [3][rows][hd] tables, the rotated key and raw
// value appended at cache row `ct` (append_decoder_kv_cache :1420-1450), and
// decode GQA over ct + 1 rows.
int decoder_layer_decode(Vec& h, const DecoderGeom& g, const float* cos_t, const float* sin_t,
                         size_t rows, size_t row, const DecoderWeights& w, bool f16,
                         float* k_cache, float* v_cache, size_t ct) {
  const size_t D = g.hidden, QW = g.qh * g.hd, KW = g.kvh * g.hd;
  Vec n1(D);
  rms_norm(h.data(), 1, D, w.input_norm, g.eps, n1.data());
  store(n1, f16);
  Vec q = linear_v(n1, 1, D, w.q, nullptr, QW, f16);
  Vec k = linear_v(n1, 1, D, w.k, nullptr, KW, f16);
  Vec v = linear_v(n1, 1, D, w.v, nullptr, KW, f16);
  Vec c1(3 * g.hd), s1(3 * g.hd);
  for (size_t a = 0; a < 3; ++a) {
    std::memcpy(&c1[a * g.hd], cos_t + (a * rows + row) * g.hd, g.hd * sizeof(float));
    std::memcpy(&s1[a * g.hd], sin_t + (a * rows + row) * g.hd, g.hd * sizeof(float));
  }
  Vec mq(QW), mk(KW);
  int st = pvlc_oracle_apply_multimodal_rope(q.data(), k.data(), 1, (uint32_t)g.qh,
                                             (uint32_t)g.kvh, (uint32_t)g.hd, c1.data(),
                                             s1.data(), g.sections, mq.data(), mk.data());
  if (st) return st;
  store(mq, f16);
  store(mk, f16);
  std::memcpy(k_cache + ct * KW, mk.data(), KW * sizeof(float));
  std::memcpy(v_cache + ct * KW, v.data(), KW * sizeof(float));
  Vec ctx(QW);
  st = pvlc_oracle_decode_gqa(mq.data(), k_cache, v_cache, (uint32_t)(ct + 1), (uint32_t)g.qh,
                              (uint32_t)g.kvh, (uint32_t)g.hd, ctx.data());
  if (st) return st;
  store(ctx, f16);
  Vec ao = linear_v(ctx, 1, QW, w.o, nullptr, D, f16);
  add_into(h, ao);
  Vec n2(D);
  rms_norm(h.data(), 1, D, w.post_norm, g.eps, n2.data());
  store(n2, f16);
  Vec gate = linear_v(n2, 1, D, w.gate, nullptr, g.inter, f16);
  Vec up = linear_v(n2, 1, D, w.up, nullptr, g.inter, f16);
  Vec act(g.inter);
  silu_gate(gate, up, act);
  store(act, f16);
  Vec down = linear_v(act, 1, g.inter, w.down, nullptr, D, f16);
  add_into(h, down);
  return OK;
}

// ---------------------------------------------------------------- vision
// Vision encoder: patch projection with bias (lib.rs:88-129), interpolated
// position embedding (:156-217), then per layer the composition of
// vision_encoder_layer_identity_rope_f32 (:2880-2987) with the engine's 2-D
// RoPE of q and k (vision_rope_2d tables, web/engine/multimodal_ocr.mjs:98-155)
// before segmented attention, and the post LayerNorm of the stack (:3050-3060).
int vision_encoder(const pvlc_oracle_model_dims& d, const uint16_t* const* vw,
                   const float* patches, size_t n, const uint32_t* grids, size_t n_grids,
                   bool f16, Vec& out) {
  const size_t H = d.vision_hidden, I = d.vision_intermediate, P = d.patch_input;
  const size_t heads = d.vision_heads, hd = d.vision_head_dim;
  Vec x(patches, patches + n * P);
  store(x, f16);
  Vec wpe = widen(vw[0], H * P), bpe = widen(vw[1], H);
  Vec h = linear_v(x, n, P, wpe.data(), bpe.data(), H, f16);
  Vec pos = widen(vw[2], (size_t)d.pos_side * d.pos_side * H);
  add_position_embedding(h, H, pos, d.pos_side, grids, n_grids);
  Vec cos_t(n * hd / 2), sin_t(n * hd / 2);
  int st = pvlc_oracle_vision_rope_tables(grids, (uint32_t)n_grids, (uint32_t)hd, d.vision_theta,
                                          cos_t.data(), sin_t.data());
  if (st) return st;
  std::vector<uint32_t> cu(1, 0);
  for (size_t g = 0; g < n_grids; ++g)
    cu.push_back(cu.back() + grids[3 * g] * grids[3 * g + 1] * grids[3 * g + 2]);
  for (size_t l = 0; l < d.vision_layers; ++l) {
    const uint16_t* const* lw = vw + 3 + 16 * l;
    Vec ln1w = widen(lw[0], H), ln1b = widen(lw[1], H);
    Vec n1(n * H);
    layer_norm(h.data(), n, H, ln1w.data(), ln1b.data(), d.vision_eps, n1.data());
    store(n1, f16);
    Vec q, k, v;
    {
      Vec w = widen(lw[2], H * H), b = widen(lw[3], H);
      q = linear_v(n1, n, H, w.data(), b.data(), H, f16);
    }
    {
      Vec w = widen(lw[4], H * H), b = widen(lw[5], H);
      k = linear_v(n1, n, H, w.data(), b.data(), H, f16);
    }
    {
      Vec w = widen(lw[6], H * H), b = widen(lw[7], H);
      v = linear_v(n1, n, H, w.data(), b.data(), H, f16);
    }
    Vec rq(n * H), rk(n * H);
    st = pvlc_oracle_vision_rope_apply_tables(q.data(), k.data(), (uint32_t)n, (uint32_t)heads,
                                              (uint32_t)hd, cos_t.data(), sin_t.data(),
                                              rq.data(), rk.data());
    if (st) return st;
    store(rq, f16);
    store(rk, f16);
    Vec ctx(n * H);
    st = pvlc_oracle_segmented_attention(rq.data(), rk.data(), v.data(), (uint32_t)n,
                                         (uint32_t)heads, (uint32_t)hd, cu.data(),
                                         (uint32_t)cu.size(), ctx.data());
    if (st) return st;
    store(ctx, f16);
    {
      Vec w = widen(lw[8], H * H), b = widen(lw[9], H);
      Vec ao = linear_v(ctx, n, H, w.data(), b.data(), H, f16);
      add_into(h, ao);
    }
    Vec ln2w = widen(lw[10], H), ln2b = widen(lw[11], H);
    Vec n2(n * H);
    layer_norm(h.data(), n, H, ln2w.data(), ln2b.data(), d.vision_eps, n2.data());
    store(n2, f16);
    Vec f1;
    {
      // the engine applies the GELU in the fc1 GEMM's epilogue, to the f32
      // result: the one fp16 storage point is after it
      Vec w = widen(lw[12], I * H), b = widen(lw[13], I);
      f1 = linear_v(n2, n, H, w.data(), b.data(), I, false);
    }
    apply(f1, gelu_tanh);
    store(f1, f16);
    {
      Vec w = widen(lw[14], H * I), b = widen(lw[15], H);
      Vec f2 = linear_v(f1, n, I, w.data(), b.data(), H, f16);
      add_into(h, f2);
    }
  }
  const uint16_t* const* pw = vw + 3 + 16 * d.vision_layers;
  Vec pw_ = widen(pw[0], H), pb_ = widen(pw[1], H);
  out.assign(n * H, 0.0f);
  layer_norm(h.data(), n, H, pw_.data(), pb_.data(), d.vision_eps, out.data());
  store(out, f16);
  return OK;
}

// crates/pvlc-cpu-ref/src/lib.rs:2598-2678 (projector_f32)
int projector(const pvlc_oracle_model_dims& d, const uint16_t* const* pw, const Vec& feats,
              size_t n, const uint32_t* grids, size_t n_grids, bool f16, Vec& out) {
  const size_t H = d.vision_hidden, M = H * d.merge * d.merge, D = d.decoder_hidden;
  Vec lw = widen(pw[0], H), lb = widen(pw[1], H);
  Vec pre(n * H);
  layer_norm(feats.data(), n, H, lw.data(), lb.data(), d.projector_eps, pre.data());
  store(pre, f16);
  Vec merged = merge_2x2(pre, H, grids, n_grids);
  const size_t m = merged.size() / M;
  Vec l1;
  {
    Vec w = widen(pw[2], M * M), b = widen(pw[3], M);
    l1 = linear_v(merged, m, M, w.data(), b.data(), M, f16);
  }
  apply(l1, gelu_erf);
  store(l1, f16);
  Vec w2 = widen(pw[4], D * M), b2 = widen(pw[5], D);
  out = linear_v(l1, m, M, w2.data(), b2.data(), D, f16);
  return OK;
}

}  // namespace

extern "C" {

// f32 primitives exposed for the known-answer tests.
int pvlc_oracle_linear(const float* in, uint32_t rows, uint32_t in_width, const float* weight,
                       const float* bias, uint32_t out_width, float* out) {
  if (rows == 0 || in_width == 0 || out_width == 0) return DIMENSION_MISMATCH;
  linear(in, rows, in_width, weight, bias, out_width, out);
  return OK;
}

int pvlc_oracle_rms_norm(const float* in, uint32_t rows, uint32_t width, const float* weight,
                         float eps, float* out) {
  if (rows == 0 || width == 0) return DIMENSION_MISMATCH;
  rms_norm(in, rows, width, weight, eps, out);
  return OK;
}

int pvlc_oracle_layer_norm(const float* in, uint32_t rows, uint32_t width, const float* weight,
                           const float* bias, float eps, float* out) {
  if (rows == 0 || width == 0) return DIMENSION_MISMATCH;
  layer_norm(in, rows, width, weight, bias, eps, out);
  return OK;
}

// crates/pvlc-cpu-ref/src/lib.rs:1469-1490 (prefill_last_logits_f32): the last
// row of a token-major final-norm output through the output-major LM head.
int pvlc_oracle_prefill_last_logits(const float* final_norm, uint32_t tokens, uint32_t hidden,
                                    const float* lm_head, uint32_t vocab, float* logits) {
  if (tokens == 0 || hidden == 0 || vocab == 0) return DIMENSION_MISMATCH;
  linear(final_norm + (size_t)(tokens - 1) * hidden, 1, hidden, lm_head, nullptr, vocab, logits);
  return OK;
}

// One decoder prefill layer with f32 weights (crates/pvlc-cpu-ref/src/lib.rs:1592-1627),
// general geometry.  weights: input_norm, q, k, v, o, post_norm, gate, up, down.
// raw cos/sin: [3][tokens][head_dim].  trace: 15 output pointers (norm1, query,
// key, value, mrope_query, mrope_key, attention_context, attention_output,
// attention_residual, norm2, mlp_gate, mlp_up, mlp_activation, mlp_down, output).
int pvlc_oracle_decoder_layer_prefill(const float* input, uint32_t tokens, uint32_t hidden,
                                      uint32_t intermediate, uint32_t query_heads,
                                      uint32_t kv_heads, uint32_t head_dim, float eps,
                                      const uint32_t* sections, const float* raw_cos,
                                      const float* raw_sin, const float* const* weights,
                                      float* const* trace) {
  if (tokens == 0 || hidden == 0 || intermediate == 0 || query_heads == 0 || kv_heads == 0 ||
      head_dim == 0)
    return DIMENSION_MISMATCH;
  DecoderGeom g{hidden, intermediate, query_heads, kv_heads, head_dim, eps, sections};
  DecoderWeights w{weights[0], weights[1], weights[2], weights[3], weights[4],
                   weights[5], weights[6], weights[7], weights[8]};
  Vec h(input, input + (size_t)tokens * hidden);
  return decoder_layer_prefill(h, tokens, g, raw_cos, raw_sin, w, false, trace, nullptr,
                               nullptr);
}

// One PaddleOCR-VL request end to end: vision encoder -> projector ->
// multimodal embedding assembly (crates/pvlc-cpu-ref/src/multimodal.rs:115-163)
// -> decoder prefill over the prompt (M-RoPE ids multimodal.rs:28-78, tables
// multimodal_ocr.mjs:937-986) -> final RMSNorm and LM head of the last row
// (lib.rs:1469-1490) -> greedy top-1 generation (lib.rs:2201-2305, EOS kept,
// stop at max_new_tokens) with one decode layer stack per step.
//
// Weights are fp16 (bit patterns), output-major, in the order:
//  vision:    patch_embed.w [H,P], patch_embed.b [H], pos_embed [side^2,H], then per
//             layer ln1.w, ln1.b, q.w, q.b, k.w, k.b, v.w, v.b, o.w, o.b, ln2.w, ln2.b,
//             fc1.w [I,H], fc1.b, fc2.w [H,I], fc2.b; then post_ln.w, post_ln.b
//  projector: pre_ln.w, pre_ln.b, linear1.w [4H,4H], linear1.b, linear2.w [D,4H], linear2.b
//  decoder:   embed [V,D], per layer input_norm, q.w, k.w, v.w, o.w, post_norm, gate.w,
//             up.w, down.w; then final_norm, lm_head [V,D]
// grids are pre-merge (t, h, w) patch grids, one per image of the prompt.
// Outputs: tokens_out [max_new_tokens] and *n_out; optional logits_out
// [max_new_tokens][vocab] (the logits each token was chosen from), vision_out
// [patches][H] and projector_out [image tokens][D].
int pvlc_oracle_generate(const pvlc_oracle_model_dims* dims, const uint16_t* const* vision_w,
                         const uint16_t* const* projector_w, const uint16_t* const* decoder_w,
                         const float* patches, const uint32_t* grids, uint32_t n_grids,
                         const uint32_t* input_ids, uint32_t n_ids, uint32_t max_new_tokens,
                         int fp16_storage, uint32_t* tokens_out, uint32_t* n_out,
                         float* logits_out, float* vision_out, float* projector_out) {
  const pvlc_oracle_model_dims& d = *dims;
  const bool f16 = fp16_storage != 0;
  if (n_grids == 0 || n_ids == 0 || max_new_tokens == 0 || d.eos_token_id >= d.vocab)
    return DIMENSION_MISMATCH;
  size_t n_patches = 0;
  for (size_t g = 0; g < n_grids; ++g) n_patches += (size_t)grids[3 * g] * grids[3 * g + 1] *
                                                    grids[3 * g + 2];
  Vec feats;
  int st = vision_encoder(d, vision_w, patches, n_patches, grids, n_grids, f16, feats);
  if (st) return st;
  if (vision_out) std::memcpy(vision_out, feats.data(), feats.size() * sizeof(float));
  Vec proj;
  st = projector(d, projector_w, feats, n_patches, grids, n_grids, f16, proj);
  if (st) return st;
  if (projector_out) std::memcpy(projector_out, proj.data(), proj.size() * sizeof(float));

  const size_t D = d.decoder_hidden, T = n_ids, L = d.decoder_layers;
  const size_t KW = (size_t)d.kv_heads * d.head_dim;
  // multimodal.rs:115-163 (assemble_multimodal_embeddings_f32)
  Vec h(T * D);
  size_t image_row = 0;
  for (size_t t = 0; t < T; ++t) {
    if (input_ids[t] == d.image_token_id) {
      if ((image_row + 1) * D > proj.size()) return DIMENSION_MISMATCH;
      std::memcpy(&h[t * D], &proj[image_row * D], D * sizeof(float));
      ++image_row;
    } else {
      if (input_ids[t] >= d.vocab) return DIMENSION_MISMATCH;
      const uint16_t* row = decoder_w[0] + (size_t)input_ids[t] * D;
      for (size_t c = 0; c < D; ++c) h[t * D + c] = widen_half(row[c]);
    }
  }
  if (image_row * D != proj.size()) return DIMENSION_MISMATCH;

  std::vector<int64_t> positions(3 * T);
  int64_t delta = 0;
  st = pvlc_oracle_mrope_position_ids(input_ids, (uint32_t)T, grids, n_grids, d.image_token_id,
                                      d.vision_start_token_id, d.merge, positions.data(), &delta);
  if (st) return st;
  const size_t cap = T + max_new_tokens;
  Vec cos_t(3 * cap * d.head_dim), sin_t(3 * cap * d.head_dim);
  st = pvlc_oracle_rope_tables(positions.data(), (uint32_t)T, delta, (uint32_t)cap,
                               d.decoder_theta, d.head_dim, cos_t.data(), sin_t.data());
  if (st) return st;
  Vec pc(3 * T * d.head_dim), ps(3 * T * d.head_dim);
  for (size_t a = 0; a < 3; ++a) {
    std::memcpy(&pc[a * T * d.head_dim], &cos_t[a * cap * d.head_dim],
                T * d.head_dim * sizeof(float));
    std::memcpy(&ps[a * T * d.head_dim], &sin_t[a * cap * d.head_dim],
                T * d.head_dim * sizeof(float));
  }

  DecoderGeom g{D, d.decoder_intermediate, d.query_heads, d.kv_heads, d.head_dim,
                d.decoder_eps, d.sections};
  const size_t QW = (size_t)d.query_heads * d.head_dim, I = d.decoder_intermediate;
  std::vector<Vec> lws(L * 9);
  std::vector<DecoderWeights> layers(L);
  for (size_t l = 0; l < L; ++l) {
    const uint16_t* const* lw = decoder_w + 1 + 9 * l;
    const size_t sizes[9] = {D, QW * D, KW * D, KW * D, D * QW, D, I * D, I * D, D * I};
    for (int j = 0; j < 9; ++j) lws[9 * l + j] = widen(lw[j], sizes[j]);
    layers[l] = DecoderWeights{lws[9 * l].data(),     lws[9 * l + 1].data(), lws[9 * l + 2].data(),
                               lws[9 * l + 3].data(), lws[9 * l + 4].data(), lws[9 * l + 5].data(),
                               lws[9 * l + 6].data(), lws[9 * l + 7].data(), lws[9 * l + 8].data()};
  }
  Vec final_norm = widen(decoder_w[1 + 9 * L], D);
  Vec lm_head = widen(decoder_w[2 + 9 * L], (size_t)d.vocab * D);
  std::vector<Vec> kc(L, Vec(cap * KW)), vc(L, Vec(cap * KW));

  for (size_t l = 0; l < L; ++l) {
    st = decoder_layer_prefill(h, T, g, pc.data(), ps.data(), layers[l], f16, nullptr,
                               kc[l].data(), vc[l].data());
    if (st) return st;
  }
  Vec logits(d.vocab), fn(D);
  auto head = [&](const float* last) {
    rms_norm(last, 1, D, final_norm.data(), d.decoder_eps, fn.data());
    store(fn, f16);
    linear(fn.data(), 1, D, lm_head.data(), nullptr, d.vocab, logits.data());
  };
  head(&h[(T - 1) * D]);
  size_t produced = 0, ct = T;
  for (;;) {
    uint32_t i1, i2;
    float v1, v2;
    top2(logits.data(), d.vocab, &i1, &v1, &i2, &v2);
    if (logits_out)
      std::memcpy(logits_out + produced * d.vocab, logits.data(), d.vocab * sizeof(float));
    tokens_out[produced++] = i1;
    if (i1 == d.eos_token_id || produced == max_new_tokens) break;
    Vec x(D);
    const uint16_t* row = decoder_w[0] + (size_t)i1 * D;
    for (size_t c = 0; c < D; ++c) x[c] = widen_half(row[c]);
    for (size_t l = 0; l < L; ++l) {
      st = decoder_layer_decode(x, g, cos_t.data(), sin_t.data(), cap, ct, layers[l], f16,
                                kc[l].data(), vc[l].data(), ct);
      if (st) return st;
    }
    ++ct;
    head(x.data());
  }
  *n_out = (uint32_t)produced;
  return OK;
}

}  // extern "C"
