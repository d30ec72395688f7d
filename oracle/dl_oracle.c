/*
 * dl_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the arithmetic laws of Dolittle's Qwen3 token loop, used
 * by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg as
 * the checker.  Nothing in the product (dolittle_b200/) links, loads or calls
 * this file; the product path fails loudly when its CUDA library is missing.
 *
 * Each function follows one reference kernel's reduction order exactly (the
 * reference compiles with --fmad=false and fixes every FP32 order), so that
 * integer/FP results without elementary functions are bit-identical to the
 * reference.  Elementary functions (expf, sinf, cosf, rsqrtf, pow) come from
 * the host libm; CUDA's versions may differ in the last unit, so comparisons
 * that pass through them are tolerance-gated on the CPU and bit-exact only
 * against the reference's own kernels run on the GPU (oracle/_ref).
 *
 * Citations are paths inside plainsight-systems/dolittle.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* BF16 storage: src/tensors/representations/bf16.cpp:43-60 (RNE narrowing
 * bits + 0x7fff + lsb, NaN -> 0x7fc0), src/kernels/cuda/common.cuh:67-89.   */
/* ------------------------------------------------------------------------ */
static inline float bf(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t to_bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u = u + 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float rnd(float f) { return bf(to_bf(f)); }

OR_API uint16_t or_bf16_from_float(float f) { return to_bf(f); }
OR_API float or_bf16_to_float(uint16_t b) { return bf(b); }
OR_API void or_bf16_from_float_array(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = to_bf(in[i]);
}
OR_API void or_bf16_to_float_array(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = bf(in[i]);
}

/* ------------------------------------------------------------------------ */
/* Projection: src/kernels/cuda/projection.cu:367-426 (dispatch) with the
 * decode/shared/tiled/pairs kernels :139-361.  Law: P = 16 when
 * I <= 4096 && O > 1024, else 32.  Partial j is the serial FMA chain over
 * features j, j+P, j+2P, ... (ascending); features in [I, ceil16(I)) add one
 * fma(0,0,partial) to partial f%P (the tiled path's zero padding,
 * :296-306); then a halving tree (offset P/2 .. 1) and one BF16 rounding.  */
/* ------------------------------------------------------------------------ */
static inline int projection_partials(size_t I, size_t O) {
  return (I <= 4096 && O > 1024) ? 16 : 32;
}

#define DEFINE_DOT(P)                                                         \
  static float dot_p##P(const float* x, const uint16_t* w, size_t I) {       \
    float acc[P];                                                             \
    for (int j = 0; j < P; ++j) acc[j] = 0.0f;                                \
    size_t full = I / P * P;                                                  \
    for (size_t base = 0; base < full; base += P) {                           \
      for (int j = 0; j < P; ++j)                                             \
        acc[j] = fmaf(x[base + j], bf(w[base + j]), acc[j]);                 \
    }                                                                         \
    for (size_t f = full; f < I; ++f)                                         \
      acc[f - full] = fmaf(x[f], bf(w[f]), acc[f - full]);                    \
    size_t padded = (I + 15) / 16 * 16;                                       \
    for (size_t f = I; f < padded; ++f)                                       \
      acc[f % P] = fmaf(0.0f, 0.0f, acc[f % P]);                              \
    for (int off = P / 2; off != 0; off /= 2)                                 \
      for (int j = 0; j < off; ++j) acc[j] = acc[j] + acc[j + off];           \
    return acc[0];                                                            \
  }
DEFINE_DOT(16)
DEFINE_DOT(32)

static float projection_dot(const float* x, const uint16_t* w, size_t I,
                            int P) {
  return P == 16 ? dot_p16(x, w, I) : dot_p32(x, w, I);
}

/* y[r][o] = round(sum_k x[r][k] * W[o][k]) under the reference partition. */
OR_API void or_projection(const uint16_t* x, const uint16_t* w, uint16_t* y,
                          size_t rows, size_t I, size_t O) {
  const int P = projection_partials(I, O);
  float* xf = (float*)malloc(sizeof(float) * rows * I);
  for (size_t i = 0; i < rows * I; ++i) xf[i] = bf(x[i]);
#pragma omp parallel for schedule(static)
  for (long long o = 0; o < (long long)O; ++o) {
    for (size_t r = 0; r < rows; ++r)
      y[r * O + (size_t)o] = to_bf(projection_dot(xf + r * I, w + (size_t)o * I, I, P));
  }
  free(xf);
}

/* Same law, FP32 output before the storage rounding (diagnostics). */
OR_API void or_projection_f32(const uint16_t* x, const uint16_t* w, float* y,
                              size_t rows, size_t I, size_t O) {
  const int P = projection_partials(I, O);
  float* xf = (float*)malloc(sizeof(float) * rows * I);
  for (size_t i = 0; i < rows * I; ++i) xf[i] = bf(x[i]);
#pragma omp parallel for schedule(static)
  for (long long o = 0; o < (long long)O; ++o) {
    for (size_t r = 0; r < rows; ++r)
      y[r * O + (size_t)o] = projection_dot(xf + r * I, w + (size_t)o * I, I, P);
  }
  free(xf);
}

/* ------------------------------------------------------------------------ */
/* RMSNorm: src/kernels/cuda/normalization.cu.  width <= 128 uses the warp
 * kernel (:82-132): lane l owns columns l+32c (c<4), squares with fmul, sums
 * its four components in order, then a shuffle-down tree with offsets
 * 1,2,4,...,16.  128 < width <= 8192 uses the staged kernel (:134-186):
 * thread t<128 serially adds fmul(v,v) over columns t+128k, groups of four
 * adjacent threads add in order, then the same 32-lane shuffle tree.  Both:
 * mean = total * (1/width), inv = rsqrtf(mean + eps),
 * y = round(round(x * inv) * w).                                           */
/* ------------------------------------------------------------------------ */
static float shuffle_down_tree32(float* s) {
  /* Lane 0's value after value += shfl_down(value, off), off = 1..16. */
  for (int off = 1; off < 32; off *= 2)
    for (int l = 0; l + off < 32; ++l) s[l] = s[l] + s[l + off];
  return s[0];
}

static float rms_inverse(const float* x, size_t width, float eps) {
  float lanes[32];
  if (width <= 128) {
    for (int l = 0; l < 32; ++l) {
      float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int c = 0; c < 4; ++c) {
        size_t col = (size_t)l + 32u * (size_t)c;
        if (col < width) part[c] = x[col] * x[col];
      }
      lanes[l] = ((part[0] + part[1]) + part[2]) + part[3];
    }
  } else {
    float part[128];
    for (int t = 0; t < 128; ++t) {
      float p = 0.0f;
      for (size_t col = (size_t)t; col < width; col += 128) {
        float sq = x[col] * x[col];
        p = p + sq;
      }
      part[t] = p;
    }
    for (int l = 0; l < 32; ++l)
      lanes[l] = ((part[4 * l] + part[4 * l + 1]) + part[4 * l + 2]) +
                 part[4 * l + 3];
  }
  float total = shuffle_down_tree32(lanes);
  float mean = total * (1.0f / (float)width);
  return 1.0f / sqrtf(mean + eps);
}

OR_API void or_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* y,
                        size_t rows, size_t width, float eps) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    float* xf = (float*)malloc(sizeof(float) * width);
    for (size_t i = 0; i < width; ++i) xf[i] = bf(x[(size_t)r * width + i]);
    float inv = rms_inverse(xf, width, eps);
    for (size_t i = 0; i < width; ++i)
      y[(size_t)r * width + i] = to_bf(rnd(xf[i] * inv) * bf(w[i]));
    free(xf);
  }
}

/* ------------------------------------------------------------------------ */
/* RoPE: src/kernels/cuda/rotary.cu:84-126.  Split-half pairs; row index
 * r = position_row*heads + head.  exponent = float(2i)/float(width),
 * inv = float(1/pow(theta, double(exponent))), angle = float(pos)*inv,
 * cos/sin rounded to storage, four rounded products, then -/+ rounded.     */
/* ------------------------------------------------------------------------ */
OR_API float or_rope_inverse_frequency(size_t feature, size_t width,
                                       double theta) {
  float exponent = (float)(2 * feature) / (float)width;
  return (float)(1.0 / pow(theta, (double)exponent));
}

OR_API void or_rotary(const uint16_t* x, uint16_t* y, size_t positions,
                      size_t heads, size_t width, size_t first_position,
                      double theta) {
  const size_t half = width / 2;
  for (size_t f = 0; f < half; ++f) {
    float inv = or_rope_inverse_frequency(f, width, theta);
    for (size_t p = 0; p < positions; ++p) {
      float angle = (float)(first_position + p) * inv;
      float c = rnd(cosf(angle)), s = rnd(sinf(angle));
      for (size_t h = 0; h < heads; ++h) {
        size_t row = p * heads + h;
        float a = bf(x[row * width + f]), b = bf(x[row * width + f + half]);
        float ac = rnd(a * c), bs = rnd(b * s), bc = rnd(b * c),
              as = rnd(a * s);
        y[row * width + f] = to_bf(ac - bs);
        y[row * width + f + half] = to_bf(bc + as);
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Causal GQA attention: src/kernels/cuda/attention.cu:231-383
 * (attention_retained; the 3-pass kernel :142-229 differs only in where the
 * division happens, see or_attention_three_pass).  Query row r sits at
 * absolute position first+r and reads keys [0, first+r].  K/V rows are
 * [position][kv_heads][width].                                              */
/* ------------------------------------------------------------------------ */
OR_API float or_attention_scale(size_t width) {
  return (float)(1.0 / sqrt((double)width));
}

static float attention_dot(const float* q, const uint16_t* k, size_t width) {
  /* 8 lanes own contiguous spans; shuffle-down tree 4,2,1 (:300-352).     */
  const size_t span = width / 8 + (width % 8 != 0);
  float p[8];
  for (int l = 0; l < 8; ++l) {
    size_t begin = (size_t)l * span;
    size_t end = begin + span < width ? begin + span : width;
    float acc = 0.0f;
    for (size_t f = begin; f < end; ++f) acc = fmaf(q[f], bf(k[f]), acc);
    p[l] = acc;
  }
  for (int off = 4; off != 0; off /= 2)
    for (int l = 0; l + off < 8; ++l) p[l] = p[l] + p[l + off];
  return p[0];
}

static float halving_sum256(float* s) {
  /* common.cuh:93-104 block_sum over 256 lanes. */
  for (int stride = 128; stride != 0; stride /= 2)
    for (int t = 0; t < stride; ++t) s[t] = s[t] + s[t + stride];
  return s[0];
}

static void attention_task(const float* q, const uint16_t* key,
                           const uint16_t* value, uint16_t* out, size_t count,
                           size_t kv_heads, size_t kv_head, size_t width,
                           float scale, float* scores) {
  for (size_t j = 0; j < count; ++j)
    scores[j] =
        attention_dot(q, key + (j * kv_heads + kv_head) * width, width) * scale;
  float maximum = scores[0];
  for (size_t j = 0; j < count; ++j) maximum = fmaxf(maximum, scores[j]);
  float lanes[256];
  for (int t = 0; t < 256; ++t) lanes[t] = 0.0f;
  for (int t = 0; t < 32; ++t) {
    float acc = 0.0f;
    for (size_t j = (size_t)t; j < count; j += 32) {
      float e = expf(scores[j] - maximum);
      scores[j] = e;
      acc = acc + e;
    }
    lanes[t] = acc;
  }
  float denominator = halving_sum256(lanes);
  for (size_t j = 0; j < count; ++j) scores[j] = scores[j] / denominator;
  const size_t split = (count - 1) / 2 + 1;
  for (size_t f = 0; f < width; ++f) {
    float first = 0.0f, second = 0.0f;
    for (size_t j = 0; j < split; ++j)
      first = fmaf(scores[j], bf(value[(j * kv_heads + kv_head) * width + f]),
                   first);
    for (size_t j = split; j < count; ++j)
      second = fmaf(scores[j], bf(value[(j * kv_heads + kv_head) * width + f]),
                    second);
    out[f] = to_bf(first + second);
  }
}

OR_API void or_attention(const uint16_t* q, const uint16_t* k,
                         const uint16_t* v, uint16_t* y, size_t rows,
                         size_t query_heads, size_t kv_heads, size_t width,
                         size_t first_position) {
  const float scale = or_attention_scale(width);
  const size_t group = query_heads / kv_heads;
#pragma omp parallel for schedule(dynamic)
  for (long long task = 0; task < (long long)(rows * query_heads); ++task) {
    size_t r = (size_t)task / query_heads, h = (size_t)task % query_heads;
    size_t count = first_position + r + 1;
    float* qf = (float*)malloc(sizeof(float) * width);
    float* scores = (float*)malloc(sizeof(float) * count);
    for (size_t f = 0; f < width; ++f) qf[f] = bf(q[(size_t)task * width + f]);
    attention_task(qf, k, v, y + (size_t)task * width, count, kv_heads,
                   h / group, width, scale, scores);
    free(scores);
    free(qf);
  }
}

/* ------------------------------------------------------------------------ */
/* Elementwise: src/kernels/cuda/elementwise.cu:62-87; embedding.cu:60-80.   */
/* ------------------------------------------------------------------------ */
static inline float silu_law(float a, float b) {
  float e = expf(a >= 0.0f ? -a : a);
  float sigmoid = a >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return rnd(rnd(a * sigmoid) * b);
}
OR_API void or_add(const uint16_t* a, const uint16_t* b, uint16_t* y,
                   size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = to_bf(bf(a[i]) + bf(b[i]));
}
OR_API void or_silu_multiply(const uint16_t* g, const uint16_t* u, uint16_t* y,
                             size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = to_bf(silu_law(bf(g[i]), bf(u[i])));
}
OR_API void or_embedding(const uint32_t* tokens, const uint16_t* table,
                         uint16_t* y, size_t rows, size_t width) {
  for (size_t r = 0; r < rows; ++r)
    memcpy(y + r * width, table + (size_t)tokens[r] * width, width * 2);
}

/* ------------------------------------------------------------------------ */
/* Steering one-row edit: src/kernels/cuda/steering.cu:106-159.  8 strided
 * lane sums of fmul(v,v), serial lane total, beta = strength*sqrt(sum),
 * h' = round(h + beta*u); state = {invalid, count}.                         */
/* ------------------------------------------------------------------------ */
OR_API void or_intervene(uint16_t* residual, const float* direction,
                         size_t width, size_t selected, size_t first,
                         size_t rows, float strength, uint32_t* state) {
  if (selected < first || selected - first >= rows) return;
  uint32_t invalid = (state[0] || state[1] != 0) ? 1u : 0u;
  state[1] += 1;
  uint16_t* row = residual + (selected - first) * width;
  float sums[8];
  for (int l = 0; l < 8; ++l) {
    float s = 0.0f;
    for (size_t i = (size_t)l; i < width; i += 8) {
      float v = bf(row[i]);
      s = s + v * v;
    }
    sums[l] = s;
  }
  float sum = 0.0f;
  for (int l = 0; l < 8; ++l) sum = sum + sums[l];
  float beta = strength * sqrtf(sum);
  if (!isfinite(beta)) invalid = 1;
  if (!invalid) {
    for (size_t i = 0; i < width; ++i) {
      float value = bf(row[i]) + beta * direction[i];
      uint16_t stored = to_bf(value);
      if (!isfinite(value) || !isfinite(bf(stored))) invalid = 1;
      row[i] = stored;
    }
  }
  state[0] = invalid;
}

/* Steering direction from two reconstructions: src/kernels/cuda/
 * steering.cu:68-98 (DeviceDirection::submit/finish :200-258).  delta =
 * FP32(edited) - FP32(original); lane L of 8 sums delta*delta (rounded) over
 * i = L + 8k in order; lanes added 0..7 in order; norm = sqrt (correctly
 * rounded); returns 1 and leaves out untouched on a zero or non-finite
 * norm, else out[i] = delta_i / norm.  Inputs are BF16 bits (bf16 != 0) or
 * FP32 values.                                                              */
OR_API uint32_t or_direction(int bf16, const void* original, const void* edited,
                             size_t width, float* out) {
  const uint16_t* ob = (const uint16_t*)original;
  const uint16_t* eb = (const uint16_t*)edited;
  const float* of = (const float*)original;
  const float* ef = (const float*)edited;
#define OR_DELTA(i) (bf16 ? bf(eb[i]) - bf(ob[i]) : ef[i] - of[i])
  float sums[8];
  for (int l = 0; l < 8; ++l) {
    float s = 0.0f;
    for (size_t i = (size_t)l; i < width; i += 8) {
      float delta = OR_DELTA(i);
      s = s + delta * delta;
    }
    sums[l] = s;
  }
  float sum = 0.0f;
  for (int l = 0; l < 8; ++l) sum = sum + sums[l];
  float norm = sqrtf(sum);
  if (!isfinite(norm) || norm == 0.0f) return 1u;
  for (size_t i = 0; i < width; ++i) out[i] = OR_DELTA(i) / norm;
#undef OR_DELTA
  return 0u;
}

/* Fixed-strength steering (no reference counterpart; the reference edits one
 * row once, or_intervene): beta = alpha * sqrt(8-lane sum of v*v) of a source
 * row, the one-row edit's norm law; then every row at a position >= first gets
 * h' = round(h + beta * u).  Returns 1 if a value or beta is not finite.     */
OR_API float or_steer_beta(const uint16_t* row, size_t width, float alpha) {
  float sums[8];
  for (int l = 0; l < 8; ++l) {
    float s = 0.0f;
    for (size_t i = (size_t)l; i < width; i += 8) {
      float v = bf(row[i]);
      s = s + v * v;
    }
    sums[l] = s;
  }
  float sum = 0.0f;
  for (int l = 0; l < 8; ++l) sum = sum + sums[l];
  return alpha * sqrtf(sum);
}

OR_API uint32_t or_steer_rows(uint16_t* residual, const float* direction, size_t width, size_t rows,
                              size_t first_position, size_t steer_from, float beta) {
  uint32_t bad = isfinite(beta) ? 0u : 1u;
  for (size_t r = 0; r < rows && !bad; ++r) {
    if (first_position + r < steer_from) continue;
    uint16_t* row = residual + r * width;
    for (size_t i = 0; i < width; ++i) {
      float value = bf(row[i]) + beta * direction[i];
      uint16_t stored = to_bf(value);
      if (!isfinite(value) || !isfinite(bf(stored))) bad = 1;
      row[i] = stored;
    }
  }
  return bad;
}

/* Injection normalisation: src/kernels/cuda/injection.cu:48-102.           */
OR_API uint32_t or_normalize_injection(const uint16_t* source, uint16_t* out,
                                       size_t width, float scale,
                                       float* norm_out) {
  uint32_t invalid = 0;
  float sums[8];
  for (int l = 0; l < 8; ++l) {
    float s = 0.0f;
    for (size_t i = (size_t)l; i < width; i += 8) {
      float v = bf(source[i]);
      if (!isfinite(v)) invalid = 1;
      s = s + v * v;
    }
    sums[l] = s;
  }
  float sum = 0.0f;
  for (int l = 0; l < 8; ++l) sum = sum + sums[l];
  float norm = sqrtf(sum);
  *norm_out = norm;
  if (!isfinite(norm) || norm == 0.0f) invalid = 1;
  if (!invalid) {
    for (size_t i = 0; i < width; ++i) {
      float value = (bf(source[i]) / norm) * scale;
      uint16_t stored = to_bf(value);
      if (!isfinite(value) || !isfinite(bf(stored))) invalid = 1;
      out[i] = stored;
    }
  }
  return invalid;
}

/* ------------------------------------------------------------------------ */
/* MT19937-64 (the std::mt19937_64 sequence the reference uses):
 * src/kernels/cuda/sampling.cu:106-137, src/inference/sampling/sampler.h.  */
/* ------------------------------------------------------------------------ */
typedef struct {
  uint64_t words[312];
  uint32_t index;
} or_mt64;

OR_API void or_mt64_seed(or_mt64* s, uint64_t seed) {
  s->words[0] = seed;
  for (unsigned i = 1; i < 312; ++i) {
    uint64_t p = s->words[i - 1];
    s->words[i] = 6364136223846793005ULL * (p ^ (p >> 62)) + i;
  }
  s->index = 312;
}
OR_API uint64_t or_mt64_next(or_mt64* s) {
  if (s->index == 312) {
    for (unsigned i = 0; i < 312; ++i) {
      uint64_t x = (s->words[i] & 0xffffffff80000000ULL) |
                   (s->words[(i + 1) % 312] & 0x7fffffffULL);
      s->words[i] = s->words[(i + 156) % 312] ^ (x >> 1) ^
                    ((x & 1) ? 0xb5026f5aa96619e9ULL : 0);
    }
    s->index = 0;
  }
  uint64_t x = s->words[s->index++];
  x ^= (x >> 29) & 0x5555555555555555ULL;
  x ^= (x << 17) & 0x71d67fffeda60000ULL;
  x ^= (x << 37) & 0xfff7eee000000000ULL;
  x ^= x >> 43;
  return x;
}
OR_API size_t or_mt64_state_bytes(void) { return sizeof(or_mt64); }

/* ------------------------------------------------------------------------ */
/* Selection laws.  Key: src/inference/sampling/categorical.cpp:73-77
 * (descending key, -0 == +0); order = (value desc, id asc).                 */
/* ------------------------------------------------------------------------ */
static inline uint32_t descending_key(float value) {
  float v = value == 0.0f ? 0.0f : value;
  uint32_t bits;
  memcpy(&bits, &v, 4);
  uint32_t mask = (0u - (bits >> 31)) | 0x80000000u;
  return ~(bits ^ mask);
}

typedef struct {
  uint32_t key, id;
} cand;

static int cand_cmp(const void* a, const void* b) {
  const cand* x = (const cand*)a;
  const cand* y = (const cand*)b;
  if (x->key != y->key) return x->key < y->key ? -1 : 1;
  return x->id < y->id ? -1 : (x->id > y->id ? 1 : 0);
}

/* Host law: src/inference/sampling/categorical.cpp:146-201.
 * Returns 0 and writes *token, or 1 when the reference throws
 * invalid_argument (NaN/+inf logit, everything masked, bad settings).
 * A categorical draw consumes the given 64-bit word.                        */
OR_API int or_select_host(const float* logits, size_t n, int categorical,
                          double temperature, size_t top_k, double top_p,
                          uint64_t word, uint32_t* token) {
  if (!(isfinite(temperature) && temperature > 0 && isfinite(top_p) &&
        top_p > 0 && top_p <= 1))
    return 1;
  if (!categorical && (temperature != 1 || top_k != 0 || top_p != 1)) return 1;
  if (top_k > n) return 1;
  cand* c = (cand*)malloc(sizeof(cand) * (n ? n : 1));
  size_t m = 0;
  for (size_t i = 0; i < n; ++i) {
    float v = logits[i];
    if (isnan(v) || v == INFINITY) {
      free(c);
      return 1;
    }
    if (isfinite(v)) c[m++] = (cand){descending_key(v), (uint32_t)i};
  }
  if (!m) {
    free(c);
    return 1;
  }
  if (!categorical) {
    size_t best = 0;
    for (size_t i = 1; i < m; ++i) {
      float a = logits[c[i].id], b = logits[c[best].id];
      if (a > b || (a == b && c[i].id < c[best].id)) best = i;
    }
    *token = c[best].id;
    free(c);
    return 0;
  }
  qsort(c, m, sizeof(cand), cand_cmp);
  if (top_k && m > top_k) m = top_k;
  double* w = (double*)malloc(sizeof(double) * m);
  const double maximum = (double)logits[c[0].id];
  double total = 0;
  for (size_t i = 0; i < m; ++i) {
    w[i] = exp(((double)logits[c[i].id] - maximum) / temperature);
    total += w[i];
  }
  double retained = 0;
  size_t count = 0;
  for (;;) {
    retained += w[count++];
    if (!(count < m && retained / total < top_p)) break;
  }
  const double u = (double)(word >> 11) * 0x1.0p-53;
  double cumulative = 0;
  uint32_t chosen = c[count - 1].id;
  for (size_t i = 0; i < count; ++i) {
    cumulative += w[i] / retained;
    if (u < cumulative) {
      chosen = c[i].id;
      break;
    }
  }
  *token = chosen;
  free(w);
  free(c);
  return 0;
}

/* Device law: src/kernels/cuda/sampling.cu:152-376 (greedy_blocks/finish,
 * initialize + stable radix order, weights with 256-entry serial tiles,
 * serial tile-total scan, cutoff/select_prefix minima).  Returns the
 * {token, status} pair the device writes; status 1 = NaN/+inf seen,
 * status 2 = no positive mass / no finite best.                             */
OR_API void or_select_device(const float* logits, size_t n, int categorical,
                             double temperature, size_t top_k, double top_p,
                             uint64_t word, uint32_t* token_out,
                             uint32_t* status_out) {
  uint32_t status = 0, token = 0;
  for (size_t i = 0; i < n; ++i)
    if (isnan(logits[i]) || logits[i] == INFINITY) status = 1;
  if (!categorical) {
    float best = -INFINITY;
    uint32_t id = 0xffffffffu;
    for (size_t i = 0; i < n; ++i) {
      float v = logits[i];
      if (v > best || (v == best && (uint32_t)i < id)) {
        best = v;
        id = (uint32_t)i;
      }
    }
    /* NaNs never win a comparison; a NaN row still latches status 1. */
    if (!status) {
      if (!isfinite(best))
        status = 2;
      else
        token = id;
    }
    *token_out = token;
    *status_out = status;
    return;
  }
  cand* c = (cand*)malloc(sizeof(cand) * n);
  for (size_t i = 0; i < n; ++i)
    c[i] = (cand){descending_key(logits[i]), (uint32_t)i};
  qsort(c, n, sizeof(cand), cand_cmp);
  const size_t keep = top_k ? top_k : n;
  if (keep == 0) {
    free(c);
    *token_out = 0;
    *status_out = 2;
    return;
  }
  const size_t tiles = (keep + 255) / 256;
  double* prefix = (double*)malloc(sizeof(double) * keep);
  double* totals = (double*)malloc(sizeof(double) * tiles);
  const double best = (double)logits[c[0].id];
  for (size_t b = 0; b < tiles; ++b) {
    double sum = 0.0;
    for (size_t j = 0; j < 256; ++j) {
      size_t i = b * 256 + j;
      double weight = 0.0;
      if (i < keep) {
        double v = (double)logits[c[i].id];
        if (isfinite(v)) weight = exp((v - best) / temperature);
      }
      sum += weight;
      if (i < keep) prefix[i] = sum;
    }
    totals[b] = sum;
  }
  double total = 0.0;
  for (size_t b = 0; b < tiles; ++b) {
    double value = totals[b];
    totals[b] = total;
    total += value;
  }
  size_t cutoff = keep - 1, selected = keep - 1;
  if (!(total > 0.0)) status = 2;
  for (size_t i = 0; i < keep; ++i) {
    if ((totals[i / 256] + prefix[i]) / total >= top_p) {
      cutoff = i;
      break;
    }
  }
  const size_t last = cutoff;
  const double retained = totals[last / 256] + prefix[last];
  const double u = (double)(word >> 11) * 0x1.0p-53;
  for (size_t i = 0; i <= last; ++i) {
    if (u < (totals[i / 256] + prefix[i]) / retained) {
      selected = i;
      break;
    }
  }
  if (!status) token = c[selected < cutoff ? selected : cutoff].id;
  *token_out = token;
  *status_out = status;
  free(prefix);
  free(totals);
  free(c);
}

/* ------------------------------------------------------------------------ */
/* Synthetic weights: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) as a
 * counter-based stream; each element is the Irwin-Hall sum of the eight
 * 16-bit halves of one Philox block, centred and scaled by one FP32
 * multiply, then rounded to BF16.  Integer-only up to that multiply, so the
 * CUDA generator in the product produces identical bits.                    */
/* ------------------------------------------------------------------------ */
static inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int round = 0; round < 10; ++round) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

OR_API void or_philox(uint64_t seed, uint32_t stream, uint64_t index,
                      uint32_t out[4]) {
  uint32_t c[4] = {(uint32_t)index, (uint32_t)(index >> 32), stream, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  memcpy(out, c, 16);
}

/* Centre of the eight-half sum; scale = sigma / sd(sum) passed as FP32. */
#define IH_CENTRE 262140
OR_API void or_fill_normal_bf16(uint16_t* out, size_t n, uint64_t seed,
                                uint32_t stream, float scale) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i) {
    uint32_t c[4] = {(uint32_t)i, (uint32_t)((uint64_t)i >> 32), stream, 0u};
    philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    int32_t s = 0;
    for (int j = 0; j < 4; ++j) s += (int32_t)(c[j] & 0xffffu) + (int32_t)(c[j] >> 16);
    out[i] = to_bf((float)(s - IH_CENTRE) * scale);
  }
}

OR_API void or_fill_uniform_ids(uint32_t* out, size_t n, uint64_t seed,
                                uint32_t stream, uint32_t bound) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t c[4] = {(uint32_t)i, (uint32_t)((uint64_t)i >> 32), stream, 0u};
    philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
    uint64_t wide = ((uint64_t)c[1] << 32) | c[0];
    out[i] = (uint32_t)(wide % bound);
  }
}

/* ------------------------------------------------------------------------ */
/* Qwen3 forward in the reference recipe order: src/models/qwen3/model.cpp
 * :343-409 (norm, q, k, v, norm(q), rope(q), norm(k), rope(k), attention,
 * o, add, norm, gate, up, silu*, down, add; final norm + lm_head on the
 * last row).  K after RoPE and V are appended at rows first..first+n-1 of
 * each block's [capacity][kv_heads][head_width] K and V arrays
 * (src/inference/cache/contiguous.cpp:115-131).                              */
/* ------------------------------------------------------------------------ */
typedef struct {
  uint32_t hidden, query_heads, kv_heads, head_width, mlp_width, vocabulary,
      layers;
  float epsilon;
  double theta;
} or_config;

enum {
  R_IN_NORM = 0,
  R_WQ,
  R_WK,
  R_WV,
  R_QNORM,
  R_KNORM,
  R_WO,
  R_POST_NORM,
  R_WG,
  R_WU,
  R_WD,
  ROLES
};
/* tensors[0] = embedding [V][D], [1] = final norm [D], [2] = lm_head [V][D],
 * tensors[3 + layer*ROLES + role] per block.                                */
#define T_LAYER(t, l, r) ((t)[3 + (size_t)(l) * ROLES + (r)])

typedef struct {
  int32_t layer;          /* block whose output row is edited/captured; -1 none */
  uint64_t selected;      /* absolute position of the edited row */
  float strength;         /* alpha: beta = alpha * ||h|| */
  const float* direction; /* unit vector [D], FP32 */
  uint32_t* state;        /* {invalid, count} */
} or_intervention;

OR_API void or_forward(const or_config* cfg, const uint16_t* const* tensors,
                       uint16_t* const* cache, size_t capacity,
                       const uint32_t* tokens, size_t rows,
                       size_t first_position, uint16_t* logits_last,
                       int32_t capture_layer, uint16_t* capture_rows,
                       const or_intervention* edit) {
  (void)capacity;
  const size_t D = cfg->hidden, H = cfg->query_heads, G = cfg->kv_heads,
               d = cfg->head_width, F = cfg->mlp_width, V = cfg->vocabulary;
  const size_t n = rows;
  uint16_t* residual = (uint16_t*)malloc(2 * n * D);
  uint16_t* normed = (uint16_t*)malloc(2 * n * D);
  uint16_t* q = (uint16_t*)malloc(2 * n * H * d);
  uint16_t* q2 = (uint16_t*)malloc(2 * n * H * d);
  uint16_t* k = (uint16_t*)malloc(2 * n * G * d);
  uint16_t* k2 = (uint16_t*)malloc(2 * n * G * d);
  uint16_t* att = (uint16_t*)malloc(2 * n * H * d);
  uint16_t* proj = (uint16_t*)malloc(2 * n * D);
  uint16_t* gate = (uint16_t*)malloc(2 * n * F);
  uint16_t* up = (uint16_t*)malloc(2 * n * F);
  or_embedding(tokens, tensors[0], residual, n, D);
  for (uint32_t l = 0; l < cfg->layers; ++l) {
    uint16_t* kc = cache[2 * l];
    uint16_t* vc = cache[2 * l + 1];
    or_rms_norm(residual, T_LAYER(tensors, l, R_IN_NORM), normed, n, D,
                cfg->epsilon);
    or_projection(normed, T_LAYER(tensors, l, R_WQ), q, n, D, H * d);
    or_projection(normed, T_LAYER(tensors, l, R_WK), k, n, D, G * d);
    or_projection(normed, T_LAYER(tensors, l, R_WV),
                  vc + first_position * G * d, n, D, G * d);
    or_rms_norm(q, T_LAYER(tensors, l, R_QNORM), q2, n * H, d, cfg->epsilon);
    or_rotary(q2, q, n, H, d, first_position, cfg->theta);
    or_rms_norm(k, T_LAYER(tensors, l, R_KNORM), k2, n * G, d, cfg->epsilon);
    or_rotary(k2, kc + first_position * G * d, n, G, d, first_position,
              cfg->theta);
    or_attention(q, kc, vc, att, n, H, G, d, first_position);
    or_projection(att, T_LAYER(tensors, l, R_WO), proj, n, H * d, D);
    or_add(residual, proj, residual, n * D);
    or_rms_norm(residual, T_LAYER(tensors, l, R_POST_NORM), normed, n, D,
                cfg->epsilon);
    or_projection(normed, T_LAYER(tensors, l, R_WG), gate, n, D, F);
    or_projection(normed, T_LAYER(tensors, l, R_WU), up, n, D, F);
    or_silu_multiply(gate, up, gate, n * F);
    or_projection(gate, T_LAYER(tensors, l, R_WD), proj, n, F, D);
    or_add(residual, proj, residual, n * D);
    if (edit && edit->layer == (int32_t)l)
      or_intervene(residual, edit->direction, D, edit->selected,
                   first_position, n, edit->strength, edit->state);
    if (capture_rows && capture_layer == (int32_t)l)
      memcpy(capture_rows, residual, 2 * n * D);
    if (capture_rows && capture_layer == -2) /* every block, [L][n][D] */
      memcpy(capture_rows + (size_t)l * n * D, residual, 2 * n * D);
  }
  if (logits_last) {
    or_rms_norm(residual + (n - 1) * D, tensors[1], normed, 1, D,
                cfg->epsilon);
    or_projection(normed, tensors[2], logits_last, 1, D, V);
  }
  free(residual);
  free(normed);
  free(q);
  free(q2);
  free(k);
  free(k2);
  free(att);
  free(proj);
  free(gate);
  free(up);
}

OR_API int or_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
OR_API void or_set_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n);
#else
  (void)n;
#endif
}
