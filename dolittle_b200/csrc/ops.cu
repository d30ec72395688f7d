// Per-operation kernels of the Qwen3 block other than the streaming GEMV:
// fused QK-norm + RoPE + KV-append, causal GQA attention (scores, then
// softmax + PV), embedding, add, SwiGLU, RMSNorm, RoPE, and the seeded weight
// generator.  Every kernel keeps the reference's FP32 order and BF16 rounding
// points (file:line citations are into the reference tree).
#include <cmath>

#include "launch.h"
#include "qknorm.cuh"

namespace dl {
namespace {

__device__ __forceinline__ int row_position(RowPositions p, int r) {
  return int((p.device ? *p.device : p.host) + r);
}

cudaLaunchConfig_t make_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                               cudaLaunchAttribute* attr, bool pdl) {
  cudaLaunchConfig_t c = {};
  c.gridDim = grid;
  c.blockDim = block;
  c.dynamicSmemBytes = smem;
  c.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE + K append.  One warp per (row, head); heads [0, Hq) are
// queries (written to q_out), [Hq, Hq+Hkv) keys (written into the K cache at
// the row's absolute position).  Norm law: normalization.cu:82-132 (warp,
// width <= 128).  RoPE law: rotary.cu:84-126 with the precomputed
// inverse-frequency table (same expression, same CUDA pow).
// ---------------------------------------------------------------------------
constexpr int kNormWarps = 8;

__global__ void qk_norm_rope_kernel(const bf16* __restrict__ q_raw, const bf16* __restrict__ k_raw,
                                    const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                    const float* __restrict__ inv_freq, bf16* __restrict__ q_out,
                                    bf16* __restrict__ k_cache, RowPositions pos, int query_heads,
                                    int kv_heads, int width, float eps) {
  __shared__ float vals[kNormWarps][128];
  __shared__ float co[64], si[64];
  allow_next();
  wait_prior();
  const int warp = threadIdx.x >> 5;
  const int r = blockIdx.x;
  const int p = row_position(pos, r);
  // One warp per head (kNormWarps heads per block): the block computes its
  // row's RoPE factors once for its heads.
  rope_factors(inv_freq, p, width, co, si);
  __syncthreads();
  const int head = blockIdx.y * kNormWarps + warp;
  if (head >= query_heads + kv_heads) return;
  const bool is_q = head < query_heads;
  const bf16* src = is_q ? q_raw + (size_t(r) * query_heads + head) * width
                         : k_raw + (size_t(r) * kv_heads + (head - query_heads)) * width;
  bf16* dst = is_q ? q_out + (size_t(r) * query_heads + head) * width
                   : k_cache + (size_t(p) * kv_heads + (head - query_heads)) * width;
  qk_norm_rope_warp_table(src, is_q ? qw : kw, co, si, dst, width, eps, vals[warp]);
}

// ---------------------------------------------------------------------------
// Attention scores: score[r][h][j] = round-free FP32 dot of q_h and k_j under
// the 8-lane law of attention.cu:300-352 (lane l owns the contiguous span
// [l*s, l*s+s), s = ceil(d/8); serial FMA; tree 4,2,1), times the scale.
// One CTA per (key-block slice, kv head, row): the GQA group's query heads
// share every K load.  Keys are split across CTAs freely: scores are
// independent, so the split changes no arithmetic.
// ---------------------------------------------------------------------------
constexpr int kScoreThreads = 256;
constexpr int kKeysPerIter = kScoreThreads / 8;   // 32
constexpr int kMaxGroup = 8;

__global__ void attention_scores_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                        float* __restrict__ scores, RowPositions pos,
                                        int query_heads, int kv_heads, int width, int capacity,
                                        float scale) {
  extern __shared__ float qs[];  // [group][width]
  allow_next();
  wait_prior();
  const int g = blockIdx.y, r = blockIdx.z;
  const int group = query_heads / kv_heads;
  const int count = row_position(pos, r) + 1;
  for (int i = threadIdx.x; i < group * width; i += blockDim.x)
    qs[i] = widen(q[(size_t(r) * query_heads + g * group) * width + i]);
  __syncthreads();
  const int lane8 = threadIdx.x & 7;
  const int span = width / 8 + (width % 8 != 0);
  const int begin = lane8 * span;
  const int end = min(begin + span, width);
  const int slices = gridDim.x;
  // Contiguous key chunk per CTA.
  const int per = (count + slices - 1) / slices;
  const int j0 = blockIdx.x * per, j1 = min(count, j0 + per);
  for (int base = j0; base < j1; base += kKeysPerIter) {
    const int j = base + (threadIdx.x >> 3);
    const bool live = j < j1;
    float part[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) part[h] = 0.f;
    if (live) {
      const bf16* kr = k + (size_t(j) * kv_heads + g) * width;
      if (width == 128) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(kr + begin);
        const uint4 w1 = *reinterpret_cast<const uint4*>(kr + begin + 8);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
          if (h < group) {
            const float* qh = qs + h * width + begin;
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float kv = (i & 1) ? bf_hi(words[i >> 1]) : bf_lo(words[i >> 1]);
              acc = __fmaf_rn(qh[i], kv, acc);
            }
            part[h] = acc;
          }
        }
      } else {
        for (int h = 0; h < group && h < kMaxGroup; ++h) {
          float acc = 0.f;
          for (int f = begin; f < end; ++f) acc = __fmaf_rn(qs[h * width + f], widen(kr[f]), acc);
          part[h] = acc;
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      float v = part[h];
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
      part[h] = v;
    }
    if (live && lane8 == 0) {
      for (int h = 0; h < group; ++h)
        scores[(size_t(r) * query_heads + g * group + h) * capacity + j] = __fmul_rn(part[h], scale);
    }
  }
}

// ---------------------------------------------------------------------------
// Softmax + PV for one (row, query head): attention.cu:354-383.  Maximum
// (exact), e = expf(s - max), denominator = 32 strided serial partials then
// the 256-lane halving tree (only lanes < 32 non-zero), p = e / den, then
// two contiguous key halves [0, split) and [split, count) summed serially per
// feature and added once.
// ---------------------------------------------------------------------------
constexpr int kPvThreads = 256;

__global__ void attention_pv_kernel(const float* __restrict__ scores, const bf16* __restrict__ v,
                                    bf16* __restrict__ out, RowPositions pos, int query_heads,
                                    int kv_heads, int width, int capacity) {
  extern __shared__ float p[];       // [count]
  __shared__ float red[kPvThreads];
  __shared__ float stat[2];
  allow_next();
  wait_prior();
  const int h = blockIdx.x, r = blockIdx.y;
  const int g = h / (query_heads / kv_heads);
  const int count = row_position(pos, r) + 1;
  const float* srow = scores + (size_t(r) * query_heads + h) * capacity;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < count; j += kPvThreads) {
    const float s = srow[j];
    p[j] = s;
    m = j == threadIdx.x ? s : fmaxf(m, s);
  }
  red[threadIdx.x] = threadIdx.x < count ? m : -INFINITY;
  __syncthreads();
  for (int off = kPvThreads / 2; off; off >>= 1) {
    if (threadIdx.x < off) red[threadIdx.x] = fmaxf(red[threadIdx.x], red[threadIdx.x + off]);
    __syncthreads();
  }
  const float maximum = red[0];
  __syncthreads();
  for (int j = threadIdx.x; j < count; j += kPvThreads) p[j] = expf(p[j] - maximum);
  __syncthreads();
  if (threadIdx.x < 32) {
    float acc = 0.f;
    for (int j = threadIdx.x; j < count; j += 32) acc = __fadd_rn(acc, p[j]);
#pragma unroll
    for (int off = 16; off; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
    if (threadIdx.x == 0) stat[0] = acc;
  }
  __syncthreads();
  const float den = stat[0];
  for (int j = threadIdx.x; j < count; j += kPvThreads) p[j] = p[j] / den;
  __syncthreads();
  const int split = (count - 1) / 2 + 1;
  const bf16* vbase = v + size_t(g) * width;
  const size_t vstride = size_t(kv_heads) * width;
  bf16* orow = out + (size_t(r) * query_heads + h) * width;
  if (width <= kPvThreads / 2) {
    const int f = threadIdx.x % (kPvThreads / 2), half = threadIdx.x / (kPvThreads / 2);
    const int jb = half == 0 ? 0 : split, je = half == 0 ? split : count;
    float acc = 0.f;
    if (f < width) {
      const bf16* col = vbase + f;
      int j = jb;
      for (; j + 4 <= je; j += 4) {
        const float v0 = widen(col[size_t(j) * vstride]);
        const float v1 = widen(col[size_t(j + 1) * vstride]);
        const float v2 = widen(col[size_t(j + 2) * vstride]);
        const float v3 = widen(col[size_t(j + 3) * vstride]);
        acc = __fmaf_rn(p[j], v0, acc);
        acc = __fmaf_rn(p[j + 1], v1, acc);
        acc = __fmaf_rn(p[j + 2], v2, acc);
        acc = __fmaf_rn(p[j + 3], v3, acc);
      }
      for (; j < je; ++j) acc = __fmaf_rn(p[j], widen(col[size_t(j) * vstride]), acc);
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < width)
      orow[threadIdx.x] = narrow(__fadd_rn(red[threadIdx.x], red[threadIdx.x + kPvThreads / 2]));
  } else {
    for (int f = threadIdx.x; f < width; f += kPvThreads) {
      float first = 0.f, second = 0.f;
      for (int j = 0; j < split; ++j) first = __fmaf_rn(p[j], widen(vbase[size_t(j) * vstride + f]), first);
      for (int j = split; j < count; ++j)
        second = __fmaf_rn(p[j], widen(vbase[size_t(j) * vstride + f]), second);
      orow[f] = narrow(__fadd_rn(first, second));
    }
  }
}

// ---------------------------------------------------------------------------
// Small elementwise kernels (embedding.cu:60-80, elementwise.cu:62-87).
// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const uint32_t* __restrict__ tokens, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int width) {
  allow_next();
  wait_prior();
  const uint32_t t = tokens[blockIdx.x];
  const bf16* src = table + size_t(t) * width;
  bf16* dst = out + size_t(blockIdx.x) * width;
  if ((width & 7) == 0) {
    for (int i = threadIdx.x; i < width / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int i = threadIdx.x; i < width; i += blockDim.x) dst[i] = src[i];
  }
}

__global__ void add_kernel(const bf16* a, const bf16* b, bf16* out, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = narrow(__fadd_rn(widen(a[i]), widen(b[i])));
}

__global__ void silu_multiply_kernel(const bf16* g, const bf16* u, bf16* out, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const float a = widen(g[i]), b = widen(u[i]);
    const float e = expf(a >= 0.0f ? -a : a);
    const float s = a >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
    out[i] = narrow(__fmul_rn(round_bf16(__fmul_rn(a, s)), b));
  }
}

// RMSNorm rows; one warp per row (normalization.cu laws by width).
__global__ void rms_norm_kernel(const bf16* x, const bf16* w, bf16* out, size_t rows, int width,
                                float eps) {
  extern __shared__ float row[];  // [warps][width]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t r = blockIdx.x * size_t(blockDim.x / 32) + warp;
  if (r >= rows) return;
  float* xs = row + size_t(warp) * width;
  for (int i = lane; i < width; i += 32) xs[i] = widen(x[r * width + i]);
  __syncwarp();
  const float inv = rms_inverse_warp(xs, width, eps);
  for (int i = lane; i < width; i += 32)
    out[r * width + i] = narrow(__fmul_rn(round_bf16(__fmul_rn(xs[i], inv)), widen(w[i])));
}

// One row per CTA for rows of width % 8 == 0 (at most 8192): the row comes
// in with 16-byte loads and is held as FP32 in shared memory, one warp runs
// the reference reduction (rms_inverse_warp: same order as above), and the
// normalisation goes out with 16-byte stores.  Bit-identical to
// rms_norm_kernel.
__global__ void rms_norm_rows_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ out,
                                     int width, float eps) {
  extern __shared__ float xs[];  // [width]
  __shared__ float chains[129];
  __shared__ float inv_s;
  allow_next();
  wait_prior();
  const size_t r = blockIdx.x;
  const int n8 = width / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x + r * width);
  for (int q = threadIdx.x; q < n8; q += blockDim.x) {
    const uint4 v = src[q];
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xs[8 * q + 2 * i] = bf_lo(wd[i]);
      xs[8 * q + 2 * i + 1] = bf_hi(wd[i]);
    }
  }
  __syncthreads();
  if (width > 128) {
    // The staged law's component sums run as 128 independent chains, one
    // per thread (chain t = 4 * lane + c sums columns t, t + 128, ...); warp
    // 0 then adds each lane's four in order and runs the shuffle tree.
    const float inv = rms_inverse_block(xs, width, eps, chains);
    if (threadIdx.x == 0) inv_s = inv;
  } else if (threadIdx.x < 32) {
    const float inv = rms_inverse_warp(xs, width, eps);
    if (threadIdx.x == 0) inv_s = inv;
  }
  __syncthreads();
  const float inv = inv_s;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4* dst = reinterpret_cast<uint4*>(out + r * width);
  for (int q = threadIdx.x; q < n8; q += blockDim.x) {
    const uint4 g = wv[q];
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bf16 lo = narrow(__fmul_rn(round_bf16(__fmul_rn(xs[8 * q + 2 * i], inv)), bf_lo(gw[i])));
      const bf16 hi = narrow(__fmul_rn(round_bf16(__fmul_rn(xs[8 * q + 2 * i + 1], inv)), bf_hi(gw[i])));
      o[i] = uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
    }
    dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void rotary_kernel(const bf16* x, bf16* out, size_t pairs, int heads, int width,
                              RowPositions pos, double theta, bool positioned) {
  const int half = width / 2;
  const int first = int(pos.device ? *pos.device : pos.host);
  bf16* o = out + (positioned ? size_t(first) * heads * width : 0);
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < pairs; i += size_t(gridDim.x) * blockDim.x) {
    const int f = int(i % half);
    const size_t row = i / half;
    const int p = first + int(row / heads);
    const float exponent = static_cast<float>(2 * f) / static_cast<float>(width);
    const float inv = static_cast<float>(1.0 / pow(theta, static_cast<double>(exponent)));
    const float angle = __fmul_rn(static_cast<float>(p), inv);
    const float co = round_bf16(cosf(angle)), si = round_bf16(sinf(angle));
    const float a = widen(x[row * width + f]), b = widen(x[row * width + f + half]);
    const float ac = round_bf16(__fmul_rn(a, co)), bs = round_bf16(__fmul_rn(b, si));
    const float bc = round_bf16(__fmul_rn(b, co)), as = round_bf16(__fmul_rn(a, si));
    o[row * width + f] = narrow(__fsub_rn(ac, bs));
    o[row * width + f + half] = narrow(__fadd_rn(bc, as));
  }
}

__global__ void inv_freq_kernel(float* out, int width, double theta) {
  const int f = threadIdx.x + blockIdx.x * blockDim.x;
  if (f < width / 2) {
    const float exponent = static_cast<float>(2 * f) / static_cast<float>(width);
    out[f] = static_cast<float>(1.0 / pow(theta, static_cast<double>(exponent)));
  }
}

// ---------------------------------------------------------------------------
// Seeded synthetic weights: Philox4x32-10 (Salmon et al., SC'11) per element,
// Irwin-Hall sum of the block's eight 16-bit halves, one FP32 scale multiply,
// BF16 rounding.  Integer-only up to the multiply, so a host restatement of
// the same algorithm reproduces the bits.
// ---------------------------------------------------------------------------
// Element i of a logical [rows][cols] tensor lands at row (i/cols) of a
// resident layout with `row_stride` elements per row.
__global__ void fill_normal_kernel(bf16* out, size_t n, size_t cols, size_t row_stride, uint64_t seed,
                                   uint32_t stream_id, float scale) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[(i / cols) * row_stride + i % cols] = normal_bf16(uint64_t(i), seed, stream_id, scale);
}

__global__ void fill_const_kernel(bf16* out, size_t n, float value) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = narrow(value);
}

__global__ void uniform_ids_kernel(uint32_t* out, size_t n, uint64_t seed, uint32_t stream_id,
                                   uint32_t bound) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    uint32_t c[4] = {uint32_t(i), uint32_t(uint64_t(i) >> 32), stream_id, 0u};
    philox4x32_10(c, uint32_t(seed), uint32_t(seed >> 32));
    const uint64_t wide = (uint64_t(c[1]) << 32) | c[0];
    out[i] = uint32_t(wide % bound);
  }
}

__global__ void add_position_kernel(long long* value, long long delta) { *value += delta; }

unsigned blocks_for(size_t n, unsigned threads) {
  const size_t b = (n + threads - 1) / threads;
  return unsigned(b < 148 * 32 ? (b ? b : 1) : 148 * 32);
}

}  // namespace

cudaError_t launch_qk_norm_rope(const bf16* q_raw, const bf16* k_raw, const bf16* q_norm_w,
                                const bf16* k_norm_w, const float* inv_freq, bf16* q_out,
                                bf16* k_cache, RowPositions pos, int rows, int query_heads,
                                int kv_heads, int width, float eps, cudaStream_t stream, bool pdl) {
  if (width > 128 || width % 2) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  const int heads = query_heads + kv_heads;
  auto cfg = make_config(dim3(rows, (heads + kNormWarps - 1) / kNormWarps), dim3(32 * kNormWarps), 0, stream, attr,
                         pdl);
  return cudaLaunchKernelEx(&cfg, qk_norm_rope_kernel, q_raw, k_raw, q_norm_w, k_norm_w, inv_freq, q_out,
                            k_cache, pos, query_heads, kv_heads, width, eps);
}

cudaError_t launch_attention_scores(const bf16* q, const bf16* k_cache, float* scores,
                                    RowPositions pos, int rows, int query_heads, int kv_heads,
                                    int width, int capacity, float scale, int ctas_per_head,
                                    cudaStream_t stream, bool pdl) {
  if (query_heads % kv_heads || query_heads / kv_heads > kMaxGroup) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  const size_t smem = size_t(query_heads / kv_heads) * width * sizeof(float);
  auto cfg = make_config(dim3(ctas_per_head, kv_heads, rows), dim3(kScoreThreads), smem, stream, attr, pdl);
  return cudaLaunchKernelEx(&cfg, attention_scores_kernel, q, k_cache, scores, pos, query_heads, kv_heads,
                            width, capacity, scale);
}

cudaError_t launch_attention_pv(const float* scores, const bf16* v_cache, bf16* out, RowPositions pos,
                                int rows, int query_heads, int kv_heads, int width, int capacity,
                                cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  const size_t smem = size_t(capacity) * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaFuncSetAttribute(attention_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  auto cfg = make_config(dim3(query_heads, rows), dim3(kPvThreads), smem, stream, attr, pdl);
  return cudaLaunchKernelEx(&cfg, attention_pv_kernel, scores, v_cache, out, pos, query_heads, kv_heads,
                            width, capacity);
}

cudaError_t launch_embedding(const uint32_t* tokens, const bf16* table, bf16* out, int rows, int width,
                             cudaStream_t stream, bool pdl) {
  cudaLaunchAttribute attr[1];
  auto cfg = make_config(dim3(rows), dim3(256), 0, stream, attr, pdl);
  return cudaLaunchKernelEx(&cfg, embedding_kernel, tokens, table, out, width);
}

cudaError_t launch_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t stream) {
  add_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(a, b, out, n);
  return cudaGetLastError();
}

cudaError_t launch_silu_multiply(const bf16* g, const bf16* u, bf16* out, size_t n, cudaStream_t stream) {
  silu_multiply_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(g, u, out, n);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm(const bf16* x, const bf16* w, bf16* out, size_t rows, int width, float eps,
                            cudaStream_t stream, bool pdl) {
  if (width > 32768) return cudaErrorInvalidValue;
  if (width % 8 == 0 && width <= 8192 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const size_t smem = size_t(width) * sizeof(float);
    cudaLaunchAttribute attr[1];
    auto cfg = make_config(dim3(unsigned(rows)), dim3(128), smem, stream, attr, pdl);
    return cudaLaunchKernelEx(&cfg, rms_norm_rows_kernel, x, w, out, width, eps);
  }
  const int warps = width > 8192 ? 1 : (width > 2048 ? 2 : 4);
  const size_t smem = size_t(warps) * width * sizeof(float);
  cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rms_norm_kernel<<<unsigned((rows + warps - 1) / warps), 32 * warps, smem, stream>>>(x, w, out, rows, width,
                                                                                     eps);
  return cudaGetLastError();
}

cudaError_t launch_rotary(const bf16* x, bf16* out, size_t positions, int heads, int width, RowPositions pos,
                          double theta, bool positioned_output, cudaStream_t stream) {
  const size_t pairs = positions * heads * (width / 2);
  rotary_kernel<<<blocks_for(pairs, 256), 256, 0, stream>>>(x, out, pairs, heads, width, pos, theta,
                                                           positioned_output);
  return cudaGetLastError();
}

cudaError_t launch_inv_freq(float* out, int width, double theta, cudaStream_t stream) {
  inv_freq_kernel<<<(width / 2 + 127) / 128, 128, 0, stream>>>(out, width, theta);
  return cudaGetLastError();
}

cudaError_t launch_fill_normal(bf16* out, size_t rows, size_t cols, size_t row_stride, uint64_t seed,
                               uint32_t stream_id, float scale, cudaStream_t stream) {
  const size_t n = rows * cols;
  fill_normal_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(out, n, cols, row_stride, seed, stream_id, scale);
  return cudaGetLastError();
}

cudaError_t launch_fill_const(bf16* out, size_t n, float value, cudaStream_t stream) {
  fill_const_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(out, n, value);
  return cudaGetLastError();
}

cudaError_t launch_uniform_ids(uint32_t* out, size_t n, uint64_t seed, uint32_t stream_id, uint32_t bound,
                               cudaStream_t stream) {
  uniform_ids_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(out, n, seed, stream_id, bound);
  return cudaGetLastError();
}

cudaError_t launch_add_position(long long* value, long long delta, cudaStream_t stream) {
  add_position_kernel<<<1, 1, 0, stream>>>(value, delta);
  return cudaGetLastError();
}

}  // namespace dl
