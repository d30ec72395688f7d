// Batched serving kernels (see serve_kernels.h).  The batched step is the fast
// path: tensor-core projections and an online-softmax attention, checked
// against the reference within tolerance; QK-norm + RoPE keep the reference
// law exactly (the shared warp routine of the per-operation kernel).
#include <algorithm>
#include <cmath>

#include "qknorm.cuh"
#include "serve_kernels.h"

namespace dl {
namespace {

__global__ void fill_normal_slice_kernel(bf16* out, size_t rows, size_t cols, size_t out_stride, size_t full_cols,
                                         size_t r0, size_t c0, uint64_t seed, uint32_t stream_id, float scale) {
  const size_t n = rows * cols;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const size_t r = i / cols, c = i % cols;
    out[r * out_stride + c] = normal_bf16(uint64_t((r0 + r) * full_cols + c0 + c), seed, stream_id, scale);
  }
}

constexpr int kRopeWarps = 8;

// Heads [0, Hq): queries; [Hq, Hq+Hkv): keys; [Hq+Hkv, Hq+2Hkv): values
// (copied).  One warp per (row, head).
__global__ void norm_rope_append_rows_kernel(const bf16* __restrict__ qkv, int ld, const bf16* __restrict__ qw,
                                             const bf16* __restrict__ kw, const float* __restrict__ inv_freq,
                                             bf16* __restrict__ q_out, KvPlanes planes,
                                             const long long* __restrict__ position, int query_heads, int kv_heads,
                                             int width, float eps) {
  __shared__ float vals[kRopeWarps][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int head = blockIdx.y * kRopeWarps + warp;
  if (head >= query_heads + 2 * kv_heads) return;
  const int p = int(*position);
  const bf16* row = qkv + size_t(b) * ld;
  const size_t G = size_t(kv_heads) * width;
  bf16* seq = planes.kv + size_t(b) * planes.seq_stride;
  if (head < query_heads) {
    qk_norm_rope_warp(row + size_t(head) * width, qw, inv_freq, p,
                      q_out + (size_t(b) * query_heads + head) * width, width, eps, vals[warp]);
  } else if (head < query_heads + kv_heads) {
    const int g = head - query_heads;
    qk_norm_rope_warp(row + size_t(query_heads) * width + size_t(g) * width, kw, inv_freq, p,
                      seq + planes.k_off + size_t(p) * G + size_t(g) * width, width, eps, vals[warp]);
  } else {
    const int g = head - query_heads - kv_heads;
    const bf16* src = row + size_t(query_heads) * width + G + size_t(g) * width;
    bf16* dst = seq + planes.v_off + size_t(p) * G + size_t(g) * width;
    for (int f = lane; f < width; f += 32) dst[f] = src[f];
  }
}

// ---------------------------------------------------------------------------
// Split-K flash decoding.  CTA (split s, kv head g, sequence b) streams keys
// [j0, j1) of b's cache in tiles of 64 through a two-stage cp.async ring
// (K and V rows padded to 272 bytes: conflict-free 16-byte reads), computes
// the group's scores (one (key, head) per thread), keeps a running max and
// sum per head and rescales the per-thread output pairs.
// ---------------------------------------------------------------------------
constexpr int kAdThreads = 256;
constexpr int kAdKeys = 64;
constexpr int kAdPitch = 136;   // BF16 per smem row (128 + 8)
constexpr int kAdQPitch = 132;  // FP32 per query row
constexpr int kAdMaxGroup = 8;
constexpr int kAdWs = 130;      // m, l, 128 outputs
constexpr int kAdStageElems = 2 * kAdKeys * kAdPitch;  // K then V
constexpr size_t kAdSmem =
    size_t(2) * kAdStageElems * 2 + size_t(kAdMaxGroup) * kAdQPitch * 4 + size_t(kAdMaxGroup) * kAdKeys * 4 +
    3 * kAdMaxGroup * 4;

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(kAdThreads) attention_decode_split_kernel(
    const bf16* __restrict__ q, KvPlanes planes, const long long* __restrict__ position, int query_heads,
    int kv_heads, int splits, float scale, float* __restrict__ ws) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* stage = reinterpret_cast<bf16*>(smem);
  float* qs = reinterpret_cast<float*>(smem + size_t(2) * kAdStageElems * 2);
  float* ps = qs + kAdMaxGroup * kAdQPitch;
  float* mrun = ps + kAdMaxGroup * kAdKeys;
  float* lrun = mrun + kAdMaxGroup;
  float* alpha = lrun + kAdMaxGroup;
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z, t = threadIdx.x;
  const int group = query_heads / kv_heads;
  const int count = int(*position) + 1;
  const int per = ((count + splits - 1) / splits + kAdKeys - 1) / kAdKeys * kAdKeys;
  const int j0 = min(count, s * per), j1 = min(count, j0 + per);
  const size_t G = size_t(kv_heads) * 128;
  const bf16* kbase = planes.kv + size_t(b) * planes.seq_stride + planes.k_off + size_t(g) * 128;
  const bf16* vbase = planes.kv + size_t(b) * planes.seq_stride + planes.v_off + size_t(g) * 128;
  for (int i = t; i < group * 128; i += kAdThreads) {
    const int h = i / 128, f = i % 128;
    qs[h * kAdQPitch + f] = widen(q[(size_t(b) * query_heads + g * group + h) * 128 + f]);
  }
  if (t < group) {
    mrun[t] = -INFINITY;
    lrun[t] = 0.f;
  }
  auto load_tile = [&](int tile, int slot) {
    const int base = j0 + tile * kAdKeys;
    const int n = min(kAdKeys, j1 - base);
    bf16* ks = stage + slot * kAdStageElems;
    bf16* vs = ks + kAdKeys * kAdPitch;
    for (int i = t; i < n * 16; i += kAdThreads) {
      const int kk = i >> 4, c = i & 15;
      cp16(ks + kk * kAdPitch + 8 * c, kbase + size_t(base + kk) * G + 8 * c);
      cp16(vs + kk * kAdPitch + 8 * c, vbase + size_t(base + kk) * G + 8 * c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int tiles = (j1 - j0 + kAdKeys - 1) / kAdKeys;
  constexpr int kMaxPairs = kAdMaxGroup * 64 / kAdThreads;  // output feature pairs per thread
  float acc[kMaxPairs][2] = {};
  if (tiles > 0) load_tile(0, 0);
  for (int tile = 0; tile < tiles; ++tile) {
    const int slot = tile & 1;
    if (tile + 1 < tiles) {
      load_tile(tile + 1, slot ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const bf16* ks = stage + slot * kAdStageElems;
    const bf16* vs = ks + kAdKeys * kAdPitch;
    const int n = min(kAdKeys, j1 - (j0 + tile * kAdKeys));
    // Scores of (key kk, head h), scaled; masked keys are -inf.
    for (int i = t; i < group * kAdKeys; i += kAdThreads) {
      const int h = i % group, kk = i / group;
      float sc = -INFINITY;
      if (kk < n) {
        const bf16* kr = ks + kk * kAdPitch;
        const float* qh = qs + h * kAdQPitch;
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(kr + 8 * c);
          const float4 qa = *reinterpret_cast<const float4*>(qh + 8 * c);
          const float4 qb = *reinterpret_cast<const float4*>(qh + 8 * c + 4);
          d = fmaf(qa.x, bf_lo(w.x), d);
          d = fmaf(qa.y, bf_hi(w.x), d);
          d = fmaf(qa.z, bf_lo(w.y), d);
          d = fmaf(qa.w, bf_hi(w.y), d);
          d = fmaf(qb.x, bf_lo(w.z), d);
          d = fmaf(qb.y, bf_hi(w.z), d);
          d = fmaf(qb.z, bf_lo(w.w), d);
          d = fmaf(qb.w, bf_hi(w.w), d);
        }
        sc = d * scale;
      }
      ps[h * kAdKeys + kk] = sc;
    }
    __syncthreads();
    // Running max / sum per head: warp h.
    const int warp = t >> 5, lane = t & 31;
    if (warp < group) {
      float* row = ps + warp * kAdKeys;
      const float s0 = row[lane], s1 = row[lane + 32];
      float m = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float m_old = mrun[warp];
      const float m_new = fmaxf(m_old, m);
      const float p0 = s0 == -INFINITY ? 0.f : expf(s0 - m_new);
      const float p1 = s1 == -INFINITY ? 0.f : expf(s1 - m_new);
      row[lane] = p0;
      row[lane + 32] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      __syncwarp();
      if (lane == 0) {
        const float a = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        alpha[warp] = a;
        lrun[warp] = lrun[warp] * a + sum;
        mrun[warp] = m_new;
      }
    }
    __syncthreads();
    // Output pairs: (head, features 2f, 2f+1).
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int pair = t + i * kAdThreads;
      if (pair < group * 64) {
        const int h = pair / 64, f = (pair % 64) * 2;
        const float a = alpha[h];
        float x = acc[i][0] * a, y = acc[i][1] * a;
        const float* ph = ps + h * kAdKeys;
        for (int kk = 0; kk < n; ++kk) {
          const uint32_t v2 = *reinterpret_cast<const uint32_t*>(vs + kk * kAdPitch + f);
          x = fmaf(ph[kk], bf_lo(v2), x);
          y = fmaf(ph[kk], bf_hi(v2), y);
        }
        acc[i][0] = x;
        acc[i][1] = y;
      }
    }
    __syncthreads();  // the next tile's loads reuse this slot
  }
  float* w = ws + ((size_t(b) * query_heads + g * group) * splits + s) * kAdWs;
  if (t < group) {
    w[size_t(t) * splits * kAdWs + 0] = mrun[t];
    w[size_t(t) * splits * kAdWs + 1] = lrun[t];
  }
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) {
    const int pair = t + i * kAdThreads;
    if (pair < group * 64) {
      const int h = pair / 64, f = (pair % 64) * 2;
      w[size_t(h) * splits * kAdWs + 2 + f] = acc[i][0];
      w[size_t(h) * splits * kAdWs + 3 + f] = acc[i][1];
    }
  }
}

__global__ void attention_decode_combine_kernel(const float* __restrict__ ws, int query_heads, int splits,
                                                bf16* __restrict__ out) {
  const int h = blockIdx.x, b = blockIdx.y, f = threadIdx.x;
  const float* w = ws + (size_t(b) * query_heads + h) * splits * kAdWs;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, w[size_t(s) * kAdWs]);
  float L = 0.f, o = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = w[size_t(s) * kAdWs];
    if (m == -INFINITY) continue;
    const float e = expf(m - M);
    L += w[size_t(s) * kAdWs + 1] * e;
    o += w[size_t(s) * kAdWs + 2 + f] * e;
  }
  out[(size_t(b) * query_heads + h) * 128 + f] = narrow(o / L);
}

__global__ void add_fp32_residual_kernel(const float* __restrict__ sum, bf16* __restrict__ residual, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    residual[i] = narrow(__fadd_rn(widen(residual[i]), round_bf16(sum[i])));
}

unsigned grid_for(size_t n) { return unsigned(std::min<size_t>((n + 255) / 256, 148 * 32)); }

}  // namespace

cudaError_t launch_fill_normal_slice(bf16* out, size_t rows, size_t cols, size_t out_stride, size_t full_cols,
                                     size_t r0, size_t c0, uint64_t seed, uint32_t stream_id, float scale,
                                     cudaStream_t stream) {
  if (!rows || !cols) return cudaSuccess;
  fill_normal_slice_kernel<<<grid_for(rows * cols), 256, 0, stream>>>(out, rows, cols, out_stride, full_cols, r0,
                                                                       c0, seed, stream_id, scale);
  return cudaGetLastError();
}

cudaError_t launch_norm_rope_append_rows(const bf16* qkv, int ld, const bf16* q_norm_w, const bf16* k_norm_w,
                                         const float* inv_freq, bf16* q_out, KvPlanes planes,
                                         const long long* position, int batch, int query_heads, int kv_heads,
                                         int width, float eps, cudaStream_t stream) {
  if (width > 128 || width % 2 || batch < 1) return cudaErrorInvalidValue;
  const int heads = query_heads + 2 * kv_heads;
  norm_rope_append_rows_kernel<<<dim3(batch, (heads + kRopeWarps - 1) / kRopeWarps), 32 * kRopeWarps, 0, stream>>>(
      qkv, ld, q_norm_w, k_norm_w, inv_freq, q_out, planes, position, query_heads, kv_heads, width, eps);
  return cudaGetLastError();
}

size_t attention_decode_ws_floats(int batch, int query_heads, int splits) {
  return size_t(batch) * query_heads * splits * kAdWs;
}

int attention_decode_splits(int batch, int kv_heads, int capacity, int sms) {
  const int units = std::max(1, batch * kv_heads);
  const int want = (4 * sms + units - 1) / units;
  return std::clamp(want, 1, std::clamp((capacity + kAdKeys - 1) / kAdKeys, 1, 64));
}

cudaError_t launch_attention_decode_batched(const bf16* q, KvPlanes planes, const long long* position, int batch,
                                            int query_heads, int kv_heads, int splits, float scale, float* ws,
                                            bf16* out, cudaStream_t stream) {
  if (query_heads % kv_heads || query_heads / kv_heads > kAdMaxGroup || splits < 1 || splits > 64 || batch < 1)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(attention_decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(kAdSmem));
  if (e != cudaSuccess) return e;
  attention_decode_split_kernel<<<dim3(splits, kv_heads, batch), kAdThreads, kAdSmem, stream>>>(
      q, planes, position, query_heads, kv_heads, splits, scale, ws);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attention_decode_combine_kernel<<<dim3(query_heads, batch), 128, 0, stream>>>(ws, query_heads, splits, out);
  return cudaGetLastError();
}

cudaError_t launch_add_fp32_residual(const float* sum, bf16* residual, size_t n, cudaStream_t stream) {
  add_fp32_residual_kernel<<<grid_for(n), 256, 0, stream>>>(sum, residual, n);
  return cudaGetLastError();
}

}  // namespace dl
