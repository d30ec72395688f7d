// Device helpers shared by the per-operation kernels (ops.cu) and the batched
// serving kernels (serve_kernels.cu): the seeded weight generator and the
// per-head QK-norm + RoPE law.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace dl {

// Philox-4x32-10 (Salmon et al., SC'11), counter c, key (k0, k1).
__device__ __forceinline__ void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint64_t p0 = uint64_t(0xD2511F53u) * c[0];
    const uint64_t p1 = uint64_t(0xCD9E8D57u) * c[2];
    const uint32_t n0 = uint32_t(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n1 = uint32_t(p1);
    const uint32_t n2 = uint32_t(p0 >> 32) ^ c[3] ^ k1;
    const uint32_t n3 = uint32_t(p0);
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Element i of a seeded tensor: Irwin-Hall sum of the Philox block's eight
// 16-bit halves, one FP32 scale multiply, BF16 rounding.  Integer-only up to
// the multiply, so a host restatement of the same algorithm reproduces the
// bits, and any slice of a tensor can be generated on its own.
__device__ __forceinline__ bf16 normal_bf16(uint64_t i, uint64_t seed, uint32_t stream_id, float scale) {
  uint32_t c[4] = {uint32_t(i), uint32_t(i >> 32), stream_id, 0u};
  philox4x32_10(c, uint32_t(seed), uint32_t(seed >> 32));
  int s = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) s += int(c[j] & 0xffffu) + int(c[j] >> 16);
  return narrow(__fmul_rn(static_cast<float>(s - 262140), scale));
}

// QK-norm + RoPE of one head (width <= 128, even) by one warp: norm law of
// normalization.cu:82-132 (warp, width <= 128), RoPE law of rotary.cu:84-126
// at absolute position p with the precomputed inverse-frequency table.
// `vals` is this warp's 128-float scratch.
__device__ __forceinline__ void qk_norm_rope_warp(const bf16* src, const bf16* w, const float* inv_freq, int p,
                                                  bf16* dst, int width, float eps, float* vals) {
  const int lane = threadIdx.x & 31;
  float x[4];
  float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int col = lane + 32 * c;
    x[c] = col < width ? widen(src[col]) : 0.f;
    if (col < width) part[c] = __fmul_rn(x[c], x[c]);
  }
  float sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  sum = shuffle_down_tree32(sum);
  const float total = __shfl_sync(0xffffffffu, sum, 0);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / static_cast<float>(width)), eps));
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int col = lane + 32 * c;
    if (col < width) vals[col] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[c], inv)), widen(w[col])));
  }
  __syncwarp();
  const int half = width / 2;
  for (int f = lane; f < half; f += 32) {
    const float angle = __fmul_rn(static_cast<float>(p), inv_freq[f]);
    const float co = round_bf16(cosf(angle));
    const float si = round_bf16(sinf(angle));
    const float a = vals[f], b = vals[f + half];
    const float ac = round_bf16(__fmul_rn(a, co)), bs = round_bf16(__fmul_rn(b, si));
    const float bc = round_bf16(__fmul_rn(b, co)), as = round_bf16(__fmul_rn(a, si));
    dst[f] = narrow(__fsub_rn(ac, bs));
    dst[f + half] = narrow(__fadd_rn(bc, as));
  }
}

// qk_norm_rope_warp with the row's rounded cosine / sine factors already in
// co[f] / si[f] (f < width / 2): every head of a row shares them, so a block
// serving all heads of one row computes them once.  Same arithmetic.
__device__ __forceinline__ void qk_norm_rope_warp_table(const bf16* src, const bf16* w, const float* co,
                                                        const float* si, bf16* dst, int width, float eps,
                                                        float* vals) {
  const int lane = threadIdx.x & 31;
  float x[4];
  float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int col = lane + 32 * c;
    x[c] = col < width ? widen(src[col]) : 0.f;
    if (col < width) part[c] = __fmul_rn(x[c], x[c]);
  }
  float sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  sum = shuffle_down_tree32(sum);
  const float total = __shfl_sync(0xffffffffu, sum, 0);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / static_cast<float>(width)), eps));
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int col = lane + 32 * c;
    if (col < width) vals[col] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[c], inv)), widen(w[col])));
  }
  __syncwarp();
  const int half = width / 2;
  for (int f = lane; f < half; f += 32) {
    const float a = vals[f], b = vals[f + half];
    const float ac = round_bf16(__fmul_rn(a, co[f])), bs = round_bf16(__fmul_rn(b, si[f]));
    const float bc = round_bf16(__fmul_rn(b, co[f])), as = round_bf16(__fmul_rn(a, si[f]));
    dst[f] = narrow(__fsub_rn(ac, bs));
    dst[f + half] = narrow(__fadd_rn(bc, as));
  }
  __syncwarp();
}

// The rounded RoPE factors of position p for f < width / 2 (threads of the
// block stride over f).
__device__ __forceinline__ void rope_factors(const float* inv_freq, int p, int width, float* co, float* si) {
  for (int f = threadIdx.x; f < width / 2; f += blockDim.x) {
    const float angle = __fmul_rn(static_cast<float>(p), inv_freq[f]);
    co[f] = round_bf16(cosf(angle));
    si[f] = round_bf16(sinf(angle));
  }
}

}  // namespace dl
