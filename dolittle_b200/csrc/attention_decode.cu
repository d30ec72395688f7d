// Decode attention (one query row per sequence step), two kernels:
//
//  1. attn_decode_scores: QK-norm + RoPE for the GQA group's query heads and
//     the new key (reference normalization.cu:82-132 warp law, rotary.cu
//     :84-126), appends the key to the K cache, then the scaled scores of the
//     group's query heads against its slice of keys (attention.cu:300-352:
//     8 lanes per key over contiguous 16-feature spans, serial FMA, tree
//     4,2,1, times the scale).  Grid (key slices, kv heads): every key's K row
//     is read once for all query heads of the group.
//  2. attn_decode_pv: per (kv head, feature slice), the reference softmax law
//     for each query head of the group (exact max, e = expf(s - max), 32
//     strided serial partials + halving tree, p = e / den) and the two
//     contiguous key halves of the PV sum, serial per feature, added once
//     (attention.cu:354-383).  The group's query heads share every V load.
// The results are bit-identical to the three-kernel path in ops.cu.
#include "attention_decode.h"

namespace dl {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) attn_decode_scores_kernel(
    const bf16* __restrict__ q_raw, const bf16* __restrict__ k_raw, const bf16* __restrict__ qw,
    const bf16* __restrict__ kw, const float* __restrict__ inv_freq, bf16* __restrict__ k_cache,
    float* __restrict__ scores, const long long* __restrict__ position, int query_heads, int kv_heads,
    int width, int capacity, float scale, float eps) {
  __shared__ float qs[8][128];
  __shared__ float ks[128];
  __shared__ float norm_vals[8][128];
  allow_next();
  wait_prior();
  const int g = blockIdx.y;
  const int group = query_heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = int(*position);
  const int count = S + 1;
  const int slices = gridDim.x;
  const int per = (count + slices - 1) / slices;
  const int j0 = blockIdx.x * per, j1 = min(count, j0 + per);
  const bool owns_new_key = S >= j0 && S < j1;
  // Warps 0..group-1: query heads of this group; warp 7: the new key.
  if (warp < group || warp == 7) {
    const bool is_q = warp < group;
    const bf16* src = is_q ? q_raw + size_t(g * group + warp) * width : k_raw + size_t(g) * width;
    const bf16* w = is_q ? qw : kw;
    float x[4], part[4] = {0.f, 0.f, 0.f, 0.f};
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
    float* nv = norm_vals[warp];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = lane + 32 * c;
      if (col < width) nv[col] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[c], inv)), widen(w[col])));
    }
    __syncwarp();
    const int half = width / 2;
    float* dst = is_q ? qs[warp] : ks;
    for (int f = lane; f < half; f += 32) {
      const float angle = __fmul_rn(static_cast<float>(S), inv_freq[f]);
      const float co = round_bf16(cosf(angle)), si = round_bf16(sinf(angle));
      const float a = nv[f], b = nv[f + half];
      const float lo = round_bf16(__fsub_rn(round_bf16(__fmul_rn(a, co)), round_bf16(__fmul_rn(b, si))));
      const float hi = round_bf16(__fadd_rn(round_bf16(__fmul_rn(b, co)), round_bf16(__fmul_rn(a, si))));
      dst[f] = lo;
      dst[f + half] = hi;
      if (!is_q && owns_new_key) {
        bf16* kc = k_cache + (size_t(S) * kv_heads + g) * width;
        kc[f] = narrow(lo);
        kc[f + half] = narrow(hi);
      }
    }
  }
  __syncthreads();
  const int lane8 = threadIdx.x & 7;
  const int span = width / 8 + (width % 8 != 0);
  const int begin = lane8 * span, end = min(begin + span, width);
  for (int base = j0; base < j1; base += kThreads / 8) {
    const int j = base + (threadIdx.x >> 3);
    const bool live = j < j1;
    float part[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) part[h] = 0.f;
    if (live && width == 128) {
      float kv[16];
      if (j == S) {
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = ks[begin + i];
      } else {
        const bf16* kr = k_cache + (size_t(j) * kv_heads + g) * width + begin;
        const uint4 w0 = *reinterpret_cast<const uint4*>(kr);
        const uint4 w1 = *reinterpret_cast<const uint4*>(kr + 8);
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = (i & 1) ? bf_hi(words[i >> 1]) : bf_lo(words[i >> 1]);
      }
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        if (h < group) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) acc = __fmaf_rn(qs[h][begin + i], kv[i], acc);
          part[h] = acc;
        }
      }
    } else if (live) {
      const bf16* kr = k_cache + (size_t(j) * kv_heads + g) * width;
      for (int h = 0; h < group; ++h) {
        float acc = 0.f;
        for (int f = begin; f < end; ++f) acc = __fmaf_rn(qs[h][f], j == S ? ks[f] : widen(kr[f]), acc);
        part[h] = acc;
      }
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      float v = part[h];
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
      v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
      part[h] = v;
    }
    if (live && lane8 == 0)
      for (int h = 0; h < group; ++h) scores[size_t(g * group + h) * capacity + j] = __fmul_rn(part[h], scale);
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// Shared memory: V slice [capacity][fpc] BF16, then p [group][capacity] FP32.
__global__ void __launch_bounds__(kThreads) attn_decode_pv_kernel(
    const float* __restrict__ scores, const bf16* __restrict__ v, bf16* __restrict__ out,
    const long long* __restrict__ position, int query_heads, int kv_heads, int width, int capacity,
    int slice_width) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ float red[kThreads];
  __shared__ float wmax[8];
  __shared__ float den_s[4];
  allow_next();
  wait_prior();
  const int g = blockIdx.x;
  const int group = query_heads / kv_heads;
  const int count = int(*position) + 1;
  const int fpc = slice_width;                       // features per CTA (multiple of 8)
  const int f0 = blockIdx.y * fpc;
  bf16* vs = reinterpret_cast<bf16*>(dyn);
  float* p = reinterpret_cast<float*>(dyn + ((size_t(capacity) * fpc * 2 + 15) / 16) * 16);
  // 1. Prefetch this CTA's V slice for all keys (16-byte async copies).
  const int chunks = fpc / 8;
  for (int c = threadIdx.x; c < count * chunks; c += kThreads) {
    const int j = c / chunks, q = c % chunks;
    cp_async16(vs + size_t(j) * fpc + 8 * q, v + (size_t(j) * kv_heads + g) * width + f0 + 8 * q);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // 2. Softmax law per query head while the copies land: warps 2h, 2h+1.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = warp >> 1, t64 = threadIdx.x & 63;
  if (h < group) {
    const float* srow = scores + size_t(g * group + h) * capacity;
    float* ph = p + size_t(h) * capacity;
    float m = -INFINITY;
    for (int j = t64; j < count; j += 64) {
      const float s = srow[j];
      ph[j] = s;
      m = fmaxf(m, s);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) wmax[warp] = m;
    named_sync(1 + h, 64);
    const float maximum = fmaxf(wmax[2 * h], wmax[2 * h + 1]);
    for (int j = t64; j < count; j += 64) ph[j] = expf(ph[j] - maximum);
    named_sync(1 + h, 64);
    if (warp == 2 * h) {
      float acc = 0.f;
      for (int j = lane; j < count; j += 32) acc = __fadd_rn(acc, ph[j]);
#pragma unroll
      for (int off = 16; off; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
      if (lane == 0) den_s[h] = acc;
    }
    named_sync(1 + h, 64);
    const float den = den_s[h];
    for (int j = t64; j < count; j += 64) ph[j] = ph[j] / den;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // 3. PV chains from shared memory: thread = (half, head, feature).
  const int t = threadIdx.x;
  const int half = t / (group * fpc);
  const int hh = (t / fpc) % group;
  const int fl = t % fpc;
  const int f = f0 + fl;
  const int split = (count - 1) / 2 + 1;
  const int jb = half == 0 ? 0 : split, je = half == 0 ? split : count;
  float acc = 0.f;
  const bool live = half < 2 && f < width;
  if (live) {
    const float* ph = p + size_t(hh) * capacity;
    const bf16* col = vs + fl;
    int j = jb;
    for (; j + 4 <= je; j += 4) {
      acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
      acc = __fmaf_rn(ph[j + 1], widen(col[size_t(j + 1) * fpc]), acc);
      acc = __fmaf_rn(ph[j + 2], widen(col[size_t(j + 2) * fpc]), acc);
      acc = __fmaf_rn(ph[j + 3], widen(col[size_t(j + 3) * fpc]), acc);
    }
    for (; j < je; ++j) acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
  }
  red[t] = acc;
  __syncthreads();
  if (live && half == 0) {
    const float second = red[t + group * fpc];
    out[size_t(g * group + hh) * width + f] = narrow(__fadd_rn(acc, second));
  }
}

}  // namespace

namespace {
int slice_width(int group, int width) { return std::min(kThreads / (2 * group), width); }
size_t pv_smem(int group, int width, int capacity) {
  const int fpc = slice_width(group, width);
  return (size_t(capacity) * fpc * 2 + 15) / 16 * 16 + size_t(group) * capacity * 4;
}
}  // namespace

bool attention_decode_supported(int query_heads, int kv_heads, int width, int capacity) {
  if (query_heads % kv_heads) return false;
  const int group = query_heads / kv_heads;
  if (group > 4 || width > 128 || width % 8) return false;
  if (slice_width(group, width) % 8 || width % slice_width(group, width)) return false;
  return pv_smem(group, width, capacity) <= 200 * 1024;
}

cudaError_t launch_attention_decode(const bf16* q_raw, const bf16* k_raw, const bf16* q_norm_w,
                                    const bf16* k_norm_w, const float* inv_freq, bf16* k_cache,
                                    const bf16* v_cache, float* scores, bf16* out, const long long* position,
                                    int query_heads, int kv_heads, int width, int capacity, float eps,
                                    int key_slices, cudaStream_t stream, bool pdl) {
  const int group = query_heads / kv_heads;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(key_slices, kv_heads);
  c.blockDim = dim3(kThreads);
  c.stream = stream;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&c, attn_decode_scores_kernel, q_raw, k_raw, q_norm_w, k_norm_w, inv_freq,
                                     k_cache, scores, position, query_heads, kv_heads, width, capacity,
                                     attention_scale(width), eps);
  if (e != cudaSuccess) return e;
  const int fpc = slice_width(group, width);
  const size_t smem = pv_smem(group, width, capacity);
  cudaFuncSetAttribute(attn_decode_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaLaunchConfig_t c2 = c;
  c2.gridDim = dim3(kv_heads, (width + fpc - 1) / fpc);
  c2.dynamicSmemBytes = smem;
  return cudaLaunchKernelEx(&c2, attn_decode_pv_kernel, static_cast<const float*>(scores), v_cache, out, position,
                            query_heads, kv_heads, width, capacity, fpc);
}

}  // namespace dl
