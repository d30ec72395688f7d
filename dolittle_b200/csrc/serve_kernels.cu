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
  allow_next();
  wait_prior();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int head = blockIdx.y * kRopeWarps + warp;
  if (head >= query_heads + 2 * kv_heads) return;
  const int p = int(*position);
  const size_t G = size_t(kv_heads) * width;
  const bf16* src = qkv + size_t(b) * ld + size_t(head) * width;  // q, k and v heads are consecutive
  bf16* seq = planes.kv + size_t(b) * planes.seq_stride;
  if (head < query_heads) {
    qk_norm_rope_warp(src, qw, inv_freq, p, q_out + (size_t(b) * query_heads + head) * width, width, eps,
                      vals[warp]);
  } else if (head < query_heads + kv_heads) {
    const int g = head - query_heads;
    qk_norm_rope_warp(src, kw, inv_freq, p, seq + planes.k_off + size_t(p) * G + size_t(g) * width, width, eps,
                      vals[warp]);
  } else {
    const int g = head - query_heads - kv_heads;
    bf16* dst = seq + planes.v_off + size_t(p) * G + size_t(g) * width;
    for (int f = lane; f < width; f += 32) dst[f] = src[f];
  }
}

// Residual epilogue of a row-parallel projection and the next RMSNorm in
// one pass: CTA m adds the split-K parts [splits][M][N] of row m in part
// order, applies residual = round(residual + round(sum)) (the split-K
// residual epilogue's law), keeps the new row as FP32 in shared memory and
// writes xn = RMSNorm(row) * w with rms_norm_rows_kernel's law (staged
// chains, width > 128).  Up to 1024 threads, PER float4 columns each, every
// part's loads issued together.
template <int PER>
__global__ void __launch_bounds__(1024) residual_norm_rows_kernel(const float* __restrict__ parts, int splits, int M,
                                                                  int N, bf16* __restrict__ residual,
                                                                  const bf16* __restrict__ w, bf16* __restrict__ xn,
                                                                  float eps) {
  extern __shared__ float xs[];  // [N]
  __shared__ float chains[129];
  // The norm weight is constant: its loads start before waiting for the parts.
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4 wq[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int q = threadIdx.x + i * blockDim.x;
    wq[i] = q < N / 8 ? wv[q] : make_uint4(0, 0, 0, 0);
  }
  allow_next();
  wait_prior();
  const int m = blockIdx.x, n4 = N / 4;
  bf16* res = residual + size_t(m) * N;
  const float4* p0 = reinterpret_cast<const float4*>(parts) + size_t(m) * n4;
  const size_t part_stride = size_t(M) * n4;
  float4 acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = threadIdx.x + i * blockDim.x;
    if (q < n4) acc[i] = __ldcg(p0 + q);
  }
#pragma unroll 4
  for (int s = 1; s < splits; ++s) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int q = threadIdx.x + i * blockDim.x;
      if (q < n4) {
        const float4 v = __ldcg(p0 + size_t(s) * part_stride + q);
        acc[i].x = __fadd_rn(acc[i].x, v.x);
        acc[i].y = __fadd_rn(acc[i].y, v.y);
        acc[i].z = __fadd_rn(acc[i].z, v.z);
        acc[i].w = __fadd_rn(acc[i].w, v.w);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = threadIdx.x + i * blockDim.x;
    if (q >= n4) continue;
    __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(res + 4 * q);
    const float2 a = __bfloat1622float2(r2[0]), b = __bfloat1622float2(r2[1]);
    const __nv_bfloat162 n0 =
        __floats2bfloat162_rn(__fadd_rn(a.x, round_bf16(acc[i].x)), __fadd_rn(a.y, round_bf16(acc[i].y)));
    const __nv_bfloat162 n1 =
        __floats2bfloat162_rn(__fadd_rn(b.x, round_bf16(acc[i].z)), __fadd_rn(b.y, round_bf16(acc[i].w)));
    r2[0] = n0;
    r2[1] = n1;
    const float2 f0 = __bfloat1622float2(n0), f1 = __bfloat1622float2(n1);
    *reinterpret_cast<float4*>(xs + 4 * q) = make_float4(f0.x, f0.y, f1.x, f1.y);
  }
  __syncthreads();
  const float inv = rms_inverse_block(xs, N, eps, chains);
  uint4* dst = reinterpret_cast<uint4*>(xn + size_t(m) * N);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int q = threadIdx.x + j * blockDim.x;
    if (q >= N / 8) continue;
    const uint4 g = wq[j];
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

// ---------------------------------------------------------------------------
// Split-K flash decoding on the tensor cores (mma.sync m16n8k16, BF16 in,
// FP32 accumulate).  CTA (kv head g, split s, sequence b) streams keys
// [j0, j1) of b's cache in tiles of 64 through a three-stage cp.async ring
// (K and V rows padded to 272 bytes so fragment reads are conflict-free; two
// CTAs fit on an SM).  The GQA group's query heads are the rows of a 16-row
// A operand (rows >= group are zero):
//   S = Q K^T: warp w computes keys 8w .. 8w+7 (8 MMAs over the 128
//   features); the running max / sum per head and p = exp(s - max) follow,
//   p goes to shared memory as BF16;
//   O += P V: warp w computes features 16w .. 16w+15 (2 n-tiles x 4 MMAs
//   over the 64 keys, V fragments by ldmatrix.trans), after rescaling its
//   accumulator rows by exp(max_old - max_new).
// Kernel fast enough to stream the cache at the HBM rate: the CUDA-core form
// spent ~4 FLOP per cache byte plus conversions and ran instruction-bound.
// ---------------------------------------------------------------------------
constexpr int kAdThreads = 256;
constexpr int kAdKeys = 64;
constexpr int kAdPitch = 136;   // BF16 per K / V smem row (128 + 8)
constexpr int kAdPPitch = 72;   // BF16 per P row (64 + 8)
constexpr int kAdMaxGroup = 8;
constexpr int kAdWs = 130;      // m, l, 128 outputs
constexpr int kAdStages = 3;
constexpr int kAdStageElems = 2 * kAdKeys * kAdPitch;  // K then V
constexpr size_t kAdSmem = size_t(kAdStages) * kAdStageElems * 2 + size_t(16) * kAdPPitch * 2 + 2 * 8 * 8 * 4;

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// Zero-filled 16 bytes (no global read): rows past the last key.
__device__ __forceinline__ void cp16_zero(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, 0;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t& b0, uint32_t& b1, const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(b0), "=r"(b1)
               : "r"(smem_addr(row_addr)));
}

__device__ __forceinline__ uint32_t lds32(const bf16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Merge of the splits of one (sequence, query head) for output feature f:
// the global max, then the rescaled sums in split order; w points at the
// head's [splits][130] workspace (L2 reads: written by other CTAs).
__device__ __forceinline__ float combine_splits(const float* w, int splits, int f) {
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, __ldcg(w + size_t(s) * kAdWs));
  float L = 0.f, o = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = __ldcg(w + size_t(s) * kAdWs);
    if (m == -INFINITY) continue;
    const float e = expf(m - M);
    L += __ldcg(w + size_t(s) * kAdWs + 1) * e;
    o += __ldcg(w + size_t(s) * kAdWs + 2 + f) * e;
  }
  return o / L;
}

// tickets (optional, [B][Hkv] zeroed): the last split CTA of each (sequence,
// KV head) to finish merges the group's splits into out itself (ticket reset
// for the next launch) instead of a separate combine launch.  Under a
// programmatic dependent launch the key tiles that end before the newest
// position (written by the previous kernel) are requested before waiting.
// qi.parts (optional): the queries, the new key and the new value come from
// the qkv projection's split-K parts instead (see AttnQkvIn).
__global__ void __launch_bounds__(kAdThreads) attention_decode_split_kernel(
    const bf16* __restrict__ q, KvPlanes planes, const long long* __restrict__ position, int query_heads,
    int kv_heads, int splits, int lead_q10, float scale, float* __restrict__ ws, int* __restrict__ tickets,
    bf16* __restrict__ out, AttnQkvIn qi) {
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* stage = reinterpret_cast<bf16*>(smem);
  bf16* ps = reinterpret_cast<bf16*>(smem + size_t(kAdStages) * kAdStageElems * 2);  // [16][72]
  float* wred = reinterpret_cast<float*>(ps + 16 * kAdPPitch);                          // [2][8 warps][8 heads]
  // KV head fastest: the heads of one (sequence, split) run side by side and
  // together read whole cache rows (Hkv x 256 bytes per position).  Even
  // ranges: grid (KV head, split, sequence).  A leading range (lead_q10 > 0,
  // two splits): grid (KV head, sequence, split), so every sequence's long
  // first range is launched before any short second one.
  const bool lead = lead_q10 > 0;
  const int g = blockIdx.x, s = lead ? blockIdx.z : blockIdx.y, b = lead ? blockIdx.y : blockIdx.z, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31, r = lane >> 2, c2 = (lane & 3) * 2;
  const int group = query_heads / kv_heads;
  const int count = int(*position) + 1;
  int j0, j1;
  if (lead) {
    // The first range holds lead_q10 / 1024 of the keys, rounded up to whole
    // tiles; the second range the rest (empty when that covers them all).
    const long long c = (static_cast<long long>(count) * lead_q10 + 1023) >> 10;
    const long long up = (c + kAdKeys - 1) / kAdKeys * kAdKeys;
    const int cut = up < count ? int(up) : count;
    j0 = s == 0 ? 0 : cut;
    j1 = s == 0 ? cut : count;
  } else {
    const int per = ((count + splits - 1) / splits + kAdKeys - 1) / kAdKeys * kAdKeys;
    j0 = min(count, s * per);
    j1 = min(count, j0 + per);
  }
  const size_t G = size_t(kv_heads) * 128;
  const bf16* kbase = planes.kv + size_t(b) * planes.seq_stride + planes.k_off + size_t(g) * 128;
  const bf16* vbase = planes.kv + size_t(b) * planes.seq_stride + planes.v_off + size_t(g) * 128;
  // P rows >= group stay zero.
  for (int i = t; i < 16 * kAdPPitch / 2; i += kAdThreads) reinterpret_cast<uint32_t*>(ps)[i] = 0u;
  const bool qrow = r < group;
  auto load_tile = [&](int tile, int slot) {
    const int base = j0 + tile * kAdKeys;
    const int n = min(kAdKeys, j1 - base);
    bf16* ks = stage + slot * kAdStageElems;
    bf16* vs = ks + kAdKeys * kAdPitch;
    for (int i = t; i < kAdKeys * 16; i += kAdThreads) {
      const int kk = i >> 4, c = i & 15;
      if (kk < n) {
        cp16(ks + kk * kAdPitch + 8 * c, kbase + size_t(base + kk) * G + 8 * c);
        cp16(vs + kk * kAdPitch + 8 * c, vbase + size_t(base + kk) * G + 8 * c);
      } else {
        cp16_zero(ks + kk * kAdPitch + 8 * c, kbase);
        cp16_zero(vs + kk * kAdPitch + 8 * c, vbase);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int tiles = (j1 - j0 + kAdKeys - 1) / kAdKeys;
  float o[2][4] = {};                // this warp's 2 n-tiles (rows r and r + 8)
  float m_run = -INFINITY, l_run = 0.f;  // head r (identical in every warp)
  // Tiles t+1 and t+2 load while tile t is processed (one commit group per
  // tile; an empty group keeps the count when fewer tiles remain).  Tiles
  // wholly before key count - 1 (appended by the previous kernel) go first.
  int pre = 0;
  for (; pre < kAdStages - 1 && pre < tiles; ++pre) {
    if (j0 + pre * kAdKeys + min(kAdKeys, j1 - (j0 + pre * kAdKeys)) > count - 1) break;
    load_tile(pre, pre);
  }
  allow_next();
  wait_prior();
  // The third ring slot is not loaded before the main loop: scratch for the
  // queries built from the qkv parts ([8][128] BF16 rotated queries, [8][128]
  // BF16 staged sums, [8][128] FP32 norm values).
  bf16* qsm = stage + 2 * kAdStageElems;
  if (qi.parts) {
    bf16* staged = qsm + 8 * 128;
    float* vals = reinterpret_cast<float*>(staged + 8 * 128);
    const int p = count - 1;
    const bool owns = j0 <= p && p < j1;  // this split holds the newest key
    const int Qw = query_heads * 128;
    // Jobs: query heads 0 .. group-1 of the group, then its key and value
    // (only for the split holding them); warp w takes jobs w and w + 8.
    for (int job = warp; job < group + 2; job += kAdThreads / 32) {
      if (job >= group && !owns) continue;
      const int col = job < group ? (g * group + job) * 128 : Qw + (job - group) * int(G) + g * 128;
      const float* src = qi.parts + size_t(b) * qi.ld + col + 4 * lane;
      float4 acc = *reinterpret_cast<const float4*>(src);
      for (int sp = 1; sp < qi.splits; ++sp) {
        const float4 v = *reinterpret_cast<const float4*>(src + size_t(sp) * qi.M * qi.ld);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
      }
      bf16* st = staged + (job & 7) * 128;
      __nv_bfloat162* d2 = reinterpret_cast<__nv_bfloat162*>(st + 4 * lane);
      d2[0] = __floats2bfloat162_rn(acc.x, acc.y);
      d2[1] = __floats2bfloat162_rn(acc.z, acc.w);
      __syncwarp();
      bf16* seq = planes.kv + size_t(b) * planes.seq_stride;
      if (job < group) {
        qk_norm_rope_warp(st, qi.q_norm, qi.inv_freq, p, qsm + job * 128, 128, qi.eps, vals + (job & 7) * 128);
      } else if (job == group) {
        qk_norm_rope_warp(st, qi.k_norm, qi.inv_freq, p, seq + planes.k_off + size_t(p) * G + size_t(g) * 128, 128,
                          qi.eps, vals + (job & 7) * 128);
      } else {
        bf16* dst = seq + planes.v_off + size_t(p) * G + size_t(g) * 128;
        reinterpret_cast<uint2*>(dst)[lane] = reinterpret_cast<const uint2*>(st)[lane];
      }
      __syncwarp();
    }
    __threadfence();  // the new K / V row is read back through the cache loads below
    __syncthreads();
  }
  for (; pre < kAdStages - 1; ++pre) {
    if (pre < tiles) load_tile(pre, pre);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // Q fragments of the 8 k-steps (rows r < group; rows 8..15 are zero).
  uint32_t qa[8][2];
  const bf16* qh = qi.parts ? qsm + (qrow ? r : 0) * 128
                            : q + (size_t(b) * query_heads + g * group + (qrow ? r : 0)) * 128;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    qa[kk][0] = qrow ? *reinterpret_cast<const uint32_t*>(qh + 16 * kk + c2) : 0u;
    qa[kk][1] = qrow ? *reinterpret_cast<const uint32_t*>(qh + 16 * kk + 8 + c2) : 0u;
  }
  if (qi.parts) __syncthreads();  // every fragment read before slot 2 is loaded
  for (int tile = 0; tile < tiles; ++tile) {
    const int slot = tile % kAdStages;
    asm volatile("cp.async.wait_group %0;" ::"n"(kAdStages - 2) : "memory");
    __syncthreads();  // tile landed; every thread is done with tile - 1, whose slot refills now
    if (tile + kAdStages - 1 < tiles) load_tile(tile + kAdStages - 1, (tile + kAdStages - 1) % kAdStages);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    const bf16* ks = stage + slot * kAdStageElems;
    const bf16* vs = ks + kAdKeys * kAdPitch;
    const int n = min(kAdKeys, j1 - (j0 + tile * kAdKeys));
    // S for keys 8 warp .. 8 warp + 7.
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    const bf16* krow = ks + (8 * warp + r) * kAdPitch + c2;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t a[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
      mma16816(sc, a, lds32(krow + 16 * kk), lds32(krow + 16 * kk + 8));
    }
    const int key = 8 * warp + c2;
    const float s0 = key < n ? sc[0] * scale : -INFINITY;
    const float s1 = key + 1 < n ? sc[1] * scale : -INFINITY;
    float wm = fmaxf(s0, s1);
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 1));
    wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, 2));
    if ((lane & 3) == 0) wred[warp * 8 + r] = wm;
    __syncthreads();
    float tmax = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) tmax = fmaxf(tmax, wred[w * 8 + r]);
    const float m_new = fmaxf(m_run, tmax);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    const float p0 = s0 == -INFINITY ? 0.f : expf(s0 - m_new);
    const float p1 = s1 == -INFINITY ? 0.f : expf(s1 - m_new);
    const __nv_bfloat162 p2 = __floats2bfloat162_rn(p0, p1);
    if (qrow) *reinterpret_cast<__nv_bfloat162*>(ps + r * kAdPPitch + key) = p2;
    float psum = __low2float(p2) + __high2float(p2);  // the BF16 weights the MMA multiplies
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    if ((lane & 3) == 0) wred[64 + warp * 8 + r] = psum;
    __syncthreads();  // P and the partial sums complete
    float tsum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tsum += wred[64 + w * 8 + r];
    l_run = l_run * alpha + tsum;
    m_run = m_new;
    // O = O * alpha + P V for features 16 warp .. 16 warp + 15.
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
    }
    const bf16* prow = ps + r * kAdPPitch + c2;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {lds32(prow + 16 * kk), 0u, lds32(prow + 16 * kk + 8), 0u};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t b0, b1;
        // Lanes 0..15 address keys 16 kk + lane (rows of the two 8x8 matrices).
        ldsm_x2_trans(b0, b1, vs + (16 * kk + (lane & 15)) * kAdPitch + 16 * warp + 8 * j);
        mma16816(o[j], a, b0, b1);
      }
    }
  }
  if (splits == 1 && tickets) {
    // One split: merging is the identity (weight expf(0) = 1), so the output
    // is O / l directly, with no workspace round trip.
    if (qrow) {
      bf16* orow = out + (size_t(b) * query_heads + g * group + r) * 128 + 16 * warp + c2;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        *reinterpret_cast<__nv_bfloat162*>(orow + 8 * j) = __floats2bfloat162_rn(o[j][0] / l_run, o[j][1] / l_run);
    }
    return;
  }
  if (qrow) {
    float* w = ws + ((size_t(b) * query_heads + g * group + r) * splits + s) * kAdWs;
    if (warp == 0 && (lane & 3) == 0) {
      w[0] = m_run;
      w[1] = l_run;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      w[2 + 16 * warp + 8 * j + c2] = o[j][0];
      w[3 + 16 * warp + 8 * j + c2] = o[j][1];
    }
  }
  if (!tickets) return;
  // Publish this split (every writer fences), then count it.
  __shared__ int last_s;
  __threadfence();
  __syncthreads();
  if (t == 0) last_s = atomicAdd(tickets + size_t(b) * kv_heads + g, 1) == splits - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  for (int i = t; i < group * 128; i += kAdThreads) {
    const int h = g * group + i / 128, f = i % 128;
    out[(size_t(b) * query_heads + h) * 128 + f] =
        narrow(combine_splits(ws + (size_t(b) * query_heads + h) * splits * kAdWs, splits, f));
  }
  if (t == 0) tickets[size_t(b) * kv_heads + g] = 0;
}

__global__ void attention_decode_combine_kernel(const float* __restrict__ ws, int query_heads, int splits,
                                                bf16* __restrict__ out) {
  allow_next();  // the o projection may request its weights meanwhile
  const int h = blockIdx.x, b = blockIdx.y, f = threadIdx.x;
  out[(size_t(b) * query_heads + h) * 128 + f] =
      narrow(combine_splits(ws + (size_t(b) * query_heads + h) * splits * kAdWs, splits, f));
}

__global__ void add_fp32_residual_kernel(const float* __restrict__ sum, bf16* __restrict__ residual, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    residual[i] = narrow(__fadd_rn(widen(residual[i]), round_bf16(sum[i])));
}

unsigned grid_for(size_t n) { return unsigned(std::min<size_t>((n + 255) / 256, 148 * 32)); }

__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr long long kPeerSpin = 1ll << 31;  // ~1 s of SM cycles

// CTA `row` owns row `row` of the [M][N] output (M <= kPeerChunks): it sums
// this rank's split-K parts of the row in part order, writes the FP32 row
// into slot `rank` of every rank's buffer, raises flag (rank, row) on each,
// waits (bounded) for every rank's flag on its own buffer, adds the slots in
// rank order and applies the residual epilogue; with NORM it then writes
// xn = RMSNorm(row) * w by the RMSNorm rows law (the row is in shared memory).
template <bool NORM>
__global__ void __launch_bounds__(1024) peer_allreduce_rows_kernel(PeerBuffers pb, const float* __restrict__ parts,
                                                                   int splits, int M, int N,
                                                                   bf16* __restrict__ residual,
                                                                   const bf16* __restrict__ w, bf16* __restrict__ xn,
                                                                   float eps) {
  extern __shared__ float xs[];  // [N] (NORM)
  __shared__ float chains[129];
  __shared__ unsigned epoch_s;
  __shared__ int ok_s;
  allow_next();
  wait_prior();
  const int row = blockIdx.x, R = pb.ranks, n4 = N / 4;
  // CTA `row` counts its own calls: every rank runs the same calls, so the
  // epochs of row `row` agree across ranks without any ordering between CTAs.
  if (threadIdx.x == 0) epoch_s = pb.epoch[row] + 1;
  __syncthreads();
  const unsigned epoch = epoch_s, par = epoch & 1u;
  const size_t off4 = size_t(row) * n4, all4 = size_t(M) * n4;
  // 1. This rank's row (split-K parts in part order) into slot `rank` of
  // every rank's buffer.
  const float4* src = reinterpret_cast<const float4*>(parts);
  for (int j = threadIdx.x; j < n4; j += blockDim.x) {
    float4 acc = src[off4 + j];
    for (int s = 1; s < splits; ++s) {
      const float4 v = src[size_t(s) * all4 + off4 + j];
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    for (int p = 0; p < R; ++p)
      reinterpret_cast<float4*>(pb.data[p] + (size_t(par) * R + pb.rank) * pb.capacity)[off4 + j] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < R; ++p) st_release_sys(pb.flags[p] + (size_t(par) * R + pb.rank) * kPeerChunks + row, epoch);
  }
  // 2. Every rank's row has arrived here (bounded wait).
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned* mine = pb.flags[pb.rank] + size_t(par) * R * kPeerChunks;
    for (int r = 0; r < R && ok; ++r) {
      const long long start = clock64();
      while (ld_relaxed_sys(mine + r * kPeerChunks + row) != epoch) {
        if (clock64() - start > kPeerSpin) {
          ok = 0;
          atomicOr(pb.err, kErrWaitFull);
          break;
        }
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // the acquire of the flags seen
    ok_s = ok;
  }
  __syncthreads();
  // 3. Sum in rank order, residual add (the residual epilogue law).
  const bool ok = ok_s != 0;
  if (ok) {
    const float* slots = pb.data[pb.rank] + size_t(par) * R * pb.capacity;
    for (int j = threadIdx.x; j < n4; j += blockDim.x) {
      float4 sum = __ldcv(reinterpret_cast<const float4*>(slots) + off4 + j);
      for (int r = 1; r < R; ++r) {
        const float4 v = __ldcv(reinterpret_cast<const float4*>(slots + size_t(r) * pb.capacity) + off4 + j);
        sum.x = __fadd_rn(sum.x, v.x);
        sum.y = __fadd_rn(sum.y, v.y);
        sum.z = __fadd_rn(sum.z, v.z);
        sum.w = __fadd_rn(sum.w, v.w);
      }
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(residual) + 2 * (off4 + j);
      const float2 a = __bfloat1622float2(r2[0]), b = __bfloat1622float2(r2[1]);
      const __nv_bfloat162 n0 =
          __floats2bfloat162_rn(__fadd_rn(a.x, round_bf16(sum.x)), __fadd_rn(a.y, round_bf16(sum.y)));
      const __nv_bfloat162 n1 =
          __floats2bfloat162_rn(__fadd_rn(b.x, round_bf16(sum.z)), __fadd_rn(b.y, round_bf16(sum.w)));
      r2[0] = n0;
      r2[1] = n1;
      if constexpr (NORM) {
        const float2 f0 = __bfloat1622float2(n0), f1 = __bfloat1622float2(n1);
        *reinterpret_cast<float4*>(xs + 4 * j) = make_float4(f0.x, f0.y, f1.x, f1.y);
      }
    }
  }
  if (threadIdx.x == 0) pb.epoch[row] = epoch;
  if constexpr (NORM) {
    if (!ok) return;  // CTA-uniform
    __syncthreads();
    const float inv = rms_inverse_block(xs, N, eps, chains);
    const uint4* wv = reinterpret_cast<const uint4*>(w);
    uint4* dst = reinterpret_cast<uint4*>(xn + size_t(row) * N);
    for (int q = threadIdx.x; q < N / 8; q += blockDim.x) {
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
}

}  // namespace

cudaError_t launch_fill_normal_slice(bf16* out, size_t rows, size_t cols, size_t out_stride, size_t full_cols,
                                     size_t r0, size_t c0, uint64_t seed, uint32_t stream_id, float scale,
                                     cudaStream_t stream) {
  if (!rows || !cols) return cudaSuccess;
  fill_normal_slice_kernel<<<grid_for(rows * cols), 256, 0, stream>>>(out, rows, cols, out_stride, full_cols, r0,
                                                                       c0, seed, stream_id, scale);
  return cudaGetLastError();
}

namespace {
cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, cudaLaunchAttribute* attr,
                              bool pdl) {
  cudaLaunchConfig_t c = {};
  c.gridDim = grid;
  c.blockDim = block;
  c.dynamicSmemBytes = smem;
  c.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}
}  // namespace

cudaError_t launch_norm_rope_append_rows(const bf16* qkv, int ld, const bf16* q_norm_w, const bf16* k_norm_w,
                                         const float* inv_freq, bf16* q_out, KvPlanes planes,
                                         const long long* position, int batch, int query_heads, int kv_heads,
                                         int width, float eps, cudaStream_t stream, bool pdl) {
  if (width > 128 || width % 2 || batch < 1 || !qkv) return cudaErrorInvalidValue;
  const int heads = query_heads + 2 * kv_heads;
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_config(dim3(batch, (heads + kRopeWarps - 1) / kRopeWarps), dim3(32 * kRopeWarps), 0, stream, attr,
                        pdl);
  return cudaLaunchKernelEx(&cfg, norm_rope_append_rows_kernel, qkv, ld, q_norm_w, k_norm_w, inv_freq, q_out, planes,
                            position, query_heads, kv_heads, width, eps);
}

cudaError_t launch_residual_norm_rows(const float* parts, int splits, int M, int N, bf16* residual, const bf16* w,
                                      bf16* xn, float eps, cudaStream_t stream, bool pdl) {
  if (N <= 128 || N % 8 || N > 8192 || splits < 1 || M < 1 ||
      (reinterpret_cast<uintptr_t>(parts) | reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(xn)) % 16)
    return cudaErrorInvalidValue;
  const int n4 = N / 4;
  const int threads = std::max(128, std::min(1024, (n4 + 31) / 32 * 32));
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_config(dim3(M), dim3(threads), size_t(N) * 4, stream, attr, pdl);
  if (n4 <= threads)
    return cudaLaunchKernelEx(&cfg, residual_norm_rows_kernel<1>, parts, splits, M, N, residual, w, xn, eps);
  return cudaLaunchKernelEx(&cfg, residual_norm_rows_kernel<2>, parts, splits, M, N, residual, w, xn, eps);
}

size_t attention_decode_ws_floats(int batch, int query_heads, int splits) {
  return size_t(batch) * query_heads * splits * kAdWs;
}

// Estimated time of `s` even splits per (sequence, KV head), in 64-key tiles:
// waves of two resident CTAs per SM x (tiles per split + ~3 tiles of fixed
// cost per CTA: query load, pipeline fill, partial write).
static long long even_split_cost(long long units, long long slots, int tiles, int s) {
  const long long waves = (units * s + slots - 1) / slots;
  return waves * ((tiles + s - 1) / s + 3);
}

int attention_decode_splits(int batch, int kv_heads, int capacity, int sms) {
  // Measured on the batch-32 step: one split per (sequence, KV head) at 1K
  // and 2K context (5.36 -> 5.08 and 6.18 -> 5.92 ms per step against 2 and
  // 4 splits), about even from 1 to 4 splits at 8K.
  const long long units = std::max(1, batch * kv_heads), slots = 2ll * std::max(1, sms);
  const int tiles = std::max(1, (capacity + kAdKeys - 1) / kAdKeys);
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= std::min(64, tiles); ++s) {
    const long long cost = even_split_cost(units, slots, tiles, s);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

AttnPlan attention_decode_plan(int batch, int kv_heads, int capacity, int sms) {
  AttnPlan plan{attention_decode_splits(batch, kv_heads, capacity, sms), 0};
  const long long units = std::max(1, batch * kv_heads), slots = 2ll * std::max(1, sms);
  const int tiles = std::max(1, (capacity + kAdKeys - 1) / kAdKeys);
  if (units >= slots || tiles < 2) return plan;
  // Fewer (sequence, KV head) units than slots: a long first range per unit
  // keeps `units` slots busy for the whole launch while the spare slots run
  // the short second ranges one after another (ceil(units / spare) each);
  // +2 tiles for merging the two ranges.
  long long best = even_split_cost(units, slots, tiles, plan.splits);
  const long long spare = slots - units, chain = (units + spare - 1) / spare;
  for (int first = 1; first < tiles; ++first) {
    const long long cost = std::max<long long>(first + 3, chain * (tiles - first + 3)) + 2;
    if (cost < best) {
      best = cost;
      plan.splits = 2;
      plan.lead_q10 = int(std::min<long long>(1023, std::max<long long>(1, (first * 1024ll + tiles / 2) / tiles)));
    }
  }
  return plan;
}

cudaError_t launch_attention_decode_batched(const bf16* q, KvPlanes planes, const long long* position, int batch,
                                            int query_heads, int kv_heads, int splits, int lead_q10, float scale,
                                            float* ws, bf16* out, cudaStream_t stream, int* tickets, bool pdl,
                                            const AttnQkvIn* qkv) {
  if (query_heads % kv_heads || query_heads / kv_heads > kAdMaxGroup || splits < 1 || splits > 64 || batch < 1 ||
      lead_q10 < 0 || lead_q10 > 1023 || (lead_q10 > 0 && splits != 2) || batch > 65535)
    return cudaErrorInvalidValue;
  AttnQkvIn qi = {};
  if (qkv) {
    qi = *qkv;
    if (!qi.parts || qi.splits < 1 || qi.M < batch || qi.ld % 4 || qi.ld != (query_heads + 2 * kv_heads) * 128 ||
        reinterpret_cast<uintptr_t>(qi.parts) % 16)
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaFuncSetAttribute(attention_decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(kAdSmem));
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  const dim3 grid = lead_q10 > 0 ? dim3(kv_heads, batch, 2) : dim3(kv_heads, splits, batch);
  auto cfg = pdl_config(grid, dim3(kAdThreads), kAdSmem, stream, attr, pdl);
  e = cudaLaunchKernelEx(&cfg, attention_decode_split_kernel, q, planes, position, query_heads, kv_heads, splits,
                         lead_q10, scale, ws, tickets, out, qi);
  if (e != cudaSuccess || tickets) return e;
  attention_decode_combine_kernel<<<dim3(query_heads, batch), 128, 0, stream>>>(ws, query_heads, splits, out);
  return cudaGetLastError();
}

size_t peer_buffer_bytes(int ranks, size_t capacity) {
  return size_t(2) * ranks * capacity * 4 + size_t(2) * ranks * kPeerChunks * 4;
}

cudaError_t launch_peer_allreduce_residual(const PeerBuffers& pb, const float* parts, int splits, int M, int N,
                                           bf16* residual, const bf16* norm_w, bf16* xn, float eps,
                                           cudaStream_t stream, bool pdl) {
  if (M < 1 || M > kPeerChunks || N % 8 || size_t(M) * N > pb.capacity || splits < 1 || pb.ranks < 1 ||
      pb.ranks > kPeerMaxRanks || (norm_w && (N <= 128 || N > 8192 || !xn)))
    return cudaErrorInvalidValue;
  const int threads = std::max(128, std::min(1024, (N / 4 + 31) / 32 * 32));
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_config(dim3(M), dim3(threads), norm_w ? size_t(N) * 4 : 0, stream, attr, pdl);
  if (norm_w)
    return cudaLaunchKernelEx(&cfg, peer_allreduce_rows_kernel<true>, pb, parts, splits, M, N, residual, norm_w, xn,
                              eps);
  return cudaLaunchKernelEx(&cfg, peer_allreduce_rows_kernel<false>, pb, parts, splits, M, N, residual, norm_w, xn,
                            eps);
}

__global__ void gather_vocab_slices_kernel(const bf16* src, bf16* dst, int ranks, int batch, int vl, int vp) {
  // 16-byte moves: vl and vp are multiples of 8 (checked by the launcher).
  const int per_row = vl / 8;
  const size_t n = size_t(ranks) * batch * per_row;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const int c = int(i % per_row);
    const size_t rb = i / per_row;
    const int b = int(rb % batch), r = int(rb / batch);
    const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t(r) * batch + b) * vp + 8 * c);
    *reinterpret_cast<uint4*>(dst + size_t(b) * ranks * vl + size_t(r) * vl + 8 * c) = v;
  }
}

cudaError_t launch_gather_vocab_slices(const bf16* src, bf16* dst, int ranks, int batch, int vl, int vp,
                                       cudaStream_t stream) {
  if (vl % 8 || vp % 8 || vl > vp) return cudaErrorInvalidValue;
  const size_t n = size_t(ranks) * batch * (vl / 8);
  gather_vocab_slices_kernel<<<int(std::min<size_t>((n + 255) / 256, 1184)), 256, 0, stream>>>(src, dst, ranks, batch,
                                                                                               vl, vp);
  return cudaGetLastError();
}

cudaError_t launch_add_fp32_residual(const float* sum, bf16* residual, size_t n, cudaStream_t stream) {
  add_fp32_residual_kernel<<<grid_for(n), 256, 0, stream>>>(sum, residual, n);
  return cudaGetLastError();
}

}  // namespace dl
