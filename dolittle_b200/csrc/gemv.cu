// Streaming GEMV kernel (see gemv.cuh for the law and the B200 mapping).
#include <algorithm>
#include <cmath>

#include "gemv.cuh"
#include "launch.h"

namespace dl {
namespace {

// Lane layout inside a warp: a quarter-warp (8 lanes) holds 8 different rows
// with the same slot, so padded shared rows give conflict-free LDS.128.
template <int P>
struct Layout {
  static constexpr int kSlots = P / 8;                 // threads per row
  static constexpr int kRowsPerWarp = 32 / kSlots;     // 16 or 8
  static constexpr int kMaxRows = kGemvConsumers / kSlots;
  __device__ static int slot(int lane) { return P == 16 ? (lane >> 3) & 1 : lane >> 3; }
  __device__ static int row(int warp, int lane) {
    return warp * kRowsPerWarp + (P == 16 ? (lane & 7) + 8 * (lane >> 4) : (lane & 7));
  }
};

// Halving tree over the P partials held 8 per thread (slot-major).
template <int P>
__device__ __forceinline__ float reduce_partials(float (&acc)[8]) {
  if constexpr (P == 32) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, acc[i], 16);
      acc[i] = __fadd_rn(acc[i], other);   // p[j] + p[j+16] (slots 0,1)
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float other = __shfl_xor_sync(0xffffffffu, acc[i], 8);
    acc[i] = __fadd_rn(acc[i], other);     // p[j] + p[j+8] (slot 0)
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], acc[i + 4]);
#pragma unroll
  for (int i = 0; i < 2; ++i) acc[i] = __fadd_rn(acc[i], acc[i + 2]);
  return __fadd_rn(acc[0], acc[1]);
}

// RMSNorm inverse of one global BF16 row by one warp (reference law).
__device__ float rms_inverse_global(const bf16* x, int width, float eps) {
  const unsigned lane = threadIdx.x & 31u;
  float sum;
  if (width <= 128) {
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (unsigned c = 0; c < 4; ++c) {
      const unsigned col = lane + 32u * c;
      if (col < static_cast<unsigned>(width)) {
        const float v = widen(x[col]);
        part[c] = __fmul_rn(v, v);
      }
    }
    sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  } else {
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    for (int base = 4 * lane; base < width; base += 128) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (base + c < width) {
          const float v = widen(x[base + c]);
          part[c] = __fadd_rn(part[c], __fmul_rn(v, v));
        }
      }
    }
    sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  }
  sum = shuffle_down_tree32(sum);
  const float total = __shfl_sync(0xffffffffu, sum, 0);
  const float mean = __fmul_rn(total, 1.0f / static_cast<float>(width));
  return rsqrtf(__fadd_rn(mean, eps));
}

// SwiGLU law (reference elementwise.cu:62-87 with Silu): gate and up are
// BF16 values; the activation is rounded to storage before the product.
__device__ __forceinline__ float swiglu(float a, float b) {
  const float e = expf(a >= 0.0f ? -a : a);
  const float s = a >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return round_bf16(__fmul_rn(round_bf16(__fmul_rn(a, s)), b));
}

__device__ __forceinline__ bool better(float v, unsigned id, float bv, unsigned bid) {
  return v > bv || (v == bv && id < bid);
}

template <int ROWS>
struct XStore {
  // ROWS == 1: FP32 row; ROWS > 1: BF16 rows.
  static constexpr bool kF32 = ROWS == 1;
  __device__ static size_t bytes(int width) {
    return kF32 ? size_t(width) * 4 : size_t(width) * 2 * ROWS;
  }
};

template <int ROWS, int P>
__device__ void consume(const GemvArgs& a, const GemvSegment& sg, int r0, int r1, int ntiles,
                        int tile_rows, unsigned char* ring, int stage_bytes, int row_stride,
                        uint64_t* full, uint64_t* empty, const void* xs, uint4* cta_best,
                        bool& failed) {
  using L = Layout<P>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = L::slot(lane);
  const int my_row = L::row(warp, lane);
  const int I = a.in_width;
  const int kc = a.kc;
  const int nk = (I + kc - 1) / kc;
  const int padded = (I + 15) / 16 * 16;
  float best_v = -INFINITY;
  unsigned best_id = 0xffffffffu, flags = 0;
  int g = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int tr0 = r0 + t * tile_rows;
    const int trows = min(tile_rows, r1 - tr0);
    const bool active = my_row < trows;
    float acc[ROWS][8];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[r][i] = 0.0f;
    for (int ks = 0; ks < nk; ++ks, ++g) {
      const int st = g % a.stages;
      if (!failed && !mbar_wait(&full[st], (g / a.stages) & 1)) {
        failed = true;
        record_error(a.err, kErrWaitFull);
      }
      if (active && !failed) {
        const int k0 = ks * kc;
        const int nfeat = min(kc, I - k0);
        const unsigned char* wrow = ring + st * stage_bytes + my_row * row_stride;
#pragma unroll 4
        for (int m = 0; m < kc / P; ++m) {
          const int f = P * m + 8 * slot;          // feature offset inside stage
          if (f < nfeat) {
            const uint4 w = lds128(wrow + 2 * f);
            const float w0 = bf_lo(w.x), w1 = bf_hi(w.x), w2 = bf_lo(w.y), w3 = bf_hi(w.y);
            const float w4 = bf_lo(w.z), w5 = bf_hi(w.z), w6 = bf_lo(w.w), w7 = bf_hi(w.w);
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              float x0, x1, x2, x3, x4, x5, x6, x7;
              if constexpr (ROWS == 1) {
                const float* xf = static_cast<const float*>(xs) + k0 + f;
                const float4 xa = lds128f(xf), xb = lds128f(xf + 4);
                x0 = xa.x; x1 = xa.y; x2 = xa.z; x3 = xa.w;
                x4 = xb.x; x5 = xb.y; x6 = xb.z; x7 = xb.w;
              } else {
                const uint4 xv = lds128(static_cast<const bf16*>(xs) + size_t(r) * I + k0 + f);
                x0 = bf_lo(xv.x); x1 = bf_hi(xv.x); x2 = bf_lo(xv.y); x3 = bf_hi(xv.y);
                x4 = bf_lo(xv.z); x5 = bf_hi(xv.z); x6 = bf_lo(xv.w); x7 = bf_hi(xv.w);
              }
              acc[r][0] = __fmaf_rn(x0, w0, acc[r][0]);
              acc[r][1] = __fmaf_rn(x1, w1, acc[r][1]);
              acc[r][2] = __fmaf_rn(x2, w2, acc[r][2]);
              acc[r][3] = __fmaf_rn(x3, w3, acc[r][3]);
              acc[r][4] = __fmaf_rn(x4, w4, acc[r][4]);
              acc[r][5] = __fmaf_rn(x5, w5, acc[r][5]);
              acc[r][6] = __fmaf_rn(x6, w6, acc[r][6]);
              acc[r][7] = __fmaf_rn(x7, w7, acc[r][7]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // Zero padding to a multiple of 16 features (ragged I only).
    if (padded != I) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = 8 * slot + i;  // partial index
        bool hit = false;
        for (int f = I; f < padded; ++f) hit |= (f % P) == j;
        if (hit)
#pragma unroll
          for (int r = 0; r < ROWS; ++r) acc[r][i] = __fmaf_rn(0.0f, 0.0f, acc[r][i]);
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float y = reduce_partials<P>(acc[r]);
      if (!active || slot != 0 || failed || r >= a.nrows) continue;
      const int o = tr0 + my_row;
      const bf16 yb = narrow(y);
      bf16* out = sg.out + (sg.out_row ? size_t(*sg.out_row) * sg.out_stride : 0);
      const size_t idx = size_t(r) * sg.out_stride + o;
      if (a.epilogue == kEpilogueResidual) {
        const bf16 nv = narrow(__fadd_rn(widen(out[idx]), widen(yb)));
        out[idx] = nv;
        if (a.capture)
          a.capture[(size_t(*a.capture_row) + r) * a.capture_stride + o] = nv;
      } else {
        out[idx] = yb;
        if (a.epilogue == kEpilogueArgmax) {
          const float v = widen(yb);
          if (isnan(v) || v == INFINITY) flags |= 1u;
          if (better(v, static_cast<unsigned>(o), best_v, best_id)) {
            best_v = v;
            best_id = static_cast<unsigned>(o);
          }
        }
      }
    }
  }
  if (a.epilogue == kEpilogueArgmax) {
    // Warp then CTA reduction of (value, lowest id); flags OR.
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, off);
      const unsigned oid = __shfl_xor_sync(0xffffffffu, best_id, off);
      flags |= __shfl_xor_sync(0xffffffffu, flags, off);
      if (better(ov, oid, best_v, best_id)) {
        best_v = ov;
        best_id = oid;
      }
    }
    if (lane == 0) cta_best[warp] = make_uint4(__float_as_uint(best_v), best_id, flags, 0);
  }
}

template <int ROWS>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint4 cta_best[kGemvConsumers / 32];
  __shared__ bool last_cta;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + a.stages;
  unsigned char* xs = smem + 256;
  const size_t xbytes = (XStore<ROWS>::bytes(a.in_width) + 127) / 128 * 128;
  unsigned char* ring = xs + xbytes;

  // Segment and row range of this CTA.
  int si = 0;
  for (int i = 1; i < a.nseg; ++i)
    if (static_cast<int>(blockIdx.x) >= a.seg[i].cta_begin) si = i;
  const GemvSegment& sg = a.seg[si];
  const int P = sg.partials;
  const int local = blockIdx.x - sg.cta_begin;
  const int per = (sg.rows + sg.cta_count - 1) / sg.cta_count;
  const int r0 = min(sg.rows, local * per), r1 = min(sg.rows, r0 + per);
  const int max_rows = kGemvConsumers / (P / 8);
  const int ntiles = r1 > r0 ? (r1 - r0 + max_rows - 1) / max_rows : 0;
  const int tile_rows = ntiles ? (r1 - r0 + ntiles - 1) / ntiles : 0;
  const int I = a.in_width;
  const int kc = a.kc;
  const int nk = (I + kc - 1) / kc;
  const int row_stride = 2 * kc + 16;
  const int stage_bytes = a.max_tile_rows * row_stride;
  const int total = ntiles * nk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumers / 32);
    }
    fence_barrier_init();
  }
  __syncthreads();
  allow_next();

  const int warp = threadIdx.x >> 5;
  if (warp == kGemvConsumers / 32) {
    // ---------------- producer warp: stream this CTA's weight slab ----------
    const int lane = threadIdx.x & 31;
    const uint64_t policy = evict_first_policy();
    bool failed = false;
    int g = 0;
    for (int t = 0; t < ntiles && !failed; ++t) {
      const int tr0 = r0 + t * tile_rows;
      const int trows = min(tile_rows, r1 - tr0);
      for (int ks = 0; ks < nk; ++ks, ++g) {
        const int st = g % a.stages;
        if (g >= a.stages && !mbar_wait(&empty[st], ((g / a.stages) - 1) & 1)) {
          failed = true;
          record_error(a.err, kErrWaitEmpty);
          break;
        }
        const int k0 = ks * kc;
        const unsigned bytes = 2u * min(kc, I - k0);
        if (lane == 0) mbar_arrive_expect_tx(&full[st], bytes * trows);
        __syncwarp();
        unsigned char* dst = ring + st * stage_bytes;
        for (int r = lane; r < trows; r += 32)
          bulk_g2s(dst + r * row_stride, sg.w + size_t(tr0 + r) * I + k0, bytes, &full[st], policy);
      }
    }
    (void)total;
    return;
  }

  // ---------------- consumers: build x, then stream-multiply -----------------
  wait_prior();
  const int nrows = a.nrows;
  if (a.prologue == kPrologueRmsNorm) {
    for (int r = warp; r < nrows; r += kGemvConsumers / 32) {
      const bf16* xr = a.x + size_t(r) * a.x_stride;
      const float inv = rms_inverse_global(xr, I, a.eps);
      for (int f = threadIdx.x & 31; f < I; f += 32) {
        const float v = round_bf16(__fmul_rn(round_bf16(__fmul_rn(widen(xr[f]), inv)), widen(a.norm_w[f])));
        if constexpr (ROWS == 1)
          reinterpret_cast<float*>(xs)[f] = v;
        else
          reinterpret_cast<bf16*>(xs)[size_t(r) * I + f] = narrow(v);
      }
    }
  } else {
    for (int idx = threadIdx.x; idx < nrows * I; idx += kGemvConsumers) {
      const int r = idx / I, f = idx % I;
      const bf16* xr = a.x + size_t(r) * a.x_stride;
      float v;
      if (a.prologue == kPrologueSwiGLU)
        v = swiglu(widen(xr[f]), widen(xr[I + f]));
      else
        v = widen(xr[f]);
      if constexpr (ROWS == 1)
        reinterpret_cast<float*>(xs)[f] = v;
      else
        reinterpret_cast<bf16*>(xs)[size_t(r) * I + f] = narrow(v);
    }
  }
  if constexpr (ROWS > 1) {
    // Zero the unused rows so the loop can run all ROWS.
    for (int idx = nrows * I + threadIdx.x; idx < ROWS * I; idx += kGemvConsumers)
      reinterpret_cast<bf16*>(xs)[idx] = narrow(0.0f);
  }
  named_sync(1, kGemvConsumers);

  bool failed = false;
  if (P == 16)
    consume<ROWS, 16>(a, sg, r0, r1, ntiles, tile_rows, ring, stage_bytes, row_stride, full, empty,
                      xs, cta_best, failed);
  else
    consume<ROWS, 32>(a, sg, r0, r1, ntiles, tile_rows, ring, stage_bytes, row_stride, full, empty,
                      xs, cta_best, failed);

  if (a.epilogue != kEpilogueArgmax) return;
  named_sync(1, kGemvConsumers);
  if (threadIdx.x == 0) {
    uint4 b = cta_best[0];
    for (int w = 1; w < kGemvConsumers / 32; ++w) {
      const uint4 c = cta_best[w];
      if (better(__uint_as_float(c.x), c.y, __uint_as_float(b.x), b.y)) { b.x = c.x; b.y = c.y; }
      b.z |= c.z;
    }
    a.partials[blockIdx.x] = b;
    __threadfence();
    last_cta = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  }
  named_sync(1, kGemvConsumers);
  if (!last_cta) return;
  __threadfence();
  // Last CTA: reduce the per-CTA partials, publish, feed the next step.
  float bv = -INFINITY;
  unsigned bid = 0xffffffffu, fl = 0;
  for (unsigned i = threadIdx.x; i < gridDim.x; i += kGemvConsumers) {
    const uint4 c = __ldcg(&a.partials[i]);
    fl |= c.z;
    if (better(__uint_as_float(c.x), c.y, bv, bid)) { bv = __uint_as_float(c.x); bid = c.y; }
  }
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const unsigned oid = __shfl_xor_sync(0xffffffffu, bid, off);
    fl |= __shfl_xor_sync(0xffffffffu, fl, off);
    if (better(ov, oid, bv, bid)) { bv = ov; bid = oid; }
  }
  if (lane == 0) cta_best[warp] = make_uint4(__float_as_uint(bv), bid, fl, 0);
  named_sync(1, kGemvConsumers);
  __shared__ unsigned chosen;
  if (threadIdx.x == 0) {
    uint4 b = cta_best[0];
    for (int w = 1; w < kGemvConsumers / 32; ++w) {
      const uint4 c = cta_best[w];
      if (better(__uint_as_float(c.x), c.y, __uint_as_float(b.x), b.y)) { b.x = c.x; b.y = c.y; }
      b.z |= c.z;
    }
    unsigned status = b.z ? 1u : 0u, token = 0;
    if (!status) {
      if (!isfinite(__uint_as_float(b.x))) status = 2;
      else token = b.y;
    }
    const SelectOutput& so = a.select;
    so.result[0] = token;
    so.result[1] = status;
    if (so.history) so.history[so.step ? *so.step : 0] = token;
    if (so.step) ++*so.step;
    if (so.terminal) *so.terminal |= (status != 0) || (so.stop_mask && so.stop_mask[token]);
    if (so.position) ++*so.position;
    *a.ticket = 0;
    chosen = token;
  }
  named_sync(1, kGemvConsumers);
  const SelectOutput& so = a.select;
  if (so.embed) {
    const bf16* src = so.embed + size_t(chosen) * so.width;
    for (int f = threadIdx.x; f < so.width; f += kGemvConsumers) so.residual[f] = src[f];
  }
}

}  // namespace

size_t gemv_smem_bytes(int rows, int in_width, int kc, int stages, int max_tile_rows) {
  const size_t x = rows == 1 ? size_t(in_width) * 4 : size_t(in_width) * 2 * rows;
  return 256 + (x + 127) / 128 * 128 + size_t(stages) * max_tile_rows * (2 * kc + 16);
}

// Plan + launch.  Segments get CTAs in proportion to their bytes.
cudaError_t launch_gemv(GemvArgs a, int rows_template, int grid, cudaStream_t stream, bool pdl) {
  const int I = a.in_width;
  long long total_bytes = 0;
  for (int i = 0; i < a.nseg; ++i) total_bytes += (long long)a.seg[i].rows * I;
  int assigned = 0;
  int max_tile_rows = 1;
  for (int i = 0; i < a.nseg; ++i) {
    int c = a.nseg == 1 ? grid
                        : std::max(1, (int)std::llround((double)grid * a.seg[i].rows * I / total_bytes));
    if (i == a.nseg - 1) c = std::max(1, grid - assigned);
    c = std::min(c, a.seg[i].rows);
    a.seg[i].cta_begin = assigned;
    a.seg[i].cta_count = c;
    assigned += c;
    const int per = (a.seg[i].rows + c - 1) / c;
    const int maxr = kGemvConsumers / (a.seg[i].partials / 8);
    const int nt = (per + maxr - 1) / maxr;
    max_tile_rows = std::max(max_tile_rows, (per + nt - 1) / nt);
  }
  a.max_tile_rows = max_tile_rows;
  const size_t xbytes = rows_template == 1 ? size_t(I) * 4 : size_t(I) * 2 * rows_template;
  a.kc = max_tile_rows <= 32 ? 256 : 128;
  if (a.kc > ((I + 31) / 32) * 32) a.kc = ((I + 31) / 32) * 32;
  const size_t stage = size_t(max_tile_rows) * (2 * a.kc + 16);
  const size_t avail = kGemvSmemBudget - 256 - (xbytes + 127) / 128 * 128;
  a.stages = (int)std::min<size_t>(16, avail / stage);
  if (a.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = gemv_smem_bytes(rows_template, I, a.kc, a.stages, max_tile_rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(assigned);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (rows_template) {
#define DL_GEMV_CASE(R)                                                                          \
  case R: {                                                                                      \
    cudaFuncSetAttribute(gemv_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    return cudaLaunchKernelEx(&cfg, gemv_kernel<R>, a);                                          \
  }
    DL_GEMV_CASE(1)
    DL_GEMV_CASE(2)
    DL_GEMV_CASE(4)
    DL_GEMV_CASE(8)
#undef DL_GEMV_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

int gemv_rows_template(int rows, int in_width) {
  // x for all rows must fit next to the ring: BF16 rows when rows > 1.
  for (int r : {1, 2, 4, 8})
    if (rows <= r && (r == 1 || size_t(in_width) * 2 * r <= 64 * 1024)) return r;
  if (size_t(in_width) * 2 * 8 <= 64 * 1024) return 8;
  if (size_t(in_width) * 2 * 4 <= 64 * 1024) return 4;
  if (size_t(in_width) * 2 * 2 <= 64 * 1024) return 2;
  return 1;
}

}  // namespace dl
