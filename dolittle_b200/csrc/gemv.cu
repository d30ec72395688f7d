// Streaming GEMV kernel (see gemv.cuh for the law and the B200 mapping).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "gemv_device.cuh"
#include "launch.h"

namespace dl {
namespace {

using namespace gemv_dev;

__host__ __device__ __forceinline__ size_t x_bytes(int rows_template, int width) {
  return (size_t(width) * 2 * rows_template + 127) / 128 * 128;
}

template <int ROWS, int P, bool MAP, int KC>
__device__ void consume(const GemvArgs& a, const GemvSegment& sg, int r0, int r1, int ntiles,
                        unsigned char* ring, uint64_t* full, uint64_t* empty, const bf16* xs, uint4* cta_best,
                        bool& failed) {
  using L = Layout<P>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = L::slot(lane);
  const int my_row = L::row(warp, lane);
  const int I = a.in_width;
  const int kc = MAP ? KC : a.kc;
  const int nk = (I + kc - 1) / kc;
  const int padded = (I + 15) / 16 * 16;
  const int tile_rows = sg.tile_rows;
  const int box_bytes = ((tile_rows + 7) / 8) * 8 * 128;
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
        const unsigned char* stage = ring + st * a.stage_bytes;
        if (MAP && nfeat == KC)
          stage_map<ROWS, P, KC>(stage, box_bytes, my_row, slot, xs, I, k0, acc);
        else
          stage_generic<ROWS, P, MAP>(stage, box_bytes, a.row_stride, my_row, slot, xs, I, k0, kc, nfeat, acc);
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
      const int row = tr0 + my_row;
      if (a.epilogue == kEpilogueSwiGLU) {
        // Even row = gate o, odd row = up o; both rounded to storage first.
        const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
        if (!active || slot != 0 || failed || r >= a.nrows || (row & 1)) continue;
        const float act = swiglu(round_bf16(y), round_bf16(partner));
        sg.out[size_t(r) * sg.out_stride + (row >> 1)] = narrow(act);
        continue;
      }
      if (!active || slot != 0 || failed || r >= a.nrows) continue;
      const bf16 yb = narrow(y);
      bf16* out = sg.out + (sg.out_row ? size_t(*sg.out_row) * sg.out_stride : 0);
      const size_t idx = size_t(r) * sg.out_stride + row;
      if (a.epilogue == kEpilogueResidual) {
        const bf16 nv = narrow(__fadd_rn(widen(out[idx]), widen(yb)));
        out[idx] = nv;
        if (a.capture) a.capture[(size_t(*a.capture_row) + r) * a.capture_stride + row] = nv;
      } else {
        out[idx] = yb;
        if (a.epilogue == kEpilogueArgmax) {
          const float v = widen(yb);
          if (isnan(v) || v == INFINITY) flags |= 1u;
          if (better(v, static_cast<unsigned>(row), best_v, best_id)) {
            best_v = v;
            best_id = static_cast<unsigned>(row);
          }
        }
      }
    }
  }
  if (a.epilogue == kEpilogueArgmax) {
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
__device__ void consume_dispatch(const GemvArgs& a, const GemvSegment& sg, int r0, int r1, int ntiles,
                                 unsigned char* ring, uint64_t* full, uint64_t* empty, const bf16* xs,
                                 uint4* cta_best, bool& failed) {
  const int P = sg.partials;
  if (a.use_map) {
    if (a.kc == 256) {
      if (P == 16)
        consume<ROWS, 16, true, 256>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
      else
        consume<ROWS, 32, true, 256>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
    } else {
      if (P == 16)
        consume<ROWS, 16, true, 128>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
      else
        consume<ROWS, 32, true, 128>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
    }
  } else {
    if (P == 16)
      consume<ROWS, 16, false, 0>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
    else
      consume<ROWS, 32, false, 0>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);
  }
}

template <int ROWS>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint4 cta_best[kGemvConsumers / 32];
  __shared__ float row_inv[8];
  __shared__ bool last_cta;
  __shared__ unsigned chosen;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + a.stages;
  bf16* xs = reinterpret_cast<bf16*>(smem + 256);
  const size_t xb = x_bytes(ROWS, a.in_width);
  unsigned char* xend = smem + 256 + xb;
  // The swizzled boxes need 1024-byte alignment of every stage.
  const uint32_t ring_s = (smem_addr(xend) + 1023u) & ~1023u;
  unsigned char* ring = xend + (ring_s - smem_addr(xend));

  int si = 0;
  for (int i = 1; i < a.nseg; ++i)
    if (static_cast<int>(blockIdx.x) >= a.seg[i].cta_begin) si = i;
  const GemvSegment& sg = a.seg[si];
  const int local = blockIdx.x - sg.cta_begin;
  const int r0 = min(sg.rows, local * sg.rows_per_cta), r1 = min(sg.rows, r0 + sg.rows_per_cta);
  const int tile_rows = sg.tile_rows;
  const int ntiles = r1 > r0 ? (r1 - r0 + tile_rows - 1) / tile_rows : 0;
  const int I = a.in_width;
  const int kc = a.kc;
  const int nk = (I + kc - 1) / kc;

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
    const int box_bytes = ((tile_rows + 7) / 8) * 8 * 128;
    int g = 0;
    for (int t = 0; t < ntiles; ++t) {
      const int tr0 = r0 + t * tile_rows;
      const int trows = min(tile_rows, r1 - tr0);
      for (int ks = 0; ks < nk; ++ks, ++g) {
        const int st = g % a.stages;
        if (g >= a.stages && !mbar_wait(&empty[st], ((g / a.stages) - 1) & 1)) {
          record_error(a.err, kErrWaitEmpty);
          return;
        }
        const int k0 = ks * kc;
        const int nfeat = min(kc, I - k0);
        unsigned char* dst = ring + st * a.stage_bytes;
        if (a.use_map) {
          const int nbox = (nfeat + kGemvBox - 1) / kGemvBox;
          if (lane == 0) mbar_arrive_expect_tx(&full[st], unsigned(nbox) * tile_rows * 128u);
          __syncwarp();
          if (lane < nbox) tma_load_2d(dst + lane * box_bytes, &sg.map, k0 + lane * kGemvBox, tr0, &full[st], policy);
        } else {
          const unsigned bytes = 2u * nfeat;
          if (lane == 0) mbar_arrive_expect_tx(&full[st], bytes * trows);
          __syncwarp();
          for (int r = lane; r < trows; r += 32)
            bulk_g2s(dst + r * a.row_stride, sg.w + size_t(tr0 + r) * I + k0, bytes, &full[st], policy);
        }
      }
    }
    return;
  }

  // ---------------- consumers: build x (BF16 rows in smem), then multiply ----
  wait_prior();
  const int nrows = a.nrows;
  {
    // Cooperative 16-byte copies of the input rows.
    const int v8 = I / 8;
    for (int idx = threadIdx.x; idx < nrows * v8; idx += kGemvConsumers) {
      const int r = idx / v8, q = idx % v8;
      reinterpret_cast<uint4*>(xs + size_t(r) * I)[q] = reinterpret_cast<const uint4*>(a.x + size_t(r) * a.x_stride)[q];
    }
    for (int idx = nrows * I + threadIdx.x; idx < ROWS * I; idx += kGemvConsumers) xs[idx] = narrow(0.0f);
  }
  named_sync(1, kGemvConsumers);
  if (a.prologue == kPrologueRmsNorm) {
    if (warp < nrows) row_inv[warp] = rms_inverse_smem(xs + size_t(warp) * I, I, a.eps);
    named_sync(1, kGemvConsumers);
    for (int idx = threadIdx.x; idx < nrows * I; idx += kGemvConsumers) {
      const int r = idx / I, f = idx % I;
      const float v = __fmul_rn(round_bf16(__fmul_rn(widen(xs[idx]), row_inv[r])), widen(a.norm_w[f]));
      xs[idx] = narrow(v);
    }
    named_sync(1, kGemvConsumers);
  }

  bool failed = false;
  consume_dispatch<ROWS>(a, sg, r0, r1, ntiles, ring, full, empty, xs, cta_best, failed);

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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

bool encode_weight_map(CUtensorMap* map, const void* w, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {uint32_t(kGemvBox), box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_weight_map3d(CUtensorMap* map, const void* w, uint64_t rows, uint64_t cols, uint32_t box_rows,
                         uint32_t blocks) {
  auto fn = encode_fn();
  if (!fn || cols % kGemvBox || blocks < 1 || blocks > 8) return false;
  // Element (f, r, b) = w[r][64 b + f]: one box is [blocks][box_rows][64].
  cuuint64_t dims[3] = {uint64_t(kGemvBox), rows, cols / kGemvBox};
  cuuint64_t strides[2] = {cols * 2, uint64_t(kGemvBox) * 2};
  cuuint32_t box[3] = {uint32_t(kGemvBox), box_rows, blocks};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

// Tuning overrides (features per stage, ring depth) read once from
// DOLITTLE_GEMV_KC / DOLITTLE_GEMV_STAGES.
struct GemvTuning {
  int kc = 0, stages = 16;
  GemvTuning() {
    if (const char* v = std::getenv("DOLITTLE_GEMV_KC")) kc = std::atoi(v) >= 256 ? 256 : 128;
    if (const char* v = std::getenv("DOLITTLE_GEMV_STAGES")) stages = std::max(2, std::min(16, std::atoi(v)));
  }
};
const GemvTuning& tuning() {
  static GemvTuning t;
  return t;
}

}  // namespace

size_t gemv_smem_bytes(int rows, int in_width, int stage_bytes, int stages) {
  return 256 + x_bytes(rows, in_width) + 1024 + size_t(stages) * stage_bytes;
}

// Plan + launch.  Segments get CTAs in proportion to their bytes; each
// segment's rows are split evenly over its CTAs (even counts for the SwiGLU
// pairing) and into tiles of at most 256/(P/8) rows (the consumer threads).
cudaError_t launch_gemv(GemvArgs a, int rows_template, int grid, cudaStream_t stream, bool pdl) {
  const int I = a.in_width;
  if (I % 8) return cudaErrorInvalidValue;
  const GemvTuning& tune = tuning();
  const bool pairs = a.epilogue == kEpilogueSwiGLU;
  long long total_bytes = 0;
  for (int i = 0; i < a.nseg; ++i) total_bytes += (long long)a.seg[i].rows * I;
  int assigned = 0;
  a.use_map = I >= kGemvBox ? 1 : 0;
  int max_box_rows = 0;
  for (int i = 0; i < a.nseg; ++i) {
    GemvSegment& s = a.seg[i];
    if (pairs && s.rows % 2) return cudaErrorInvalidValue;
    int c = a.nseg == 1 ? grid : std::max(1, (int)std::llround((double)grid * s.rows * I / total_bytes));
    if (i == a.nseg - 1) c = std::max(1, grid - assigned);
    c = std::min(c, s.rows);
    int per = (s.rows + c - 1) / c;
    if (pairs) per += per & 1;
    c = (s.rows + per - 1) / per;
    s.cta_begin = assigned;
    s.cta_count = c;
    s.rows_per_cta = per;
    assigned += c;
    const int maxr = kGemvConsumers / (s.partials / 8);
    const int nt = (per + maxr - 1) / maxr;
    s.tile_rows = (per + nt - 1) / nt;
    if (pairs) s.tile_rows += s.tile_rows & 1;
    max_box_rows = std::max(max_box_rows, ((s.tile_rows + 7) / 8) * 8);
  }
  if (a.use_map) {
    a.kc = tune.kc ? tune.kc : (4 * max_box_rows * 128 <= 40 * 1024 ? 256 : 128);
    for (int i = 0; i < a.nseg; ++i)
      if (!encode_weight_map(&a.seg[i].map, a.seg[i].w, uint64_t(a.seg[i].rows), uint64_t(I),
                             uint32_t(a.seg[i].tile_rows)))
        return cudaErrorInvalidValue;
    a.stage_bytes = (a.kc / kGemvBox) * max_box_rows * 128;
  } else {
    a.kc = ((I + 31) / 32) * 32;
    a.row_stride = 2 * a.kc + 16;
    int maxt = 0;
    for (int i = 0; i < a.nseg; ++i) maxt = std::max(maxt, a.seg[i].tile_rows);
    a.stage_bytes = maxt * a.row_stride;
  }
  const size_t fixed = gemv_smem_bytes(rows_template, I, 0, 0);
  if (kGemvSmemBudget <= fixed) return cudaErrorInvalidValue;
  a.stages = (int)std::min<size_t>(tune.stages, (kGemvSmemBudget - fixed) / a.stage_bytes);
  if (a.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = gemv_smem_bytes(rows_template, I, a.stage_bytes, a.stages);
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
  // x for all rows (BF16) must fit next to the ring.
  for (int r : {1, 2, 4, 8})
    if (rows <= r && size_t(in_width) * 2 * r <= 64 * 1024) return r;
  if (size_t(in_width) * 2 * 8 <= 64 * 1024) return 8;
  if (size_t(in_width) * 2 * 4 <= 64 * 1024) return 4;
  if (size_t(in_width) * 2 * 2 <= 64 * 1024) return 2;
  return 1;
}

}  // namespace dl
