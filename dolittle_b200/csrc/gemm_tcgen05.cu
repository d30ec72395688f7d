// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   Y[M][N] = X[M][K] * W[N][K]^T, BF16 operands, FP32 accumulation in TMEM,
//   one BF16 rounding in the epilogue (plus the recipe's own rounding points:
//   residual add, SwiGLU on interleaved gate/up columns).
//
// One CTA computes one BM x BN output tile (BM = 128, BN = 128 or 256):
//  * a producer thread streams K-slices of X and W with 2D TMA boxes
//    ([64 features] x [rows], 128-byte swizzle) into a ring of stages;
//  * one MMA thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN,
//    K=16 per instruction) on shared-memory descriptors and commits each stage
//    back to the producer through an mbarrier (tcgen05.commit);
//  * after the last K-slice, all four warps read the accumulator with
//    tcgen05.ld (warp w owns TMEM lanes 32w..32w+31 = rows), round, apply the
//    epilogue and store.
// This path does not keep the reference's FP32 summation order (tensor-core
// accumulation); it is the fast prefill path, checked against the reference
// within tolerance, while the parity path keeps bit-identical prefill.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm_tcgen05.h"
#include "tcgen05.cuh"

namespace dl {
namespace {

using namespace tc;

constexpr int kBM = 128;
constexpr int kBK = 64;   // one 128-byte swizzle atom of BF16
constexpr int kThreads = 192;  // producer warp, MMA warp, 4 epilogue warps
// Ring depth of the single-SM kernel.  The few-row split-K form streams
// weights only, so it takes as many stages as fit in 224 KB (five 40 KB
// stages of two k-steps at 32 rows).
constexpr int kMaxStages = 12;
// Tile choice, in units of one 256-wide k-step (~0.5 us on a B200): a
// 128-wide k-step takes nearly as long (the narrow MMA is bound by shared
// memory reads), and split-K costs a fixed ~8 us plus its FP32 partials'
// traffic at ~3 TB/s.  Fitted to a sweep of M = 512 / 2048 x the Qwen3-8B
// projections (qkv, o, gate|up, down) over tile widths 128 / 256 and 1-4
// parts: the estimate ranks the measured times in the same order.
constexpr double kStep128 = 0.95;
// 256 x 256 on two SMs (32 KB of loads per SM and k-step, against 48 KB) measured
// 1.13-1.4x the single-SM step: one accumulator, so the epilogue does not
// overlap the next tile, and each step waits for both SMs' loads.
constexpr double kStepPair = 1.25;
constexpr double kSplitFixed = 16.0;
constexpr double kSplitPerByte = 1.0 / 1.5e6;
// Stream-K (every CTA an equal share of the k-steps) is available on request
// only: measured against the tile choices above it never won by more than
// 2 % (down at M = 2048: 176 vs 180 us) and lost up to 12 % at M = 512 (qkv
// 47 vs 42, gate|up 119 vs 109, down 78 vs 70 us with 2 K parts).  The
// k-steps it saves in the last wave are spent on the partial tiles' stores,
// the finishers' sums and restarting the pipeline per unit.

struct alignas(64) GemmArgs {
  CUtensorMap map_a;
  CUtensorMap map_b;
  int M, N, K;
  int epilogue;
  int stages;
  int nseg;
  int seg_n0[3];
  bf16* seg_out[3];
  int seg_ld[3];
  unsigned* err;
  int split;           // K parts per tile
  float* partial;      // [split][M][N] FP32
  unsigned* tickets;   // per tile (split >= 2 with the epilogue in the kernel)
  int partial_only;    // every part stores its FP32 partial; no epilogue
  int streamk;         // stream-K: equal (tile, k-step) ranges per CTA (see WorkIter)
};

// The units of work of one CTA.  Split mode: units b, b + grid, ... of
// tiles x split, unit u = K part u / tiles of tile u % tiles.  Stream-K mode:
// the CTAs form one group per row of M tiles (CTA b serves M tile b % mt, as
// rank b / mt of its group); each group cuts its row's flattened
// (N tile, k-step) space into equal contiguous ranges, and a CTA walks its
// range tile by tile from the END, so each unit is a k-range of one tile.
// CTAs b .. b + mt - 1 cover the same k-steps of the same N tiles of all M
// rows at the same time, so a weight tile is read from DRAM once and shared
// through L2, as in the tile mode.  A tile cut between CTAs is summed by the
// CTA that holds its last k-step, in k order (see tile_epilogue_streamk).
// Walking backwards puts a CTA's contribution to the next tile (the end of
// its range) first and its finishing work (the start of its range) last: no
// CTA waits on a partial that is itself queued behind a wait.
struct Work {
  int tile, k_lo, k_hi, part;
};
// Stream-K range of group rank r of R over a row of nt N tiles x kt k-steps.
__device__ __forceinline__ long long sk_bound(int r, int R, int nt, int kt) {
  return (long long)r * nt * kt / R;
}

template <bool SK>
struct WorkIter {
  int u, units, stride, tiles, kt, split, mt, m;
  long long w, w1;
  __device__ WorkIter(const GemmArgs& a, int tiles_, int kt_all, int mt_)
      : u(blockIdx.x), units(tiles_ * a.split), stride(gridDim.x), tiles(tiles_), kt(kt_all), split(a.split), mt(mt_),
        m(int(blockIdx.x) % mt_) {
    if constexpr (SK) {
      const int R = int(gridDim.x) / mt_, r = int(blockIdx.x) / mt_, nt = tiles_ / mt_;
      w = sk_bound(r, R, nt, kt_all);
      w1 = sk_bound(r + 1, R, nt, kt_all);
    }
  }
  __device__ bool next(Work& o) {
    if constexpr (SK) {
      if (w1 <= w) return false;
      const int n = int((w1 - 1) / kt);  // N tile of this row
      const long long t0 = (long long)n * kt;
      o.tile = n * mt + m;
      o.k_hi = int(w1 - t0);
      o.k_lo = int(max(w, t0) - t0);
      o.part = 0;
      w1 = t0 + o.k_lo;
      return true;
    }
    if (u >= units) return false;
    o.tile = u % tiles;
    o.part = u / tiles;
    o.k_lo = o.part * kt / split;
    o.k_hi = (o.part + 1) * kt / split;
    u += stride;
    return true;
  }
};

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// {64 features, rows from y, feature blocks from z} box of a 3D map (see
// encode_3d): consecutive [rows][64] tiles in shared memory.
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ float swiglu_law(float a, float b) {
  const float e = expf(a >= 0.0f ? -a : a);
  const float s = a >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return round_bf16(__fmul_rn(round_bf16(__fmul_rn(a, s)), b));
}

// Epilogue of one accumulator row chunk: 32 FP32 columns of output row `row`
// starting at column `col` (of the output segment).
// The residual epilogue's 32 old values of the chunk (four 16-byte words),
// loaded one chunk ahead so the round trip overlaps the previous chunk.
__device__ __forceinline__ void load_residual(const bf16* out, int ld, int row, int col, uint4 (&old)[4]) {
  const uint4* src = reinterpret_cast<const uint4*>(out + size_t(row) * ld + col);
#pragma unroll
  for (int q = 0; q < 4; ++q) old[q] = src[q];
}

__device__ __forceinline__ void store_chunk(const GemmArgs& a, bf16* out, int ld, int row, int col,
                                            const uint32_t (&r)[32], const uint4 (&res)[4]) {
  if (a.epilogue == kGemmSwiGLU) {
    // Columns (2o, 2o+1) = (gate o, up o).
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float v0 = swiglu_law(round_bf16(__uint_as_float(r[2 * i])), round_bf16(__uint_as_float(r[2 * i + 1])));
      const float v1 =
          swiglu_law(round_bf16(__uint_as_float(r[2 * i + 2])), round_bf16(__uint_as_float(r[2 * i + 3])));
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
      packed[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + size_t(row) * ld + col / 2);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    return;
  }
  uint32_t packed[16];
  bf16* dst = out + size_t(row) * ld + col;
  if (a.epilogue == kGemmResidual) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 old = res[q];
      const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e = q * 8 + 2 * i;
        const float y0 = round_bf16(__uint_as_float(r[e])), y1 = round_bf16(__uint_as_float(r[e + 1]));
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(__fadd_rn(bf_lo(ow[i]), y0), __fadd_rn(bf_hi(ow[i]), y1));
        packed[q * 4 + i] = *reinterpret_cast<const uint32_t*>(&h2);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
      packed[i] = *reinterpret_cast<const uint32_t*>(&h2);
    }
  }
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) d4[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
}

// Epilogue of one 128-row x BN tile held in TMEM at `acc` (this warp's lane
// group): the store / residual / SwiGLU epilogue of output row `row`, columns
// c0.. of `out`; or, with K split in parts, this part's FP32 partial
// (block `tile` of `tiles`) and, for the last part to finish, the sum in
// part order followed by the epilogue.  Run by the 4 epilogue warps (threads
// 64-191, named barrier 1).
template <int BN>
__device__ __forceinline__ void tile_epilogue(const GemmArgs& a, uint32_t acc, bf16* out, int ld, int row, int c0,
                                              int tile, int tiles, int half, int q, int lane, bool& last_half) {
  if (a.split == 1) {
    const bool resid = a.epilogue == kGemmResidual && row < a.M;
    uint4 res[4] = {};
    if (resid) load_residual(out, ld, row, c0, res);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(acc + uint32_t(c * 32), r);
      uint4 next[4] = {};
      if (resid && c + 1 < BN / 32) load_residual(out, ld, row, c0 + (c + 1) * 32, next);
      if (row < a.M) store_chunk(a, out, ld, row, c0 + c * 32, r, res);
#pragma unroll
      for (int q = 0; q < 4; ++q) res[q] = next[q];
    }
  } else {
    // Every K part publishes its FP32 partial; the last part to finish
    // adds all parts in part order (p0 + p1 + ... whichever finished
    // last, so the result is deterministic) and applies the epilogue.
    // Partial block of (part, tile): [BN columns][128 rows], so each warp
    // store covers one 128-byte line (lanes = consecutive rows).
    const size_t blk = size_t(BN) * kBM;
    float* mine = a.partial + (size_t(half) * tiles + tile) * blk + q * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(acc + uint32_t(c * 32), r);
#pragma unroll
      for (int i = 0; i < 32; ++i) mine[size_t(c * 32 + i) * kBM] = __uint_as_float(r[i]);
    }
    __threadfence();
    named_sync(1, 128);
    if (threadIdx.x == 64) last_half = atomicAdd(&a.tickets[tile], 1u) == unsigned(a.split - 1);
    named_sync(1, 128);
    if (last_half) {
      __threadfence();
      const float* first = a.partial + size_t(tile) * blk + q * 32 + lane;
      const size_t part_stride = size_t(tiles) * blk;
      const bool resid = a.epilogue == kGemmResidual && row < a.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        // One round trip per chunk: the other parts' values and the
        // residual words are all loaded before the sums.
        float pv[kGemmMaxSplit][32];
#pragma unroll
        for (int h = 0; h < kGemmMaxSplit; ++h)
          if (h < a.split && h != half) {
            const float* ph = first + size_t(h) * part_stride + size_t(c * 32) * kBM;
#pragma unroll
            for (int i = 0; i < 32; ++i) pv[h][i] = __ldcg(ph + size_t(i) * kBM);
          }
        uint4 res[4] = {};
        if (resid) load_residual(out, ld, row, c0 + c * 32, res);
        uint32_t r[32];
        tmem_ld32(acc + uint32_t(c * 32), r);
#pragma unroll
        for (int h = 0; h < kGemmMaxSplit; ++h)
          if (h == half) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pv[h][i] = __uint_as_float(r[i]);
          }
        // Sum in part order.
#pragma unroll
        for (int h = 1; h < kGemmMaxSplit; ++h)
          if (h < a.split) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pv[0][i] = __fadd_rn(pv[0][i], pv[h][i]);
          }
        if (row < a.M) {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(pv[0][i]);
          store_chunk(a, out, ld, row, c0 + c * 32, r, res);
        }
      }
      if (threadIdx.x == 64) a.tickets[tile] = 0;
    }
  }
}

// Stream-K epilogue of one unit (tile `tile`, k-steps [k_lo, k_hi) of kt):
//  * the whole tile: the plain epilogue;
//  * a unit without the tile's last k-step (a contributor; only a CTA's last
//    unit can be one): its FP32 partial into this CTA's slot, a block
//    [BN columns][128 rows] so a warp store is one 128-byte line; then one
//    ticket on the tile;
//  * the unit holding the last k-step (the finisher): waits (bounded) until
//    every contributor -- the CTAs before this one whose ranges reach into
//    the tile -- has ticked, adds their partials in k order and its own
//    accumulator last, applies the epilogue and resets the ticket.
// Contributors hold a tile's early k-steps, which they reach at the start of
// their ranges, so the finisher rarely waits; the sum order is fixed, so
// repeated runs are bit-identical.
template <int BN>
__device__ __forceinline__ void tile_epilogue_streamk(const GemmArgs& a, uint32_t acc, bf16* out, int ld, int row,
                                                      int c0, const Work& wk, int tiles, int kt, int mt, int q,
                                                      int lane, int* shared_flag) {
  if (wk.k_lo == 0 && wk.k_hi == kt) {
    bool unused = false;
    GemmArgs one = a;
    one.split = 1;
    tile_epilogue<BN>(one, acc, out, ld, row, c0, wk.tile, tiles, 0, q, lane, unused);
    return;
  }
  const size_t blk = size_t(BN) * kBM;
  if (wk.k_hi < kt) {
    float* mine = a.partial + size_t(blockIdx.x) * blk + q * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(acc + uint32_t(c * 32), r);
#pragma unroll
      for (int i = 0; i < 32; ++i) mine[size_t(c * 32 + i) * kBM] = __uint_as_float(r[i]);
    }
    __threadfence();
    named_sync(1, 128);
    if (threadIdx.x == 64) atomicAdd(&a.tickets[wk.tile], 1u);
    return;
  }
  // Finisher: the contributors are the lower ranks of this CTA's group whose
  // ranges reach into this tile (CTAs (r - 1) mt + m, (r - 2) mt + m, ...).
  const int m = int(blockIdx.x) % mt;
  const int R = int(gridDim.x) / mt, r = int(blockIdx.x) / mt, nt = tiles / mt;
  const long long tile_w0 = (long long)(wk.tile / mt) * kt;
  int first_r = r;
  while (first_r > 0 && sk_bound(first_r, R, nt, kt) > tile_w0) --first_r;  // rank whose range holds k-step 0
  const unsigned contrib = unsigned(r - first_r);
  if (threadIdx.x == 64) {
    int ok = 1;
    const long long start = clock64();
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&a.tickets[wk.tile]) : "memory");
      if (v >= contrib) break;
      if (clock64() - start > (1ll << 32)) {
        ok = 0;
        record_error(a.err, kErrWaitFull);
        break;
      }
    }
    *shared_flag = ok;
  }
  named_sync(1, 128);
  const bool ok = *shared_flag != 0;
  __threadfence();
  const bool resid = a.epilogue == kGemmResidual && row < a.M;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float sum[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) sum[i] = 0.f;
    for (int rr = first_r; rr < r && ok; ++rr) {
      const float* src = a.partial + size_t(rr * mt + m) * blk + size_t(c * 32) * kBM + q * 32 + lane;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __ldcg(src + size_t(i) * kBM);
      if (rr == first_r) {
#pragma unroll
        for (int i = 0; i < 32; ++i) sum[i] = v[i];
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) sum[i] = __fadd_rn(sum[i], v[i]);
      }
    }
    uint4 res[4] = {};
    if (resid) load_residual(out, ld, row, c0 + c * 32, res);
    uint32_t r[32];
    tmem_ld32(acc + uint32_t(c * 32), r);
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__fadd_rn(sum[i], __uint_as_float(r[i])));
    if (row < a.M && ok) store_chunk(a, out, ld, row, c0 + c * 32, r, res);
  }
  named_sync(1, 128);
  if (threadIdx.x == 64) a.tickets[wk.tile] = 0;
}

// Persistent, warp-specialized: CTA b processes tiles b, b + grid, ... with
// M tiles varying fastest (the CTAs that share a weight tile run together,
// so it is read from DRAM once).  Warp 0 streams A/B stages by TMA through
// the ring, warp 1 issues the MMAs into one of two TMEM accumulators, and
// warps 2-5 (TMEM lane groups 2, 3, 0, 1) drain the other accumulator, so a
// tile's epilogue overlaps the next tile's main loop.
// SWAP (a few rows, split-K partials only): the weights are the 128-row A
// operand and the M <= BN input rows the N side, D = W X^T lands in TMEM as
// [128 output features][BN rows]; a stage then carries 16 KB of weights and
// BN x 128 bytes of inputs instead of a mostly zero-filled 128-row input tile.
// NB (SWAP only): k-steps per stage, loaded as one 3D box per operand
// ({64 features, rows, NB feature blocks}), so each weight row is read NB x
// 128 contiguous bytes at a time.
template <int BN, bool SWAP = false, bool SK = false, int NB = 1>
__global__ void __launch_bounds__(kThreads, 1) gemm_tcgen05_kernel(const __grid_constant__ GemmArgs a) {
  static_assert(NB == 1 || SWAP, "multi-block stages are for the swapped form");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t full[kMaxStages], empty[kMaxStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ bool last_half;
  constexpr int kABlock = kBM * kBK * 2, kBBlock = BN * kBK * 2;
  constexpr int kABytes = kABlock * NB;
  constexpr int kBBytes = kBBlock * NB;
  constexpr int kStageBytes = kABytes + kBBytes;
  constexpr uint32_t kCols = 2 * BN;
  const uint32_t base_s = (smem_addr(smem_raw) + 1023u) & ~1023u;
  unsigned char* ring = smem_raw + (base_s - smem_addr(smem_raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = SWAP ? 1 : (a.M + kBM - 1) / kBM;
  const int tiles = SWAP ? a.N / kBM : mt * (a.N / BN);
  // Units: (tile, K part) in split mode, k-ranges of tiles under stream-K.
  const int kt_all = a.K / (kBK * NB);
  const int S = a.stages;
  __shared__ int sk_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, kCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;
  allow_next();
  const bool producer = warp == 0 && lane == 0;
  if (!producer) wait_prior();

  if (warp == 0) {
    if (lane == 0) {
      // Producer.  A rows m0.. (inputs; SWAP: weights), B rows n0.. (weights;
      // SWAP: inputs).  The weight halves of the first S stages are requested
      // before waiting for the previous kernel (programmatic dependent launch):
      // no kernel writes the weights, so they stream in during its tail.
      int pre = 0;
      {
        WorkIter<SK> it(a, tiles, kt_all, mt);
        Work wk;
        while (pre < S && it.next(wk)) {
          const int tile = wk.tile;
          const int m0 = SWAP ? tile * kBM : (tile % mt) * kBM, n0 = SWAP ? 0 : (tile / mt) * BN;
          for (int kt = wk.k_lo; kt < wk.k_hi && pre < S; ++kt, ++pre) {
            unsigned char* st = ring + pre * kStageBytes;
            mbar_arrive_expect_tx(&full[pre], kStageBytes);
            if constexpr (NB > 1)
              tma_3d(st, &a.map_a, m0, kt * NB, &full[pre]);
            else if (SWAP)
              tma_2d(st, &a.map_a, kt * kBK, m0, &full[pre]);
            else
              tma_2d(st + kABytes, &a.map_b, kt * kBK, n0, &full[pre]);
          }
        }
      }
      wait_prior();
      int g = 0;
      WorkIter<SK> it(a, tiles, kt_all, mt);
      Work wk;
      while (!*reinterpret_cast<volatile int*>(&abort_flag) && it.next(wk)) {
        const int tile = wk.tile;
        const int m0 = SWAP ? tile * kBM : (tile % mt) * kBM, n0 = SWAP ? 0 : (tile / mt) * BN;
        for (int kt = wk.k_lo; kt < wk.k_hi; ++kt, ++g) {
          const int s = g % S;
          unsigned char* st = ring + s * kStageBytes;
          if (g < pre) {
            // Weights already requested: the input half completes the stage.
            if constexpr (NB > 1)
              tma_3d(st + kABytes, &a.map_b, n0, kt * NB, &full[s]);
            else if (SWAP)
              tma_2d(st + kABytes, &a.map_b, kt * kBK, n0, &full[s]);
            else
              tma_2d(st, &a.map_a, kt * kBK, m0, &full[s]);
            continue;
          }
          if (g >= S && !mbar_wait(&empty[s], ((g / S) - 1) & 1)) {
            record_error(a.err, kErrWaitEmpty);
            atomicExch(&abort_flag, 1);
            break;
          }
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          if constexpr (NB > 1) {
            tma_3d(st, &a.map_a, m0, kt * NB, &full[s]);
            tma_3d(st + kABytes, &a.map_b, n0, kt * NB, &full[s]);
          } else {
            tma_2d(st, &a.map_a, kt * kBK, m0, &full[s]);
            tma_2d(st + kABytes, &a.map_b, kt * kBK, n0, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.
      constexpr uint32_t idesc = instr_desc_bf16(kBM, BN);
      int g = 0, t = 0;
      WorkIter<SK> it(a, tiles, kt_all, mt);
      Work wk;
      for (; !*reinterpret_cast<volatile int*>(&abort_flag) && it.next(wk); ++t) {
        const int buf = t & 1;
        if (t >= 2 && !mbar_wait(&acc_empty[buf], ((t >> 1) - 1) & 1)) {
          record_error(a.err, kErrWaitEmpty);
          atomicExch(&abort_flag, 1);
          break;
        }
        fence_after_sync();
        const uint32_t acc = tmem + uint32_t(buf * BN);
        bool ok = true;
        const int kt_n = wk.k_hi - wk.k_lo;
        for (int kt = 0; kt < kt_n; ++kt, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1)) {
            record_error(a.err, kErrWaitFull);
            atomicExch(&abort_flag, 1);
            ok = false;
            break;
          }
          fence_after_sync();
          const uint32_t sa = smem_addr(ring + s * kStageBytes);
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            const uint64_t adesc = smem_desc_sw128(sa + j * kABlock);
            const uint64_t bdesc = smem_desc_sw128(sa + kABytes + j * kBBlock);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_bf16(acc, adesc + uint64_t(kk * 2), bdesc + uint64_t(kk * 2), idesc, (kt | j | kk) != 0);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // Epilogue warps: TMEM lane group q = warp % 4 holds accumulator rows
    // 32q .. 32q+31 of the tile.
    const int q = warp & 3;
    int t = 0;
    WorkIter<SK> it(a, tiles, kt_all, mt);
    Work wk;
    for (; it.next(wk); ++t) {
      const int tile = wk.tile, half = wk.part;
      const int buf = t & 1;
      if (!mbar_wait(&acc_full[buf], (t >> 1) & 1)) {
        record_error(a.err, kErrWaitFull);
        atomicExch(&abort_flag, 1);
        break;
      }
      fence_after_sync();
      const int m0 = SWAP ? tile * kBM : (tile % mt) * kBM, n0 = SWAP ? 0 : (tile / mt) * BN;
      const int row = m0 + q * 32 + lane;  // SWAP: the output feature
      int si = 0;
      for (int i = 1; i < a.nseg; ++i)
        if (n0 >= a.seg_n0[i]) si = i;
      bf16* out = a.seg_out[si];
      const int ld = a.seg_ld[si];
      const int c0 = n0 - a.seg_n0[si];
      const uint32_t acc = tmem + uint32_t(buf * BN) + (uint32_t(q * 32) << 16);
      if (SWAP) {
        // D[feature row][input m]: part `half`, FP32, [part][M][N] as below;
        // for each m the warp's 32 features are 128 contiguous bytes.
        float* mine = a.partial + size_t(half) * a.M * a.N + row;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + uint32_t(c * 32), r);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < a.M) mine[size_t(c * 32 + i) * a.N] = __uint_as_float(r[i]);
        }
      } else if (a.partial_only) {
        // K part `half` of the tile as FP32; the split-K epilogue kernel adds
        // the parts in order.
        float* mine = a.partial + (size_t(half) * a.M + row) * a.N + n0;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(acc + uint32_t(c * 32), r);
          if (row < a.M) {
            uint4* d = reinterpret_cast<uint4*>(mine + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
          }
        }
      } else if constexpr (SK) {
        tile_epilogue_streamk<BN>(a, acc, out, ld, row, c0, wk, tiles, kt_all, mt, q, lane, &sk_flag);
      } else {
        tile_epilogue<BN>(a, acc, out, ld, row, c0, tile, tiles, half, q, lane, last_half);
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

// TMA load into this CTA's shared memory whose completion is counted on the
// pair's even-CTA barrier (`bar`, a cluster address).
__device__ __forceinline__ void tma_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// CTA-pair GEMM: 256 x 256 output tiles on two SMs (tcgen05 cta_group::2).
// Per k-step each CTA loads its 128 input rows and 128 of the tile's 256
// weight rows (32 KB, against 48 KB for a 128 x 256 tile on one SM), and
// the even CTA's MMA thread issues one M = 256, N = 256 MMA per 16 features
// over both CTAs' shared memory.  Both CTAs' loads complete on the even
// CTA's stage barrier; each MMA batch is committed to both CTAs' stage-free
// barriers, each finished tile to both CTAs' accumulator barriers; the
// epilogue warps of both CTAs drain their 128 TMEM rows and report to the
// even CTA.  Two 256-column accumulators per CTA, so a tile's epilogue
// overlaps the next tile's MMAs.  Units are (tile, K part)
// as in the single-CTA kernel; pair p takes units p, p + pairs, ...
constexpr int kPairN = 256;
constexpr uint32_t kPairCols = 2 * kPairN;  // two 256-column accumulators per CTA

__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t full[8], empty[8], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ bool last_half;
  constexpr int kABytes = kBM * kBK * 2;
  constexpr int kBBytes = (kPairN / 2) * kBK * 2;
  constexpr int kStageBytes = kABytes + kBBytes;
  const uint32_t base_s = (smem_addr(smem_raw) + 1023u) & ~1023u;
  unsigned char* ring = smem_raw + (base_s - smem_addr(smem_raw));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int mt = (a.M + 2 * kBM - 1) / (2 * kBM);
  const int tiles = mt * (a.N / kPairN);
  const int units = tiles * a.split;
  const int kt_all = a.K / kBK;
  const int S = a.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // 4 epilogue warps in each CTA
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc_pair(&tmem_base, kPairCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  // Both CTAs' barriers exist before either signals the other's.
  cluster_sync();
  const uint32_t tmem = tmem_base;
  allow_next();
  wait_prior();

  if (warp == 0) {
    if (lane == 0) {
      // Producer (both CTAs): this CTA's A rows and B rows of each k-step,
      // completing on the even CTA's stage barrier.
      int g = 0;
      for (int u = pair; u < units && !*reinterpret_cast<volatile int*>(&abort_flag); u += pairs) {
        const int tile = u % tiles, part = u / tiles;
        const int m0 = (tile % mt) * 2 * kBM + int(rank) * kBM;
        const int nb = (tile / mt) * kPairN + int(rank) * (kPairN / 2);
        for (int kt = part * kt_all / a.split; kt < (part + 1) * kt_all / a.split; ++kt, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait_cluster(&empty[s], ((g / S) - 1) & 1)) {
            record_error(a.err, kErrWaitEmpty);
            atomicExch(&abort_flag, 1);
            break;
          }
          unsigned char* st = ring + s * kStageBytes;
          const uint32_t bar = mapa_shared(smem_addr(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
          tma_2d_pair(st, &a.map_a, kt * kBK, m0, bar);
          tma_2d_pair(st + kABytes, &a.map_b, kt * kBK, nb, bar);
        }
      }
      // Drain: the last commits onto this CTA's stage barriers have landed
      // before the CTA can leave.
      if (!*reinterpret_cast<volatile int*>(&abort_flag))
        for (int h = g - S < 0 ? 0 : g - S; h < g; ++h)
          if (!mbar_wait_cluster(&empty[h % S], (h / S) & 1)) {
            record_error(a.err, kErrWaitEmpty);
            break;
          }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // MMA issuer (even CTA).
      constexpr uint32_t idesc = instr_desc_bf16(2 * kBM, kPairN);
      int g = 0, t = 0;
      for (int u = pair; u < units && !*reinterpret_cast<volatile int*>(&abort_flag); u += pairs, ++t) {
        // Two accumulators: tile t's MMAs run while tile t - 1 drains.
        const int buf = t & 1;
        if (t >= 2 && !mbar_wait_cluster(&acc_empty[buf], ((t >> 1) - 1) & 1)) {
          record_error(a.err, kErrWaitEmpty);
          atomicExch(&abort_flag, 1);
          break;
        }
        fence_after_sync();
        const uint32_t acc = tmem + uint32_t(buf * kPairN);
        bool ok = true;
        const int part = u / tiles;
        const int kt_n = (part + 1) * kt_all / a.split - part * kt_all / a.split;
        for (int kt = 0; kt < kt_n; ++kt, ++g) {
          const int s = g % S;
          if (!mbar_wait_cluster(&full[s], (g / S) & 1)) {
            record_error(a.err, kErrWaitFull);
            atomicExch(&abort_flag, 1);
            ok = false;
            break;
          }
          fence_after_sync();
          const uint32_t sa = smem_addr(ring + s * kStageBytes);
          const uint64_t adesc = smem_desc_sw128(sa);
          const uint64_t bdesc = smem_desc_sw128(sa + kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_pair(acc, adesc + uint64_t(kk * 2), bdesc + uint64_t(kk * 2), idesc, (kt | kk) != 0);
          mma_commit_pair(mapa_shared(smem_addr(&empty[s]), 0));
          mma_commit_pair(mapa_shared(smem_addr(&empty[s]), 1));
        }
        if (!ok) break;
        mma_commit_pair(mapa_shared(smem_addr(&acc_full[buf]), 0));
        mma_commit_pair(mapa_shared(smem_addr(&acc_full[buf]), 1));
      }
    }
  } else {
    // Epilogue warps (both CTAs): TMEM lane group q = warp % 4 holds rows
    // 32q .. 32q+31 of this CTA's 128 rows of the tile.
    const int q = warp & 3;
    int t = 0;
    for (int u = pair; u < units; u += pairs, ++t) {
      const int tile = u % tiles, half = u / tiles;
      const int buf = t & 1;
      if (!mbar_wait_cluster(&acc_full[buf], (t >> 1) & 1)) {
        record_error(a.err, kErrWaitFull);
        atomicExch(&abort_flag, 1);
        break;
      }
      fence_after_sync();
      const int m0 = (tile % mt) * 2 * kBM + int(rank) * kBM, n0 = (tile / mt) * kPairN;
      const int row = m0 + q * 32 + lane;
      int si = 0;
      for (int i = 1; i < a.nseg; ++i)
        if (n0 >= a.seg_n0[i]) si = i;
      // Split-K blocks and tickets per 128-row half tile.
      tile_epilogue<kPairN>(a, tmem + uint32_t(buf * kPairN) + (uint32_t(q * 32) << 16), a.seg_out[si],
                            a.seg_ld[si], row, n0 - a.seg_n0[si], tile * 2 + int(rank), tiles * 2, half, q, lane,
                            last_half);
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_addr(&acc_empty[buf]), 0));
    }
  }
  fence_before_sync();
  __syncthreads();
  // Neither CTA leaves while the pair may still touch its shared memory or TMEM.
  cluster_sync();
  if (warp == 0) tmem_dealloc_pair(tmem, kPairCols);
}

}  // namespace

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {uint32_t(kBK), box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows][cols] BF16 (row stride ld elements) as {64 features, rows, cols /
// 64 feature blocks}: a box of `blocks` blocks holds `blocks` consecutive
// 128-byte-swizzled [box_rows][64] tiles.
bool encode_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
               uint32_t blocks) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {uint64_t(kBK), rows, cols / kBK};
  cuuint64_t strides[2] = {ld * 2, uint64_t(kBK) * 2};
  cuuint32_t box[3] = {uint32_t(kBK), box_rows, blocks};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool gemm_tcgen05_supported(int M, int N, int K) { return M > 0 && K % kBK == 0 && N % 128 == 0; }

size_t gemm_split_floats(int M, int N, int parts) {
  return size_t(parts) * size_t((M + 2 * kBM - 1) / (2 * kBM)) * 2 * kBM * N;  // 256-row tiles (CTA pairs) included
}

namespace {

// Sum of the K parts in part order, then the epilogue of the un-split kernel
// (store / residual / SwiGLU), or the FP32 sum itself.  One thread per pair
// of columns.
__global__ void splitk_epilogue_kernel(const float* __restrict__ parts, int splits, int M, int N, int epilogue,
                                       bf16* out, int ld, float* sum_out) {
  allow_next();  // a dependent GEMM may request its weights meanwhile
  wait_prior();
  const size_t pairs = size_t(M) * (N / 2);
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < pairs; i += size_t(gridDim.x) * blockDim.x) {
    const int m = int(i / (N / 2)), n = int(i % (N / 2)) * 2;
    float2 acc = *reinterpret_cast<const float2*>(parts + size_t(m) * N + n);
    for (int s = 1; s < splits; ++s) {
      const float2 v = *reinterpret_cast<const float2*>(parts + (size_t(s) * M + m) * N + n);
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
    }
    if (sum_out) {
      *reinterpret_cast<float2*>(sum_out + size_t(m) * N + n) = acc;
      continue;
    }
    if (epilogue == kGemmSwiGLU) {
      out[size_t(m) * ld + n / 2] = narrow(swiglu_law(round_bf16(acc.x), round_bf16(acc.y)));
    } else if (epilogue == kGemmResidual) {
      bf16* d = out + size_t(m) * ld + n;
      const float y0 = round_bf16(acc.x), y1 = round_bf16(acc.y);
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(__fadd_rn(widen(d[0]), y0), __fadd_rn(widen(d[1]), y1));
      *reinterpret_cast<__nv_bfloat162*>(d) = h2;
    } else {
      *reinterpret_cast<__nv_bfloat162*>(out + size_t(m) * ld + n) = __floats2bfloat162_rn(acc.x, acc.y);
    }
  }
}

}  // namespace

int gemm_splitk_parts(int M, int N, int K, int sms) {
  // Parts (uneven when K/64 is not a multiple) that fill whole waves of the
  // SMs best, with at least 8 k-steps each; ties go to fewer parts.
  const int mt = (M + kBM - 1) / kBM, tiles = mt * (N / 128), kt = K / kBK;
  int best = 1;
  double best_fill = 0.0;
  for (int s = 1; s <= 16 && kt / s >= 8; ++s) {
    const long long units = (long long)tiles * s;
    const long long waves = (units + sms - 1) / sms;
    const double fill = double(units) / double(waves * sms);
    if (fill > best_fill + 0.02) {
      best = s;
      best_fill = fill;
    }
  }
  return best;
}

cudaError_t launch_gemm_tcgen05_parts(const GemmProblem& p, int splits, float* parts, cudaStream_t stream,
                                      bool pdl) {
  if (!gemm_tcgen05_supported(p.M, p.N, p.K) || splits < 1 || splits > 16 || p.K / kBK < splits || !parts)
    return cudaErrorInvalidValue;
  GemmArgs a = {};
  // Up to 128 rows: the swapped form (weights as the 128-row operand).
  const bool swap = p.M <= 128;
  const int BN = swap ? (p.M <= 32 ? 32 : p.M <= 64 ? 64 : 128) : 128;
  if (swap) {
    if (!encode_2d(&a.map_a, p.w, uint64_t(p.N), uint64_t(p.K), uint64_t(p.K), kBM)) return cudaErrorInvalidValue;
    if (!encode_2d(&a.map_b, p.x, uint64_t(p.M), uint64_t(p.K), uint64_t(p.ldx), uint32_t(BN)))
      return cudaErrorInvalidValue;
  } else {
    if (!encode_2d(&a.map_a, p.x, uint64_t(p.M), uint64_t(p.K), uint64_t(p.ldx), kBM)) return cudaErrorInvalidValue;
    if (!encode_2d(&a.map_b, p.w, uint64_t(p.N), uint64_t(p.K), uint64_t(p.K), uint32_t(BN)))
      return cudaErrorInvalidValue;
  }
  // Two feature blocks per stage in the swapped form (32 rows): 256
  // contiguous bytes of each weight row per request.  Measured on the batch-32
  // decode step at 2K context: 6.56 -> 6.18 ms (four blocks: 6.19 ms, with
  // only two 80 KB stages in flight).
  int nb = swap && BN == 32 ? 2 : 1;
  if (nb > 1 && ((p.K / kBK) % nb || p.K / kBK / nb < splits)) nb = 1;
  if (nb > 1) {
    if (!encode_3d(&a.map_a, p.w, uint64_t(p.N), uint64_t(p.K), uint64_t(p.K), kBM, uint32_t(nb)) ||
        !encode_3d(&a.map_b, p.x, uint64_t(p.M), uint64_t(p.K), uint64_t(p.ldx), uint32_t(BN), uint32_t(nb)))
      return cudaErrorInvalidValue;
  }
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.epilogue = kGemmStore;
  a.nseg = 1;
  a.err = p.err;
  a.split = splits;
  a.partial = parts;
  a.partial_only = 1;
  const int stage_bytes = (kBM + BN) * kBK * 2 * nb;
  a.stages = std::min(kMaxStages, (224 * 1024) / stage_bytes);
  const size_t smem = size_t(a.stages) * stage_bytes + 1024;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = swap ? p.N / kBM : (long long)((p.M + kBM - 1) / kBM) * (p.N / BN);
  const long long units = tiles * splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(std::min<long long>(units, sms)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  auto go = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cudaLaunchKernelEx(&cfg, kernel, a);
  };
  if (!swap) return go(gemm_tcgen05_kernel<128>);
  if (BN == 32) return nb == 2 ? go(gemm_tcgen05_kernel<32, true, false, 2>) : go(gemm_tcgen05_kernel<32, true>);
  if (BN == 64) return go(gemm_tcgen05_kernel<64, true>);
  return go(gemm_tcgen05_kernel<128, true>);
}

cudaError_t launch_gemm_splitk_epilogue(const float* parts, int splits, int M, int N, int epilogue, bf16* out,
                                        int ld, float* sum_out, cudaStream_t stream, bool pdl) {
  if (N % 2 || splits < 1 || (!out && !sum_out)) return cudaErrorInvalidValue;
  const size_t pairs = size_t(M) * (N / 2);
  const unsigned blocks = unsigned(std::min<size_t>((pairs + 255) / 256, 148 * 16));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, splitk_epilogue_kernel, parts, splits, M, N, epilogue, out, ld, sum_out);
}

// CTA pairs that fit on the device at once (clusters of 2 at one CTA per SM).
int gemm_pair_clusters(int sms) {
  static int cached = -1;
  static std::once_flag once;
  std::call_once(once, [sms] {
    const size_t smem = size_t(std::min(8, (225 * 1024) / ((kBM + kPairN / 2) * kBK * 2))) *
                            ((kBM + kPairN / 2) * kBK * 2) + 1024;
    cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * unsigned(sms / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    cached = cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg) == cudaSuccess ? n : 0;
    cudaGetLastError();
  });
  return cached;
}

cudaError_t launch_gemm_tcgen05(const GemmProblem& p, cudaStream_t stream, bool pdl) {
  if (!gemm_tcgen05_supported(p.M, p.N, p.K) || p.nseg < 1 || p.nseg > 3) return cudaErrorInvalidValue;
  GemmArgs a = {};
  // Tile width and K parts by estimated time: waves over the SMs x k-steps
  // per unit x the cost of one k-step, plus the partial sums' traffic.  A
  // 128-wide k-step moves 2/3 of a 256-wide one's bytes for half the MMA work.
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long mt = (p.M + kBM - 1) / kBM;
  const int kt = p.K / kBK;
  bool aligned256 = p.N % 256 == 0;
  for (int i = 0; i < p.nseg; ++i) aligned256 = aligned256 && p.seg_n0[i] % 256 == 0;
  const bool workspace = p.partial && p.tickets;
  int BN = 0, split = 0;
  bool pair = false;
  double best = 1e30;
  // Single-CTA tiles 128 x 256 / 128 x 128, and 256 x 256 tiles on CTA pairs.
  struct Shape {
    int bm, bn;
  };
  const Shape shapes[3] = {{128, 256}, {128, 128}, {256, 256}};
  const int pair_slots = gemm_pair_clusters(sms);
  for (const Shape& sh : shapes) {
    const bool is_pair = sh.bm == 256;
    if (sh.bn == 256 && !(aligned256 && p.wide_tiles)) continue;
    if (p.force_bn && sh.bn != p.force_bn) continue;
    if (p.force_bm && sh.bm != p.force_bm) continue;
    if (is_pair && pair_slots < 1) continue;
    const long long mtiles = (p.M + sh.bm - 1) / sh.bm;
    const long long tiles = mtiles * (p.N / sh.bn);
    const long long slots = is_pair ? pair_slots : sms;
    for (int sp = 1; sp <= kGemmMaxSplit; ++sp) {
      if (p.force_split && sp != p.force_split) continue;
      const size_t split_floats = size_t(sp) * size_t(mtiles) * sh.bm * size_t(p.N);
      if (sp > 1 && (!workspace || kt / sp < 4 || split_floats > p.partial_floats ||
                     tiles * (sh.bm / kBM) > p.n_tickets))
        continue;
      const long long waves = (tiles * sp + slots - 1) / slots;
      const double step = is_pair ? kStepPair : sh.bn == 256 ? 1.0 : kStep128;
      const double split_cost = sp > 1 ? kSplitFixed + kSplitPerByte * 4.0 * double(split_floats) : 0.0;
      const double cost = double(waves) * double((kt + sp - 1) / sp) * step + split_cost;
      if (cost < best * 0.98) {
        best = cost;
        BN = sh.bn;
        split = sp;
        pair = is_pair;
      }
    }
  }
  // Stream-K on single-SM tiles: one partial block per CTA in the workspace,
  // one ticket per tile.
  int sk_grid = 0;
  if (workspace && p.force_streamk > 0 && !p.force_split && p.force_bm != 256) {
    for (const int bn : {256, 128}) {
      if (bn == 256 && !(aligned256 && p.wide_tiles)) continue;
      if (p.force_bn && bn != p.force_bn) continue;
      const long long tiles = mt * (p.N / bn);
      // One group of CTAs per row of M tiles, at least 8 k-steps per CTA.
      const long long per_row = std::min<long long>(sms / mt, (p.N / bn) * kt / 8);
      const int G = int(per_row * mt);
      if (per_row < 1 || G < 2 || tiles > p.n_tickets || size_t(G) * bn * kBM > p.partial_floats) continue;
      if (BN == 0 || sk_grid == 0) {
        BN = bn;
        split = 1;
        pair = false;
        sk_grid = G;
      }
    }
  }
  if (!BN) return cudaErrorInvalidValue;
  for (int i = 0; i < p.nseg; ++i)
    if (p.seg_n0[i] % BN) return cudaErrorInvalidValue;  // tiles never straddle outputs
  if (!encode_2d(&a.map_a, p.x, uint64_t(p.M), uint64_t(p.K), uint64_t(p.ldx), kBM)) return cudaErrorInvalidValue;
  if (!encode_2d(&a.map_b, p.w, uint64_t(p.N), uint64_t(p.K), uint64_t(p.K), uint32_t(pair ? BN / 2 : BN)))
    return cudaErrorInvalidValue;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.epilogue = p.epilogue;
  a.nseg = p.nseg;
  for (int i = 0; i < p.nseg; ++i) {
    a.seg_n0[i] = p.seg_n0[i];
    a.seg_out[i] = p.seg_out[i];
    a.seg_ld[i] = p.seg_ld[i];
  }
  a.err = p.err;
  const int stage_bytes = (kBM + (pair ? BN / 2 : BN)) * kBK * 2;
  a.stages = std::min(8, (225 * 1024) / stage_bytes);
  const size_t smem = size_t(a.stages) * stage_bytes + 1024;
  cudaLaunchConfig_t cfg = {};
  a.split = split;
  a.partial = p.partial;
  a.tickets = p.tickets;
  if (pair) {
    const long long units = (long long)((p.M + 2 * kBM - 1) / (2 * kBM)) * (p.N / kPairN) * split;
    cfg.gridDim = dim3(unsigned(2 * std::min<long long>(units, pair_slots)));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cudaLaunchKernelEx(&cfg, gemm_pair_kernel, a);
  }
  const long long units = mt * (p.N / BN) * split;
  a.streamk = sk_grid > 0 ? 1 : 0;
  cfg.gridDim = dim3(unsigned(sk_grid > 0 ? sk_grid : std::min<long long>(units, sms)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  auto go = [&](auto kernel) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cudaLaunchKernelEx(&cfg, kernel, a);
  };
  if (a.streamk) return BN == 256 ? go(gemm_tcgen05_kernel<256, false, true>) : go(gemm_tcgen05_kernel<128, false, true>);
  return BN == 256 ? go(gemm_tcgen05_kernel<256>) : go(gemm_tcgen05_kernel<128>);
}

}  // namespace dl
