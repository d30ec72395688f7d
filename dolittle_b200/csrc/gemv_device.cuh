// Device building blocks of the streaming projection law, shared by the
// stand-alone GEMV kernel (gemv.cu) and the persistent decode kernel
// (decode_persistent.cu).  The law itself is described in gemv.cuh.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemv.cuh"

namespace dl {
namespace gemv_dev {

// Lane layout inside a warp: a quarter-warp (8 lanes) holds 8 consecutive
// rows with the same slot, so the 8 swizzle phases (or the 16-byte row
// padding) give conflict-free LDS.128.  Rows 2k and 2k+1 sit in lanes l and
// l^1 (used by the SwiGLU epilogue).
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

// Shared-memory loads as plain C++ loads (not volatile asm), so the compiler
// can issue a stage's loads ahead of the FMAs that use them; they stay
// ordered after the stage's mbarrier wait, whose asm clobbers memory.
__device__ __forceinline__ uint4 sld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 sld8(const void* p) { return *reinterpret_cast<const uint2*>(p); }

// Halving tree over the P partials held 8 per thread (slot-major).
template <int P>
__device__ __forceinline__ float reduce_partials(float (&acc)[8]) {
  if constexpr (P == 32) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 16));
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 8));
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], acc[i + 4]);
#pragma unroll
  for (int i = 0; i < 2; ++i) acc[i] = __fadd_rn(acc[i], acc[i + 2]);
  return __fadd_rn(acc[0], acc[1]);
}

// acc[0] += x.lo * w.lo, acc[1] += x.hi * w.hi: one rounding each (the
// product of two BF16 values is exact in FP32).
__device__ __forceinline__ void fma_pair(float& a0, float& a1, uint32_t x2, uint32_t w2) {
  asm("{\n\t.reg .b16 xl, xh, wl, wh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "mov.b32 {wl, wh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, xl, wl, %0;\n\t"
      "fma.rn.f32.bf16 %1, xh, wh, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(x2), "r"(w2));
}

__device__ __forceinline__ void fma8(float (&acc)[8], const uint4& x, const uint4& w) {
  fma_pair(acc[0], acc[1], x.x, w.x);
  fma_pair(acc[2], acc[3], x.y, w.y);
  fma_pair(acc[4], acc[5], x.z, w.z);
  fma_pair(acc[6], acc[7], x.w, w.w);
}

// RMSNorm inverse of one BF16 row held in shared memory, by one warp, with
// the reference law (normalization.cu:82-186, by width).
__device__ __forceinline__ float rms_inverse_smem(const bf16* x, int width, float eps) {
  const int lane = threadIdx.x & 31;
  float part[4] = {0.f, 0.f, 0.f, 0.f};
  if (width <= 128) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = lane + 32 * c;
      if (col < width) {
        const float v = widen(x[col]);
        part[c] = __fmul_rn(v, v);
      }
    }
  } else {
    for (int base = 4 * lane; base < width; base += 128) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (base + c < width) {
          const float v = widen(x[base + c]);
          part[c] = __fadd_rn(part[c], __fmul_rn(v, v));
        }
      }
    }
  }
  float sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  sum = shuffle_down_tree32(sum);
  const float total = __shfl_sync(0xffffffffu, sum, 0);
  const float mean = __fmul_rn(total, 1.0f / static_cast<float>(width));
  return rsqrtf(__fadd_rn(mean, eps));
}

// SwiGLU law (reference elementwise.cu:62-87 with Silu) on BF16 gate/up.
__device__ __forceinline__ float swiglu(float a, float b) {
  const float e = expf(a >= 0.0f ? -a : a);
  const float s = a >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
  return round_bf16(__fmul_rn(round_bf16(__fmul_rn(a, s)), b));
}

// Greedy order: larger value first, then the smaller ID.
__device__ __forceinline__ bool better(float v, unsigned id, float bv, unsigned bid) {
  return v > bv || (v == bv && id < bid);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// One full tensor-map stage: KC features of this thread's row.  Boxes are
// [tile rows x 64 features] with the 128-byte swizzle, box_bytes apart.
template <int ROWS, int P, int KC>
__device__ __forceinline__ void stage_map(const unsigned char* stage, int box_bytes, int row, int slot,
                                          const bf16* xs, int I, int k0, float (&acc)[ROWS][8]) {
  const unsigned char* rbase = stage + row * 128;
  const int swz = row & 7;
#pragma unroll
  for (int m = 0; m < KC / P; ++m) {
    const int b = (P * m) >> 6;                              // box (compile-time)
    const int c = (((P * m) & 63) >> 3) + slot;              // chunk within the 128-byte row
    const uint4 w = sld16(rbase + b * box_bytes + ((c ^ swz) << 4));
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const uint4 xv = sld16(xs + size_t(r) * I + k0 + P * m + 8 * slot);
      fma8(acc[r], xv, w);
    }
  }
}

// One full stage loaded through a 3D map as a dense [blocks][tile_rows][128 B]
// box: the 128-byte swizzle follows the shared-memory address, so 128-byte
// line L = b * tile_rows + row has its 16-byte chunks permuted by L & 7
// (stage base 1024-byte aligned).  A quarter-warp reads 8 consecutive lines.
template <int ROWS, int P, int KC>
__device__ __forceinline__ void stage_dense(const unsigned char* stage, int tile_rows, int row, int slot,
                                            const bf16* xs, int I, int k0, float (&acc)[ROWS][8]) {
  // Partly unrolled: the persistent kernel inlines one copy per (P, KC) and
  // fully unrolled copies do not fit the instruction cache together.
#pragma unroll 4
  for (int m = 0; m < KC / P; ++m) {
    const int b = (P * m) >> 6;                              // feature block (compile-time)
    const int c = (((P * m) & 63) >> 3) + slot;              // 16-byte chunk within the line
    const int line = b * tile_rows + row;
    const uint4 w = sld16(stage + line * 128 + ((c ^ (line & 7)) << 4));
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const uint4 xv = sld16(xs + size_t(r) * I + k0 + P * m + 8 * slot);
      fma8(acc[r], xv, w);
    }
  }
}

// Generic stage (ragged tail or padded-row layout): guarded per 8 features.
template <int ROWS, int P, bool MAP>
__device__ __forceinline__ void stage_generic(const unsigned char* stage, int box_bytes, int row_stride,
                                              int row, int slot, const bf16* xs, int I, int k0, int kc,
                                              int nfeat, float (&acc)[ROWS][8]) {
  for (int m = 0; m < kc / P; ++m) {
    const int f = P * m + 8 * slot;
    if (f >= nfeat) continue;
    const unsigned char* wp;
    if constexpr (MAP) {
      const int c = (f & 63) >> 3;
      wp = stage + (f >> 6) * box_bytes + row * 128 + ((c ^ (row & 7)) << 4);
    } else {
      wp = stage + row * row_stride + 2 * f;
    }
    const uint4 w = sld16(wp);
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const uint4 xv = sld16(xs + size_t(r) * I + k0 + f);
      fma8(acc[r], xv, w);
    }
  }
}

}  // namespace gemv_dev

// Host: 2D tensor map of a row-major BF16 matrix [rows][cols] with boxes of
// [box_rows][64] and the 128-byte swizzle (gemv.cu).
bool encode_weight_map(CUtensorMap* map, const void* w, uint64_t rows, uint64_t cols, uint32_t box_rows);
// Host: 3D view {64 features, rows, cols/64 feature blocks} of the same
// matrix; one box is `blocks` feature blocks of [box_rows][64], written to
// shared memory densely as [blocks][box_rows][128 bytes] with the 128-byte
// swizzle, so one copy moves a whole stage.
bool encode_weight_map3d(CUtensorMap* map, const void* w, uint64_t rows, uint64_t cols, uint32_t box_rows,
                         uint32_t blocks);

}  // namespace dl
