// Streaming BF16 GEMV/skinny-GEMM with the reference's projection law.
//
// Law (reference src/kernels/cuda/projection.cu:277-426): output o of input
// row r is the halving-tree sum of P strided partial chains; partial j is the
// serial __fmaf_rn chain over features j, j+P, j+2P, ... in ascending order;
// features in [I, ceil16(I)) add one fma(0,0,p) (the tiled path's zero
// padding); P = 16 when I <= 4096 and O > 1024, else 32; one BF16 rounding.
// Products of two BF16 values are exact in FP32, so the mixed-precision
// fma.rn.f32.bf16 (BF16 operands, FP32 addend, one rounding) computes exactly
// __fmaf_rn(float(x), float(w), acc).
//
// B200 mapping.  Each CTA owns a contiguous range of weight rows and streams
// it through a ring of shared-memory stages.  Each stage is loaded by the TMA
// engine as 2D tensor-map boxes of [tile rows x 64 features] with the 128-byte
// swizzle (one instruction moves a whole box; the swizzle makes the consumer's
// 128-bit shared loads conflict-free), with an L2 evict-first policy.  A
// producer warp keeps the ring full; consumer threads each own 8 consecutive
// partials of one row, so a row is worked by P/8 threads and every chain keeps
// its order.  Lanes are laid out so that each quarter-warp reads 8 different
// rows (the 8 swizzle phases).  The producer starts streaming before
// griddepcontrol.wait, so with PDL the weight fetch overlaps the previous
// kernel's tail.  Matrices narrower than 64 features use per-row bulk copies
// into 16-byte-padded rows instead.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace dl {

constexpr int kGemvConsumers = 256;             // consumer threads (8 warps)
constexpr int kGemvThreads = kGemvConsumers + 32;
constexpr int kGemvMaxSegs = 3;
constexpr int kGemvSmemBudget = 200 * 1024;
constexpr int kGemvBox = 64;                     // features per TMA box (128 B)

enum GemvPrologue : int {
  kProloguePlain = 0,    // x rows are BF16 in global memory
  kPrologueRmsNorm = 1,  // x = RMSNorm(x_rows, norm_w) with the reference law
};

enum GemvEpilogue : int {
  kEpilogueStore = 0,     // out[r*stride + o] = bf16(y)
  kEpilogueResidual = 1,  // out[r*stride + o] = round(out + round(y)) in place
  kEpilogueArgmax = 2,    // store logits + greedy selection (one input row)
  kEpilogueSwiGLU = 3,    // rows (2o, 2o+1) = (gate o, up o):
                          // out[r*stride + o] = round(round(g*sigmoid(g))*u)
};

struct alignas(64) GemvSegment {
  CUtensorMap map;        // 2D map of w, box [tile_rows][64] (tensor-map path)
  const bf16* w;          // [rows][I] row-major, contiguous
  bf16* out;              // output base
  const long long* out_row;  // optional device row index: out += (*out_row) * out_stride
  int rows;               // weight rows of this segment
  int partials;           // P: 16 or 32
  int cta_begin;          // first CTA of this segment
  int cta_count;          // CTAs assigned to it
  int out_stride;         // elements between input rows in the output
  int tile_rows;          // rows per tile (= TMA box rows)
  int rows_per_cta;       // contiguous rows owned by one CTA
};

inline GemvSegment make_segment(const bf16* w, bf16* out, const long long* out_row, int rows, int partials,
                                int out_stride) {
  GemvSegment s{};
  s.w = w;
  s.out = out;
  s.out_row = out_row;
  s.rows = rows;
  s.partials = partials;
  s.out_stride = out_stride;
  return s;
}

// Greedy selection finish (argmax epilogue), run by the last CTA.
struct SelectOutput {
  unsigned* result;       // {token, status}; status 1 = NaN/+inf, 2 = no finite best
  unsigned* history;      // optional: history[*step] = token
  int* step;              // optional counter, incremented
  const bf16* embed;      // optional: next residual row = embed[token]
  bf16* residual;
  int width;
  long long* position;    // optional: ++*position after the step
  const unsigned char* stop_mask;  // optional stop-ID latch
  unsigned* terminal;     // latched terminal flag (stop ID or error)
};

struct alignas(64) GemvArgs {
  GemvSegment seg[kGemvMaxSegs];
  const bf16* x;          // input rows (or residual for RMSNorm)
  int x_stride;           // elements between input rows
  int in_width;           // I
  int nrows;              // input rows this launch (<= ROWS template)
  int prologue;
  const bf16* norm_w;
  float eps;
  int epilogue;
  bf16* capture;          // optional second copy of residual outputs
  const long long* capture_row;  // device row index of the capture copy
  int capture_stride;
  int nseg;
  int use_map;            // 1: tensor-map boxes, 0: per-row bulk copies
  int kc;                 // features per stage
  int stages;             // ring depth
  int stage_bytes;        // bytes per stage
  int row_stride;         // padded row bytes (bulk-copy path)
  uint4* partials;        // argmax: per-CTA {value bits, id, flags, 0}
  unsigned* ticket;       // argmax: completion counter (self-resetting)
  SelectOutput select;
  unsigned* err;
};

}  // namespace dl
