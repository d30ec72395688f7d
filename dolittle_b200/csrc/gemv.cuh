// Streaming BF16 GEMV/skinny-GEMM with the reference's projection law.
//
// Law (reference src/kernels/cuda/projection.cu:277-426): output o of input
// row r is the halving-tree sum of P strided partial chains; partial j is the
// serial __fmaf_rn chain over features j, j+P, j+2P, ... in ascending order;
// features in [I, ceil16(I)) add one fma(0,0,p) (the tiled path's zero
// padding); P = 16 when I <= 4096 and O > 1024, else 32; one BF16 rounding.
//
// B200 mapping.  Each CTA owns a contiguous range of weight rows (so its work
// is one contiguous slab of HBM) and streams it through a ring of shared-
// memory stages with the TMA engine (cp.async.bulk, one piece per row per
// stage, L2 evict-first).  A producer warp keeps the ring full; consumer
// threads each own 8 consecutive partials of one row (128-bit shared loads),
// so a row is worked by P/8 threads and every chain keeps its order.  Rows
// are padded by 16 B in shared memory and lanes are laid out so that each
// quarter-warp reads 8 different rows: conflict-free LDS.128.  The producer
// starts streaming before griddepcontrol.wait, so with PDL the weight fetch
// overlaps the previous kernel's tail.
#pragma once

#include "common.cuh"

namespace dl {

constexpr int kGemvConsumers = 128;             // consumer threads (4 warps)
constexpr int kGemvThreads = kGemvConsumers + 32;
constexpr int kGemvMaxSegs = 3;
constexpr int kGemvSmemBudget = 200 * 1024;

enum GemvPrologue : int {
  kProloguePlain = 0,    // x rows are BF16 in global memory
  kPrologueRmsNorm = 1,  // x = RMSNorm(x_rows, norm_w) with the reference law
  kPrologueSwiGLU = 2,   // x = round(round(g*sigmoid(g))*u), g = x[0:I], u = x[I:2I]
};

enum GemvEpilogue : int {
  kEpilogueStore = 0,     // out[r*stride + o] = bf16(y)
  kEpilogueResidual = 1,  // out[r*stride + o] = round(out + round(y)) in place
  kEpilogueArgmax = 2,    // store logits + greedy selection (one input row)
};

struct GemvSegment {
  const bf16* w;          // [rows][I] row-major, contiguous
  bf16* out;              // output base
  const long long* out_row;  // optional device row index: out += (*out_row) * out_stride
  int rows;               // output width of this segment
  int partials;           // P: 16 or 32
  int cta_begin;          // first CTA of this segment
  int cta_count;          // CTAs assigned to it
  int out_stride;         // elements between input rows in the output
};

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

struct GemvArgs {
  const bf16* x;          // input rows (or residual for RMSNorm, or gate|up)
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
  GemvSegment seg[kGemvMaxSegs];
  int kc;                 // features per stage (multiple of 32)
  int stages;             // ring depth
  int max_tile_rows;
  uint4* partials;        // argmax: per-CTA {value bits, id, flags, 0}
  unsigned* ticket;       // argmax: completion counter (self-resetting)
  SelectOutput select;
  unsigned* err;
};

}  // namespace dl
