// tcgen05/TMEM GEMM for prefill projections (see gemm_tcgen05.cu).
#pragma once

#include "launch.h"

namespace dl {

enum GemmEpilogue : int {
  kGemmStore = 0,     // out = bf16(acc)
  kGemmResidual = 1,  // out = round(out + round(acc)) in place
  kGemmSwiGLU = 3,    // columns (2o, 2o+1) = (gate o, up o): out[o] = SwiGLU law
};

struct GemmProblem {
  const bf16* x;      // [M][K], row stride ldx
  int ldx;
  const bf16* w;      // [N][K] contiguous
  int M, N, K;
  int epilogue;
  int nseg;           // outputs by column range: columns [seg_n0[i], seg_n0[i+1])
  int seg_n0[3];
  bf16* seg_out[3];   // output of segment i (column 0 of the segment)
  int seg_ld[3];      // output row stride (elements)
  bool wide_tiles;    // allow 128 x 256 tiles
  unsigned* err;
  // Optional split-K workspace (both or neither): room for FP32 partials
  // (partial_floats >= gemm_split_floats(M, N, parts)) and n_tickets per-tile tickets (zeroed,
  // left zeroed).  With them, shapes that would leave SMs idle run as up to
  // kGemmMaxSplit K parts whose last finisher adds the parts in part order
  // and applies the epilogue.
  float* partial;
  size_t partial_floats;
  unsigned* tickets;
  int n_tickets;
  // Tuning overrides (0 = chosen by the launcher): tile height 128 (one SM)
  // or 256 (a CTA pair, 256 wide), tile width 128 / 256, the number of K parts.
  int force_bm, force_bn, force_split;
  // Stream-K (single-SM tiles, needs the workspace): 0 = by the cost model,
  // 1 = always, -1 = never.
  int force_streamk;
};

constexpr int kGemmMaxSplit = 4;

bool gemm_tcgen05_supported(int M, int N, int K);
// FP32 workspace of `parts` K parts: one plane of N columns x M rows rounded
// up to 256 per part.
size_t gemm_split_floats(int M, int N, int parts);
cudaError_t launch_gemm_tcgen05(const GemmProblem& p, cudaStream_t stream, bool pdl);

// Split-K for few rows (batched decode): the K extent in `splits` parts
// (k-steps [h kt / splits, (h + 1) kt / splits) for part h),
// each (tile, part) unit storing its FP32 partial into parts[splits][M][N];
// then the epilogue kernel adds the parts in part order and applies
// `epilogue` into out (row stride ld), or writes the FP32 sum to sum_out.
// Only p.x, p.ldx, p.w, M, N, K and err are read from p.
int gemm_splitk_parts(int M, int N, int K, int sms);  // parts that fill the SMs
// pdl: programmatic dependent launch (weights stream in before the kernel
// waits for its predecessor).
cudaError_t launch_gemm_tcgen05_parts(const GemmProblem& p, int splits, float* parts, cudaStream_t stream,
                                      bool pdl = false);
cudaError_t launch_gemm_splitk_epilogue(const float* parts, int splits, int M, int N, int epilogue, bf16* out,
                                        int ld, float* sum_out, cudaStream_t stream, bool pdl = false);

}  // namespace dl
