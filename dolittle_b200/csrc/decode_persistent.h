// Persistent decode step: one cooperative launch runs a whole single-row
// forward pass (every block and the vocabulary head) on one CTA per SM.
//
// Why: a batch-1 decode step streams 15.1 GB of weights and does little else.
// As separate kernels, every projection pays a ramp-up and a drain, and HBM
// idles through the attention kernels and launch gaps.  Here a producer warp
// per SM streams that SM's share of every weight matrix, phase after phase,
// through one TMA ring that never drains: it runs ahead across grid barriers,
// attention and norms, so the next projection's weights are already in shared
// memory when its input vector is ready.
//
// Phases per block (grid barrier after each):
//   qkv   RMSNorm prologue; q, k rows -> scratch, v rows -> V cache row S
//   score QK-norm + RoPE for each GQA group, new key -> K cache, scaled scores
//   pv    softmax law per query head, two-halves PV chains -> attention rows
//   o     projection + residual epilogue (in place)
//   gu    RMSNorm prologue; interleaved gate|up rows, SwiGLU epilogue
//   down  projection + residual epilogue (+ block-output capture)
//   edit  (steered block only) one-shot steering edit of the selected row
// then the vocabulary head (final RMSNorm, logits, greedy selection with
// token feedback, or logits only for the categorical sampler).
//
// Every phase computes exactly the reference's arithmetic (the same device
// functions as the stand-alone kernels), so the results are bit-identical to
// the multi-kernel path.  Grid barriers and ring waits are bounded: a barrier
// that does not complete in ~2 s records an error word and the kernel unwinds.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gemv.cuh"

namespace dl {

constexpr int kPersistSlots = 6;
constexpr int kPersistSlotBytes = 32 * 1024;
constexpr int kPersistHeaderBytes = 2048;
constexpr int kPersistUnionBytes = 30 * 1024;  // x row, or attention scratch
constexpr int kPersistSmem =
    kPersistHeaderBytes + kPersistUnionBytes + 1024 /* ring alignment */ + kPersistSlots * kPersistSlotBytes;
constexpr int kPersistMaxInput = 12288;     // projection input width (features)
constexpr int kPersistMaxNormInput = 4096;  // width of an RMSNorm prologue input
// L2 prefetch burst (stages past the ring) per attention stall.  The phases
// already stream at the HBM read rate (~7.8 TB/s) and L2 hits do not arrive
// faster, so longer bursts only compete with the attention loads: 12 measured
// best (0 to 40 span ~1 %).
constexpr int kPersistPrefetchStages = 12;

struct PSeg {
  const CUtensorMap* map;    // device copy, 3D box {64, tile_rows, kc / 64}
  bf16* out;
  const long long* out_row;  // optional device row index: out += (*out_row) * out_stride
  int rows, partials, cta_begin, cta_count;
  int rows_per_cta, tile_rows, out_stride, kc;
};

struct alignas(16) PGemv {
  const bf16* x;       // input row
  const bf16* norm_w;  // RMSNorm prologue weight (nullptr: plain input)
  int in_width, epilogue, nseg, pad;
  PSeg seg[kGemvMaxSegs];
};

struct PLayer {
  PGemv qkv, o, gu, down;
  // Attention operands (16-byte aligned: copied to shared memory together).
  const bf16* q_norm;
  const bf16* k_norm;
  bf16* k_cache;
  const bf16* v_cache;
};

struct PersistArgs {
  const PLayer* layers;
  int nlayers;
  PGemv head;
  const bf16* q_raw;
  const bf16* k_raw;
  float* scores;        // [Hq][score_stride]
  bf16* att;            // [Hq * d]
  bf16* residual;       // [D]
  const float* inv_freq;
  const long long* position;
  int hidden, query_heads, kv_heads, width, capacity;
  float scale, eps;
  int score_stride;     // capacity rounded up to 4 (16-byte score rows)
  int score_slices, pv_features;
  int prefetch_stages;  // producer L2 prefetch distance
  // block-output capture and one-shot steering
  bf16* capture;        // arena [capacity][D] or nullptr
  int capture_layer;
  int edit_layer;
  long long edit_row;
  float edit_strength;
  const float* edit_direction;
  unsigned* edit_state;
  // greedy selection in the head epilogue
  uint4* partials;
  unsigned* ticket;
  SelectOutput select;
  unsigned* barrier;       // grid barrier arrivals (reset by the last CTA)
  unsigned* exit_ticket;
  unsigned* err;
};

// Host planning of one projection phase over `grid` CTAs: CTA ranges by
// bytes, tile rows, features per stage, and the tensor maps (written to
// maps[0..nseg), host memory; the caller copies them to the device and
// points seg[i].map at the copies).  Returns false when the shape does not
// fit the persistent kernel.
struct PSegSpec {
  const bf16* w;
  bf16* out;
  const long long* out_row;
  int rows, partials, out_stride;
};
bool plan_persist_gemv(PGemv& g, const PSegSpec* specs, int nseg, const bf16* x, const bf16* norm_w,
                       int in_width, int epilogue, int grid, CUtensorMap* maps);

// True when the kernel can run `grid` co-resident CTAs on this device.
bool decode_persistent_fits(int grid);
cudaError_t launch_decode_persistent(const PersistArgs& a, int grid, cudaStream_t stream);

}  // namespace dl
