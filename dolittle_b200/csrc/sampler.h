// Device token selection (role of the reference's DeviceCategorical,
// src/inference/sampling/device.h:54-85).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/dolittle_b200.h"
#include "common.cuh"

namespace dl {

struct SamplerState;  // device-resident MT19937-64 words + latches

// One sampler serves `rows` logits rows at once (every kernel launches with
// gridDim.y = rows); row r owns the arena slice at r * stride bytes and draws
// from the device-owned stream (MT19937-64, or Philox4x32-10 when selected)
// seeded with seed + r.
struct Sampler {
  size_t vocabulary = 0;
  bool bf16_input = true;
  unsigned rows = 1;
  size_t stride = 0;           // bytes per row's arena slice
  void* arena = nullptr;       // device scratch (rows * stride)
  SamplerState* state = nullptr;
  unsigned* result = nullptr;  // {token, status} of row 0 (sampler_result for row r)
  unsigned char* stop_mask = nullptr;
  dl_sampling settings = {0, 1.0, 0, 1.0};
  bool started = false;
  unsigned engine = DL_RNG_MT19937_64;  // draw source of the device-owned stream (set before start)
};

// Settings law of src/inference/sampling/categorical.cpp:37-47; throws
// std::invalid_argument like the reference.
void validate_sampling(const dl_sampling& s, size_t vocabulary);

size_t sampler_required_bytes(size_t vocabulary);
cudaError_t sampler_init(Sampler& s, size_t vocabulary, bool bf16_input, unsigned rows = 1);
void sampler_free(Sampler& s);
cudaError_t sampler_start(Sampler& s, const dl_sampling& settings, uint64_t seed, const uint32_t* stop_ids,
                          size_t n_stop, cudaStream_t stream);
// owned = device-owned MT stream (submit_next); otherwise `bits` is the draw.
// Row r's logits are at row + r * row_stride elements.
cudaError_t sampler_submit(Sampler& s, const void* row, const dl_sampling& settings, uint64_t bits, bool owned,
                           cudaStream_t stream, size_t row_stride = 0);
// Kernels one sampler_submit enqueues (for launch accounting).
int sampler_launch_count(const Sampler& s, const dl_sampling& settings, bool owned);
// After a selection, per row r: history[r * history_stride + step[r]] =
// token, ++step[r], residual row r = embed[token]; ++*position once (each
// optional).
cudaError_t sampler_feed(Sampler& s, unsigned* history, int* step, const bf16* embed, bf16* residual,
                         int width, long long* position, cudaStream_t stream, size_t history_stride = 0);
unsigned* sampler_result(const Sampler& s, unsigned row);

}  // namespace dl
