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

struct Sampler {
  size_t vocabulary = 0;
  bool bf16_input = true;
  void* arena = nullptr;       // device scratch (sampler_required_bytes)
  SamplerState* state = nullptr;
  unsigned* result = nullptr;  // {token, status}
  unsigned char* stop_mask = nullptr;
  dl_sampling settings = {0, 1.0, 0, 1.0};
  bool started = false;
};

// Settings law of src/inference/sampling/categorical.cpp:37-47; throws
// std::invalid_argument like the reference.
void validate_sampling(const dl_sampling& s, size_t vocabulary);

size_t sampler_required_bytes(size_t vocabulary);
cudaError_t sampler_init(Sampler& s, size_t vocabulary, bool bf16_input);
void sampler_free(Sampler& s);
cudaError_t sampler_start(Sampler& s, const dl_sampling& settings, uint64_t seed, const uint32_t* stop_ids,
                          size_t n_stop, cudaStream_t stream);
// owned = device-owned MT stream (submit_next); otherwise `bits` is the draw.
cudaError_t sampler_submit(Sampler& s, const void* row, const dl_sampling& settings, uint64_t bits, bool owned,
                           cudaStream_t stream);
// Kernels one sampler_submit enqueues (for launch accounting).
int sampler_launch_count(const Sampler& s, const dl_sampling& settings, bool owned);
// After a selection: history[*step] = token, ++*step, residual = embed[token],
// ++*position (each optional).
cudaError_t sampler_feed(Sampler& s, unsigned* history, int* step, const bf16* embed, bf16* residual,
                         int width, long long* position, cudaStream_t stream);

}  // namespace dl
