// Launchers for steering.cu.
#pragma once

#include <algorithm>

#include "common.cuh"

namespace dl {
cudaError_t launch_intervene(bf16* residual, const float* direction, const long long* position, unsigned* state,
                             int width, long long selected, int rows, float strength, cudaStream_t stream,
                             bool pdl);
cudaError_t launch_copy_rows(const bf16* src, bf16* arena, const long long* position, int width, int rows,
                             cudaStream_t stream, bool pdl);
cudaError_t launch_direction(bool bf16_input, const void* original, const void* edited, float* out,
                             unsigned* status, int width, cudaStream_t stream);
cudaError_t launch_normalize_injection(const bf16* source, bf16* out, float* norm, unsigned* status,
                                       int width, float scale, cudaStream_t stream);
}  // namespace dl
