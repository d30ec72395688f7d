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
// Fixed-strength steering (steering.cu): beta = alpha * ||row|| (intervene
// norm law); rows at positions >= first of the masked sequences get
// h' = round(h + beta * u).  Row r is at (position ? *position : base) + r
// of sequence 0 of mask, or (per_sequence) at *position of sequence r.
cudaError_t launch_steer_beta(const bf16* row, int width, float alpha, float* beta, unsigned* err,
                              cudaStream_t stream);
cudaError_t launch_steer_rows(bf16* residual, int width, int rows, const long long* position, long long base,
                              bool per_sequence, const unsigned char* mask, long long first, const float* beta,
                              const float* direction, unsigned* err, cudaStream_t stream);
// arena[b * seq_stride + (*position) * width ...] = rows[b] for b < batch.
cudaError_t launch_capture_batch(const bf16* rows, bf16* arena, size_t seq_stride, const long long* position,
                                 int width, int batch, cudaStream_t stream);
cudaError_t launch_direction(bool bf16_input, const void* original, const void* edited, float* out,
                             unsigned* status, int width, cudaStream_t stream);
cudaError_t launch_normalize_injection(const bf16* source, bf16* out, float* norm, unsigned* status,
                                       int width, float scale, cudaStream_t stream);
}  // namespace dl
