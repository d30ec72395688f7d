// Host-side launch helpers shared by the C ABI (capi.cu) and the engine.
// All launches enqueue on the given stream only: no allocation, transfer or
// host wait (the contract of the reference's src/kernels/cuda/launch.h).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "common.cuh"

namespace dl {

struct GemvArgs;

// gemv.cu
size_t gemv_smem_bytes(int rows, int in_width, int stage_bytes, int stages);
cudaError_t launch_gemv(GemvArgs a, int rows_template, int grid, cudaStream_t stream, bool pdl);
int gemv_rows_template(int rows, int in_width);
inline int projection_partials(size_t in_width, size_t out_width) {
  return (in_width <= 4096 && out_width > 1024) ? 16 : 32;
}

// ops.cu
struct RowPositions {
  const long long* device;  // device position of row 0 (nullptr: use host)
  long long host;
};

cudaError_t launch_qk_norm_rope(const bf16* q_raw, const bf16* k_raw, const bf16* q_norm_w,
                                const bf16* k_norm_w, const float* inv_freq, bf16* q_out,
                                bf16* k_cache, RowPositions pos, int rows, int query_heads,
                                int kv_heads, int width, float eps, cudaStream_t stream, bool pdl);
cudaError_t launch_attention_scores(const bf16* q, const bf16* k_cache, float* scores,
                                    RowPositions pos, int rows, int query_heads, int kv_heads,
                                    int width, int capacity, float scale, int ctas_per_head,
                                    cudaStream_t stream, bool pdl);
cudaError_t launch_attention_pv(const float* scores, const bf16* v_cache, bf16* out,
                                RowPositions pos, int rows, int query_heads, int kv_heads,
                                int width, int capacity, cudaStream_t stream, bool pdl);
cudaError_t launch_embedding(const uint32_t* tokens, const bf16* table, bf16* out, int rows,
                             int width, cudaStream_t stream, bool pdl);
cudaError_t launch_add(const bf16* a, const bf16* b, bf16* out, size_t n, cudaStream_t stream);
cudaError_t launch_silu_multiply(const bf16* g, const bf16* u, bf16* out, size_t n,
                                 cudaStream_t stream);
cudaError_t launch_rms_norm(const bf16* x, const bf16* w, bf16* out, size_t rows, int width,
                            float eps, cudaStream_t stream, bool pdl = false);
cudaError_t launch_rotary(const bf16* x, bf16* out, size_t positions, int heads, int width,
                          RowPositions pos, double theta, bool positioned_output,
                          cudaStream_t stream);
cudaError_t launch_inv_freq(float* out, int width, double theta, cudaStream_t stream);
cudaError_t launch_fill_normal(bf16* out, size_t rows, size_t cols, size_t row_stride, uint64_t seed,
                               uint32_t stream_id, float scale, cudaStream_t stream);
cudaError_t launch_fill_const(bf16* out, size_t n, float value, cudaStream_t stream);
cudaError_t launch_uniform_ids(uint32_t* out, size_t n, uint64_t seed, uint32_t stream_id,
                               uint32_t bound, cudaStream_t stream);
cudaError_t launch_add_position(long long* value, long long delta, cudaStream_t stream);

// capi.cu: message returned by dl_last_error() on the calling thread.
void set_last_error(const std::string& message);

inline float attention_scale(int width) {
  return static_cast<float>(1.0 / __builtin_sqrt(static_cast<double>(width)));
}

}  // namespace dl
