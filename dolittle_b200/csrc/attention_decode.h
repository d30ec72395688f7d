// Decode attention (one query row): fused QK-norm/RoPE/K-append + scores,
// then softmax + PV sharing V loads across the GQA group.
#pragma once

#include "launch.h"

namespace dl {

bool attention_decode_supported(int query_heads, int kv_heads, int width, int capacity);
cudaError_t launch_attention_decode(const bf16* q_raw, const bf16* k_raw, const bf16* q_norm_w,
                                    const bf16* k_norm_w, const float* inv_freq, bf16* k_cache,
                                    const bf16* v_cache, float* scores, bf16* out, const long long* position,
                                    int query_heads, int kv_heads, int width, int capacity, float eps,
                                    int key_slices, cudaStream_t stream, bool pdl);

}  // namespace dl
