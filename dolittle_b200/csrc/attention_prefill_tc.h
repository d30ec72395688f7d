// Causal GQA prompt attention on tcgen05 tensor cores (attention_prefill_tc.cu).
#pragma once

#include "launch.h"

namespace dl {

struct AttnTcMaps;

bool attention_prefill_tc_supported(int query_heads, int kv_heads, int width);
// Tensor maps over the rotated queries [max_rows][Hq][d], the KV arena
// (block l's K at 2l * kv_block_bytes, V at (2l + 1) * kv_block_bytes, each
// [capacity][Hkv][d]) and the transposed-V scratch [Hkv][d][vt_stride].
// nullptr when unsupported.
AttnTcMaps* attention_prefill_tc_maps(const bf16* q, int max_rows, int query_heads, const bf16* kv_arena,
                                      size_t kv_block_bytes, int capacity, int layers, int kv_heads, int width,
                                      const bf16* vt, int vt_stride);
void attention_prefill_tc_free(AttnTcMaps* maps);
// pdl: programmatic dependent launch (both kernels wait for the previous
// kernel's completion before reading its results).
cudaError_t launch_vt_transpose(const bf16* v_cache, bf16* vt, int keys, int kv_heads, int width, int vt_stride,
                                cudaStream_t stream, bool pdl = false);
// out[rows][Hq * d] for query rows at absolute positions first .. first+rows-1
// of block `layer`; keys 0 .. first+rows-1 (the cache already holds them).
cudaError_t launch_attention_prefill_tc(const AttnTcMaps* maps, bf16* out, int rows, long long first, int layer,
                                        int query_heads, int kv_heads, float scale, unsigned* err,
                                        cudaStream_t stream, bool pdl = false);

}  // namespace dl
