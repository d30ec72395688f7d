// Kernels of the batched serving step (serve_kernels.cu): lockstep batches of
// sequences, each with its own KV arena, and tensor-parallel slices.
#pragma once

#include "launch.h"

namespace dl {

// Where block l's K / V rows of sequence b live: kv + b * seq_stride + k_off
// (or v_off) + position * (kv_heads * width), elements.
struct KvPlanes {
  bf16* kv;
  size_t seq_stride;
  size_t k_off, v_off;
};

// Rows [r0, r0 + rows) x columns [c0, c0 + cols) of the seeded tensor with
// `full_cols` columns (element index r * full_cols + c), into out (row stride
// out_stride): any tensor-parallel slice of the same weights.
cudaError_t launch_fill_normal_slice(bf16* out, size_t rows, size_t cols, size_t out_stride, size_t full_cols,
                                     size_t r0, size_t c0, uint64_t seed, uint32_t stream_id, float scale,
                                     cudaStream_t stream);

// Batched decode: row b of qkv [B][Hq*d + 2*Hkv*d] (row stride ld) is
// sequence b's token at the shared position *position.  Queries get QK-norm
// + RoPE into q_out [B][Hq][d]; keys get QK-norm + RoPE and values are copied,
// both into sequence b's cache at that position.  pdl: launched as a
// programmatic dependent of the previous kernel.
cudaError_t launch_norm_rope_append_rows(const bf16* qkv, int ld, const bf16* q_norm_w, const bf16* k_norm_w,
                                         const float* inv_freq, bf16* q_out, KvPlanes planes,
                                         const long long* position, int batch, int query_heads, int kv_heads,
                                         int width, float eps, cudaStream_t stream, bool pdl = false);

// residual[m] = round(residual[m] + round(sum of parts [splits][M][N] in part
// order)), then xn[m] = RMSNorm(residual[m]) * w (the RMSNorm rows law, N >
// 128, N % 8 == 0, N <= 8192): the row-parallel projection's residual
// epilogue and the following norm as one launch of M CTAs.
cudaError_t launch_residual_norm_rows(const float* parts, int splits, int M, int N, bf16* residual, const bf16* w,
                                      bf16* xn, float eps, cudaStream_t stream, bool pdl);

// Split-K flash decoding: for every sequence b and query head h, attention of
// q [B][Hq][128] over keys 0 .. *position of b's cache, the keys cut into
// `splits` ranges whose (max, sum, unnormalised output) go to ws
// [B][Hq][splits][130] FP32, merged into out [B][Hq*128] BF16 by the combine
// kernel.  Online softmax: not the reference's reduction order.  The ranges
// are even, or (lead_q10 > 0, two splits) a first range of lead_q10 / 1024
// of the keys (rounded up to 64-key tiles) and the rest.
size_t attention_decode_ws_floats(int batch, int query_heads, int splits);
// Even splits by a wave-cost model (two resident CTAs per SM).
int attention_decode_splits(int batch, int kv_heads, int capacity, int sms);
struct AttnPlan {
  int splits;
  int lead_q10;  // 0: even ranges
};
// The even splits, or a leading range when fewer (sequence, KV head) units
// than CTA slots would leave slots idle for the whole launch.
AttnPlan attention_decode_plan(int batch, int kv_heads, int capacity, int sms);
// tickets ([B][Hkv] int, zeroed once; each launch leaves them zero): the
// last split of each (sequence, KV head) merges the splits itself, no
// combine launch (with one split the CTA writes O / l directly).  pdl:
// programmatic dependent launch (the key tiles before the newest position
// are requested before waiting for the previous kernel).
// qkv (optional): the batch's qkv projection as split-K parts [splits][M][ld]
// FP32 (ld = (Hq + 2 Hkv) * 128).  Each CTA then builds its group's queries
// itself (parts summed in part order and rounded to BF16, QK-norm + RoPE with
// the same warp routine as launch_norm_rope_append_rows), and the split that
// holds the newest position appends that position's key (QK-norm + RoPE) and
// value to the cache before reading it; q is not read.
struct AttnQkvIn {
  const float* parts;
  int splits, M, ld;
  const bf16* q_norm;
  const bf16* k_norm;
  const float* inv_freq;
  float eps;
};
cudaError_t launch_attention_decode_batched(const bf16* q, KvPlanes planes, const long long* position, int batch,
                                            int query_heads, int kv_heads, int splits, int lead_q10, float scale,
                                            float* ws, bf16* out, cudaStream_t stream, int* tickets = nullptr,
                                            bool pdl = false, const AttnQkvIn* qkv = nullptr);

// Vocabulary-split head: src [t][B][Vp] (rank r's logits of vocabulary rows
// [r Vl, (r+1) Vl) in its first Vl columns) -> dst [B][t Vl].
cudaError_t launch_gather_vocab_slices(const bf16* src, bf16* dst, int ranks, int batch, int vl, int vp,
                                       cudaStream_t stream);

// residual[m][n] = round(residual + round(sum[m][n])): the residual epilogue
// applied to an FP32 sum (after the tensor-parallel all-reduce).
cudaError_t launch_add_fp32_residual(const float* sum, bf16* residual, size_t n, cudaStream_t stream);

// Tensor-parallel all-reduce of the row-parallel projections over NVLink peer
// memory, fused with the split-K sum, the residual add and (norm_w) the next
// RMSNorm: CTA `row` sums this rank's split-K parts of its row [splits][M][N]
// in part order and writes the FP32 row into slot `rank` of every rank's
// buffer (peer pointers from CUDA IPC), raises flag (rank, row) on each with
// the call's epoch, waits (bounded) for every rank's flag `row` on its own
// buffer, then adds the slots in rank order (the same sum on every rank) and
// applies residual = round(residual + round(sum)); with norm_w it writes xn =
// RMSNorm(residual row) * norm_w (the RMSNorm rows law).  Buffers alternate by
// epoch parity so a rank running one call ahead never overwrites a slot still
// being read.  M <= kPeerChunks; pdl: programmatic dependent launch.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerChunks = 128;  // rows per call (one CTA each)
struct PeerBuffers {
  float* data[kPeerMaxRanks];       // [2][ranks][capacity] FP32 on each rank
  unsigned* flags[kPeerMaxRanks];   // [2][ranks][kPeerChunks] on each rank
  unsigned* epoch;                  // this rank: calls so far, per CTA [kPeerChunks]
  unsigned* err;
  int ranks, rank;
  size_t capacity;                  // floats per slot
};
size_t peer_buffer_bytes(int ranks, size_t capacity);  // data + flags, one rank
cudaError_t launch_peer_allreduce_residual(const PeerBuffers& pb, const float* parts, int splits, int M, int N,
                                           bf16* residual, const bf16* norm_w, bf16* xn, float eps,
                                           cudaStream_t stream, bool pdl);

}  // namespace dl
