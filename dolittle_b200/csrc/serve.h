// Server: lockstep batched serving of B sequences on one GPU, or on one rank
// of a tensor-parallel group over KV-head groups.  The long-context serving
// workload of the reference runs each sequence through CachedForwardPlan
// (src/inference/executor.cpp:1482-1716) one at a time; here the B sequences
// share every weight read:
//  * prompt pass per sequence in chunks: tcgen05 GEMMs (M = chunk rows),
//    the tcgen05 causal attention over that sequence's cache;
//  * decode step for all B rows at once: split-K tcgen05 GEMMs (M = B), the
//    exact QK-norm + RoPE + KV append, split-K flash decoding over each
//    sequence's cache, per-row sampling;
//  * tensor parallelism over KV-head groups (rank r of t holds query heads
//    [r Hq/t, (r+1) Hq/t), the matching KV heads and MLP columns): q/k/v and
//    gate/up are column slices, o_proj and down_proj row slices whose FP32
//    partial sums meet in an NCCL all-reduce before the residual add; the
//    vocabulary head is split by rows, its logits meeting in an all-gather.
// All sequences have the same prompt length and advance together, so one
// device position serves the batch.  The decode step is one CUDA graph
// (the all-reduces included).
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <vector>

#include "../../include/dolittle_b200.h"
#include "engine.h"
#include "sampler.h"
#include "serve_kernels.h"

namespace dl {

class Server {
 public:
  Server(const dl_model_config& cfg, int device, size_t batch, size_t capacity, size_t chunk_rows, int tp_rank,
         int tp_size);
  ~Server();

  static void nccl_id(unsigned char* out128);
  void connect(const unsigned char* id128);
  // NVLink peer all-reduce of the decode step: this rank's buffer handle,
  // then every rank's handles [tp][64] (CUDA IPC).
  void ipc_handle(unsigned char* out64);
  void connect_peers(const unsigned char* handles);
  void init_random(uint64_t seed, float sigma);
  void set_sampler_engine(int engine) { sampler_.engine = unsigned(engine); }
  // Full tensor `index` (engine order) from the host; this rank keeps its slice.
  void set_tensor(size_t index, const void* host, size_t bytes);
  // This rank's slice of tensor `index` ([rows][cols] as held).
  void get_tensor(size_t index, void* host, size_t bytes);
  bool slice_shape(size_t index, size_t* rows, size_t* cols, size_t* r0, size_t* c0);
  void prefill(const uint32_t* tokens, size_t prompt_len, const dl_sampling& s, uint64_t seed, uint32_t* first_out);
  void decode(size_t steps, uint32_t* tokens_out, uint16_t* logits_out, dl_serve_stats* stats);
  size_t position();
  // Block `layer`'s output rows of every sequence and position (prompt and
  // decode) into an arena [B][capacity][D]; layer < 0 disables.
  void set_capture(int layer);
  void read_capture(size_t sequence, size_t first, size_t count, uint16_t* host);
  // Fixed-strength steering of every position >= first at block `layer` for
  // the sequences in mask[B] (see dl_serve_set_steering); layer < 0 disables.
  void set_steering(int layer, size_t first, float strength, const float* direction, const uint8_t* mask,
                    long long source_sequence, size_t source_position);
  float steering_strength();
  // Fused decode step on (default) or off; both give the same bits.
  void set_step_fusion(bool on);

 private:
  struct Slice {
    bf16* ptr;
    size_t rows, cols, stride, r0, c0, full_cols;
  };
  Slice slice(size_t index);
  KvPlanes planes(size_t layer) const;
  bf16* vcache(size_t b, size_t layer) const;
  bf16* kcache(size_t b, size_t layer) const;
  void gemm(const bf16* x, int ldx, const bf16* w, int M, int N, int K, int epi, int nseg, const int* n0s,
            bf16* const* outs, const int* lds);
  void row_projection_out(const bf16* x, int ldx, const bf16* w, int M, int K, bool decode);  // o / down
  void decode_projection_norm(const bf16* x, int K, const bf16* w, int layer, const bf16* norm_w);
  bool fused_step() const;
  bool peer_decode(int rows) const;
  void prefill_sequence(size_t b, const uint32_t* tokens, size_t n);
  void block_output_hooks(size_t l, size_t b, size_t c0, int rows);  // prompt chunk rows of sequence b
  void block_output_hooks_decode(size_t l);
  void decode_body();
  void all_reduce(float* buf, size_t n);
  void vocabulary_head(int rows);
  void check(cudaError_t e, const char* what);
  void check_nccl(ncclResult_t r, const char* what);
  void check_fault();

  dl_model_config cfg_;
  int device_, sms_ = 148;
  size_t batch_, capacity_, chunk_;
  int rank_, tp_;
  int hq_, hkv_;        // local heads
  size_t D_, Ql_, Gl_, Fl_, V_, d_, L_;
  size_t Vl_ = 0, Vp_ = 0;  // vocabulary rows of this rank, padded to the GEMM tile
  cudaStream_t stream_ = nullptr;
  ncclComm_t comm_ = nullptr;
  // peer all-reduce: this rank's slots + flags, the peers' mapped copies
  void* peer_mem_ = nullptr;
  unsigned* peer_epoch_ = nullptr;
  void* peer_open_[kPeerMaxRanks] = {};
  PeerBuffers pb_ = {};
  bool peers_ = false;
  // weights (local slices)
  void* weight_arena_ = nullptr;
  bf16 *embed_ = nullptr, *final_norm_ = nullptr, *lm_head_ = nullptr;
  std::vector<Layer> layers_;
  float* inv_freq_ = nullptr;
  // KV: [B][L][2][C][Gl]
  void* kv_arena_ = nullptr;
  size_t plane_elems_ = 0, seq_elems_ = 0;
  // scratch
  void* scratch_ = nullptr;
  bf16 *residual_, *xn_, *qkv_, *q_raw_, *k_raw_, *q_rot_, *att_, *act_, *logits_, *xlast_, *vt_;
  bf16 *head_local_ = nullptr, *head_gather_ = nullptr;  // tensor parallelism: [B][Vp], [tp][B][Vp]
  float *parts_, *attn_ws_;
  int* attn_tickets_ = nullptr;  // [B][Hkv], zero between launches
  bool fuse_ = true;             // fused decode step (set_step_fusion)
  size_t parts_floats_ = 0;
  uint32_t* tokens_dev_;
  uint32_t* history_;
  int* steps_;
  long long* position_;
  unsigned* err_;
  size_t history_cap_ = 0;
  int vt_stride_ = 0;
  AttnPlan attn_plan_{1, 0};  // key ranges of the decode attention
  std::vector<AttnTcMaps*> attn_maps_;
  Sampler sampler_;  // one row per sequence
  dl_sampling settings_ = {0, 1.0, 0, 1.0};
  bool started_ = false;
  cudaGraphExec_t step_exec_ = nullptr;
  size_t kernels_per_step_ = 0;
  size_t launches_ = 0;
  double prefill_ms_ = 0.0;
  cudaEvent_t ev_[2] = {};
  // block-output capture [B][capacity][D] and fixed-strength steering
  int capture_layer_ = -1;
  bf16* capture_ = nullptr;
  int steer_layer_ = -1;
  long long steer_first_ = 0;
  float steer_strength_ = 0.f;
  long long steer_source_ = -1;   // sequence whose row sets beta = strength * ||row||; -1: beta = strength
  size_t steer_source_pos_ = 0;
  void* steer_mem_ = nullptr;     // direction [D] FP32, beta, mask [B]
  float* steer_dir_ = nullptr;
  float* steer_beta_ = nullptr;
  unsigned char* steer_mask_ = nullptr;
};

}  // namespace dl
