// Engine: resident Qwen3 weights, contiguous KV cache, and the prefill/decode
// loop.  Role of the reference's CachedForwardPlan (src/inference/executor.h:
// 242-342) and DeviceSequence (src/inference/decoding/device.h:84-137) for the
// CUDA backend: one ordered stream, device-resident position and token
// feedback, and the per-token body captured once into a CUDA graph.
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/dolittle_b200.h"
#include "decode_persistent.h"
#include "gemv.cuh"
#include "launch.h"
#include "sampler.h"

namespace dl {

struct Layer {
  bf16 *in_norm, *wqkv, *q_norm, *k_norm, *wo, *post_norm, *wgu, *wd;
};

struct TensorView {
  bf16* ptr;
  size_t rows, cols, row_stride;  // elements
};

struct DeviceState {
  long long position;  // absolute position of the next row to consume
  int step;            // number of selections made
  unsigned result[2];  // {token, status} of the last selection
  unsigned terminal;   // stop ID or error latched
  unsigned err;        // kernel error word
  unsigned ticket;     // argmax completion counter
  unsigned barrier;    // persistent decode: grid barrier arrivals
  unsigned exit_ticket;
  unsigned limit;      // device sequence loop: selections to make
  unsigned pad[6];
};

class Engine {
 public:
  Engine(const dl_model_config& cfg, int device, size_t capacity, size_t max_rows);
  ~Engine();

  static size_t tensor_count(const dl_model_config& c) { return 3 + 11 * size_t(c.layers); }
  static bool tensor_shape(const dl_model_config& c, size_t index, size_t* rows, size_t* cols);

  void init_random(uint64_t seed, float sigma);
  void set_tensor(size_t index, const void* host, size_t bytes);
  void get_tensor(size_t index, void* host, size_t bytes);
  // Device address of a resident tensor; gate/up live interleaved (strided)
  // and are reported through their row stride.
  void* tensor_device(size_t index, size_t* row_stride) {
    const TensorView v = view(index);
    if (row_stride) *row_stride = v.row_stride;
    return v.ptr;
  }
  void reset();
  void consume(const uint32_t* tokens, size_t n, int mode, uint16_t* logits_out);
  size_t position();
  void set_capture(int layer);
  void read_capture(size_t first, size_t count, uint16_t* host);
  void set_observation(void* device_rows, size_t positions);
  void set_intervention(int layer, size_t selected, float strength, const float* direction);
  void read_kv(size_t layer, int values, size_t first, size_t count, uint16_t* host);
  void set_injection(long long position, const uint16_t* source_bits, float scale);
  void set_reconstruction_head(const uint16_t* host_bits);
  void reconstruct(const uint32_t* tokens, size_t n, uint16_t* out_host);
  void generate(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s,
                uint64_t seed, const uint32_t* stop_ids, size_t n_stop, int prefill_mode,
                uint32_t* tokens_out, size_t* n_out, uint16_t* logits_out,
                dl_generation_stats* stats);
  // Device-side generation loop (role of the reference's DeviceSequence):
  // start returns at once; the journal reports each selection.
  void start(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s, uint64_t seed,
             const uint32_t* stop_ids, size_t n_stop, int prefill_mode);
  bool collect(size_t index, long long timeout_ms, dl_sequence_event* out);
  void request_stop();
  void drain(uint32_t* tokens_out, size_t* n_out, dl_generation_stats* stats);

 private:
  TensorView view(size_t index);
  void consume_rows(const uint32_t* tokens, size_t n, bool pdl, int mode, long long first);
  void run_layers(int rows, bool pdl);
  void run_layers_fast(int rows, long long first);
  bool fast_prefill_supported() const;
  void decode_step(bool pdl);
  void lm_head_select(const bf16* last_row, bool advance_position, bool generating, bool pdl);
  void lm_head_logits(const bf16* last_row, bool pdl);
  void select(const bf16* last_row, bool advance_position, bool pdl);
  void project(const bf16* x, int x_stride, int rows, int in_width, int prologue, const bf16* norm_w,
               int epilogue, GemvSegment* segs, int nseg, bool pdl);
  void capture_decode_graph();
  void build_loop_graph();
  void begin_sequence(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s,
                      uint64_t seed, const uint32_t* stop_ids, size_t n_stop, int prefill_mode);
  bool persistent_decode_ready();
  void launch_persistent_step(bool greedy);
  void check(cudaError_t e, const char* what);
  void check_fault();
  void observe_block(size_t layer, int rows);

  dl_model_config cfg_;
  int device_;
  size_t capacity_, max_rows_;
  int sms_;
  cudaStream_t stream_ = nullptr;
  // weights
  void* weight_arena_ = nullptr;
  size_t weight_bytes_ = 0;
  bf16 *embed_ = nullptr, *final_norm_ = nullptr, *lm_head_ = nullptr;
  std::vector<Layer> layers_;
  float* inv_freq_ = nullptr;
  // sequence
  void* kv_arena_ = nullptr;
  std::vector<bf16*> kcache_, vcache_;
  // scratch
  void* scratch_ = nullptr;
  bf16 *residual_, *q_raw_, *k_raw_, *q_rot_, *att_, *gu_, *logits_, *xn_;
  float* scores_;
  uint32_t* tokens_dev_;
  uint32_t* history_;
  size_t history_cap_;
  uint4* partials_;
  DeviceState* state_;
  // capture / steering
  int capture_layer_ = -1;
  bf16* capture_arena_ = nullptr;
  bf16* observe_rows_ = nullptr;  // caller-owned [layers][observe_positions_][D]
  size_t observe_positions_ = 0;
  bool observing_ = false;  // set only inside a prompt pass
  int edit_layer_ = -1;
  size_t edit_row_ = 0;
  float edit_strength_ = 0.f;
  float* edit_direction_ = nullptr;
  uint32_t* edit_state_ = nullptr;
  // decode graph
  cudaGraphExec_t decode_exec_ = nullptr;
  int graph_capture_layer_ = -2, graph_edit_layer_ = -2;
  size_t kernels_per_step_ = 0;
  size_t launches_ = 0;
  int last_rows_ = 1;
  bool capture_target_ = false;
  const unsigned char* stop_mask_ = nullptr;
  int mode_ = 0, graph_mode_ = -1;
  Sampler sampler_;
  cudaEvent_t ev_[4] = {};
  // device-side sequence loop: journal and cancel flag in mapped host memory
  dl_sequence_event* journal_host_ = nullptr;
  dl_sequence_event* journal_dev_ = nullptr;
  size_t journal_cap_ = 0;
  unsigned* cancel_host_ = nullptr;
  unsigned* cancel_dev_ = nullptr;
  cudaGraphExec_t loop_exec_ = nullptr;
  int loop_capture_layer_ = -2, loop_edit_layer_ = -2, loop_mode_ = -1, loop_path_ = -1;
  bool seq_running_ = false;
  size_t seq_max_new_ = 0, seq_launches_ = 0;
  // persistent decode step (one cooperative launch per token)
  int decode_path_ = DL_DECODE_PERSISTENT, graph_path_ = -1;
  int persist_state_ = -1;  // -1 not planned, 0 unsupported, 1 ready
  PLayer* persist_layers_ = nullptr;
  CUtensorMap* persist_maps_ = nullptr;
  PGemv persist_head_ = {};
  // fast prompt pass: tcgen05 attention (tensor maps) and transposed-V scratch
  struct AttnTcMaps* attn_tc_ = nullptr;
  bf16* vt_ = nullptr;
  int vt_stride_ = 0;
  float* gemm_partial_ = nullptr;  // split-K partials of the prompt-pass GEMMs
  size_t gemm_partial_floats_ = 0;
  static constexpr int kGemmTickets = 4096;
  unsigned* gemm_tickets_ = nullptr;
  // verbalizer injection (marker row) and reconstruction head
  long long inject_position_ = -1;
  bf16* inject_row_ = nullptr;  // [2][D]: the row to insert, then the staged source
  float* inject_norm_ = nullptr;
  unsigned* inject_status_ = nullptr;
  void* recon_head_ = nullptr;

 public:
  void set_decode_path(int path);
  void set_sampler_engine(int engine) { sampler_.engine = unsigned(engine); }
};

}  // namespace dl
