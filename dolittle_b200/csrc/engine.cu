// Engine implementation (see engine.h).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include <atomic>
#include <chrono>
#include <thread>

#include "attention_decode.h"
#include "attention_prefill_tc.h"
#include "engine.h"
#include "gemm_tcgen05.h"
#include "sequence.h"
#include "steering.h"

namespace dl {

namespace {
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Shape {
  size_t rows, cols;
};

Shape shape_of(const dl_model_config& c, size_t index) {
  const size_t D = c.hidden, Q = size_t(c.query_heads) * c.head_width,
               G = size_t(c.kv_heads) * c.head_width, F = c.mlp_width, V = c.vocabulary,
               d = c.head_width;
  if (index == 0) return {V, D};
  if (index == 1) return {1, D};
  if (index == 2) return {V, D};
  switch ((index - 3) % 11) {
    case 0: return {1, D};
    case 1: return {Q, D};
    case 2: return {G, D};
    case 3: return {G, D};
    case 4: return {1, d};
    case 5: return {1, d};
    case 6: return {D, Q};
    case 7: return {1, D};
    case 8: return {F, D};
    case 9: return {F, D};
    default: return {D, F};
  }
}
}  // namespace

bool Engine::tensor_shape(const dl_model_config& c, size_t index, size_t* rows, size_t* cols) {
  if (index >= tensor_count(c)) return false;
  const Shape s = shape_of(c, index);
  *rows = s.rows;
  *cols = s.cols;
  return true;
}

void Engine::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

Engine::Engine(const dl_model_config& cfg, int device, size_t capacity, size_t max_rows)
    : cfg_(cfg), device_(device), capacity_(capacity), max_rows_(max_rows) {
  const size_t D = cfg.hidden, Q = size_t(cfg.query_heads) * cfg.head_width,
               G = size_t(cfg.kv_heads) * cfg.head_width, F = cfg.mlp_width, V = cfg.vocabulary,
               d = cfg.head_width, L = cfg.layers;
  if (!D || !Q || !G || !F || !V || !L || !capacity || !max_rows || max_rows > 8192 ||
      cfg.query_heads % cfg.kv_heads || d > 128 || d % 2 || D % 8 || Q % 8 || F % 8 ||
      cfg.query_heads / cfg.kv_heads > 8)
    throw std::invalid_argument("unsupported Qwen3 configuration");
  check(cudaSetDevice(device), "cudaSetDevice");
  int sms = 0;
  check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "sm count");
  sms_ = sms;
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
  for (auto& ev : ev_) check(cudaEventCreate(&ev), "event");

  // ---- weights: one arena, 256-byte aligned tensors ----
  size_t off = 0;
  auto take = [&](size_t elems) {
    const size_t o = off;
    off = align_up(off + elems * 2, 256);
    return o;
  };
  const size_t o_embed = take(V * D), o_final = take(D), o_head = take(V * D);
  std::vector<size_t> lo(L * 8);
  for (size_t l = 0; l < L; ++l) {
    lo[l * 8 + 0] = take(D);
    lo[l * 8 + 1] = take((Q + 2 * G) * D);
    lo[l * 8 + 2] = take(d);
    lo[l * 8 + 3] = take(d);
    lo[l * 8 + 4] = take(D * Q);
    lo[l * 8 + 5] = take(D);
    lo[l * 8 + 6] = take(2 * F * D);
    lo[l * 8 + 7] = take(D * F);
  }
  weight_bytes_ = off;
  check(cudaMalloc(&weight_arena_, weight_bytes_), "weights");
  auto* base = static_cast<unsigned char*>(weight_arena_);
  embed_ = reinterpret_cast<bf16*>(base + o_embed);
  final_norm_ = reinterpret_cast<bf16*>(base + o_final);
  lm_head_ = reinterpret_cast<bf16*>(base + o_head);
  layers_.resize(L);
  for (size_t l = 0; l < L; ++l) {
    Layer& y = layers_[l];
    y.in_norm = reinterpret_cast<bf16*>(base + lo[l * 8 + 0]);
    y.wqkv = reinterpret_cast<bf16*>(base + lo[l * 8 + 1]);
    y.q_norm = reinterpret_cast<bf16*>(base + lo[l * 8 + 2]);
    y.k_norm = reinterpret_cast<bf16*>(base + lo[l * 8 + 3]);
    y.wo = reinterpret_cast<bf16*>(base + lo[l * 8 + 4]);
    y.post_norm = reinterpret_cast<bf16*>(base + lo[l * 8 + 5]);
    y.wgu = reinterpret_cast<bf16*>(base + lo[l * 8 + 6]);
    y.wd = reinterpret_cast<bf16*>(base + lo[l * 8 + 7]);
  }

  // ---- KV cache: per block K[C][Hkv][d] then V[C][Hkv][d] ----
  const size_t kv_block = align_up(capacity * G * 2, 256);
  check(cudaMalloc(&kv_arena_, kv_block * 2 * L), "kv cache");
  check(cudaMemsetAsync(kv_arena_, 0, kv_block * 2 * L, stream_), "kv clear");
  for (size_t l = 0; l < L; ++l) {
    kcache_.push_back(reinterpret_cast<bf16*>(static_cast<unsigned char*>(kv_arena_) + kv_block * (2 * l)));
    vcache_.push_back(reinterpret_cast<bf16*>(static_cast<unsigned char*>(kv_arena_) + kv_block * (2 * l + 1)));
  }

  // ---- scratch ----
  const size_t R = max_rows;
  history_cap_ = capacity + 1;
  size_t s = 0;
  auto stake = [&](size_t bytes) {
    const size_t o = s;
    s = align_up(s + bytes, 256);
    return o;
  };
  const size_t o_res = stake(R * D * 2), o_qraw = stake(R * Q * 2), o_kraw = stake(R * G * 2),
               o_qrot = stake(R * Q * 2), o_att = stake(R * Q * 2), o_gu = stake(R * 2 * F * 2),
               o_logits = stake(V * 2), o_scores = stake(R * cfg.query_heads * align_up(capacity, 4) * 4),
               o_tok = stake(std::max<size_t>(R, 64) * 4), o_hist = stake(history_cap_ * 4),
               o_part = stake(size_t(4 * sms_) * 16), o_state = stake(sizeof(DeviceState)),
               o_inv = stake(d * 2), o_dir = stake(D * 4), o_edit = stake(64),
               o_cap = stake(capacity * D * 2), o_xn = stake(R * D * 2),
               o_vt = stake(size_t(cfg.kv_heads) * d * align_up(capacity, 64) * 2),
               o_split = stake(gemm_split_floats(int(std::min<size_t>(R, 1024)), int(std::max<size_t>(D, Q + 2 * G)),
                                                 kGemmMaxSplit) * 4),
               o_tickets = stake(size_t(kGemmTickets) * 4), o_inject = stake(2 * D * 2), o_inject_misc = stake(64);
  check(cudaMalloc(&scratch_, s), "scratch");
  check(cudaMemsetAsync(scratch_, 0, s, stream_), "scratch clear");
  auto* sb = static_cast<unsigned char*>(scratch_);
  residual_ = reinterpret_cast<bf16*>(sb + o_res);
  q_raw_ = reinterpret_cast<bf16*>(sb + o_qraw);
  k_raw_ = reinterpret_cast<bf16*>(sb + o_kraw);
  q_rot_ = reinterpret_cast<bf16*>(sb + o_qrot);
  att_ = reinterpret_cast<bf16*>(sb + o_att);
  gu_ = reinterpret_cast<bf16*>(sb + o_gu);
  logits_ = reinterpret_cast<bf16*>(sb + o_logits);
  scores_ = reinterpret_cast<float*>(sb + o_scores);
  tokens_dev_ = reinterpret_cast<uint32_t*>(sb + o_tok);
  history_ = reinterpret_cast<uint32_t*>(sb + o_hist);
  partials_ = reinterpret_cast<uint4*>(sb + o_part);
  state_ = reinterpret_cast<DeviceState*>(sb + o_state);
  inv_freq_ = reinterpret_cast<float*>(sb + o_inv);
  edit_direction_ = reinterpret_cast<float*>(sb + o_dir);
  edit_state_ = reinterpret_cast<uint32_t*>(sb + o_edit);
  capture_arena_ = reinterpret_cast<bf16*>(sb + o_cap);
  xn_ = reinterpret_cast<bf16*>(sb + o_xn);
  vt_ = reinterpret_cast<bf16*>(sb + o_vt);
  gemm_partial_ = reinterpret_cast<float*>(sb + o_split);
  gemm_partial_floats_ =
      gemm_split_floats(int(std::min<size_t>(R, 1024)), int(std::max<size_t>(D, Q + 2 * G)), kGemmMaxSplit);
  gemm_tickets_ = reinterpret_cast<unsigned*>(sb + o_tickets);
  inject_row_ = reinterpret_cast<bf16*>(sb + o_inject);
  inject_norm_ = reinterpret_cast<float*>(sb + o_inject_misc);
  inject_status_ = reinterpret_cast<unsigned*>(sb + o_inject_misc + 16);
  vt_stride_ = int(align_up(capacity, 64));
  attn_tc_ = attention_prefill_tc_maps(q_rot_, int(R), int(cfg.query_heads), static_cast<const bf16*>(kv_arena_),
                                       kv_block, int(capacity), int(L), int(cfg.kv_heads), int(d), vt_, vt_stride_);
  check(launch_inv_freq(inv_freq_, int(d), cfg.theta, stream_), "inv_freq");
  // Journal of the device-side loop (prompt event, a selection per token, a
  // terminal event) and its cancel flag, in mapped host memory.
  journal_cap_ = capacity + 2;
  check(cudaHostAlloc(reinterpret_cast<void**>(&journal_host_), journal_cap_ * sizeof(dl_sequence_event),
                      cudaHostAllocMapped),
        "journal");
  check(cudaHostGetDevicePointer(reinterpret_cast<void**>(&journal_dev_), journal_host_, 0), "journal map");
  check(cudaHostAlloc(reinterpret_cast<void**>(&cancel_host_), 64, cudaHostAllocMapped), "cancel flag");
  check(cudaHostGetDevicePointer(reinterpret_cast<void**>(&cancel_dev_), cancel_host_, 0), "cancel map");
  std::memset(journal_host_, 0, journal_cap_ * sizeof(dl_sequence_event));
  *cancel_host_ = 0;
  check(cudaStreamSynchronize(stream_), "init sync");
}

Engine::~Engine() {
  if (stream_) cudaStreamSynchronize(stream_);
  if (decode_exec_) cudaGraphExecDestroy(decode_exec_);
  if (loop_exec_) cudaGraphExecDestroy(loop_exec_);
  if (journal_host_) cudaFreeHost(journal_host_);
  if (cancel_host_) cudaFreeHost(cancel_host_);
  attention_prefill_tc_free(attn_tc_);
  cudaFree(recon_head_);
  cudaFree(persist_layers_);
  cudaFree(persist_maps_);
  for (auto& ev : ev_)
    if (ev) cudaEventDestroy(ev);
  cudaFree(scratch_);
  cudaFree(kv_arena_);
  cudaFree(weight_arena_);
  if (stream_) cudaStreamDestroy(stream_);
}

// Resident layout of each logical tensor.  Gate and up rows are interleaved
// in one [2F][D] matrix (row 2o = gate o, row 2o+1 = up o) so one CTA holds
// both halves of every SwiGLU pair; every other tensor is contiguous.
TensorView Engine::view(size_t index) {
  if (index >= tensor_count(cfg_)) throw std::invalid_argument("tensor index out of range");
  const Shape sh = shape_of(cfg_, index);
  TensorView v{nullptr, sh.rows, sh.cols, sh.cols};
  if (index == 0) v.ptr = embed_;
  else if (index == 1) v.ptr = final_norm_;
  else if (index == 2) v.ptr = lm_head_;
  else {
    const size_t l = (index - 3) / 11, role = (index - 3) % 11;
    const size_t D = cfg_.hidden, Q = size_t(cfg_.query_heads) * cfg_.head_width,
                 G = size_t(cfg_.kv_heads) * cfg_.head_width;
    const Layer& y = layers_[l];
    switch (role) {
      case 0: v.ptr = y.in_norm; break;
      case 1: v.ptr = y.wqkv; break;
      case 2: v.ptr = y.wqkv + Q * D; break;
      case 3: v.ptr = y.wqkv + (Q + G) * D; break;
      case 4: v.ptr = y.q_norm; break;
      case 5: v.ptr = y.k_norm; break;
      case 6: v.ptr = y.wo; break;
      case 7: v.ptr = y.post_norm; break;
      case 8: v.ptr = y.wgu; v.row_stride = 2 * D; break;
      case 9: v.ptr = y.wgu + D; v.row_stride = 2 * D; break;
      default: v.ptr = y.wd; break;
    }
  }
  return v;
}

void Engine::init_random(uint64_t seed, float sigma) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  const double sd = std::sqrt(8.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const float scale = static_cast<float>(double(sigma) / sd);
  for (size_t i = 0; i < tensor_count(cfg_); ++i) {
    const TensorView v = view(i);
    if (v.rows == 1)
      check(launch_fill_const(v.ptr, v.cols, 1.0f, stream_), "fill norm");
    else
      check(launch_fill_normal(v.ptr, v.rows, v.cols, v.row_stride, seed, uint32_t(i), scale, stream_),
            "fill normal");
  }
  check(cudaStreamSynchronize(stream_), "init_random sync");
}

void Engine::set_tensor(size_t index, const void* host, size_t bytes) {
  const TensorView v = view(index);
  if (bytes != v.rows * v.cols * 2) throw std::invalid_argument("tensor byte size mismatch");
  check(cudaMemcpy2DAsync(v.ptr, v.row_stride * 2, host, v.cols * 2, v.cols * 2, v.rows, cudaMemcpyHostToDevice,
                          stream_),
        "set_tensor");
  check(cudaStreamSynchronize(stream_), "set_tensor sync");
}

void Engine::get_tensor(size_t index, void* host, size_t bytes) {
  const TensorView v = view(index);
  if (bytes != v.rows * v.cols * 2) throw std::invalid_argument("tensor byte size mismatch");
  check(cudaMemcpy2DAsync(host, v.cols * 2, v.ptr, v.row_stride * 2, v.cols * 2, v.rows, cudaMemcpyDeviceToHost,
                          stream_),
        "get_tensor");
  check(cudaStreamSynchronize(stream_), "get_tensor sync");
}

void Engine::reset() {
  DeviceState z = {};
  check(cudaMemcpyAsync(state_, &z, sizeof(z), cudaMemcpyHostToDevice, stream_), "reset");
  const uint32_t zero[2] = {0, 0};
  check(cudaMemcpyAsync(edit_state_, zero, sizeof(zero), cudaMemcpyHostToDevice, stream_), "reset edit");
  check(cudaStreamSynchronize(stream_), "reset sync");
}

size_t Engine::position() {
  DeviceState s;
  check(cudaMemcpyAsync(&s, state_, sizeof(s), cudaMemcpyDeviceToHost, stream_), "position");
  check(cudaStreamSynchronize(stream_), "position sync");
  return size_t(s.position);
}

void Engine::check_fault() {
  unsigned err = 0;
  check(cudaMemcpyAsync(&err, &state_->err, 4, cudaMemcpyDeviceToHost, stream_), "fault read");
  check(cudaStreamSynchronize(stream_), "fault sync");
  if (err) throw std::runtime_error("device fault word " + std::to_string(err));
}

// One projection (possibly several segments sharing the input) over `rows`
// input rows, split into row groups the streaming kernel holds in smem.
void Engine::project(const bf16* x, int x_stride, int rows, int in_width, int prologue,
                     const bf16* norm_w, int epilogue, GemvSegment* segs, int nseg, bool pdl) {
  const int rt = gemv_rows_template(rows, in_width);
  for (int g0 = 0; g0 < rows; g0 += rt) {
    GemvArgs a = {};
    a.x = x + size_t(g0) * x_stride;
    a.x_stride = x_stride;
    a.in_width = in_width;
    a.nrows = std::min(rt, rows - g0);
    a.prologue = prologue;
    a.norm_w = norm_w;
    a.eps = cfg_.epsilon;
    a.epilogue = epilogue;
    a.nseg = nseg;
    for (int i = 0; i < nseg; ++i) {
      a.seg[i] = segs[i];
      a.seg[i].out = segs[i].out + size_t(g0) * segs[i].out_stride;
    }
    if (epilogue == kEpilogueResidual && capture_arena_ && capture_target_) {
      a.capture = capture_arena_ + size_t(g0) * cfg_.hidden;
      a.capture_row = &state_->position;
      a.capture_stride = int(cfg_.hidden);
    }
    a.err = &state_->err;
    check(launch_gemv(a, rt, sms_, stream_, pdl), "gemv");
    ++launches_;
  }
}

void Engine::run_layers(int rows, bool pdl) {
  const int D = int(cfg_.hidden), Q = int(cfg_.query_heads * cfg_.head_width),
            G = int(cfg_.kv_heads * cfg_.head_width), F = int(cfg_.mlp_width),
            d = int(cfg_.head_width), H = int(cfg_.query_heads), Hk = int(cfg_.kv_heads);
  const RowPositions pos{&state_->position, 0};
  const float scale = attention_scale(d);
  const int cap = int(capacity_);
  const int score_ctas = rows == 1 ? std::clamp((cap + 63) / 64, 1, 16) : std::clamp((cap + 255) / 256, 1, 8);
  for (size_t l = 0; l < layers_.size(); ++l) {
    const Layer& y = layers_[l];
    GemvSegment qkv[3];
    qkv[0] = make_segment(y.wqkv, q_raw_, nullptr, Q, projection_partials(D, Q), Q);
    qkv[1] = make_segment(y.wqkv + size_t(Q) * D, k_raw_, nullptr, G, projection_partials(D, G), G);
    qkv[2] = make_segment(y.wqkv + size_t(Q + G) * D, vcache_[l], &state_->position, G, projection_partials(D, G), G);
    capture_target_ = false;
    project(residual_, D, rows, D, kPrologueRmsNorm, y.in_norm, kEpilogueStore, qkv, 3, pdl);
    if (rows == 1 && attention_decode_supported(H, Hk, d, cap)) {
      // One query row: QK-norm/RoPE/K-append fused into the score kernel.
      check(launch_attention_decode(q_raw_, k_raw_, y.q_norm, y.k_norm, inv_freq_, kcache_[l], vcache_[l], scores_,
                                    att_, &state_->position, H, Hk, d, cap, cfg_.epsilon, score_ctas, stream_, pdl),
            "attention decode");
      launches_ += 2;
    } else {
      check(launch_qk_norm_rope(q_raw_, k_raw_, y.q_norm, y.k_norm, inv_freq_, q_rot_, kcache_[l], pos, rows,
                                H, Hk, d, cfg_.epsilon, stream_, pdl),
            "qk_norm_rope");
      check(launch_attention_scores(q_rot_, kcache_[l], scores_, pos, rows, H, Hk, d, cap, scale, score_ctas,
                                    stream_, pdl),
            "attention scores");
      check(launch_attention_pv(scores_, vcache_[l], att_, pos, rows, H, Hk, d, cap, stream_, pdl),
            "attention pv");
      launches_ += 3;
    }
    GemvSegment o = make_segment(y.wo, residual_, nullptr, D, projection_partials(Q, D), D);
    project(att_, Q, rows, Q, kProloguePlain, nullptr, kEpilogueResidual, &o, 1, pdl);
    // Interleaved gate|up rows; the epilogue writes the SwiGLU activation.
    GemvSegment gu = make_segment(y.wgu, gu_, nullptr, 2 * F, projection_partials(D, F), F);
    project(residual_, D, rows, D, kPrologueRmsNorm, y.post_norm, kEpilogueSwiGLU, &gu, 1, pdl);
    const bool edit_here = edit_layer_ == int(l);
    capture_target_ = capture_layer_ == int(l) && !edit_here;
    GemvSegment dn = make_segment(y.wd, residual_, nullptr, D, projection_partials(F, D), D);
    project(gu_, F, rows, F, kProloguePlain, nullptr, kEpilogueResidual, &dn, 1, pdl);
    capture_target_ = false;
    if (edit_here) {
      check(launch_intervene(residual_, edit_direction_, &state_->position, edit_state_, D,
                             (long long)edit_row_, rows, edit_strength_, stream_, pdl),
            "intervene");
      ++launches_;
      if (capture_layer_ == int(l)) {
        check(launch_copy_rows(residual_, capture_arena_, &state_->position, D, rows, stream_, pdl),
              "capture copy");
        ++launches_;
      }
    }
    observe_block(l, rows);
  }
}

void Engine::lm_head_select(const bf16* last_row, bool advance, bool generating, bool pdl) {
  const int D = int(cfg_.hidden), V = int(cfg_.vocabulary);
  GemvArgs a = {};
  a.x = last_row;
  a.x_stride = D;
  a.in_width = D;
  a.nrows = 1;
  a.prologue = kPrologueRmsNorm;
  a.norm_w = final_norm_;
  a.eps = cfg_.epsilon;
  a.epilogue = kEpilogueArgmax;
  a.nseg = 1;
  a.seg[0] = make_segment(lm_head_, logits_, nullptr, V, projection_partials(D, V), V);
  a.partials = partials_;
  a.ticket = &state_->ticket;
  a.select.result = state_->result;
  if (generating) {
    a.select.history = history_;
    a.select.step = &state_->step;
    a.select.embed = embed_;
    a.select.residual = residual_;
    a.select.width = D;
    a.select.terminal = &state_->terminal;
    a.select.stop_mask = stop_mask_;
  }
  if (advance) a.select.position = &state_->position;
  a.err = &state_->err;
  check(launch_gemv(a, 1, sms_, stream_, pdl), "lm_head");
  ++launches_;
}

bool Engine::fast_prefill_supported() const {
  const int D = int(cfg_.hidden), Q = int(cfg_.query_heads * cfg_.head_width),
            G = int(cfg_.kv_heads * cfg_.head_width), F = int(cfg_.mlp_width);
  return gemm_tcgen05_supported(1, Q + 2 * G, D) && gemm_tcgen05_supported(1, D, Q) &&
         gemm_tcgen05_supported(1, 2 * F, D) && gemm_tcgen05_supported(1, D, F) && Q % 256 == 0 &&
         (Q + G) % 256 == 0;
}

// Prompt rows on the tensor cores: RMSNorm, then tcgen05 GEMMs for QKV (V
// rows appended to the cache by the epilogue), o (+residual), gate|up
// (+SwiGLU) and down (+residual); QK-norm/RoPE and causal attention use the
// same kernels as the parity path.  `first` is the absolute position of row 0.
// Every kernel of the chain is a programmatic dependent launch: each waits
// (griddepcontrol.wait) for its predecessor before reading, so its launch and
// prologue overlap the predecessor's tail.

void Engine::run_layers_fast(int rows, long long first) {
  const int D = int(cfg_.hidden), Q = int(cfg_.query_heads * cfg_.head_width),
            G = int(cfg_.kv_heads * cfg_.head_width), F = int(cfg_.mlp_width), d = int(cfg_.head_width),
            H = int(cfg_.query_heads), Hk = int(cfg_.kv_heads);
  const RowPositions pos{&state_->position, 0};
  const int cap = int(capacity_);
  const int score_ctas = std::clamp((cap + 255) / 256, 1, 8);
  auto gemm = [&](const bf16* x, int ldx, const bf16* w, int N, int K, int epi, int nseg, const int* n0s,
                  bf16* const* outs, const int* lds) {
    GemmProblem p = {};
    p.x = x;
    p.ldx = ldx;
    p.w = w;
    p.M = rows;
    p.N = N;
    p.K = K;
    p.epilogue = epi;
    p.nseg = nseg;
    for (int i = 0; i < nseg; ++i) {
      p.seg_n0[i] = n0s[i];
      p.seg_out[i] = outs[i];
      p.seg_ld[i] = lds[i];
    }
    p.wide_tiles = true;
    p.err = &state_->err;
    // Split-K where the parts fit the workspace (the launcher checks).
    p.partial = gemm_partial_;
    p.partial_floats = gemm_partial_floats_;
    p.tickets = gemm_tickets_;
    p.n_tickets = kGemmTickets;
    check(launch_gemm_tcgen05(p, stream_, true), "gemm");
    ++launches_;
  };
  for (size_t l = 0; l < layers_.size(); ++l) {
    const Layer& y = layers_[l];
    check(launch_rms_norm(residual_, y.in_norm, xn_, size_t(rows), D, cfg_.epsilon, stream_, true), "rms_norm");
    {
      const int n0s[3] = {0, Q, Q + G};
      bf16* outs[3] = {q_raw_, k_raw_, vcache_[l] + size_t(first) * G};
      const int lds[3] = {Q, G, G};
      gemm(xn_, D, y.wqkv, Q + 2 * G, D, kGemmStore, 3, n0s, outs, lds);
    }
    check(launch_qk_norm_rope(q_raw_, k_raw_, y.q_norm, y.k_norm, inv_freq_, q_rot_, kcache_[l], pos, rows, H, Hk,
                              d, cfg_.epsilon, stream_, true),
          "qk_norm_rope");
    if (attn_tc_) {
      // Tensor-core causal attention over keys 0 .. first+rows-1.
      check(launch_vt_transpose(vcache_[l], vt_, int(first) + rows, Hk, d, vt_stride_, stream_, true), "v transpose");
      check(launch_attention_prefill_tc(attn_tc_, att_, rows, first, int(l), H, Hk, attention_scale(d), &state_->err,
                                        stream_, true),
            "attention prefill");
    } else {
      check(launch_attention_scores(q_rot_, kcache_[l], scores_, pos, rows, H, Hk, d, cap, attention_scale(d),
                                    score_ctas, stream_, false),
            "attention scores");
      check(launch_attention_pv(scores_, vcache_[l], att_, pos, rows, H, Hk, d, cap, stream_, false), "attention pv");
    }
    launches_ += 4;
    {
      const int n0s[1] = {0};
      bf16* outs[1] = {residual_};
      const int lds[1] = {D};
      gemm(att_, Q, y.wo, D, Q, kGemmResidual, 1, n0s, outs, lds);
    }
    check(launch_rms_norm(residual_, y.post_norm, xn_, size_t(rows), D, cfg_.epsilon, stream_, true), "rms_norm");
    ++launches_;
    {
      const int n0s[1] = {0};
      bf16* outs[1] = {gu_};
      const int lds[1] = {F};
      gemm(xn_, D, y.wgu, 2 * F, D, kGemmSwiGLU, 1, n0s, outs, lds);
    }
    {
      const int n0s[1] = {0};
      bf16* outs[1] = {residual_};
      const int lds[1] = {D};
      gemm(gu_, F, y.wd, D, F, kGemmResidual, 1, n0s, outs, lds);
    }
    if (edit_layer_ == int(l)) {
      check(launch_intervene(residual_, edit_direction_, &state_->position, edit_state_, D, (long long)edit_row_,
                             rows, edit_strength_, stream_, false),
            "intervene");
      ++launches_;
    }
    if (capture_layer_ == int(l)) {
      check(launch_copy_rows(residual_, capture_arena_, &state_->position, D, rows, stream_, false), "capture copy");
      ++launches_;
    }
    observe_block(l, rows);
  }
}

void Engine::consume_rows(const uint32_t* tokens, size_t n, bool pdl, int mode, long long first) {
  const bool fast = mode == DL_PREFILL_FAST && fast_prefill_supported();
  if (observe_rows_ && size_t(first) + n > observe_positions_)
    throw std::invalid_argument("prompt pass reaches past the observation rows");
  observing_ = observe_rows_ != nullptr;
  struct Off {
    bool& flag;
    ~Off() { flag = false; }
  } off{observing_};
  for (size_t c0 = 0; c0 < n; c0 += max_rows_) {
    const int rows = int(std::min(max_rows_, n - c0));
    check(cudaMemcpyAsync(tokens_dev_, tokens + c0, rows * 4, cudaMemcpyHostToDevice, stream_), "tokens");
    check(launch_embedding(tokens_dev_, embed_, residual_, rows, int(cfg_.hidden), stream_, false), "embed");
    // Verbalizer injection: the marker row's embedding is replaced by the
    // normalized vector (reference src/kernels/cuda/decode.cu:221-230).
    if (inject_position_ >= first && inject_position_ < first + rows)
      check(cudaMemcpyAsync(residual_ + size_t(inject_position_ - first) * cfg_.hidden, inject_row_,
                            cfg_.hidden * 2, cudaMemcpyDeviceToDevice, stream_),
            "inject");
    if (fast)
      run_layers_fast(rows, first);
    else
      run_layers(rows, pdl);
    check(launch_add_position(&state_->position, rows, stream_), "advance");
    first += rows;
    last_rows_ = rows;
  }
}

void Engine::consume(const uint32_t* tokens, size_t n, int mode, uint16_t* logits_out) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!n) throw std::invalid_argument("empty consume");
  const size_t first = position();
  if (first + n > capacity_) throw std::length_error("sequence exceeds KV capacity");
  if (mode != DL_PREFILL_PARITY && mode != DL_PREFILL_FAST) throw std::invalid_argument("unknown prefill mode");
  consume_rows(tokens, n, true, mode, (long long)first);
  lm_head_select(residual_ + size_t(last_rows_ - 1) * cfg_.hidden, false, false, true);
  if (logits_out)
    check(cudaMemcpyAsync(logits_out, logits_, size_t(cfg_.vocabulary) * 2, cudaMemcpyDeviceToHost, stream_),
          "logits");
  check(cudaStreamSynchronize(stream_), "consume sync");
  check_fault();
}

void Engine::set_injection(long long position, const uint16_t* source_bits, float scale) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (position < 0) {
    inject_position_ = -1;
    return;
  }
  if (size_t(position) >= capacity_) throw std::invalid_argument("injection position beyond capacity");
  if (!(scale > 0.f) || !std::isfinite(scale)) throw std::invalid_argument("injection scale must be finite and > 0");
  const size_t D = cfg_.hidden;
  // Source row staged in the injection row itself, normalized into a second
  // half of the buffer, then kept as the row to insert.
  check(cudaMemcpyAsync(inject_row_ + D, source_bits, D * 2, cudaMemcpyHostToDevice, stream_), "injection source");
  check(launch_normalize_injection(inject_row_ + D, inject_row_, inject_norm_, inject_status_, int(D), scale, stream_),
        "normalize injection");
  unsigned status = 0;
  check(cudaMemcpyAsync(&status, inject_status_, 4, cudaMemcpyDeviceToHost, stream_), "injection status");
  check(cudaStreamSynchronize(stream_), "injection sync");
  if (status) throw std::invalid_argument("injection source has zero or non-finite norm");
  inject_position_ = position;
}

void Engine::set_reconstruction_head(const uint16_t* host_bits) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  const size_t D = cfg_.hidden;
  if (!recon_head_) check(cudaMalloc(&recon_head_, D * D * 2), "reconstruction head");
  check(cudaMemcpyAsync(recon_head_, host_bits, D * D * 2, cudaMemcpyHostToDevice, stream_), "reconstruction head");
  check(cudaStreamSynchronize(stream_), "reconstruction head sync");
}

// AR forward-only pass (reference src/inference/executor.cpp:1750-1771,
// src/models/qwen3/model.cpp:395-404): the prompt through every block from a
// fresh sequence, then the last position's residual (no final norm) through
// the D x D reconstruction head under the projection law.
void Engine::reconstruct(const uint32_t* tokens, size_t n, uint16_t* out_host) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!recon_head_) throw std::invalid_argument("reconstruction head not set");
  if (!n || n > capacity_) throw std::invalid_argument("reconstruction prompt length");
  reset();
  consume_rows(tokens, n, true, DL_PREFILL_PARITY, 0);
  const int D = int(cfg_.hidden);
  GemvSegment seg = make_segment(static_cast<const bf16*>(recon_head_), xn_, nullptr, D, projection_partials(D, D), D);
  project(residual_ + size_t(last_rows_ - 1) * D, D, 1, D, kProloguePlain, nullptr, kEpilogueStore, &seg, 1, true);
  check(cudaMemcpyAsync(out_host, xn_, size_t(D) * 2, cudaMemcpyDeviceToHost, stream_), "reconstruction out");
  check(cudaStreamSynchronize(stream_), "reconstruct sync");
  check_fault();
}

void Engine::set_observation(void* device_rows, size_t positions) {
  if (device_rows && !positions) throw std::invalid_argument("observation needs positions");
  observe_rows_ = static_cast<bf16*>(device_rows);
  observe_positions_ = device_rows ? positions : 0;
}

void Engine::observe_block(size_t layer, int rows) {
  if (!observe_rows_ || !observing_) return;
  check(launch_copy_rows(residual_, observe_rows_ + layer * observe_positions_ * cfg_.hidden, &state_->position,
                         int(cfg_.hidden), rows, stream_, false),
        "observe copy");
  ++launches_;
}

void Engine::set_capture(int layer) {
  if (layer >= int(cfg_.layers)) throw std::invalid_argument("capture layer out of range");
  capture_layer_ = layer;
}

void Engine::read_capture(size_t first, size_t count, uint16_t* host) {
  if (first + count > capacity_) throw std::invalid_argument("capture range");
  check(cudaMemcpyAsync(host, capture_arena_ + first * cfg_.hidden, count * cfg_.hidden * 2,
                        cudaMemcpyDeviceToHost, stream_),
        "read capture");
  check(cudaStreamSynchronize(stream_), "read capture sync");
}

void Engine::set_intervention(int layer, size_t selected, float strength, const float* direction) {
  if (layer >= int(cfg_.layers)) throw std::invalid_argument("intervention layer out of range");
  // The captured step graph holds the row and strength as launch arguments.
  if (decode_exec_) {
    cudaGraphExecDestroy(decode_exec_);
    decode_exec_ = nullptr;
  }
  edit_layer_ = layer;
  edit_row_ = selected;
  edit_strength_ = strength;
  if (layer >= 0) {
    check(cudaMemcpyAsync(edit_direction_, direction, cfg_.hidden * 4, cudaMemcpyHostToDevice, stream_),
          "direction");
    const uint32_t zero[2] = {0, 0};
    check(cudaMemcpyAsync(edit_state_, zero, 8, cudaMemcpyHostToDevice, stream_), "edit state");
    check(cudaStreamSynchronize(stream_), "intervention sync");
  }
}

void Engine::read_kv(size_t layer, int values, size_t first, size_t count, uint16_t* host) {
  if (layer >= layers_.size() || first + count > capacity_) throw std::invalid_argument("kv range");
  const size_t G = size_t(cfg_.kv_heads) * cfg_.head_width;
  const bf16* src = (values ? vcache_[layer] : kcache_[layer]) + first * G;
  check(cudaMemcpyAsync(host, src, count * G * 2, cudaMemcpyDeviceToHost, stream_), "read kv");
  check(cudaStreamSynchronize(stream_), "read kv sync");
}

void Engine::lm_head_logits(const bf16* last_row, bool pdl) {
  const int D = int(cfg_.hidden), V = int(cfg_.vocabulary);
  GemvArgs a = {};
  a.x = last_row;
  a.x_stride = D;
  a.in_width = D;
  a.nrows = 1;
  a.prologue = kPrologueRmsNorm;
  a.norm_w = final_norm_;
  a.eps = cfg_.epsilon;
  a.epilogue = kEpilogueStore;
  a.nseg = 1;
  a.seg[0] = make_segment(lm_head_, logits_, nullptr, V, projection_partials(D, V), V);
  a.err = &state_->err;
  check(launch_gemv(a, 1, sms_, stream_, pdl), "lm_head");
  ++launches_;
}

// Selection after the logits of the last consumed row are in logits_.
void Engine::select(const bf16* last_row, bool advance, bool pdl) {
  if (mode_ == 0) {
    lm_head_select(last_row, advance, true, pdl);
    return;
  }
  lm_head_logits(last_row, pdl);
  check(sampler_submit(sampler_, logits_, sampler_.settings, 0, true, stream_), "sampler");
  check(sampler_feed(sampler_, history_, &state_->step, embed_, residual_, int(cfg_.hidden),
                     advance ? &state_->position : nullptr, stream_),
        "sampler feed");
  launches_ += sampler_launch_count(sampler_, sampler_.settings, true) + 1;
}

void Engine::set_decode_path(int path) {
  if (path != DL_DECODE_PERSISTENT && path != DL_DECODE_KERNELS) throw std::invalid_argument("unknown decode path");
  decode_path_ = path;
}

// Plans the persistent decode step once: per block the qkv, o, gate|up and
// down projection phases and the vocabulary head, with their tensor maps, in
// device memory.  Unsupported shapes or devices keep the per-operation path.
bool Engine::persistent_decode_ready() {
  if (persist_state_ >= 0) return persist_state_ == 1;
  persist_state_ = 0;
  const int D = int(cfg_.hidden), Q = int(cfg_.query_heads * cfg_.head_width),
            G = int(cfg_.kv_heads * cfg_.head_width), F = int(cfg_.mlp_width), V = int(cfg_.vocabulary),
            d = int(cfg_.head_width), group = int(cfg_.query_heads / cfg_.kv_heads);
  const int grid = sms_;
  if (group > 7 || d > 128 || d % 8 || 2 * group * 8 > kGemvConsumers || !decode_persistent_fits(grid)) return false;
  const size_t L = layers_.size();
  std::vector<PLayer> host(L);
  std::vector<CUtensorMap> maps(L * 6 + 1);
  for (size_t l = 0; l < L; ++l) {
    const Layer& y = layers_[l];
    PLayer& p = host[l];
    const PSegSpec qkv[3] = {
        {y.wqkv, q_raw_, nullptr, Q, projection_partials(D, Q), Q},
        {y.wqkv + size_t(Q) * D, k_raw_, nullptr, G, projection_partials(D, G), G},
        {y.wqkv + size_t(Q + G) * D, vcache_[l], &state_->position, G, projection_partials(D, G), G}};
    const PSegSpec o = {y.wo, residual_, nullptr, D, projection_partials(Q, D), D};
    const PSegSpec gu = {y.wgu, gu_, nullptr, 2 * F, projection_partials(D, F), F};
    const PSegSpec dn = {y.wd, residual_, nullptr, D, projection_partials(F, D), D};
    if (!plan_persist_gemv(p.qkv, qkv, 3, residual_, y.in_norm, D, kEpilogueStore, grid, &maps[l * 6]) ||
        !plan_persist_gemv(p.o, &o, 1, att_, nullptr, Q, kEpilogueResidual, grid, &maps[l * 6 + 3]) ||
        !plan_persist_gemv(p.gu, &gu, 1, residual_, y.post_norm, D, kEpilogueSwiGLU, grid, &maps[l * 6 + 4]) ||
        !plan_persist_gemv(p.down, &dn, 1, gu_, nullptr, F, kEpilogueResidual, grid, &maps[l * 6 + 5]))
      return false;
    p.q_norm = y.q_norm;
    p.k_norm = y.k_norm;
    p.k_cache = kcache_[l];
    p.v_cache = vcache_[l];
  }
  const PSegSpec head = {lm_head_, logits_, nullptr, V, projection_partials(D, V), V};
  if (!plan_persist_gemv(persist_head_, &head, 1, residual_, final_norm_, D, kEpilogueArgmax, grid, &maps[L * 6]))
    return false;
  check(cudaMalloc(&persist_maps_, maps.size() * sizeof(CUtensorMap)), "persistent maps");
  check(cudaMalloc(&persist_layers_, L * sizeof(PLayer)), "persistent plan");
  for (size_t l = 0; l < L; ++l) {
    PGemv* ph[4] = {&host[l].qkv, &host[l].o, &host[l].gu, &host[l].down};
    const int base[4] = {0, 3, 4, 5};
    for (int k = 0; k < 4; ++k)
      for (int i = 0; i < ph[k]->nseg; ++i) ph[k]->seg[i].map = persist_maps_ + l * 6 + base[k] + i;
  }
  persist_head_.seg[0].map = persist_maps_ + L * 6;
  check(cudaMemcpy(persist_maps_, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice),
        "persistent maps copy");
  check(cudaMemcpy(persist_layers_, host.data(), L * sizeof(PLayer), cudaMemcpyHostToDevice), "persistent plan copy");
  persist_state_ = 1;
  return true;
}

void Engine::launch_persistent_step(bool greedy) {
  PersistArgs a = {};
  a.layers = persist_layers_;
  a.nlayers = int(layers_.size());
  a.head = persist_head_;
  a.head.epilogue = greedy ? kEpilogueArgmax : kEpilogueStore;
  a.q_raw = q_raw_;
  a.k_raw = k_raw_;
  a.scores = scores_;
  a.att = att_;
  a.residual = residual_;
  a.inv_freq = inv_freq_;
  a.position = &state_->position;
  a.hidden = int(cfg_.hidden);
  a.query_heads = int(cfg_.query_heads);
  a.kv_heads = int(cfg_.kv_heads);
  a.width = int(cfg_.head_width);
  a.capacity = int(capacity_);
  a.scale = attention_scale(int(cfg_.head_width));
  a.eps = cfg_.epsilon;
  a.score_stride = int(align_up(capacity_, 4));
  a.score_slices = std::max(1, sms_ / int(cfg_.kv_heads));
  a.pv_features = 8;
  // DOLITTLE_PERSIST_PREFETCH overrides the L2 prefetch distance (stages).
  static const int prefetch = [] {
    const char* v = std::getenv("DOLITTLE_PERSIST_PREFETCH");
    return v ? std::max(0, std::min(256, std::atoi(v))) : kPersistPrefetchStages;
  }();
  a.prefetch_stages = prefetch;
  a.capture = capture_layer_ >= 0 ? capture_arena_ : nullptr;
  a.capture_layer = capture_layer_;
  a.edit_layer = edit_layer_;
  a.edit_row = (long long)edit_row_;
  a.edit_strength = edit_strength_;
  a.edit_direction = edit_direction_;
  a.edit_state = edit_state_;
  a.partials = partials_;
  a.ticket = &state_->ticket;
  if (greedy) {
    a.select.result = state_->result;
    a.select.history = history_;
    a.select.step = &state_->step;
    a.select.embed = embed_;
    a.select.residual = residual_;
    a.select.width = int(cfg_.hidden);
    a.select.terminal = &state_->terminal;
    a.select.stop_mask = stop_mask_;
    a.select.position = &state_->position;
  }
  a.barrier = &state_->barrier;
  a.exit_ticket = &state_->exit_ticket;
  a.err = &state_->err;
  check(launch_decode_persistent(a, sms_, stream_), "persistent decode");
  ++launches_;
}

void Engine::decode_step(bool pdl) {
  if (decode_path_ == DL_DECODE_PERSISTENT && persistent_decode_ready()) {
    launch_persistent_step(mode_ == 0);
    if (mode_ != 0) {
      check(sampler_submit(sampler_, logits_, sampler_.settings, 0, true, stream_), "sampler");
      check(sampler_feed(sampler_, history_, &state_->step, embed_, residual_, int(cfg_.hidden), &state_->position,
                         stream_),
            "sampler feed");
      launches_ += sampler_launch_count(sampler_, sampler_.settings, true) + 1;
    }
    return;
  }
  run_layers(1, pdl);
  select(residual_, true, pdl);
}

void Engine::capture_decode_graph() {
  if (decode_exec_ && graph_capture_layer_ == capture_layer_ && graph_edit_layer_ == edit_layer_ &&
      graph_mode_ == mode_ && graph_path_ == decode_path_)
    return;
  // Plan outside the capture (it allocates and copies).
  if (decode_path_ == DL_DECODE_PERSISTENT) persistent_decode_ready();
  if (decode_exec_) {
    cudaGraphExecDestroy(decode_exec_);
    decode_exec_ = nullptr;
  }
  cudaGraph_t graph = nullptr;
  check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
  launches_ = 0;
  try {
    decode_step(true);
  } catch (...) {
    cudaStreamEndCapture(stream_, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  check(cudaStreamEndCapture(stream_, &graph), "end capture");
  kernels_per_step_ = launches_;
  const cudaError_t e = cudaGraphInstantiate(&decode_exec_, graph, 0);
  cudaGraphDestroy(graph);
  check(e, "graph instantiate");
  graph_capture_layer_ = capture_layer_;
  graph_edit_layer_ = edit_layer_;
  graph_mode_ = mode_;
  graph_path_ = decode_path_;
}

void Engine::begin_sequence(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s,
                            uint64_t seed, const uint32_t* stop_ids, size_t n_stop, int prefill_mode) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (seq_running_) throw std::logic_error("a device sequence is running: drain it first");
  if (!n_prompt || !max_new) throw std::invalid_argument("empty prompt or budget");
  if (n_prompt + max_new > capacity_) throw std::length_error("sequence exceeds KV capacity");
  validate_sampling(s, cfg_.vocabulary);
  if (prefill_mode != DL_PREFILL_PARITY && prefill_mode != DL_PREFILL_FAST)
    throw std::invalid_argument("unknown prefill mode");
  for (size_t i = 0; i < n_stop; ++i)
    if (stop_ids[i] >= cfg_.vocabulary) throw std::invalid_argument("stop ID outside vocabulary");
  reset();
  mode_ = s.mode;
  if (!sampler_.arena) check(sampler_init(sampler_, cfg_.vocabulary, true), "sampler init");
  check(sampler_start(sampler_, s, seed, stop_ids, n_stop, stream_), "sampler start");
  stop_mask_ = sampler_.stop_mask;  // the greedy finisher latches on the same mask
}

void Engine::generate(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s,
                      uint64_t seed, const uint32_t* stop_ids, size_t n_stop, int prefill_mode,
                      uint32_t* tokens_out, size_t* n_out, uint16_t* logits_out, dl_generation_stats* stats) {
  begin_sequence(prompt, n_prompt, max_new, s, seed, stop_ids, n_stop, prefill_mode);
  capture_decode_graph();
  const size_t V = cfg_.vocabulary;
  check(cudaEventRecord(ev_[0], stream_), "event");
  launches_ = 0;
  consume_rows(prompt, n_prompt, true, prefill_mode, 0);
  select(residual_ + size_t(last_rows_ - 1) * cfg_.hidden, false, true);
  check(cudaEventRecord(ev_[1], stream_), "event");
  // DOLITTLE_DECODE_GRAPH=0 launches the same per-token kernels eagerly
  // instead of replaying the captured graph (for per-kernel profilers).
  static const bool use_graph = [] {
    const char* v = std::getenv("DOLITTLE_DECODE_GRAPH");
    return !(v && v[0] == '0');
  }();
  auto step = [&] {
    if (use_graph)
      check(cudaGraphLaunch(decode_exec_, stream_), "graph launch");
    else
      decode_step(true);
  };
  if (logits_out) {
    check(cudaMemcpyAsync(logits_out, logits_, V * 2, cudaMemcpyDeviceToHost, stream_), "logits");
    for (size_t i = 1; i < max_new; ++i) {
      step();
      check(cudaMemcpyAsync(logits_out + i * V, logits_, V * 2, cudaMemcpyDeviceToHost, stream_), "logits");
    }
  } else {
    for (size_t i = 1; i < max_new; ++i) step();
  }
  check(cudaEventRecord(ev_[2], stream_), "event");
  check(cudaMemcpyAsync(tokens_out, history_, max_new * 4, cudaMemcpyDeviceToHost, stream_), "history");
  DeviceState st;
  check(cudaMemcpyAsync(&st, state_, sizeof(st), cudaMemcpyDeviceToHost, stream_), "state");
  check(cudaStreamSynchronize(stream_), "generate sync");
  float pre = 0, dec = 0;
  check(cudaEventElapsedTime(&pre, ev_[0], ev_[1]), "elapsed");
  check(cudaEventElapsedTime(&dec, ev_[1], ev_[2]), "elapsed");
  // Stop at the first stop ID (inclusive) or failed selection, like the
  // reference's device loop (src/kernels/cuda/decode.cu:161-194).
  size_t produced = max_new;
  {
    std::vector<unsigned char> stop(cfg_.vocabulary, 0);
    for (size_t i = 0; i < n_stop; ++i) stop[stop_ids[i]] = 1;
    for (size_t i = 0; i < max_new; ++i)
      if (stop[tokens_out[i]]) {
        produced = i + 1;
        break;
      }
  }
  *n_out = produced;
  if (stats) {
    stats->prefill_ms = pre;
    stats->decode_ms = dec;
    stats->decode_steps = max_new - 1;
    stats->kernels_per_decode_step = kernels_per_step_;
    stats->kernels_total = launches_ + kernels_per_step_ * (max_new - 1);
    stats->status = st.result[1];
    stats->fault = st.err;
  }
  if (st.err) throw std::runtime_error("device fault word " + std::to_string(st.err));
}

// ---------------------------------------------------------------------------
// Device-side generation loop (DeviceSequence): one graph = journal the
// first selection and set the loop condition, then a WHILE node whose body
// is the decode step plus the journal/condition kernel.
// ---------------------------------------------------------------------------
void Engine::build_loop_graph() {
  if (loop_exec_ && loop_capture_layer_ == capture_layer_ && loop_edit_layer_ == edit_layer_ && loop_mode_ == mode_ &&
      loop_path_ == decode_path_)
    return;
  if (decode_path_ == DL_DECODE_PERSISTENT) persistent_decode_ready();  // plans outside the capture
  if (loop_exec_) {
    cudaGraphExecDestroy(loop_exec_);
    loop_exec_ = nullptr;
  }
  const unsigned* result = mode_ == 0 ? state_->result : sampler_.result;
  cudaGraph_t g = nullptr;
  check(cudaGraphCreate(&g, 0), "loop graph");
  try {
    cudaGraphConditionalHandle loop;
    check(cudaGraphConditionalHandleCreate(&loop, g, 0, 0), "loop handle");
    cudaGraph_t captured = nullptr;
    check(cudaStreamBeginCaptureToGraph(stream_, g, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal),
          "capture first selection");
    const cudaError_t e1 = launch_journal_selection(&state_->step, result, &state_->position, stop_mask_,
                                                    &state_->limit, cancel_dev_, journal_dev_, loop, true, stream_);
    check(cudaStreamEndCapture(stream_, &captured), "end capture");
    check(e1, "journal kernel");
    cudaGraphNode_t first = nullptr;
    size_t nodes = 1;
    check(cudaGraphGetNodes(g, &first, &nodes), "loop graph nodes");
    cudaGraphNodeParams cp = {};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = loop;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    cudaGraphNode_t node = nullptr;
    check(cudaGraphAddNode(&node, g, &first, 1, &cp), "while node");
    cudaGraph_t body = cp.conditional.phGraph_out[0];
    check(cudaStreamBeginCaptureToGraph(stream_, body, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal),
          "capture loop body");
    launches_ = 0;
    try {
      decode_step(false);
      check(launch_journal_selection(&state_->step, result, &state_->position, stop_mask_, &state_->limit,
                                     cancel_dev_, journal_dev_, loop, true, stream_),
            "journal kernel");
    } catch (...) {
      cudaStreamEndCapture(stream_, &captured);
      throw;
    }
    check(cudaStreamEndCapture(stream_, &captured), "end capture");
    kernels_per_step_ = launches_ + 1;
    check(cudaGraphInstantiate(&loop_exec_, g, 0), "loop graph instantiate");
  } catch (...) {
    cudaGraphDestroy(g);
    throw;
  }
  cudaGraphDestroy(g);
  loop_capture_layer_ = capture_layer_;
  loop_edit_layer_ = edit_layer_;
  loop_mode_ = mode_;
  loop_path_ = decode_path_;
}

void Engine::start(const uint32_t* prompt, size_t n_prompt, size_t max_new, const dl_sampling& s, uint64_t seed,
                   const uint32_t* stop_ids, size_t n_stop, int prefill_mode) {
  begin_sequence(prompt, n_prompt, max_new, s, seed, stop_ids, n_stop, prefill_mode);
  build_loop_graph();
  std::memset(journal_host_, 0, (max_new + 2) * sizeof(dl_sequence_event));
  *reinterpret_cast<volatile unsigned*>(cancel_host_) = 0;
  const unsigned limit = unsigned(max_new);
  check(cudaMemcpyAsync(&state_->limit, &limit, 4, cudaMemcpyHostToDevice, stream_), "limit");
  check(cudaEventRecord(ev_[0], stream_), "event");
  launches_ = 0;
  consume_rows(prompt, n_prompt, true, prefill_mode, 0);
  check(launch_journal_consumed(journal_dev_, n_prompt, stream_), "journal");
  select(residual_ + size_t(last_rows_ - 1) * cfg_.hidden, false, true);
  check(cudaEventRecord(ev_[1], stream_), "event");
  check(cudaGraphLaunch(loop_exec_, stream_), "loop launch");
  check(cudaEventRecord(ev_[2], stream_), "event");
  seq_running_ = true;
  seq_max_new_ = max_new;
  seq_launches_ = launches_ + 1;
}

bool Engine::collect(size_t index, long long timeout_ms, dl_sequence_event* out) {
  if (!seq_running_ && index >= seq_max_new_ + 2) throw std::invalid_argument("no such journal event");
  if (index >= journal_cap_) throw std::invalid_argument("journal index beyond capacity + 2");
  const volatile uint8_t* kind = &journal_host_[index].kind;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    if (*kind) {
      std::atomic_thread_fence(std::memory_order_acquire);
      std::memcpy(out, const_cast<const dl_sequence_event*>(&journal_host_[index]), sizeof(*out));
      return true;
    }
    const cudaError_t q = cudaStreamQuery(stream_);
    if (q != cudaSuccess && q != cudaErrorNotReady) check(q, "sequence");
    if (q == cudaSuccess && !*kind) return false;  // the loop ended without this event
    if (timeout_ms >= 0 &&
        std::chrono::steady_clock::now() - t0 >= std::chrono::milliseconds(timeout_ms))
      return false;
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

void Engine::request_stop() { *reinterpret_cast<volatile unsigned*>(cancel_host_) = 1; }

void Engine::drain(uint32_t* tokens_out, size_t* n_out, dl_generation_stats* stats) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!seq_running_) throw std::logic_error("no device sequence is running");
  seq_running_ = false;
  check(cudaStreamSynchronize(stream_), "drain");
  DeviceState st;
  check(cudaMemcpy(&st, state_, sizeof(st), cudaMemcpyDeviceToHost), "state");
  const size_t n = std::min(size_t(std::max(st.step, 0)), seq_max_new_);
  if (tokens_out && n) check(cudaMemcpy(tokens_out, history_, n * 4, cudaMemcpyDeviceToHost), "history");
  if (n_out) *n_out = n;
  float pre = 0, dec = 0;
  check(cudaEventElapsedTime(&pre, ev_[0], ev_[1]), "elapsed");
  check(cudaEventElapsedTime(&dec, ev_[1], ev_[2]), "elapsed");
  if (stats) {
    stats->prefill_ms = pre;
    stats->decode_ms = dec;
    stats->decode_steps = n ? n - 1 : 0;
    stats->kernels_per_decode_step = kernels_per_step_;
    stats->kernels_total = seq_launches_ + kernels_per_step_ * (n ? n - 1 : 0);
    stats->status = st.result[1];
    stats->fault = st.err;
  }
  if (st.err) throw std::runtime_error("device fault word " + std::to_string(st.err));
}

}  // namespace dl
