// Server implementation (see serve.h).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include <dlfcn.h>
#include <nvtx3/nvToolsExt.h>

#include "attention_prefill_tc.h"
#include "gemm_tcgen05.h"
#include "serve.h"
#include "steering.h"

namespace dl {

namespace {
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// NCCL is resolved at run time, only when a tensor-parallel group connects:
// a process that already loaded libnccl.so.2 (PyTorch's bundled copy, say)
// keeps using that copy, and single-GPU use never loads NCCL at all.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  const char* (*error_string)(ncclResult_t);
};

const NcclApi& nccl() {
  static const NcclApi api = [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) throw std::runtime_error("tensor parallelism needs libnccl.so.2");
    NcclApi a{};
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.all_reduce || !a.all_gather || !a.comm_destroy ||
        !a.error_string)
      throw std::runtime_error("libnccl.so.2 lacks the NCCL 2 API");
    return a;
  }();
  return api;
}
}  // namespace

void Server::check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void Server::check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + nccl().error_string(r));
}

Server::Server(const dl_model_config& cfg, int device, size_t batch, size_t capacity, size_t chunk_rows, int tp_rank,
               int tp_size)
    : cfg_(cfg), device_(device), batch_(batch), capacity_(capacity), chunk_(chunk_rows), rank_(tp_rank),
      tp_(tp_size) {
  D_ = cfg.hidden;
  d_ = cfg.head_width;
  V_ = cfg.vocabulary;
  L_ = cfg.layers;
  if (tp_ < 1 || rank_ < 0 || rank_ >= tp_ || cfg.kv_heads % tp_ || cfg.mlp_width % (size_t(tp_) * 64))
    throw std::invalid_argument("tensor-parallel size must divide the KV heads and the MLP width");
  hq_ = int(cfg.query_heads) / tp_;
  hkv_ = int(cfg.kv_heads) / tp_;
  Ql_ = size_t(hq_) * d_;
  Gl_ = size_t(hkv_) * d_;
  Fl_ = cfg.mlp_width / tp_;
  // The vocabulary head is split by rows too: rank r holds vocabulary rows
  // [r V/t, (r+1) V/t), padded with zero rows to a multiple of 128 (the GEMM
  // tile); the ranks' logits meet in an all-gather.
  if (V_ % size_t(tp_)) throw std::invalid_argument("tensor-parallel size must divide the vocabulary");
  Vl_ = V_ / tp_;
  Vp_ = tp_ == 1 ? V_ : align_up(Vl_, 128);
  if (!batch || batch > 128 || !capacity || !chunk_rows || chunk_rows > 4096 || cfg.query_heads % cfg.kv_heads ||
      d_ != 128 || D_ % 128 || V_ % 128 || Ql_ % 128 || (tp_ > 1 && Vl_ % 8) || !L_ ||
      !attention_prefill_tc_supported(hq_, hkv_, int(d_)))
    throw std::invalid_argument("unsupported serving configuration");
  check(cudaSetDevice(device), "cudaSetDevice");
  check(cudaDeviceGetAttribute(&sms_, cudaDevAttrMultiProcessorCount, device), "sm count");
  check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
  for (auto& ev : ev_) check(cudaEventCreate(&ev), "event");

  // ---- weights (this rank's slices) ----
  size_t off = 0;
  auto take = [&](size_t elems) {
    const size_t o = off;
    off = align_up(off + elems * 2, 256);
    return o;
  };
  const size_t o_embed = take(V_ * D_), o_final = take(D_), o_head = take(Vp_ * D_);
  std::vector<size_t> lo(L_ * 8);
  for (size_t l = 0; l < L_; ++l) {
    lo[l * 8 + 0] = take(D_);
    lo[l * 8 + 1] = take((Ql_ + 2 * Gl_) * D_);
    lo[l * 8 + 2] = take(d_);
    lo[l * 8 + 3] = take(d_);
    lo[l * 8 + 4] = take(D_ * Ql_);
    lo[l * 8 + 5] = take(D_);
    lo[l * 8 + 6] = take(2 * Fl_ * D_);
    lo[l * 8 + 7] = take(D_ * Fl_);
  }
  check(cudaMalloc(&weight_arena_, off), "weights");
  check(cudaMemsetAsync(weight_arena_, 0, off, stream_), "weights clear");  // zero padding rows of the head slice
  auto* base = static_cast<unsigned char*>(weight_arena_);
  embed_ = reinterpret_cast<bf16*>(base + o_embed);
  final_norm_ = reinterpret_cast<bf16*>(base + o_final);
  lm_head_ = reinterpret_cast<bf16*>(base + o_head);
  layers_.resize(L_);
  for (size_t l = 0; l < L_; ++l) {
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

  // ---- KV: sequence b, block l: K plane then V plane, each [C][Gl] ----
  plane_elems_ = align_up(capacity * Gl_ * 2, 256) / 2;
  seq_elems_ = plane_elems_ * 2 * L_;
  check(cudaMalloc(&kv_arena_, seq_elems_ * 2 * batch), "kv cache");
  check(cudaMemsetAsync(kv_arena_, 0, seq_elems_ * 2 * batch, stream_), "kv clear");

  // ---- scratch ----
  const size_t R = std::max(chunk_rows, batch), B = batch;
  history_cap_ = capacity + 1;
  // DOLITTLE_ATTN_PLAN=even keeps even key ranges (a tuning override).
  static const bool even_ranges = [] {
    const char* v = std::getenv("DOLITTLE_ATTN_PLAN");
    return v && std::string(v) == "even";
  }();
  attn_plan_ = even_ranges ? AttnPlan{attention_decode_splits(int(B), hkv_, int(capacity), sms_), 0}
                           : attention_decode_plan(int(B), hkv_, int(capacity), sms_);
  // Split-K partials of the decode projections (and the FP32 sums of the
  // row-sliced projections under tensor parallelism).
  const int Ns[4] = {int(Ql_ + 2 * Gl_), int(D_), int(2 * Fl_), int(D_)};
  const int Ks[4] = {int(D_), int(Ql_), int(D_), int(Fl_)};
  for (int i = 0; i < 4; ++i)
    parts_floats_ = std::max(parts_floats_, size_t(gemm_splitk_parts(int(B), Ns[i], Ks[i], sms_)) * B * Ns[i]);
  parts_floats_ = std::max(parts_floats_, R * D_);
  vt_stride_ = int(align_up(capacity, 64));
  size_t so = 0;
  auto grab = [&](size_t bytes) {
    const size_t o = so;
    so = align_up(so + bytes, 256);
    return o;
  };
  const size_t o_res = grab(R * D_ * 2), o_xn = grab(R * D_ * 2), o_qkv = grab(B * (Ql_ + 2 * Gl_) * 2),
               o_qraw = grab(R * Ql_ * 2), o_kraw = grab(R * Gl_ * 2), o_qrot = grab(R * Ql_ * 2),
               o_att = grab(R * Ql_ * 2), o_act = grab(R * Fl_ * 2), o_logits = grab(B * V_ * 2),
               o_hlocal = grab(tp_ > 1 ? B * Vp_ * 2 : 0), o_hgather = grab(tp_ > 1 ? size_t(tp_) * B * Vp_ * 2 : 0),
               o_xlast = grab(B * D_ * 2), o_vt = grab(size_t(hkv_) * d_ * vt_stride_ * 2),
               o_parts = grab(parts_floats_ * 4),
               o_ws = grab(attention_decode_ws_floats(int(B), hq_, attn_plan_.splits) * 4),
               o_tickets = grab(B * size_t(hkv_) * 4), o_tok = grab(R * 4),
               o_hist = grab(B * history_cap_ * 4), o_steps = grab(B * 4), o_pos = grab(8), o_err = grab(16),
               o_freq = grab(d_ / 2 * 4);
  check(cudaMalloc(&scratch_, so), "scratch");
  check(cudaMemsetAsync(scratch_, 0, so, stream_), "scratch clear");
  auto* sb = static_cast<unsigned char*>(scratch_);
  residual_ = reinterpret_cast<bf16*>(sb + o_res);
  xn_ = reinterpret_cast<bf16*>(sb + o_xn);
  qkv_ = reinterpret_cast<bf16*>(sb + o_qkv);
  q_raw_ = reinterpret_cast<bf16*>(sb + o_qraw);
  k_raw_ = reinterpret_cast<bf16*>(sb + o_kraw);
  q_rot_ = reinterpret_cast<bf16*>(sb + o_qrot);
  att_ = reinterpret_cast<bf16*>(sb + o_att);
  act_ = reinterpret_cast<bf16*>(sb + o_act);
  logits_ = reinterpret_cast<bf16*>(sb + o_logits);
  head_local_ = reinterpret_cast<bf16*>(sb + o_hlocal);
  head_gather_ = reinterpret_cast<bf16*>(sb + o_hgather);
  xlast_ = reinterpret_cast<bf16*>(sb + o_xlast);
  vt_ = reinterpret_cast<bf16*>(sb + o_vt);
  parts_ = reinterpret_cast<float*>(sb + o_parts);
  attn_ws_ = reinterpret_cast<float*>(sb + o_ws);
  attn_tickets_ = reinterpret_cast<int*>(sb + o_tickets);
  tokens_dev_ = reinterpret_cast<uint32_t*>(sb + o_tok);
  history_ = reinterpret_cast<uint32_t*>(sb + o_hist);
  steps_ = reinterpret_cast<int*>(sb + o_steps);
  position_ = reinterpret_cast<long long*>(sb + o_pos);
  err_ = reinterpret_cast<unsigned*>(sb + o_err);
  inv_freq_ = reinterpret_cast<float*>(sb + o_freq);
  for (size_t b = 0; b < B; ++b) {
    AttnTcMaps* m = attention_prefill_tc_maps(q_rot_, int(chunk_rows), hq_, kcache(b, 0), plane_elems_ * 2,
                                              int(capacity), int(L_), hkv_, int(d_), vt_, vt_stride_);
    if (!m) throw std::runtime_error("prompt attention tensor maps");
    attn_maps_.push_back(m);
  }
  check(sampler_init(sampler_, V_, true, unsigned(B)), "sampler init");
  check(launch_inv_freq(inv_freq_, int(d_), cfg.theta, stream_), "inv_freq");
  check(cudaStreamSynchronize(stream_), "init sync");
}

Server::~Server() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  if (step_exec_) cudaGraphExecDestroy(step_exec_);
  if (comm_) nccl().comm_destroy(comm_);
  for (auto* p : peer_open_)
    if (p) cudaIpcCloseMemHandle(p);
  cudaFree(peer_mem_);
  cudaFree(peer_epoch_);
  for (auto* m : attn_maps_) attention_prefill_tc_free(m);
  sampler_free(sampler_);
  for (auto& ev : ev_)
    if (ev) cudaEventDestroy(ev);
  cudaFree(scratch_);
  cudaFree(kv_arena_);
  cudaFree(weight_arena_);
  cudaFree(capture_);
  cudaFree(steer_mem_);
  if (stream_) cudaStreamDestroy(stream_);
}

void Server::nccl_id(unsigned char* out128) {
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess) throw std::runtime_error("ncclGetUniqueId failed");
  static_assert(sizeof(id) == 128, "NCCL unique id size");
  std::memcpy(out128, &id, sizeof(id));
}

void Server::connect(const unsigned char* id128) {
  if (tp_ == 1) return;
  if (comm_) throw std::logic_error("already connected");
  check(cudaSetDevice(device_), "cudaSetDevice");
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof(id));
  check_nccl(nccl().comm_init_rank(&comm_, tp_, id, rank_), "ncclCommInitRank");
  // NCCL sets up the connections of an algorithm the first time a message
  // needs it, blocking the host for a second or more.  Run each collective
  // once here, at the sizes the server uses (a prompt chunk's and a decode
  // step's all-reduce, the logits all-gather; the buffers are scratch), so
  // that cost belongs to connecting and not to the first prompt pass.
  all_reduce(parts_, chunk_ * D_);
  all_reduce(parts_, batch_ * D_);
  check_nccl(nccl().all_gather(head_local_, head_gather_, batch_ * Vp_, ncclBfloat16, comm_, stream_),
             "ncclAllGather");
  check(cudaStreamSynchronize(stream_), "connect sync");
}

void Server::ipc_handle(unsigned char* out64) {
  if (tp_ == 1) throw std::logic_error("no tensor-parallel group");
  if (tp_ > kPeerMaxRanks) throw std::invalid_argument("peer all-reduce supports up to 8 ranks");
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!peer_mem_) {
    const size_t bytes = peer_buffer_bytes(tp_, batch_ * D_);
    check(cudaMalloc(&peer_mem_, bytes), "peer buffer");
    check(cudaMemset(peer_mem_, 0, bytes), "peer buffer clear");
    check(cudaMalloc(reinterpret_cast<void**>(&peer_epoch_), kPeerChunks * 4), "peer epochs");
    check(cudaMemset(peer_epoch_, 0, kPeerChunks * 4), "peer epochs clear");
  }
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, peer_mem_), "ipc handle");
  static_assert(sizeof(h) == 64, "CUDA IPC handle size");
  std::memcpy(out64, &h, 64);
}

void Server::connect_peers(const unsigned char* handles) {
  if (!peer_mem_) throw std::logic_error("ipc_handle first");
  if (peers_) throw std::logic_error("peers already connected");
  check(cudaSetDevice(device_), "cudaSetDevice");
  const size_t cap = batch_ * D_;
  const size_t data_bytes = size_t(2) * tp_ * cap * 4;
  pb_ = PeerBuffers{};
  for (int r = 0; r < tp_; ++r) {
    void* base = peer_mem_;
    if (r != rank_) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles + size_t(r) * 64, 64);
      check(cudaIpcOpenMemHandle(&peer_open_[r], h, cudaIpcMemLazyEnablePeerAccess), "ipc open");
      base = peer_open_[r];
    }
    pb_.data[r] = static_cast<float*>(base);
    pb_.flags[r] = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(base) + data_bytes);
  }
  pb_.epoch = peer_epoch_;
  pb_.err = err_;
  pb_.ranks = tp_;
  pb_.rank = rank_;
  pb_.capacity = cap;
  peers_ = true;
  if (step_exec_) {  // the decode graph picks the peer path at capture
    cudaGraphExecDestroy(step_exec_);
    step_exec_ = nullptr;
  }
}

// Slice of tensor `index` held by this rank.  q/k/v and gate/up: row ranges
// (output columns of the projection); o and down: column ranges (its input
// features); the rest whole.
Server::Slice Server::slice(size_t index) {
  size_t fr = 0, fc = 0;
  if (!Engine::tensor_shape(cfg_, index, &fr, &fc)) throw std::invalid_argument("tensor index out of range");
  Slice s{nullptr, fr, fc, fc, 0, 0, fc};
  if (index == 0) s.ptr = embed_;
  else if (index == 1) s.ptr = final_norm_;
  else if (index == 2) {
    s.ptr = lm_head_;
    s.rows = Vl_;
    s.r0 = size_t(rank_) * Vl_;
  }
  else {
    const size_t l = (index - 3) / 11, role = (index - 3) % 11;
    const Layer& y = layers_[l];
    const size_t r = size_t(rank_);
    switch (role) {
      case 0: s.ptr = y.in_norm; break;
      case 1: s.ptr = y.wqkv; s.rows = Ql_; s.r0 = r * Ql_; break;
      case 2: s.ptr = y.wqkv + Ql_ * D_; s.rows = Gl_; s.r0 = r * Gl_; break;
      case 3: s.ptr = y.wqkv + (Ql_ + Gl_) * D_; s.rows = Gl_; s.r0 = r * Gl_; break;
      case 4: s.ptr = y.q_norm; break;
      case 5: s.ptr = y.k_norm; break;
      case 6: s.ptr = y.wo; s.cols = Ql_; s.stride = Ql_; s.c0 = r * Ql_; break;
      case 7: s.ptr = y.post_norm; break;
      case 8: s.ptr = y.wgu; s.rows = Fl_; s.r0 = r * Fl_; s.stride = 2 * D_; break;
      case 9: s.ptr = y.wgu + D_; s.rows = Fl_; s.r0 = r * Fl_; s.stride = 2 * D_; break;
      default: s.ptr = y.wd; s.cols = Fl_; s.stride = Fl_; s.c0 = r * Fl_; break;
    }
  }
  return s;
}

bool Server::slice_shape(size_t index, size_t* rows, size_t* cols, size_t* r0, size_t* c0) {
  if (index >= Engine::tensor_count(cfg_)) return false;
  const Slice s = slice(index);
  *rows = s.rows;
  *cols = s.cols;
  *r0 = s.r0;
  *c0 = s.c0;
  return true;
}

void Server::init_random(uint64_t seed, float sigma) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  const double sd = std::sqrt(8.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const float scale = static_cast<float>(double(sigma) / sd);
  for (size_t i = 0; i < Engine::tensor_count(cfg_); ++i) {
    const Slice s = slice(i);
    size_t fr = 0, fc = 0;
    Engine::tensor_shape(cfg_, i, &fr, &fc);
    if (fr == 1)
      check(launch_fill_const(s.ptr, s.cols, 1.0f, stream_), "fill norm");
    else
      check(launch_fill_normal_slice(s.ptr, s.rows, s.cols, s.stride, s.full_cols, s.r0, s.c0, seed, uint32_t(i),
                                     scale, stream_),
            "fill normal slice");
  }
  check(cudaStreamSynchronize(stream_), "init_random sync");
}

void Server::set_tensor(size_t index, const void* host, size_t bytes) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  size_t fr = 0, fc = 0;
  if (!Engine::tensor_shape(cfg_, index, &fr, &fc)) throw std::invalid_argument("tensor index out of range");
  if (bytes != fr * fc * 2) throw std::invalid_argument("tensor byte size mismatch");
  const Slice s = slice(index);
  const auto* src = static_cast<const unsigned char*>(host) + (s.r0 * fc + s.c0) * 2;
  check(cudaMemcpy2DAsync(s.ptr, s.stride * 2, src, fc * 2, s.cols * 2, s.rows, cudaMemcpyHostToDevice, stream_),
        "set_tensor");
  check(cudaStreamSynchronize(stream_), "set_tensor sync");
}

void Server::get_tensor(size_t index, void* host, size_t bytes) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  const Slice s = slice(index);
  if (bytes != s.rows * s.cols * 2) throw std::invalid_argument("tensor byte size mismatch");
  check(cudaMemcpy2DAsync(host, s.cols * 2, s.ptr, s.stride * 2, s.cols * 2, s.rows, cudaMemcpyDeviceToHost, stream_),
        "get_tensor");
  check(cudaStreamSynchronize(stream_), "get_tensor sync");
}

bf16* Server::kcache(size_t b, size_t layer) const {
  return static_cast<bf16*>(kv_arena_) + b * seq_elems_ + (2 * layer) * plane_elems_;
}
bf16* Server::vcache(size_t b, size_t layer) const {
  return static_cast<bf16*>(kv_arena_) + b * seq_elems_ + (2 * layer + 1) * plane_elems_;
}
KvPlanes Server::planes(size_t layer) const {
  return KvPlanes{static_cast<bf16*>(kv_arena_), seq_elems_, 2 * layer * plane_elems_, (2 * layer + 1) * plane_elems_};
}

size_t Server::position() {
  long long p = 0;
  check(cudaMemcpyAsync(&p, position_, 8, cudaMemcpyDeviceToHost, stream_), "position");
  check(cudaStreamSynchronize(stream_), "position sync");
  return size_t(p);
}

void Server::check_fault() {
  unsigned err = 0;
  check(cudaMemcpyAsync(&err, err_, 4, cudaMemcpyDeviceToHost, stream_), "fault read");
  check(cudaStreamSynchronize(stream_), "fault sync");
  if (err) throw std::runtime_error("device fault word " + std::to_string(err));
}

void Server::gemm(const bf16* x, int ldx, const bf16* w, int M, int N, int K, int epi, int nseg, const int* n0s,
                  bf16* const* outs, const int* lds) {
  GemmProblem p = {};
  p.x = x;
  p.ldx = ldx;
  p.w = w;
  p.M = M;
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
  p.err = err_;
  check(launch_gemm_tcgen05(p, stream_, false), "gemm");
  ++launches_;
}

// Logits [B][V] of the B normed rows in xn_.  One rank: one GEMM.  Several
// ranks: this rank's vocabulary rows [B][Vp], the all-gather of every rank's
// rows, then the ranks' valid columns into [B][V] (every rank then samples
// the same tokens from the same logits).
void Server::vocabulary_head(int B) {
  const int n0s[1] = {0};
  const int lds[1] = {int(Vp_)};
  if (tp_ == 1) {
    bf16* outs[1] = {logits_};
    gemm(xn_, int(D_), lm_head_, B, int(V_), int(D_), kGemmStore, 1, n0s, outs, lds);
    return;
  }
  bf16* outs[1] = {head_local_};
  gemm(xn_, int(D_), lm_head_, B, int(Vp_), int(D_), kGemmStore, 1, n0s, outs, lds);
  check_nccl(nccl().all_gather(head_local_, head_gather_, size_t(B) * Vp_, ncclBfloat16, comm_, stream_),
             "ncclAllGather");
  check(launch_gather_vocab_slices(head_gather_, logits_, tp_, B, int(Vl_), int(Vp_), stream_), "vocab gather");
  launches_ += 2;
}

void Server::all_reduce(float* buf, size_t n) {
  check_nccl(nccl().all_reduce(buf, buf, n, ncclFloat, ncclSum, comm_, stream_), "ncclAllReduce");
}

// o_proj / down_proj of M rows into the residual.  One rank: the GEMM adds
// into the residual (split-K for the decode rows).  Several ranks: the FP32
// partial sums of this rank's input slice, the all-reduce, then the add.
void Server::row_projection_out(const bf16* x, int ldx, const bf16* w, int M, int K, bool decode) {
  const int N = int(D_);
  GemmProblem p = {};
  p.x = x;
  p.ldx = ldx;
  p.w = w;
  p.M = M;
  p.N = N;
  p.K = K;
  p.err = err_;
  if (tp_ == 1 && !decode) {
    const int n0s[1] = {0};
    bf16* outs[1] = {residual_};
    const int lds[1] = {N};
    gemm(x, ldx, w, M, N, K, kGemmResidual, 1, n0s, outs, lds);
    return;
  }
  const int parts = decode ? gemm_splitk_parts(M, N, K, sms_) : 1;
  check(launch_gemm_tcgen05_parts(p, parts, parts_, stream_, decode), "gemm parts");
  ++launches_;
  if (tp_ == 1) {
    check(launch_gemm_splitk_epilogue(parts_, parts, M, N, kGemmResidual, residual_, N, nullptr, stream_,
                                      decode && fused_step()),
          "splitk epilogue");
    ++launches_;
    return;
  }
  // Decode rows: one kernel sums the K parts, exchanges them over NVLink peer
  // memory and adds the residual (NCCL when DOLITTLE_TP_ALLREDUCE=nccl, and
  // for the prompt pass's large messages).
  if (decode && peer_decode(M)) {
    check(launch_peer_allreduce_residual(pb_, parts_, parts, M, N, residual_, nullptr, nullptr, 0.f, stream_, false),
          "peer all-reduce");
    ++launches_;
    return;
  }
  if (parts > 1) {
    // Sum the K parts in place into part 0 (FP32), then all-reduce.
    check(launch_gemm_splitk_epilogue(parts_, parts, M, N, kGemmStore, nullptr, N, parts_, stream_), "splitk sum");
    ++launches_;
  }
  all_reduce(parts_, size_t(M) * N);
  check(launch_add_fp32_residual(parts_, residual_, size_t(M) * N, stream_), "add residual");
  launches_ += 2;
}

void Server::prefill_sequence(size_t b, const uint32_t* tokens, size_t n) {
  const int D = int(D_), Q = int(Ql_), G = int(Gl_), F = int(Fl_), d = int(d_);
  for (size_t c0 = 0; c0 < n; c0 += chunk_) {
    const int rows = int(std::min(chunk_, n - c0));
    check(cudaMemcpyAsync(tokens_dev_, tokens + c0, rows * 4, cudaMemcpyHostToDevice, stream_), "tokens");
    check(launch_embedding(tokens_dev_, embed_, residual_, rows, D, stream_, false), "embed");
    for (size_t l = 0; l < L_; ++l) {
      const Layer& y = layers_[l];
      check(launch_rms_norm(residual_, y.in_norm, xn_, size_t(rows), D, cfg_.epsilon, stream_), "rms_norm");
      {
        const int n0s[3] = {0, Q, Q + G};
        bf16* outs[3] = {q_raw_, k_raw_, vcache(b, l) + c0 * G};
        const int lds[3] = {Q, G, G};
        gemm(xn_, D, y.wqkv, rows, Q + 2 * G, D, kGemmStore, 3, n0s, outs, lds);
      }
      check(launch_qk_norm_rope(q_raw_, k_raw_, y.q_norm, y.k_norm, inv_freq_, q_rot_, kcache(b, l),
                                RowPositions{nullptr, (long long)c0}, rows, hq_, hkv_, d, cfg_.epsilon, stream_, false),
            "qk_norm_rope");
      check(launch_vt_transpose(vcache(b, l), vt_, int(c0) + rows, hkv_, d, vt_stride_, stream_), "v transpose");
      check(launch_attention_prefill_tc(attn_maps_[b], att_, rows, (long long)c0, int(l), hq_, hkv_,
                                        attention_scale(d), err_, stream_),
            "attention prefill");
      launches_ += 4;
      row_projection_out(att_, Q, y.wo, rows, Q, false);
      check(launch_rms_norm(residual_, y.post_norm, xn_, size_t(rows), D, cfg_.epsilon, stream_), "rms_norm");
      ++launches_;
      {
        const int n0s[1] = {0};
        bf16* outs[1] = {act_};
        const int lds[1] = {F};
        gemm(xn_, D, y.wgu, rows, 2 * F, D, kGemmSwiGLU, 1, n0s, outs, lds);
      }
      row_projection_out(act_, F, y.wd, rows, F, false);
      block_output_hooks(l, b, c0, rows);
    }
    if (c0 + rows == n)
      check(cudaMemcpyAsync(xlast_ + b * D_, residual_ + size_t(rows - 1) * D_, D_ * 2, cudaMemcpyDeviceToDevice,
                            stream_),
            "last row");
  }
}

void Server::prefill(const uint32_t* tokens, size_t prompt_len, const dl_sampling& s, uint64_t seed,
                     uint32_t* first_out) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!prompt_len || prompt_len >= capacity_) throw std::length_error("prompt exceeds KV capacity");
  if (tp_ > 1 && !comm_) throw std::logic_error("tensor-parallel server is not connected");
  validate_sampling(s, V_);
  settings_ = s;
  check(cudaEventRecord(ev_[0], stream_), "event");
  for (size_t b = 0; b < batch_; ++b) prefill_sequence(b, tokens + b * prompt_len, prompt_len);
  // Vocabulary head on the B last rows, then each row's first selection
  // (the sampler feeds the token's embedding row in as the next input).
  const int B = int(batch_);
  check(launch_rms_norm(xlast_, final_norm_, xn_, batch_, int(D_), cfg_.epsilon, stream_), "final norm");
  vocabulary_head(B);
  check(cudaMemsetAsync(steps_, 0, batch_ * 4, stream_), "steps");
  // Row b draws from the stream seeded with seed + b.
  check(sampler_start(sampler_, s, seed, nullptr, 0, stream_), "sampler start");
  check(sampler_submit(sampler_, logits_, s, 0, true, stream_, V_), "sampler");
  check(sampler_feed(sampler_, history_, steps_, embed_, residual_, int(D_), nullptr, stream_, history_cap_),
        "sampler feed");
  const long long pos = (long long)prompt_len;
  check(cudaMemcpyAsync(position_, &pos, 8, cudaMemcpyHostToDevice, stream_), "position");
  std::vector<uint32_t> first(batch_);
  for (size_t b = 0; b < batch_; ++b)
    check(cudaMemcpyAsync(&first[b], history_ + b * history_cap_, 4, cudaMemcpyDeviceToHost, stream_), "first");
  check(cudaEventRecord(ev_[1], stream_), "event");
  check(cudaStreamSynchronize(stream_), "prefill sync");
  check_fault();
  float ms = 0.f;
  check(cudaEventElapsedTime(&ms, ev_[0], ev_[1]), "elapsed");
  prefill_ms_ = ms;
  if (first_out) std::memcpy(first_out, first.data(), batch_ * 4);
  started_ = true;
  if (step_exec_) {
    cudaGraphExecDestroy(step_exec_);
    step_exec_ = nullptr;
  }
}

// Block-output hooks, in the reference's order: the steering edit, then the
// capture of the (edited) rows.  Prompt chunk: rows c0 .. c0+rows-1 of
// sequence b.  beta comes from the source sequence's row before its edit.
void Server::block_output_hooks(size_t l, size_t b, size_t c0, int rows) {
  const int D = int(D_);
  if (int(l) == steer_layer_) {
    if (steer_source_ == (long long)b && steer_source_pos_ >= c0 && steer_source_pos_ < c0 + size_t(rows)) {
      check(launch_steer_beta(residual_ + (steer_source_pos_ - c0) * D_, D, steer_strength_, steer_beta_, err_,
                              stream_),
            "steer beta");
      ++launches_;
    }
    check(launch_steer_rows(residual_, D, rows, nullptr, (long long)c0, false, steer_mask_ + b, steer_first_,
                            steer_beta_, steer_dir_, err_, stream_),
          "steer rows");
    ++launches_;
  }
  if (int(l) == capture_layer_) {
    check(cudaMemcpyAsync(capture_ + (b * capacity_ + c0) * D_, residual_, size_t(rows) * D_ * 2,
                          cudaMemcpyDeviceToDevice, stream_),
          "capture rows");
  }
}

void Server::block_output_hooks_decode(size_t l) {
  const int D = int(D_), B = int(batch_);
  if (int(l) == steer_layer_) {
    check(launch_steer_rows(residual_, D, B, position_, 0, true, steer_mask_, steer_first_, steer_beta_, steer_dir_,
                            err_, stream_),
          "steer rows");
    ++launches_;
  }
  if (int(l) == capture_layer_) {
    check(launch_capture_batch(residual_, capture_, capacity_ * D_, position_, D, B, stream_), "capture rows");
    ++launches_;
  }
}

void Server::set_capture(int layer) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (layer >= int(L_)) throw std::invalid_argument("capture layer out of range");
  if (layer >= 0 && !capture_) {
    check(cudaMalloc(&capture_, batch_ * capacity_ * D_ * 2), "capture arena");
    check(cudaMemsetAsync(capture_, 0, batch_ * capacity_ * D_ * 2, stream_), "capture clear");
  }
  capture_layer_ = layer < 0 ? -1 : layer;
  if (step_exec_) {
    cudaGraphExecDestroy(step_exec_);
    step_exec_ = nullptr;
  }
}

void Server::read_capture(size_t sequence, size_t first, size_t count, uint16_t* host) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!capture_ || sequence >= batch_ || first + count > capacity_) throw std::invalid_argument("capture range");
  check(cudaMemcpyAsync(host, capture_ + (sequence * capacity_ + first) * D_, count * D_ * 2, cudaMemcpyDeviceToHost,
                        stream_),
        "read capture");
  check(cudaStreamSynchronize(stream_), "read capture sync");
}

void Server::set_steering(int layer, size_t first, float strength, const float* direction, const uint8_t* mask,
                          long long source_sequence, size_t source_position) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (layer >= int(L_)) throw std::invalid_argument("steering layer out of range");
  if (step_exec_) {
    cudaGraphExecDestroy(step_exec_);
    step_exec_ = nullptr;
  }
  if (layer < 0) {
    steer_layer_ = -1;
    return;
  }
  if (!direction || !mask || !std::isfinite(strength)) throw std::invalid_argument("steering arguments");
  for (size_t i = 0; i < D_; ++i)
    if (!std::isfinite(direction[i])) throw std::invalid_argument("steering direction must be finite");
  if (source_sequence >= 0) {
    // beta comes from the source row in the prompt pass, before any masked
    // sequence prefilled after it needs it.
    if (size_t(source_sequence) >= batch_ || source_position >= capacity_)
      throw std::invalid_argument("steering source out of range");
    for (size_t b = 0; b < size_t(source_sequence); ++b)
      if (mask[b]) throw std::invalid_argument("steered sequences must follow the strength source");
  }
  if (!steer_mem_) check(cudaMalloc(&steer_mem_, D_ * 4 + 256 + batch_), "steering state");
  steer_dir_ = static_cast<float*>(steer_mem_);
  steer_beta_ = reinterpret_cast<float*>(static_cast<unsigned char*>(steer_mem_) + D_ * 4);
  steer_mask_ = static_cast<unsigned char*>(steer_mem_) + D_ * 4 + 256;
  check(cudaMemcpyAsync(steer_dir_, direction, D_ * 4, cudaMemcpyHostToDevice, stream_), "steering direction");
  check(cudaMemcpyAsync(steer_beta_, &strength, 4, cudaMemcpyHostToDevice, stream_), "steering strength");
  check(cudaMemcpyAsync(steer_mask_, mask, batch_, cudaMemcpyHostToDevice, stream_), "steering mask");
  check(cudaStreamSynchronize(stream_), "steering sync");
  steer_layer_ = layer;
  steer_first_ = (long long)first;
  steer_strength_ = strength;
  steer_source_ = source_sequence;
  steer_source_pos_ = source_position;
}

void Server::set_step_fusion(bool on) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (on == fuse_) return;
  fuse_ = on;
  if (step_exec_) {
    cudaGraphExecDestroy(step_exec_);
    step_exec_ = nullptr;
  }
}

float Server::steering_strength() {
  check(cudaSetDevice(device_), "cudaSetDevice");
  float b = 0.f;
  if (steer_beta_) {
    check(cudaMemcpyAsync(&b, steer_beta_, 4, cudaMemcpyDeviceToHost, stream_), "steering strength");
    check(cudaStreamSynchronize(stream_), "steering strength sync");
  }
  return b;
}

// o / down projection of the B decode rows into the residual, the block
// output hooks of `layer` (none for o: layer < 0), then xn_ = RMSNorm of the
// residual with norm_w.  Fused (one rank, no hook on this block): the GEMM
// and one kernel that adds the split-K parts into the residual and normalises
// the rows.
void Server::decode_projection_norm(const bf16* x, int K, const bf16* w, int layer, const bf16* norm_w) {
  const int B = int(batch_), D = int(D_);
  const bool hooks = layer >= 0 && (layer == steer_layer_ || layer == capture_layer_);
  const bool fold = fused_step() && !hooks;
  if (fold && (tp_ == 1 || peer_decode(B))) {
    GemmProblem p = {};
    p.err = err_;
    p.x = x;
    p.ldx = K;
    p.w = w;
    p.M = B;
    p.N = D;
    p.K = K;
    const int parts = gemm_splitk_parts(B, D, K, sms_);
    check(launch_gemm_tcgen05_parts(p, parts, parts_, stream_, true), "gemm parts");
    if (tp_ == 1)
      check(launch_residual_norm_rows(parts_, parts, B, D, residual_, norm_w, xn_, cfg_.epsilon, stream_, true),
            "residual norm");
    else
      check(launch_peer_allreduce_residual(pb_, parts_, parts, B, D, residual_, norm_w, xn_, cfg_.epsilon, stream_,
                                           true),
            "peer all-reduce + norm");
    launches_ += 2;
    return;
  }
  if (fold && tp_ > 1) {
    // NCCL: the parts summed in part order, the all-reduce, then one kernel
    // for the residual add and the norm (the parts kernel with one part).
    GemmProblem p = {};
    p.err = err_;
    p.x = x;
    p.ldx = K;
    p.w = w;
    p.M = B;
    p.N = D;
    p.K = K;
    const int parts = gemm_splitk_parts(B, D, K, sms_);
    check(launch_gemm_tcgen05_parts(p, parts, parts_, stream_, true), "gemm parts");
    if (parts > 1) {
      check(launch_gemm_splitk_epilogue(parts_, parts, B, D, kGemmStore, nullptr, D, parts_, stream_), "splitk sum");
      ++launches_;
    }
    all_reduce(parts_, size_t(B) * D);
    check(launch_residual_norm_rows(parts_, 1, B, D, residual_, norm_w, xn_, cfg_.epsilon, stream_, false),
          "residual norm");
    launches_ += 3;
    return;
  }
  row_projection_out(x, K, w, B, K, true);
  if (layer >= 0) block_output_hooks_decode(size_t(layer));
  check(launch_rms_norm(residual_, norm_w, xn_, batch_, D, cfg_.epsilon, stream_, fused_step()), "rms_norm");
  ++launches_;
}

// Decode all-reduces over NVLink peer memory for two ranks, NCCL for more:
// every rank writes its whole partial to every other rank, so the bytes a
// rank sends grow with t - 1 while NCCL's in-switch and tree reductions do
// not.  Measured at batch 32, 2K context: peer 4.73 / NCCL 4.55 ms per step at
// four ranks, 5.70 / 4.74 ms at eight; even at two (where the peer kernel also
// applies the next RMSNorm).  DOLITTLE_TP_ALLREDUCE=nccl or =peer overrides.
// One CTA per row, so at most kPeerChunks rows.
bool Server::peer_decode(int rows) const {
  static const int mode = [] {
    const char* v = std::getenv("DOLITTLE_TP_ALLREDUCE");
    if (v && std::string(v) == "nccl") return 1;
    if (v && std::string(v) == "peer") return 2;
    return 0;
  }();
  const bool peer = mode == 2 || (mode == 0 && tp_ == 2);
  return tp_ > 1 && peers_ && peer && rows <= kPeerChunks && size_t(rows) * D_ <= pb_.capacity && D_ % 8 == 0 &&
         D_ > 128 && D_ <= 8192;
}

// The fused decode step: split-K sums folded into the kernels that consume
// them (the attention kernel, residual + RMSNorm), the attention splits
// merged by their last CTA, and every kernel of the chain a programmatic
// dependent launch.  Same arithmetic as the unfused step, bit for bit.
bool Server::fused_step() const { return fuse_ && d_ == 128 && D_ > 128 && D_ % 8 == 0 && D_ <= 8192; }

// One decode step for all B rows at the shared position.  xn_ holds the
// normed input of block l at the top of each iteration.
void Server::decode_body() {
  const int B = int(batch_), D = int(D_), Q = int(Ql_), G = int(Gl_), F = int(Fl_), d = int(d_);
  const bool fused = fused_step();
  check(launch_rms_norm(residual_, layers_[0].in_norm, xn_, batch_, D, cfg_.epsilon, stream_, fused), "rms_norm");
  ++launches_;
  for (size_t l = 0; l < L_; ++l) {
    const Layer& y = layers_[l];
    GemmProblem p = {};
    p.err = err_;
    p.x = xn_;
    p.ldx = D;
    p.w = y.wqkv;
    p.M = B;
    p.N = Q + 2 * G;
    p.K = D;
    int parts = gemm_splitk_parts(B, p.N, p.K, sms_);
    // The split-K projections are programmatic dependent launches: their
    // weights stream in while the previous kernel finishes.
    check(launch_gemm_tcgen05_parts(p, parts, parts_, stream_, true), "qkv parts");
    if (fused) {
      // The attention kernel builds the queries and appends the new key and
      // value from the qkv parts itself.
      const AttnQkvIn qi{parts_, parts, B, Q + 2 * G, y.q_norm, y.k_norm, inv_freq_, cfg_.epsilon};
      check(launch_attention_decode_batched(q_rot_, planes(l), position_, B, hq_, hkv_, attn_plan_.splits,
                                            attn_plan_.lead_q10, attention_scale(d), attn_ws_, att_, stream_,
                                            attn_tickets_, true, &qi),
            "qkv parts + attention decode");
      launches_ += 2;
    } else {
      check(launch_gemm_splitk_epilogue(parts_, parts, B, p.N, kGemmStore, qkv_, p.N, nullptr, stream_), "qkv sum");
      check(launch_norm_rope_append_rows(qkv_, Q + 2 * G, y.q_norm, y.k_norm, inv_freq_, q_rot_, planes(l),
                                         position_, B, hq_, hkv_, d, cfg_.epsilon, stream_),
            "norm rope append");
      check(launch_attention_decode_batched(q_rot_, planes(l), position_, B, hq_, hkv_, attn_plan_.splits,
                                            attn_plan_.lead_q10, attention_scale(d), attn_ws_, att_, stream_),
            "attention decode");
      launches_ += 5;
    }
    decode_projection_norm(att_, Q, y.wo, -1, y.post_norm);
    p.w = y.wgu;
    p.N = 2 * F;
    p.K = D;
    parts = gemm_splitk_parts(B, p.N, p.K, sms_);
    check(launch_gemm_tcgen05_parts(p, parts, parts_, stream_, true), "gate/up parts");
    check(launch_gemm_splitk_epilogue(parts_, parts, B, p.N, kGemmSwiGLU, act_, F, nullptr, stream_, fused),
          "swiglu");
    launches_ += 2;
    decode_projection_norm(act_, F, y.wd, int(l), l + 1 < L_ ? layers_[l + 1].in_norm : final_norm_);
  }
  vocabulary_head(B);
  check(sampler_submit(sampler_, logits_, settings_, 0, true, stream_, V_), "sampler");
  check(sampler_feed(sampler_, history_, steps_, embed_, residual_, D, nullptr, stream_, history_cap_), "sampler feed");
  launches_ += sampler_launch_count(sampler_, settings_, true) + 1;
  check(launch_add_position(position_, 1, stream_), "advance");
  launches_ += 2;
}

void Server::decode(size_t steps, uint32_t* tokens_out, uint16_t* logits_out, dl_serve_stats* stats) {
  check(cudaSetDevice(device_), "cudaSetDevice");
  if (!started_) throw std::logic_error("decode before prefill");
  const size_t pos0 = position();
  if (pos0 + steps > capacity_) throw std::length_error("generation exceeds KV capacity");
  if (!step_exec_) {
    const size_t before = launches_;
    cudaGraph_t graph = nullptr;
    check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "capture begin");
    try {
      decode_body();
    } catch (...) {
      cudaStreamEndCapture(stream_, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    check(cudaStreamEndCapture(stream_, &graph), "capture end");
    check(cudaGraphInstantiate(&step_exec_, graph, 0), "graph instantiate");
    cudaGraphDestroy(graph);
    kernels_per_step_ = launches_ - before;
  }
  nvtxRangePushA("serve_decode");  // profilers can select the decode steps alone
  check(cudaEventRecord(ev_[0], stream_), "event");
  for (size_t i = 0; i < steps; ++i) {
    check(cudaGraphLaunch(step_exec_, stream_), "graph launch");
    if (logits_out)
      check(cudaMemcpyAsync(logits_out + i * batch_ * V_, logits_, batch_ * V_ * 2, cudaMemcpyDeviceToHost, stream_),
            "logits");
  }
  check(cudaEventRecord(ev_[1], stream_), "event");
  nvtxRangePop();
  check(cudaStreamSynchronize(stream_), "decode sync");
  check_fault();
  float ms = 0.f;
  check(cudaEventElapsedTime(&ms, ev_[0], ev_[1]), "elapsed");
  if (tokens_out) {
    // history[b][1 + i] is sequence b's token of decode step i.
    std::vector<uint32_t> h(batch_ * history_cap_);
    check(cudaMemcpy(h.data(), history_, h.size() * 4, cudaMemcpyDeviceToHost), "history");
    int step_count = 0;
    check(cudaMemcpy(&step_count, steps_, 4, cudaMemcpyDeviceToHost), "steps");
    for (size_t i = 0; i < steps; ++i)
      for (size_t b = 0; b < batch_; ++b)
        tokens_out[i * batch_ + b] = h[b * history_cap_ + size_t(step_count) - steps + i];
  }
  if (stats) {
    stats->prefill_ms = prefill_ms_;
    stats->decode_ms = ms;
    stats->decode_steps = steps;
    stats->kernels_per_decode_step = kernels_per_step_;
  }
}

}  // namespace dl
