// C ABI entry points (include/dolittle_b200.h).  Validation mirrors the
// reference's prepared-operation checks (src/kernels/operations.cpp:192-202,
// src/kernels/cuda/common.cuh:57-65): unsupported dtypes and shapes are
// rejected, never silently converted.  Exceptions become dl_status codes and
// a thread-local message.
#include <climits>
#include <cstring>
#include <exception>
#include <new>
#include <stdexcept>
#include <string>

#include "../../include/dolittle_b200.h"
#include "attention_prefill_tc.h"
#include "engine.h"
#include "gemm_tcgen05.h"
#include "gemv.cuh"
#include "launch.h"
#include "sampler.h"
#include "serve.h"
#include "serve_kernels.h"
#include "steering.h"

namespace {
thread_local std::string g_error;

dl_status fail(dl_status s, const std::string& msg) {
  g_error = msg;
  return s;
}
dl_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DL_OK;
  return fail(DL_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}
template <class F>
dl_status guarded(F&& f) {
  try {
    return f();
  } catch (const std::invalid_argument& e) {
    return fail(DL_INVALID_ARGUMENT, e.what());
  } catch (const std::length_error& e) {
    return fail(DL_OUT_OF_MEMORY, e.what());
  } catch (const std::bad_alloc& e) {
    return fail(DL_OUT_OF_MEMORY, e.what());
  } catch (const std::exception& e) {
    const std::string m = e.what();
    return fail(m.find("device fault") != std::string::npos ? DL_DEVICE_FAULT : DL_CUDA_ERROR, m);
  }
}
cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }
using dl::bf16;
}  // namespace

namespace dl {
void set_last_error(const std::string& message) { g_error = message; }
}  // namespace dl

struct dl_engine {
  dl::Engine* impl;
};
struct dl_sampler {
  dl::Sampler s;
};
struct dl_serve {
  dl::Server* impl;
};

extern "C" {

DL_API const char* dl_last_error(void) { return g_error.c_str(); }
DL_API const char* dl_version(void) { return "dolittle_b200 0.1 (sm_100a)"; }

DL_API dl_status dl_projection(dl_dtype type, const void* input, const void* weight, void* output,
                               size_t rows, size_t input_width, size_t output_width, void* stream,
                               const size_t* output_position) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "projection: only BF16 storage is supported");
  if (!input || !weight || !output || !rows || !input_width || !output_width)
    return fail(DL_INVALID_ARGUMENT, "projection: null pointer or empty shape");
  if (input_width % 8 || reinterpret_cast<uintptr_t>(weight) % 16)
    return fail(DL_UNSUPPORTED, "projection: input width must be a multiple of 8, weight 16-byte aligned");
  if (output_width > (1u << 30) || input_width > (1u << 20)) return fail(DL_UNSUPPORTED, "projection: shape");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int I = int(input_width);
  const int rt = dl::gemv_rows_template(int(rows), I);
  for (size_t g0 = 0; g0 < rows; g0 += rt) {
    dl::GemvArgs a = {};
    a.x = static_cast<const bf16*>(input) + g0 * input_width;
    a.x_stride = I;
    a.in_width = I;
    a.nrows = int(std::min<size_t>(rt, rows - g0));
    a.prologue = dl::kProloguePlain;
    a.epilogue = dl::kEpilogueStore;
    a.nseg = 1;
    a.seg[0].w = static_cast<const bf16*>(weight);
    a.seg[0].out = static_cast<bf16*>(output) + g0 * output_width;
    a.seg[0].out_row = reinterpret_cast<const long long*>(output_position);
    a.seg[0].rows = int(output_width);
    a.seg[0].partials = dl::projection_partials(input_width, output_width);
    a.seg[0].out_stride = int(output_width);
    const dl_status s = cuda_status(dl::launch_gemv(a, rt, sms, st(stream), false), "projection");
    if (s != DL_OK) return s;
  }
  return DL_OK;
}

DL_API dl_status dl_rms_norm(dl_dtype type, const void* input, const void* weight, void* output,
                             size_t rows, size_t width, float epsilon, void* stream) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "rms_norm: only BF16 storage is supported");
  if (!input || !weight || !output || !rows || !width) return fail(DL_INVALID_ARGUMENT, "rms_norm: arguments");
  if (width > 32768) return fail(DL_UNSUPPORTED, "rms_norm: width above 32768");
  return cuda_status(dl::launch_rms_norm(static_cast<const bf16*>(input), static_cast<const bf16*>(weight),
                                         static_cast<bf16*>(output), rows, int(width), epsilon, st(stream)),
                     "rms_norm");
}

DL_API dl_status dl_rotary(dl_dtype type, const void* input, void* output, size_t positions, size_t heads,
                           size_t width, size_t first_position, double theta, void* stream,
                           const size_t* device_position, int positioned_output) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "rotary: only BF16 storage is supported");
  if (!input || !output || !positions || !heads || !width || width % 2)
    return fail(DL_INVALID_ARGUMENT, "rotary: arguments");
  dl::RowPositions pos{reinterpret_cast<const long long*>(device_position), (long long)first_position};
  return cuda_status(dl::launch_rotary(static_cast<const bf16*>(input), static_cast<bf16*>(output), positions,
                                       int(heads), int(width), pos, theta, positioned_output != 0, st(stream)),
                     "rotary");
}

DL_API dl_status dl_attention_scale(float* output, size_t width, void* stream) {
  if (!output || !width) return fail(DL_INVALID_ARGUMENT, "attention_scale: arguments");
  const float v = dl::attention_scale(int(width));
  return cuda_status(cudaMemcpyAsync(output, &v, 4, cudaMemcpyHostToDevice, st(stream)), "attention_scale");
}

DL_API size_t dl_attention_workspace_bytes(size_t positions, size_t query_heads, size_t capacity) {
  return positions * query_heads * capacity * sizeof(float);
}

DL_API size_t dl_attention_prefill_fast_workspace_bytes(size_t kv_heads, size_t width, size_t capacity) {
  return kv_heads * width * ((capacity + 63) / 64 * 64) * 2;
}

DL_API dl_status dl_attention_prefill_fast(const void* query, const void* key, const void* value, void* output,
                                           size_t positions, size_t query_heads, size_t kv_heads, size_t width,
                                           void* stream, size_t first_position, size_t capacity,
                                           void* workspace) {
  if (!query || !key || !value || !output || !workspace || !positions || !kv_heads)
    return fail(DL_INVALID_ARGUMENT, "attention prefill: arguments");
  if (!dl::attention_prefill_tc_supported(int(query_heads), int(kv_heads), int(width)))
    return fail(DL_UNSUPPORTED, "attention prefill: head width 128 and whole GQA groups required");
  if (first_position + positions > capacity) return fail(DL_INVALID_ARGUMENT, "attention prefill: keys > capacity");
  const int vt_stride = int((capacity + 63) / 64 * 64);
  dl::AttnTcMaps* maps = dl::attention_prefill_tc_maps(
      static_cast<const bf16*>(query), int(positions), int(query_heads), static_cast<const bf16*>(key),
      capacity * kv_heads * width * 2, int(capacity), 1, int(kv_heads), int(width),
      static_cast<const bf16*>(workspace), vt_stride);
  if (!maps) return fail(DL_UNSUPPORTED, "attention prefill: tensor maps");
  dl_status s = cuda_status(dl::launch_vt_transpose(static_cast<const bf16*>(value), static_cast<bf16*>(workspace),
                                                    int(first_position + positions), int(kv_heads), int(width),
                                                    vt_stride, st(stream)),
                            "attention prefill: V transpose");
  if (s == DL_OK)
    s = cuda_status(dl::launch_attention_prefill_tc(maps, static_cast<bf16*>(output), int(positions),
                                                    (long long)first_position, 0, int(query_heads), int(kv_heads),
                                                    dl::attention_scale(int(width)), nullptr, st(stream)),
                    "attention prefill");
  dl::attention_prefill_tc_free(maps);  // the kernel took the maps by value
  return s;
}

DL_API dl_status dl_attention(dl_dtype type, const void* query, const void* key, const void* value,
                              void* output, size_t positions, size_t query_heads, size_t kv_heads,
                              size_t width, void* stream, size_t first_position,
                              const size_t* device_position, size_t capacity, const float* scale,
                              void* workspace) {
  (void)scale;  // the scale law float(1/sqrt(double(d))) is applied in-kernel
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "attention: only BF16 storage is supported");
  if (!query || !key || !value || !output || !workspace || !positions || !kv_heads || !width)
    return fail(DL_INVALID_ARGUMENT, "attention: arguments");
  if (query_heads % kv_heads || query_heads / kv_heads > 8 || width > 128 || width % 8)
    return fail(DL_UNSUPPORTED, "attention: GQA group <= 8 and head width <= 128 (multiple of 8)");
  const size_t cap = device_position ? capacity : first_position + positions;
  if (cap * 4 > 200 * 1024) return fail(DL_UNSUPPORTED, "attention: more than 51200 keys");
  dl::RowPositions pos{reinterpret_cast<const long long*>(device_position), (long long)first_position};
  const int ctas = positions == 1 ? 16 : 8;
  dl_status s = cuda_status(
      dl::launch_attention_scores(static_cast<const bf16*>(query), static_cast<const bf16*>(key),
                                  static_cast<float*>(workspace), pos, int(positions), int(query_heads),
                                  int(kv_heads), int(width), int(cap), dl::attention_scale(int(width)), ctas,
                                  st(stream), false),
      "attention scores");
  if (s != DL_OK) return s;
  return cuda_status(dl::launch_attention_pv(static_cast<const float*>(workspace), static_cast<const bf16*>(value),
                                             static_cast<bf16*>(output), pos, int(positions), int(query_heads),
                                             int(kv_heads), int(width), int(cap), st(stream), false),
                     "attention pv");
}

DL_API dl_status dl_embedding(dl_dtype type, const uint32_t* tokens, const void* weight, void* output,
                              size_t rows, size_t width, void* stream) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "embedding: only BF16 storage is supported");
  if (!tokens || !weight || !output || !rows || !width) return fail(DL_INVALID_ARGUMENT, "embedding: arguments");
  return cuda_status(dl::launch_embedding(tokens, static_cast<const bf16*>(weight), static_cast<bf16*>(output),
                                          int(rows), int(width), st(stream), false),
                     "embedding");
}

DL_API dl_status dl_add(dl_dtype type, const void* left, const void* right, void* output, size_t count,
                        void* stream) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "add: only BF16 storage is supported");
  if (!left || !right || !output || !count) return fail(DL_INVALID_ARGUMENT, "add: arguments");
  return cuda_status(dl::launch_add(static_cast<const bf16*>(left), static_cast<const bf16*>(right),
                                    static_cast<bf16*>(output), count, st(stream)),
                     "add");
}

DL_API dl_status dl_silu_multiply(dl_dtype type, const void* gate, const void* up, void* output, size_t count,
                                  void* stream) {
  if (type != DL_BF16) return fail(DL_UNSUPPORTED, "silu_multiply: only BF16 storage is supported");
  if (!gate || !up || !output || !count) return fail(DL_INVALID_ARGUMENT, "silu_multiply: arguments");
  return cuda_status(dl::launch_silu_multiply(static_cast<const bf16*>(gate), static_cast<const bf16*>(up),
                                              static_cast<bf16*>(output), count, st(stream)),
                     "silu_multiply");
}

DL_API dl_status dl_qkv_projection(const void* residual, const void* norm_weight, float epsilon,
                                   const void* wqkv, size_t rows, size_t input_width, size_t q_rows,
                                   size_t kv_rows, void* q_out, void* k_out, void* v_out,
                                   const int64_t* v_position, void* stream) {
  if (!residual || !norm_weight || !wqkv || !q_out || !k_out || !v_out || !rows || rows > 8)
    return fail(DL_INVALID_ARGUMENT, "qkv_projection: arguments (rows 1..8)");
  if (input_width % 8 || input_width * 2 * rows > 64 * 1024 && rows > 1)
    return fail(DL_UNSUPPORTED, "qkv_projection: input width");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  dl::GemvArgs a = {};
  const int I = int(input_width), Qr = int(q_rows), Kr = int(kv_rows);
  const bf16* w = static_cast<const bf16*>(wqkv);
  a.x = static_cast<const bf16*>(residual);
  a.x_stride = I;
  a.in_width = I;
  a.nrows = int(rows);
  a.prologue = dl::kPrologueRmsNorm;
  a.norm_w = static_cast<const bf16*>(norm_weight);
  a.eps = epsilon;
  a.epilogue = dl::kEpilogueStore;
  a.nseg = 3;
  a.seg[0] = dl::make_segment(w, static_cast<bf16*>(q_out), nullptr, Qr, dl::projection_partials(I, Qr), Qr);
  a.seg[1] = dl::make_segment(w + size_t(Qr) * I, static_cast<bf16*>(k_out), nullptr, Kr,
                              dl::projection_partials(I, Kr), Kr);
  a.seg[2] = dl::make_segment(w + size_t(Qr + Kr) * I, static_cast<bf16*>(v_out),
                              reinterpret_cast<const long long*>(v_position), Kr, dl::projection_partials(I, Kr), Kr);
  return cuda_status(dl::launch_gemv(a, dl::gemv_rows_template(int(rows), I), sms, st(stream), false),
                     "qkv_projection");
}

DL_API dl_status dl_rope_inverse_frequency(float* output, size_t width, double theta, void* stream) {
  if (!output || !width || width % 2) return fail(DL_INVALID_ARGUMENT, "rope_inverse_frequency: arguments");
  return cuda_status(dl::launch_inv_freq(output, int(width), theta, st(stream)), "rope_inverse_frequency");
}

DL_API dl_status dl_qk_norm_rope_append(const void* q_raw, const void* k_raw, const void* q_norm_weight,
                                        const void* k_norm_weight, const float* inv_freq, void* q_out,
                                        void* k_cache, const int64_t* position, size_t rows,
                                        size_t query_heads, size_t kv_heads, size_t width, float epsilon,
                                        void* stream) {
  if (!q_raw || !k_raw || !q_norm_weight || !k_norm_weight || !inv_freq || !q_out || !k_cache || !position ||
      !rows || !query_heads || !kv_heads)
    return fail(DL_INVALID_ARGUMENT, "qk_norm_rope_append: arguments");
  if (width > 128 || width % 2) return fail(DL_UNSUPPORTED, "qk_norm_rope_append: head width <= 128, even");
  dl::RowPositions pos{reinterpret_cast<const long long*>(position), 0};
  return cuda_status(dl::launch_qk_norm_rope(static_cast<const bf16*>(q_raw), static_cast<const bf16*>(k_raw),
                                             static_cast<const bf16*>(q_norm_weight),
                                             static_cast<const bf16*>(k_norm_weight), inv_freq,
                                             static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache), pos,
                                             int(rows), int(query_heads), int(kv_heads), int(width), epsilon,
                                             st(stream), false),
                     "qk_norm_rope_append");
}

DL_API dl_status dl_gemm_bf16(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M, size_t N,
                              size_t K, int epilogue, void* stream) {
  if (!x || !w || !y || !M) return fail(DL_INVALID_ARGUMENT, "gemm: null pointer or empty shape");
  if (epilogue != dl::kGemmStore && epilogue != dl::kGemmResidual && epilogue != dl::kGemmSwiGLU)
    return fail(DL_INVALID_ARGUMENT, "gemm: epilogue must be 0, 1 or 3");
  if (!dl::gemm_tcgen05_supported(int(M), int(N), int(K)) || ldx % 8 || ldy % 8 || ldx < K ||
      (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) % 16)
    return fail(DL_UNSUPPORTED, "gemm: K % 64, N % 128, 8-element row strides and 16-byte alignment required");
  dl::GemmProblem p = {};
  p.x = static_cast<const bf16*>(x);
  p.ldx = int(ldx);
  p.w = static_cast<const bf16*>(w);
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.epilogue = epilogue;
  p.nseg = 1;
  p.seg_out[0] = static_cast<bf16*>(y);
  p.seg_ld[0] = int(ldy);
  p.wide_tiles = true;
  return cuda_status(dl::launch_gemm_tcgen05(p, st(stream), false), "gemm");
}

DL_API size_t dl_gemm_bf16_split_workspace_bytes(size_t M, size_t N) {
  return dl::gemm_split_floats(int(M), int(N), dl::kGemmMaxSplit) * 4;
}

DL_API dl_status dl_gemm_bf16_config(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                     size_t N, size_t K, int epilogue, void* stream, void* workspace,
                                     unsigned* tickets, size_t n_tickets, int tile_m, int tile_n, int parts) {
  if ((workspace == nullptr) != (tickets == nullptr))
    return fail(DL_INVALID_ARGUMENT, "gemm: workspace and tickets go together");
  if (workspace && n_tickets < ((M + 127) / 128) * (N / 128))
    return fail(DL_INVALID_ARGUMENT, "gemm split: one ticket per 128 x 128 tile required");
  if ((tile_m != 0 && tile_m != 128 && tile_m != 256) || (tile_n != 0 && tile_n != 128 && tile_n != 256) ||
      (tile_m == 256 && tile_n == 128) || parts < -1 || parts > dl::kGemmMaxSplit || (parts > 1 && !workspace) ||
      (parts == -1 && (!workspace || tile_m == 256)))
    return fail(DL_INVALID_ARGUMENT,
                "gemm: tile_m 0/128/256, tile_n 0/128/256 (256 x 128 does not exist), parts -1..4 (more than 1 and "
                "stream-K (-1, single-SM tiles) need the workspace)");
  if (!x || !w || !y || !M) return fail(DL_INVALID_ARGUMENT, "gemm: null pointer or empty shape");
  if (epilogue != dl::kGemmStore && epilogue != dl::kGemmResidual && epilogue != dl::kGemmSwiGLU)
    return fail(DL_INVALID_ARGUMENT, "gemm: epilogue must be 0, 1 or 3");
  if (!dl::gemm_tcgen05_supported(int(M), int(N), int(K)) || ldx % 8 || ldy % 8 || ldx < K ||
      (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) % 16)
    return fail(DL_UNSUPPORTED, "gemm: K % 64, N % 128, 8-element row strides and 16-byte alignment required");
  if (((tile_n == 256 || tile_m == 256) && N % 256) || (parts > 1 && size_t(K / 64) < size_t(4 * parts)))
    return fail(DL_UNSUPPORTED, "gemm: 256-wide tiles need N % 256; each K part needs 4 k-steps of 64");
  dl::GemmProblem p = {};
  p.x = static_cast<const bf16*>(x);
  p.ldx = int(ldx);
  p.w = static_cast<const bf16*>(w);
  p.M = int(M);
  p.N = int(N);
  p.K = int(K);
  p.epilogue = epilogue;
  p.nseg = 1;
  p.seg_out[0] = static_cast<bf16*>(y);
  p.seg_ld[0] = int(ldy);
  p.wide_tiles = true;
  if (workspace) {
    p.partial = static_cast<float*>(workspace);
    p.partial_floats = dl::gemm_split_floats(int(M), int(N), dl::kGemmMaxSplit);
    p.tickets = tickets;
    p.n_tickets = int(std::min<size_t>(n_tickets, 1u << 30));
  }
  p.force_bm = tile_m;
  p.force_bn = tile_n;
  // parts -1: stream-K; 1..4: that many K parts (no stream-K); 0: the cost model.
  p.force_split = parts > 0 ? parts : 0;
  p.force_streamk = parts == -1 ? 1 : parts > 0 ? -1 : 0;
  return cuda_status(dl::launch_gemm_tcgen05(p, st(stream), false), "gemm");
}

DL_API dl_status dl_gemm_bf16_split(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                    size_t N, size_t K, int epilogue, void* stream, void* workspace,
                                    unsigned* tickets, size_t n_tickets) {
  if (!workspace || !tickets) return fail(DL_INVALID_ARGUMENT, "gemm split: workspace and tickets required");
  return dl_gemm_bf16_config(x, ldx, w, y, ldy, M, N, K, epilogue, stream, workspace, tickets, n_tickets, 0, 0, 0);
}

DL_API dl_status dl_projection_residual(const void* input, const void* weight, void* residual, size_t rows,
                                        size_t input_width, size_t output_width, void* stream) {
  if (!input || !weight || !residual || !rows || input_width % 8)
    return fail(DL_INVALID_ARGUMENT, "projection_residual: arguments");
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int I = int(input_width);
  const int rt = dl::gemv_rows_template(int(rows), I);
  for (size_t g0 = 0; g0 < rows; g0 += rt) {
    dl::GemvArgs a = {};
    a.x = static_cast<const bf16*>(input) + g0 * input_width;
    a.x_stride = I;
    a.in_width = I;
    a.nrows = int(std::min<size_t>(rt, rows - g0));
    a.prologue = dl::kProloguePlain;
    a.epilogue = dl::kEpilogueResidual;
    a.nseg = 1;
    a.seg[0] = dl::make_segment(static_cast<const bf16*>(weight), static_cast<bf16*>(residual) + g0 * output_width,
                                nullptr, int(output_width), dl::projection_partials(input_width, output_width),
                                int(output_width));
    const dl_status s = cuda_status(dl::launch_gemv(a, rt, sms, st(stream), false), "projection_residual");
    if (s != DL_OK) return s;
  }
  return DL_OK;
}

// ---------------------------------------------------------------------------
// Steering / injection
// ---------------------------------------------------------------------------
DL_API dl_status dl_intervene(void* residual, const float* direction, const int64_t* position, uint32_t* state,
                              size_t width, size_t selected, size_t rows, float strength, void* stream) {
  if (!residual || !direction || !position || !state || !width || !rows)
    return fail(DL_INVALID_ARGUMENT, "intervene: arguments");
  return cuda_status(dl::launch_intervene(static_cast<bf16*>(residual), direction,
                                          reinterpret_cast<const long long*>(position), state, int(width),
                                          (long long)selected, int(rows), strength, st(stream), false),
                     "intervene");
}

DL_API dl_status dl_direction(dl_dtype type, const void* original, const void* edited, size_t width,
                              float* direction, uint32_t* status, void* stream) {
  if (type != DL_BF16 && type != DL_F32) return fail(DL_UNSUPPORTED, "direction: BF16 or FP32 reconstructions");
  if (!original || !edited || !direction || !status || !width || width > 0x7fffffffu)
    return fail(DL_INVALID_ARGUMENT, "direction: arguments");
  const size_t element = type == DL_BF16 ? 2 : 4;
  if (reinterpret_cast<uintptr_t>(original) % element || reinterpret_cast<uintptr_t>(edited) % element ||
      reinterpret_cast<uintptr_t>(direction) % 4 || reinterpret_cast<uintptr_t>(status) % 4)
    return fail(DL_INVALID_ARGUMENT, "direction: misaligned pointer");
  return cuda_status(dl::launch_direction(type == DL_BF16, original, edited, direction, status, int(width), st(stream)),
                     "direction");
}

DL_API dl_status dl_normalize_injection(const void* source, void* output, float* norm, uint32_t* status,
                                        size_t width, float scale, void* stream) {
  if (!source || !output || !norm || !status || !width) return fail(DL_INVALID_ARGUMENT, "normalize: arguments");
  return cuda_status(dl::launch_normalize_injection(static_cast<const bf16*>(source), static_cast<bf16*>(output),
                                                    norm, status, int(width), scale, st(stream)),
                     "normalize_injection");
}

// ---------------------------------------------------------------------------
// Sampler
// ---------------------------------------------------------------------------
DL_API size_t dl_sampler_required_bytes(size_t vocabulary) { return dl::sampler_required_bytes(vocabulary); }

DL_API dl_status dl_sampler_create(size_t vocabulary, dl_dtype type, dl_sampler** out) {
  if (!out || !vocabulary || vocabulary > 0x7fffffffu) return fail(DL_INVALID_ARGUMENT, "sampler: vocabulary");
  auto* s = new dl_sampler;
  const dl_status r = cuda_status(dl::sampler_init(s->s, vocabulary, type == DL_BF16), "sampler_create");
  if (r != DL_OK) {
    dl::sampler_free(s->s);
    delete s;
    return r;
  }
  *out = s;
  return DL_OK;
}

DL_API void dl_sampler_destroy(dl_sampler* s) {
  if (!s) return;
  dl::sampler_free(s->s);
  delete s;
}

DL_API dl_status dl_sampler_set_engine(dl_sampler* s, int engine) {
  if (!s || (engine != DL_RNG_MT19937_64 && engine != DL_RNG_PHILOX4X32_10))
    return fail(DL_INVALID_ARGUMENT, "sampler_set_engine: unknown engine");
  if (s->s.started) return fail(DL_INVALID_ARGUMENT, "sampler_set_engine: sampler already started");
  s->s.engine = unsigned(engine);
  return DL_OK;
}

DL_API dl_status dl_sampler_start(dl_sampler* s, const dl_sampling* settings, uint64_t seed,
                                  const uint32_t* stop_ids, size_t n_stop, void* stream) {
  if (!s || !settings || (n_stop && !stop_ids)) return fail(DL_INVALID_ARGUMENT, "sampler_start: arguments");
  return guarded([&] {
    if (s->s.started) throw std::invalid_argument("invalid or repeated device sampler start");
    dl::validate_sampling(*settings, s->s.vocabulary);
    for (size_t i = 0; i < n_stop; ++i)
      if (stop_ids[i] >= s->s.vocabulary) throw std::invalid_argument("stop ID outside vocabulary");
    const dl_status r =
        cuda_status(dl::sampler_start(s->s, *settings, seed, stop_ids, n_stop, st(stream)), "sampler_start");
    return r;
  });
}

DL_API dl_status dl_sampler_submit(dl_sampler* s, const void* row, const dl_sampling* settings, uint64_t bits,
                                   void* stream, const uint32_t** result) {
  if (!s || !row || !settings) return fail(DL_INVALID_ARGUMENT, "sampler_submit: arguments");
  return guarded([&] {
    dl::validate_sampling(*settings, s->s.vocabulary);
    const dl_status r =
        cuda_status(dl::sampler_submit(s->s, row, *settings, bits, false, st(stream)), "sampler_submit");
    if (result) *result = s->s.result;
    return r;
  });
}

DL_API dl_status dl_sampler_submit_next(dl_sampler* s, const void* row, void* stream, const uint32_t** result) {
  if (!s || !row) return fail(DL_INVALID_ARGUMENT, "sampler_submit_next: arguments");
  if (!s->s.started) return fail(DL_INVALID_ARGUMENT, "device sampler not started");
  const dl_status r =
      cuda_status(dl::sampler_submit(s->s, row, s->s.settings, 0, true, st(stream)), "sampler_submit_next");
  if (result) *result = s->s.result;
  return r;
}

// ---------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------
DL_API size_t dl_engine_tensor_count(const dl_model_config* c) { return c ? dl::Engine::tensor_count(*c) : 0; }

DL_API dl_status dl_engine_tensor_shape(const dl_model_config* c, size_t index, size_t* rows, size_t* cols) {
  if (!c || !rows || !cols || !dl::Engine::tensor_shape(*c, index, rows, cols))
    return fail(DL_INVALID_ARGUMENT, "tensor_shape: index");
  return DL_OK;
}

DL_API dl_status dl_engine_create(const dl_model_config* config, int device, size_t capacity, size_t max_rows,
                                  dl_engine** out) {
  if (!config || !out) return fail(DL_INVALID_ARGUMENT, "engine_create: arguments");
  return guarded([&] {
    *out = new dl_engine{new dl::Engine(*config, device, capacity, max_rows)};
    return DL_OK;
  });
}

DL_API void dl_engine_destroy(dl_engine* e) {
  if (!e) return;
  delete e->impl;
  delete e;
}

#define DL_ENGINE_CALL(body)                                           \
  if (!e || !e->impl) return fail(DL_INVALID_ARGUMENT, "null engine"); \
  return guarded([&] {                                                 \
    body;                                                              \
    return DL_OK;                                                      \
  })

DL_API dl_status dl_engine_init_random(dl_engine* e, uint64_t seed, float sigma) {
  DL_ENGINE_CALL(e->impl->init_random(seed, sigma));
}
DL_API dl_status dl_engine_set_tensor(dl_engine* e, size_t index, const void* host_bits, size_t bytes) {
  DL_ENGINE_CALL(e->impl->set_tensor(index, host_bits, bytes));
}
DL_API dl_status dl_engine_get_tensor(dl_engine* e, size_t index, void* host_bits, size_t bytes) {
  DL_ENGINE_CALL(e->impl->get_tensor(index, host_bits, bytes));
}
DL_API dl_status dl_engine_tensor_device(dl_engine* e, size_t index, void** device_ptr, size_t* row_stride) {
  if (!device_ptr) return fail(DL_INVALID_ARGUMENT, "tensor_device: null output");
  DL_ENGINE_CALL(*device_ptr = e->impl->tensor_device(index, row_stride));
}
DL_API dl_status dl_engine_reset(dl_engine* e) { DL_ENGINE_CALL(e->impl->reset()); }
DL_API dl_status dl_engine_consume(dl_engine* e, const uint32_t* tokens, size_t n, int mode, uint16_t* logits_out) {
  DL_ENGINE_CALL(e->impl->consume(tokens, n, mode, logits_out));
}
DL_API size_t dl_engine_position(dl_engine* e) {
  if (!e || !e->impl) return 0;
  try {
    return e->impl->position();
  } catch (...) {
    return 0;
  }
}
DL_API dl_status dl_engine_set_capture(dl_engine* e, int layer) { DL_ENGINE_CALL(e->impl->set_capture(layer)); }
DL_API dl_status dl_engine_set_observation(dl_engine* e, void* device_rows, size_t positions) {
  DL_ENGINE_CALL(e->impl->set_observation(device_rows, positions));
}
DL_API dl_status dl_engine_read_capture(dl_engine* e, size_t first, size_t count, uint16_t* host) {
  DL_ENGINE_CALL(e->impl->read_capture(first, count, host));
}
DL_API dl_status dl_engine_set_intervention(dl_engine* e, int layer, size_t selected, float strength,
                                            const float* host_direction) {
  DL_ENGINE_CALL(e->impl->set_intervention(layer, selected, strength, host_direction));
}
DL_API dl_status dl_engine_set_decode_path(dl_engine* e, int path) {
  DL_ENGINE_CALL(e->impl->set_decode_path(path));
}
DL_API dl_status dl_engine_set_sampler_engine(dl_engine* e, int engine) {
  if (engine != DL_RNG_MT19937_64 && engine != DL_RNG_PHILOX4X32_10)
    return fail(DL_INVALID_ARGUMENT, "set_sampler_engine: unknown engine");
  DL_ENGINE_CALL(e->impl->set_sampler_engine(engine));
}
DL_API dl_status dl_engine_set_injection(dl_engine* e, int64_t position, const uint16_t* source_bits,
                                         float scale) {
  if (position >= 0 && !source_bits) return fail(DL_INVALID_ARGUMENT, "injection: source required");
  DL_ENGINE_CALL(e->impl->set_injection((long long)position, source_bits, scale));
}
DL_API dl_status dl_engine_set_reconstruction_head(dl_engine* e, const uint16_t* head_bits) {
  if (!head_bits) return fail(DL_INVALID_ARGUMENT, "reconstruction head: null");
  DL_ENGINE_CALL(e->impl->set_reconstruction_head(head_bits));
}
DL_API dl_status dl_engine_reconstruct(dl_engine* e, const uint32_t* tokens, size_t n, uint16_t* out_bits) {
  if (!tokens || !out_bits) return fail(DL_INVALID_ARGUMENT, "reconstruct: null");
  DL_ENGINE_CALL(e->impl->reconstruct(tokens, n, out_bits));
}
DL_API dl_status dl_engine_read_kv(dl_engine* e, size_t layer, int values, size_t first, size_t count,
                                   uint16_t* host) {
  DL_ENGINE_CALL(e->impl->read_kv(layer, values, first, count, host));
}
DL_API dl_status dl_engine_generate(dl_engine* e, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                                    const dl_sampling* settings, uint64_t seed, const uint32_t* stop_ids,
                                    size_t n_stop, int prefill_mode, uint32_t* tokens_out, size_t* n_out,
                                    uint16_t* logits_out, dl_generation_stats* stats) {
  if (!settings || !prompt || !tokens_out || !n_out) return fail(DL_INVALID_ARGUMENT, "generate: arguments");
  DL_ENGINE_CALL(e->impl->generate(prompt, n_prompt, max_new, *settings, seed, stop_ids, n_stop, prefill_mode,
                                   tokens_out, n_out, logits_out, stats));
}


// ---- device-side sequence loop ----
DL_API dl_status dl_engine_start(dl_engine* e, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                                 const dl_sampling* settings, uint64_t seed, const uint32_t* stop_ids,
                                 size_t n_stop, int prefill_mode) {
  if (!prompt || !settings || (n_stop && !stop_ids)) return fail(DL_INVALID_ARGUMENT, "engine_start: arguments");
  DL_ENGINE_CALL(e->impl->start(prompt, n_prompt, max_new, *settings, seed, stop_ids, n_stop, prefill_mode));
}

DL_API dl_status dl_engine_collect(dl_engine* e, size_t index, int64_t timeout_ms, dl_sequence_event* out) {
  if (!e || !e->impl || !out) return fail(DL_INVALID_ARGUMENT, "engine_collect: arguments");
  bool got = false;
  const dl_status st = guarded([&] {
    got = e->impl->collect(index, timeout_ms, out);
    return DL_OK;
  });
  if (st != DL_OK) return st;
  return got ? DL_OK : fail(DL_NOT_READY, "journal event not available");
}

DL_API dl_status dl_engine_request_stop(dl_engine* e) { DL_ENGINE_CALL(e->impl->request_stop()); }

DL_API dl_status dl_engine_drain(dl_engine* e, uint32_t* tokens_out, size_t* n_out, dl_generation_stats* stats) {
  DL_ENGINE_CALL(e->impl->drain(tokens_out, n_out, stats));
}

// ---- batched serving ----
DL_API dl_status dl_serve_create(const dl_model_config* config, int device, size_t batch, size_t capacity,
                                 size_t chunk_rows, int tp_rank, int tp_size, dl_serve** out) {
  if (!config || !out) return fail(DL_INVALID_ARGUMENT, "serve_create: arguments");
  return guarded([&] {
    *out = new dl_serve{new dl::Server(*config, device, batch, capacity, chunk_rows, tp_rank, tp_size)};
    return DL_OK;
  });
}

DL_API void dl_serve_destroy(dl_serve* s) {
  if (!s) return;
  delete s->impl;
  delete s;
}

DL_API dl_status dl_serve_nccl_id(unsigned char* id128) {
  if (!id128) return fail(DL_INVALID_ARGUMENT, "serve_nccl_id: null");
  return guarded([&] {
    dl::Server::nccl_id(id128);
    return DL_OK;
  });
}

#define DL_SERVE_CALL(body)                                            \
  if (!s || !s->impl) return fail(DL_INVALID_ARGUMENT, "null server"); \
  return guarded([&] {                                                 \
    body;                                                              \
    return DL_OK;                                                      \
  })

DL_API dl_status dl_serve_connect(dl_serve* s, const unsigned char* id128) {
  if (!id128) return fail(DL_INVALID_ARGUMENT, "serve_connect: null id");
  DL_SERVE_CALL(s->impl->connect(id128));
}
DL_API dl_status dl_serve_ipc_handle(dl_serve* s, unsigned char* handle64) {
  if (!handle64) return fail(DL_INVALID_ARGUMENT, "serve_ipc_handle: null");
  DL_SERVE_CALL(s->impl->ipc_handle(handle64));
}
DL_API dl_status dl_serve_connect_peers(dl_serve* s, const unsigned char* handles) {
  if (!handles) return fail(DL_INVALID_ARGUMENT, "serve_connect_peers: null");
  DL_SERVE_CALL(s->impl->connect_peers(handles));
}
DL_API dl_status dl_serve_init_random(dl_serve* s, uint64_t seed, float sigma) {
  DL_SERVE_CALL(s->impl->init_random(seed, sigma));
}
DL_API dl_status dl_serve_set_sampler_engine(dl_serve* s, int engine) {
  if (engine != DL_RNG_MT19937_64 && engine != DL_RNG_PHILOX4X32_10)
    return fail(DL_INVALID_ARGUMENT, "set_sampler_engine: unknown engine");
  DL_SERVE_CALL(s->impl->set_sampler_engine(engine));
}
DL_API dl_status dl_serve_set_tensor(dl_serve* s, size_t index, const void* host_bits, size_t bytes) {
  if (!host_bits) return fail(DL_INVALID_ARGUMENT, "serve_set_tensor: null");
  DL_SERVE_CALL(s->impl->set_tensor(index, host_bits, bytes));
}
DL_API dl_status dl_serve_get_tensor(dl_serve* s, size_t index, void* host_bits, size_t bytes) {
  if (!host_bits) return fail(DL_INVALID_ARGUMENT, "serve_get_tensor: null");
  DL_SERVE_CALL(s->impl->get_tensor(index, host_bits, bytes));
}
DL_API dl_status dl_serve_slice_shape(dl_serve* s, size_t index, size_t* rows, size_t* cols, size_t* r0,
                                      size_t* c0) {
  if (!rows || !cols || !r0 || !c0) return fail(DL_INVALID_ARGUMENT, "serve_slice_shape: null");
  DL_SERVE_CALL(if (!s->impl->slice_shape(index, rows, cols, r0, c0)) throw std::invalid_argument("tensor index"));
}
DL_API dl_status dl_serve_prefill(dl_serve* s, const uint32_t* tokens, size_t prompt_len,
                                  const dl_sampling* settings, uint64_t seed, uint32_t* first_tokens) {
  if (!tokens || !settings) return fail(DL_INVALID_ARGUMENT, "serve_prefill: null");
  DL_SERVE_CALL(s->impl->prefill(tokens, prompt_len, *settings, seed, first_tokens));
}
DL_API dl_status dl_serve_decode(dl_serve* s, size_t steps, uint32_t* tokens_out, uint16_t* logits_out,
                                 dl_serve_stats* stats) {
  DL_SERVE_CALL(s->impl->decode(steps, tokens_out, logits_out, stats));
}
DL_API dl_status dl_serve_set_capture(dl_serve* s, int layer) { DL_SERVE_CALL(s->impl->set_capture(layer)); }
DL_API dl_status dl_serve_read_capture(dl_serve* s, size_t sequence, size_t first, size_t count,
                                       uint16_t* host_bits) {
  if (!host_bits) return fail(DL_INVALID_ARGUMENT, "serve_read_capture: null");
  DL_SERVE_CALL(s->impl->read_capture(sequence, first, count, host_bits));
}
DL_API dl_status dl_serve_set_steering(dl_serve* s, int layer, size_t first_position, float strength,
                                       const float* host_direction, const uint8_t* host_sequence_mask,
                                       int64_t source_sequence, size_t source_position) {
  if (layer >= 0 && (!host_direction || !host_sequence_mask))
    return fail(DL_INVALID_ARGUMENT, "serve_set_steering: direction and mask required");
  DL_SERVE_CALL(s->impl->set_steering(layer, first_position, strength, host_direction, host_sequence_mask,
                                      (long long)source_sequence, source_position));
}
DL_API dl_status dl_serve_set_step_fusion(dl_serve* s, int on) {
  DL_SERVE_CALL(s->impl->set_step_fusion(on != 0));
}
DL_API dl_status dl_serve_steering_strength(dl_serve* s, float* beta) {
  if (!beta) return fail(DL_INVALID_ARGUMENT, "serve_steering_strength: null");
  DL_SERVE_CALL(*beta = s->impl->steering_strength());
}
DL_API size_t dl_serve_position(dl_serve* s) {
  if (!s || !s->impl) return 0;
  try {
    return s->impl->position();
  } catch (const std::exception& e) {
    fail(DL_CUDA_ERROR, e.what());
    return 0;
  }
}

DL_API size_t dl_gemm_bf16_parts_workspace_bytes(size_t M, size_t N, size_t K, size_t parts) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t p = parts ? parts : size_t(dl::gemm_splitk_parts(int(M), int(N), int(K), sms));
  return p * M * N * 4;
}

DL_API dl_status dl_gemm_bf16_parts(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                    size_t N, size_t K, int epilogue, size_t parts, void* workspace,
                                    void* stream) {
  if (!x || !w || !y || !M || !workspace) return fail(DL_INVALID_ARGUMENT, "gemm parts: null pointer or empty shape");
  if (epilogue != dl::kGemmStore && epilogue != dl::kGemmResidual && epilogue != dl::kGemmSwiGLU)
    return fail(DL_INVALID_ARGUMENT, "gemm parts: epilogue must be 0, 1 or 3");
  if (!dl::gemm_tcgen05_supported(int(M), int(N), int(K)) || ldx % 8 || ldx < K ||
      (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) % 16)
    return fail(DL_UNSUPPORTED, "gemm parts: K % 64, N % 128, 8-element row stride and 16-byte alignment required");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int p = parts ? int(parts) : dl::gemm_splitk_parts(int(M), int(N), int(K), sms);
  if (p < 1 || p > 16 || K / 64 < size_t(p)) return fail(DL_INVALID_ARGUMENT, "gemm parts: 1..16 parts, at most K/64");
  dl::GemmProblem g = {};
  g.x = static_cast<const bf16*>(x);
  g.ldx = int(ldx);
  g.w = static_cast<const bf16*>(w);
  g.M = int(M);
  g.N = int(N);
  g.K = int(K);
  const dl_status s1 = cuda_status(dl::launch_gemm_tcgen05_parts(g, p, static_cast<float*>(workspace), st(stream)),
                                   "gemm parts");
  if (s1 != DL_OK) return s1;
  return cuda_status(dl::launch_gemm_splitk_epilogue(static_cast<const float*>(workspace), p, int(M), int(N), epilogue,
                                                     static_cast<bf16*>(y), int(ldy), nullptr, st(stream)),
                     "gemm parts epilogue");
}

DL_API dl_status dl_attention_decode_batched_plan(size_t batch, size_t kv_heads, size_t capacity, int sms,
                                                  int* splits, int* lead_q10) {
  if (!splits || !lead_q10 || !batch || !kv_heads || !capacity || sms < 1 || batch > 65535 || kv_heads > 65535 ||
      capacity > size_t(INT_MAX))
    return fail(DL_INVALID_ARGUMENT, "attention decode plan: null output, empty shape or size out of range");
  const dl::AttnPlan plan = dl::attention_decode_plan(int(batch), int(kv_heads), int(capacity), sms);
  *splits = plan.splits;
  *lead_q10 = plan.lead_q10;
  return DL_OK;
}

DL_API size_t dl_attention_decode_batched_workspace_bytes(size_t batch, size_t query_heads, size_t kv_heads,
                                                          size_t capacity) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const dl::AttnPlan plan = dl::attention_decode_plan(int(batch), int(kv_heads), int(capacity), sms);
  return dl::attention_decode_ws_floats(int(batch), int(query_heads), plan.splits) * 4;
}

DL_API dl_status dl_attention_decode_batched(const void* query, const void* kv, size_t seq_stride,
                                             size_t k_offset, size_t v_offset, const int64_t* position,
                                             size_t batch, size_t query_heads, size_t kv_heads, size_t capacity,
                                             void* output, void* workspace, void* stream) {
  if (!query || !kv || !position || !output || !workspace || !batch || !kv_heads)
    return fail(DL_INVALID_ARGUMENT, "attention decode batched: null pointer or empty shape");
  if (query_heads % kv_heads || query_heads / kv_heads > 8 ||
      (seq_stride | k_offset | v_offset) % 8 || reinterpret_cast<uintptr_t>(kv) % 16)
    return fail(DL_UNSUPPORTED, "attention decode batched: group <= 8, 16-byte aligned rows");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const dl::AttnPlan plan = dl::attention_decode_plan(int(batch), int(kv_heads), int(capacity), sms);
  const dl::KvPlanes planes{static_cast<bf16*>(const_cast<void*>(kv)), seq_stride, k_offset, v_offset};
  return cuda_status(dl::launch_attention_decode_batched(static_cast<const bf16*>(query), planes,
                                                         reinterpret_cast<const long long*>(position), int(batch),
                                                         int(query_heads), int(kv_heads), plan.splits,
                                                         plan.lead_q10, dl::attention_scale(128),
                                                         static_cast<float*>(workspace),
                                                         static_cast<bf16*>(output), st(stream)),
                     "attention decode batched");
}

}  // extern "C"
