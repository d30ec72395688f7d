/*
 * dolittle_b200.h -- C ABI of the B200 (sm_100a) Qwen3 token loop.
 *
 * Plain pointers and sizes only.  Device pointers are CUDA device addresses
 * on the current device; `stream` is a cudaStream_t passed as void* (NULL =
 * legacy default stream).  Every launch entry point only enqueues work: no
 * allocation, transfer or host wait (the contract of the reference's
 * src/kernels/cuda/launch.h:1-60), and is graph-capturable.  Errors are
 * returned as dl_status; dl_last_error() gives a message for the calling
 * thread.  BF16 tensors are raw 16-bit storage (uint16_t bits).
 *
 * Reference interfaces replaced (paths inside plainsight-systems/dolittle):
 *   dl_projection ........ launch_projection       src/kernels/cuda/launch.h:79-83
 *   dl_rms_norm .......... launch_rms_norm         src/kernels/cuda/launch.h:84-86
 *   dl_rotary ............ launch_rotary           src/kernels/cuda/launch.h:87-92
 *   dl_attention_scale ... launch_attention_scale  src/kernels/cuda/launch.h:93-94
 *   dl_attention ......... launch_attention        src/kernels/cuda/launch.h:95-101
 *   dl_embedding ......... launch_embedding        src/kernels/cuda/launch.h:102-104
 *   dl_add ............... launch_add              src/kernels/cuda/launch.h:105-106
 *   dl_silu_multiply ..... launch_silu_multiply    src/kernels/cuda/launch.h:107-109
 *   dl_sampler_* ......... DeviceCategorical       src/inference/sampling/device.h:54-85
 *   dl_intervene ......... DeviceIntervention      src/inference/steering/device.h:50-68
 *                          (kernel src/kernels/cuda/steering.cu:106-159)
 *   dl_direction ......... DeviceDirection         src/inference/steering/device.h:30-48
 *                          (submit/finish src/kernels/cuda/steering.cu:200-258,
 *                           kernel :68-98)
 *   dl_normalize_injection DeviceInjection         src/inference/injection/device.h:26-47
 *                          (kernel src/kernels/cuda/injection.cu:48-102)
 *   dl_engine_* .......... CachedForwardPlan       src/inference/executor.h:242-342
 *                          (prepare_device_generation/start_sequence/
 *                           collect_sequence/consume_view) and generate()
 *                          src/inference/generation.h:129-138
 * Fused entry points (new Operation variants the Qwen3 recipe may emit):
 *   dl_qkv_projection, dl_qk_norm_rope_append, dl_projection_residual.
 */
#ifndef DOLITTLE_B200_H
#define DOLITTLE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DL_API __attribute__((visibility("default")))
#else
#define DL_API
#endif

typedef enum {
  DL_OK = 0,
  DL_INVALID_ARGUMENT = 1,  /* reference: std::invalid_argument */
  DL_UNSUPPORTED = 2,       /* unsupported dtype/shape (reference: invalid_argument) */
  DL_CUDA_ERROR = 3,        /* launch or runtime error (reference: runtime_error) */
  DL_OUT_OF_MEMORY = 4,     /* reference: length_error on budget */
  DL_DEVICE_FAULT = 5,      /* a kernel recorded a bounded-wait timeout */
  DL_NOT_READY = 6          /* dl_engine_collect: the event did not arrive in time */
} dl_status;

typedef enum { DL_BF16 = 0, DL_F32 = 1 } dl_dtype;

DL_API const char* dl_last_error(void);
DL_API const char* dl_version(void);

/* ------------------------------------------------------------------------ */
/* Operation launches (reference launch.h mirrors).  The product computes in */
/* BF16 storage with FP32 arithmetic; DL_F32 is rejected with DL_UNSUPPORTED
 * (except by dl_direction, whose reconstructions may be FP32). */
/* Positions: device_position (size_t on device) overrides first_position.  */
/* ------------------------------------------------------------------------ */

/* Y[rows][O] = X[rows][I] * W[O][I]^T under the reference projection law.
 * output_position (device, optional): output rows start at row
 * *output_position of Y (KV-cache append). I must be a multiple of 8. */
DL_API dl_status dl_projection(dl_dtype type, const void* input, const void* weight, void* output,
                               size_t rows, size_t input_width, size_t output_width, void* stream,
                               const size_t* output_position);
DL_API dl_status dl_rms_norm(dl_dtype type, const void* input, const void* weight, void* output,
                             size_t rows, size_t width, float epsilon, void* stream);
DL_API dl_status dl_rotary(dl_dtype type, const void* input, void* output, size_t positions,
                           size_t heads, size_t width, size_t first_position, double theta,
                           void* stream, const size_t* device_position, int positioned_output);
DL_API dl_status dl_attention_scale(float* output, size_t width, void* stream);
/* Causal GQA attention; query row i attends keys [0, first+i].  workspace:
 * dl_attention_workspace_bytes() bytes of device memory (scores), declared
 * at preparation time like the reference's PreparedOperation::workspace(). */
DL_API size_t dl_attention_workspace_bytes(size_t positions, size_t query_heads, size_t capacity);
DL_API dl_status dl_attention(dl_dtype type, const void* query, const void* key, const void* value,
                              void* output, size_t positions, size_t query_heads, size_t kv_heads,
                              size_t width, void* stream, size_t first_position,
                              const size_t* device_position, size_t capacity, const float* scale,
                              void* workspace);
/* dl_attention for callers that cannot allocate device memory: a host that
 * owns every device allocation through its own arena and forbids allocation
 * once generation runs, or a plugin whose process allocator does not let it
 * call cudaMalloc.  No counterpart in the reference.  Same arguments and
 * results as dl_attention, but the scores live in a fixed array inside the
 * library's device memory (DL_ATTENTION_FIXED_SCRATCH_SCORES FP32 values,
 * 4 MiB, held on every GPU that loads the library until the process exits),
 * so nothing is allocated.  positions * query_heads * key capacity above
 * that limit is rejected with DL_INVALID_ARGUMENT.  All calls on a device
 * share the array and it keeps the last call's contents; calls that overlap
 * on the GPU race on it, so serialize them.  The first call on each device
 * looks up the array's address (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture.  The address is
 * kept for the life of the process: calls must not span a cudaDeviceReset. */
#define DL_ATTENTION_FIXED_SCRATCH_SCORES ((size_t)1 << 20)
DL_API dl_status dl_attention_fixed_scratch(dl_dtype type, const void* query, const void* key,
                                            const void* value, void* output, size_t positions,
                                            size_t query_heads, size_t kv_heads, size_t width,
                                            void* stream, size_t first_position,
                                            const size_t* device_position, size_t capacity);
/* Causal GQA attention of the fast prompt pass on tcgen05 tensor cores
 * (tensor-core accumulation; not the reference reduction order): query rows
 * [positions][Hq][d] at absolute positions first .. first+positions-1 attend
 * keys 0 .. first+positions-1 of key/value [capacity][Hkv][d].  d = 128.
 * workspace: dl_attention_prefill_fast_workspace_bytes() bytes (transposed V). */
DL_API size_t dl_attention_prefill_fast_workspace_bytes(size_t kv_heads, size_t width, size_t capacity);
DL_API dl_status dl_attention_prefill_fast(const void* query, const void* key, const void* value, void* output,
                                           size_t positions, size_t query_heads, size_t kv_heads, size_t width,
                                           void* stream, size_t first_position, size_t capacity,
                                           void* workspace);
DL_API dl_status dl_embedding(dl_dtype type, const uint32_t* tokens, const void* weight,
                              void* output, size_t rows, size_t width, void* stream);
DL_API dl_status dl_add(dl_dtype type, const void* left, const void* right, void* output,
                        size_t count, void* stream);
DL_API dl_status dl_silu_multiply(dl_dtype type, const void* gate, const void* up, void* output,
                                  size_t count, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused decode operations (same arithmetic as the unfused recipe).          */
/* ------------------------------------------------------------------------ */

/* normalized = RMSNorm(residual, norm_weight); q/k/v = projections of it.
 * wqkv = [Wq; Wk; Wv] contiguous ([q_rows + 2*kv_rows][I]).  v rows are
 * written at row *v_position of v_out (KV append) when v_position != NULL. */
DL_API dl_status dl_qkv_projection(const void* residual, const void* norm_weight, float epsilon,
                                   const void* wqkv, size_t rows, size_t input_width,
                                   size_t q_rows, size_t kv_rows, void* q_out, void* k_out,
                                   void* v_out, const int64_t* v_position, void* stream);
/* QK-norm + RoPE for rows at positions *position + i; queries to q_out,
 * keys into k_cache row (*position + i).  inv_freq from dl_rope_inverse_frequency. */
DL_API dl_status dl_rope_inverse_frequency(float* output, size_t width, double theta,
                                           void* stream);
DL_API dl_status dl_qk_norm_rope_append(const void* q_raw, const void* k_raw,
                                        const void* q_norm_weight, const void* k_norm_weight,
                                        const float* inv_freq, void* q_out, void* k_cache,
                                        const int64_t* position, size_t rows, size_t query_heads,
                                        size_t kv_heads, size_t width, float epsilon,
                                        void* stream);
/* Prefill / batched projection on the tcgen05 tensor cores (TMEM FP32
 * accumulation; not the reference's summation order):
 *   epilogue 0: Y = bf16(X W^T)            (Y row stride ldy)
 *   epilogue 1: Y = round(Y + round(X W^T)) in place (residual add)
 *   epilogue 3: W rows interleaved (gate o, up o): Y[:, o] = SwiGLU law.
 * X [M][K] with row stride ldx, W [N][K] contiguous; K % 64 == 0,
 * N % 128 == 0, 16-byte aligned rows. */
DL_API dl_status dl_gemm_bf16(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                              size_t N, size_t K, int epilogue, void* stream);
/* dl_gemm_bf16 that may split K into up to 4 parts when the tile count
 * leaves SMs idle (the last part to finish adds the parts in part order):
 * workspace of dl_gemm_bf16_split_workspace_bytes(M, N) bytes (FP32
 * partials) and n_tickets >= ceil(M/128) * (N/128) zeroed words (left
 * zeroed).  Repeated calls give bit-identical results. */
DL_API size_t dl_gemm_bf16_split_workspace_bytes(size_t M, size_t N);
DL_API dl_status dl_gemm_bf16_split(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                    size_t N, size_t K, int epilogue, void* stream, void* workspace,
                                    unsigned* tickets, size_t n_tickets);
/* dl_gemm_bf16_split with the tiling chosen by the caller: tile_m 128 rows
 * per tile on one SM or 256 on a pair of SMs (then 256 columns), tile_n 128
 * or 256 output columns, and `parts` K parts (1..4), or parts = -1 for
 * stream-K (single-SM tiles: every CTA takes an equal contiguous share of
 * the tiles' k-steps; a tile cut between CTAs is summed in k order by the
 * CTA holding its last k-step, so results are bit-identical run to run);
 * 0 = chosen by the library for any of them.  workspace / tickets may be NULL
 * when parts is 0 or 1. */
DL_API dl_status dl_gemm_bf16_config(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                     size_t N, size_t K, int epilogue, void* stream, void* workspace,
                                     unsigned* tickets, size_t n_tickets, int tile_m, int tile_n, int parts);
/* residual = round(residual + round(X W^T)) in place. */
DL_API dl_status dl_projection_residual(const void* input, const void* weight, void* residual,
                                        size_t rows, size_t input_width, size_t output_width,
                                        void* stream);

/* ------------------------------------------------------------------------ */
/* Device sampler (DeviceCategorical).  Greedy or categorical with          */
/* temperature / top-k / top-p under the reference device law; the draw is */
/* explicit bits or the device-owned MT19937-64 stream.                     */
/* ------------------------------------------------------------------------ */
typedef struct dl_sampler dl_sampler;
typedef struct {
  int32_t mode;        /* 0 greedy, 1 categorical */
  double temperature;
  size_t top_k;        /* 0 disables */
  double top_p;
} dl_sampling;

DL_API size_t dl_sampler_required_bytes(size_t vocabulary);
DL_API dl_status dl_sampler_create(size_t vocabulary, dl_dtype type, dl_sampler** out);
DL_API void dl_sampler_destroy(dl_sampler* s);
/* Draw source of the device-owned stream (dl_sampler_submit_next and the
 * engine / server sequences).  DL_RNG_MT19937_64 is the reference's stream
 * (std::mt19937_64 seeded with the seed, src/kernels/cuda/sampling.cu:
 * 106-137) and the default; DL_RNG_PHILOX4X32_10 is a counter-based stream
 * with no counterpart in the reference: draw k of row r is the first two
 * 32-bit words w0, w1 of Philox4x32-10 (Salmon et al., SC'11) at counter
 * {k mod 2^32, k >> 32, 0x5A4D504C, 0} under key seed + r (low word first),
 * u = (((w1 << 32) | w0) >> 11) * 2^-53.  The selection law given u is the
 * same for both.  Set before dl_sampler_start. */
enum { DL_RNG_MT19937_64 = 0, DL_RNG_PHILOX4X32_10 = 1 };
DL_API dl_status dl_sampler_set_engine(dl_sampler* s, int engine);
/* Seed the device-owned stream and the stop-ID mask. */
DL_API dl_status dl_sampler_start(dl_sampler* s, const dl_sampling* settings, uint64_t seed,
                                  const uint32_t* stop_ids, size_t n_stop, void* stream);
/* One selection of a device logits row; result = device {token, status}. */
DL_API dl_status dl_sampler_submit(dl_sampler* s, const void* row, const dl_sampling* settings,
                                   uint64_t bits, void* stream, const uint32_t** result);
DL_API dl_status dl_sampler_submit_next(dl_sampler* s, const void* row, void* stream,
                                        const uint32_t** result);

/* ------------------------------------------------------------------------ */
/* Steering and injection                                                    */
/* ------------------------------------------------------------------------ */
/* At absolute row `selected` (if *position <= selected < *position+rows):
 * beta = strength*||h||, h' = round(h + beta*direction); state = {invalid,
 * count} in device memory. */
DL_API dl_status dl_intervene(void* residual, const float* direction, const int64_t* position,
                              uint32_t* state, size_t width, size_t selected, size_t rows,
                              float strength, void* stream);
/* Steering direction from two reconstructions (DeviceDirection::submit;
 * finish = read *status after the stream completes):
 * direction = (edited - original) / ||edited - original||, FP32 [width].
 * The norm follows the reference law: 8 lanes, lane L summing the rounded
 * squares of FP32(edited[i]) - FP32(original[i]) over i = L + 8k in order,
 * then lane sums 0..7 in order, sqrt_rn; each quotient div_rn.  *status = 1
 * (direction left untouched) on a zero or non-finite norm, else 0.
 * type: DL_BF16 or DL_F32 reconstructions; all pointers device memory. */
DL_API dl_status dl_direction(dl_dtype type, const void* original, const void* edited, size_t width,
                              float* direction, uint32_t* status, void* stream);
/* out = BF16((h/||h||)*scale); norm and status written to device memory. */
DL_API dl_status dl_normalize_injection(const void* source, void* output, float* norm,
                                        uint32_t* status, size_t width, float scale,
                                        void* stream);

/* ------------------------------------------------------------------------ */
/* Engine: resident Qwen3 weights + KV cache + prefill/decode loop.          */
/* ------------------------------------------------------------------------ */
typedef struct {
  uint32_t hidden, query_heads, kv_heads, head_width, mlp_width, vocabulary, layers;
  float epsilon;
  double theta;
} dl_model_config;

typedef struct dl_engine dl_engine;

typedef struct {
  double prefill_ms;     /* device time of the prompt pass + first selection */
  double decode_ms;      /* device time of all decode steps */
  uint64_t decode_steps; /* single-token forward passes */
  uint64_t kernels_per_decode_step;
  uint64_t kernels_total; /* kernels this library launched for the call */
  uint32_t status;       /* last selection status (0 ok) */
  uint32_t fault;        /* kernel error word (bounded waits) */
} dl_generation_stats;

enum { DL_PREFILL_PARITY = 0, DL_PREFILL_FAST = 1 };
/* Decode step implementation (identical results): one persistent
 * cooperative kernel per token (default; falls back to the per-operation
 * kernels when the model shape or device does not fit it), or the
 * per-operation kernels captured in the step graph. */
enum { DL_DECODE_PERSISTENT = 0, DL_DECODE_KERNELS = 1 };

/* Tensors are addressed by index: 0 embedding [V][D], 1 final norm [D],
 * 2 lm_head [V][D], then 3 + 11*block + role with roles input_norm, q, k,
 * v, q_norm, k_norm, o, post_norm, gate, up, down (Qwen3 recipe order,
 * src/models/qwen3/model.cpp:343-409). */
DL_API size_t dl_engine_tensor_count(const dl_model_config* config);
DL_API dl_status dl_engine_tensor_shape(const dl_model_config* config, size_t index, size_t* rows,
                                        size_t* cols);
DL_API dl_status dl_engine_create(const dl_model_config* config, int device, size_t capacity,
                                  size_t max_rows, dl_engine** out);
DL_API void dl_engine_destroy(dl_engine* e);
/* Seeded synthetic weights: N(0, sigma) approximation (Philox4x32-10,
 * Irwin-Hall of 8 halves) per tensor, norms = 1. */
DL_API dl_status dl_engine_init_random(dl_engine* e, uint64_t seed, float sigma);
DL_API dl_status dl_engine_set_tensor(dl_engine* e, size_t index, const void* host_bits,
                                      size_t bytes);
DL_API dl_status dl_engine_get_tensor(dl_engine* e, size_t index, void* host_bits, size_t bytes);
/* Device address of a resident tensor (for binding it into other kernels,
 * like the reference executor binds parameter regions) and its row stride
 * in elements: gate and up rows are stored interleaved in one [2F][D]
 * matrix, so their stride is 2*D; every other tensor is contiguous. */
DL_API dl_status dl_engine_tensor_device(dl_engine* e, size_t index, void** device_ptr,
                                         size_t* row_stride);
/* Fresh sequence: position 0, empty KV cache contents unchanged. */
DL_API dl_status dl_engine_reset(dl_engine* e);
/* Consume prompt/continuation tokens (host IDs) at the current position;
 * logits_out (host, optional) receives the BF16 logits of the last row.
 * mode: DL_PREFILL_PARITY (reference reduction order) or DL_PREFILL_FAST. */
DL_API dl_status dl_engine_consume(dl_engine* e, const uint32_t* tokens, size_t n, int mode,
                                   uint16_t* logits_out);
DL_API size_t dl_engine_position(dl_engine* e);
/* Capture block `layer`'s output rows for every consumed position into an
 * arena [capacity][D] (layer < 0 disables). */
DL_API dl_status dl_engine_set_capture(dl_engine* e, int layer);
DL_API dl_status dl_engine_read_capture(dl_engine* e, size_t first, size_t count, uint16_t* host);
/* Observe every block's output (the residual after block l, the site the
 * reference's ObservationPlan resolves per advertised block,
 * src/inference/observations.h) during later prompt passes: the BF16 row of
 * absolute position p after block l is written to
 * device_rows + (l * positions + p) * D.  device_rows is caller-owned device
 * memory of layers * positions * D BF16 values; a prompt pass reaching a
 * position >= `positions` is rejected (DL_INVALID_ARGUMENT).  Decode steps do
 * not observe.  device_rows == NULL turns observation off. */
DL_API dl_status dl_engine_set_observation(dl_engine* e, void* device_rows, size_t positions);
/* One-shot steering edit at block `layer`, absolute row `selected`. */
DL_API dl_status dl_engine_set_intervention(dl_engine* e, int layer, size_t selected,
                                            float strength, const float* host_direction);
DL_API dl_status dl_engine_set_decode_path(dl_engine* e, int path);
/* Draw source of later generations' categorical selections (DL_RNG_*, see
 * dl_sampler_set_engine); the default is the reference's MT19937-64. */
DL_API dl_status dl_engine_set_sampler_engine(dl_engine* e, int engine);
/* Verbalizer (AV) injection: every later prompt pass replaces the embedding
 * of absolute position `position` with BF16((h / ||h||) * scale) of the BF16
 * row `source_bits` [D] (DeviceInjection::normalize + the marker-row replace,
 * src/kernels/cuda/injection.cu:48-102, decode.cu:221-230).  position < 0
 * clears it.  A zero or non-finite source is rejected (DL_INVALID_ARGUMENT). */
DL_API dl_status dl_engine_set_injection(dl_engine* e, int64_t position, const uint16_t* source_bits,
                                         float scale);
/* Reconstructor (AR) forward-only pass: the D x D BF16 head, then for a
 * prompt the last position's residual after the final block (no final norm)
 * through the head under the projection law -> out_bits [D] (host).  Starts
 * a fresh sequence (executor.cpp:1750-1771, qwen3/model.cpp:395-404). */
DL_API dl_status dl_engine_set_reconstruction_head(dl_engine* e, const uint16_t* head_bits);
DL_API dl_status dl_engine_reconstruct(dl_engine* e, const uint32_t* tokens, size_t n, uint16_t* out_bits);
DL_API dl_status dl_engine_read_kv(dl_engine* e, size_t layer, int values, size_t first,
                                   size_t count, uint16_t* host);
/* Live generation: prompt pass, first selection, then decode steps replayed
 * from one captured CUDA graph per step until max_new tokens or a stop ID.
 * tokens_out receives the generated IDs (host); logits_out (optional, host,
 * [max_new][V]) the BF16 logits each selection read. */
DL_API dl_status dl_engine_generate(dl_engine* e, const uint32_t* prompt, size_t n_prompt,
                                    size_t max_new, const dl_sampling* settings, uint64_t seed,
                                    const uint32_t* stop_ids, size_t n_stop, int prefill_mode,
                                    uint32_t* tokens_out, size_t* n_out, uint16_t* logits_out,
                                    dl_generation_stats* stats);

/* ------------------------------------------------------------------------ */
/* Batched serving (the long-context serving workload): B sequences of one  */
/* prompt length advancing in lockstep, on one GPU or one rank of a        */
/* tensor-parallel group over KV-head groups.  Replaces running each       */
/* sequence through CachedForwardPlan::prepare_device_generation /         */
/* start_sequence (src/inference/executor.cpp:1482-1716) one at a time.    */
/* Fast path: tcgen05 GEMMs, online-softmax flash decoding; checked        */
/* against the reference law within tolerance.                              */
/* ------------------------------------------------------------------------ */
typedef struct dl_serve dl_serve;

typedef struct {
  double prefill_ms;      /* device time of the last dl_serve_prefill */
  double decode_ms;       /* device time of the decode steps */
  uint64_t decode_steps;
  uint64_t kernels_per_decode_step;
} dl_serve_stats;

/* Rank tp_rank of tp_size (1 = single GPU): query heads, KV heads and MLP
 * columns are split in tp_size equal slices (tp_size must divide the KV
 * heads).  chunk_rows: prompt rows per pass (<= 4096). */
DL_API dl_status dl_serve_create(const dl_model_config* config, int device, size_t batch, size_t capacity,
                                 size_t chunk_rows, int tp_rank, int tp_size, dl_serve** out);
DL_API void dl_serve_destroy(dl_serve* s);
/* NCCL communicator: rank 0 makes the 128-byte id, every rank passes the
 * same id to dl_serve_connect (all ranks concurrently). */
DL_API dl_status dl_serve_nccl_id(unsigned char* id128);
DL_API dl_status dl_serve_connect(dl_serve* s, const unsigned char* id128);
/* Fused NVLink all-reduce of the decode step (peer memory instead of NCCL
 * for o_proj / down_proj): each rank publishes a 64-byte CUDA IPC handle of
 * its buffer, then every rank passes all handles [tp_size][64] in rank order
 * (after dl_serve_connect; ranks must be separate processes). */
DL_API dl_status dl_serve_ipc_handle(dl_serve* s, unsigned char* handle64);
DL_API dl_status dl_serve_connect_peers(dl_serve* s, const unsigned char* handles);
/* Seeded weights as dl_engine_init_random; each rank generates only its
 * slice of the same tensors. */
DL_API dl_status dl_serve_init_random(dl_serve* s, uint64_t seed, float sigma);
/* Draw source of later prefills' sequences (DL_RNG_*; row r uses seed + r). */
DL_API dl_status dl_serve_set_sampler_engine(dl_serve* s, int engine);
/* Full tensor `index` (engine order, host BF16 bits); the rank keeps its
 * slice.  dl_serve_get_tensor returns the slice [rows][cols] held, at
 * rows r0.., columns c0.. of the full tensor (dl_serve_slice_shape). */
DL_API dl_status dl_serve_set_tensor(dl_serve* s, size_t index, const void* host_bits, size_t bytes);
DL_API dl_status dl_serve_get_tensor(dl_serve* s, size_t index, void* host_bits, size_t bytes);
DL_API dl_status dl_serve_slice_shape(dl_serve* s, size_t index, size_t* rows, size_t* cols, size_t* r0,
                                      size_t* c0);
/* tokens [batch][prompt_len] (host): prompt pass of every sequence, then
 * each sequence's first selection (sampler seed = seed + sequence index)
 * into first_tokens [batch] (host). */
DL_API dl_status dl_serve_prefill(dl_serve* s, const uint32_t* tokens, size_t prompt_len,
                                  const dl_sampling* settings, uint64_t seed, uint32_t* first_tokens);
/* `steps` decode steps of every sequence: tokens_out [steps][batch] (host),
 * logits_out (optional, host) [steps][batch][V] BF16. */
DL_API dl_status dl_serve_decode(dl_serve* s, size_t steps, uint32_t* tokens_out, uint16_t* logits_out,
                                 dl_serve_stats* stats);
DL_API size_t dl_serve_position(dl_serve* s);
/* Block `layer`'s output rows (after any steering edit, as the reference
 * captures, src/inference/executor.cpp:1633-1656) of every sequence at every
 * prompt and decode position into an arena [batch][capacity][D] the server
 * allocates on first use; layer < 0 disables.  Read back one sequence's rows
 * [first, first + count) as BF16 bits. */
DL_API dl_status dl_serve_set_capture(dl_serve* s, int layer);
DL_API dl_status dl_serve_read_capture(dl_serve* s, size_t sequence, size_t first, size_t count,
                                       uint16_t* host_bits);
/* Fixed-strength steering of every position from first_position on, at the
 * output of block `layer`, for the sequences whose host_sequence_mask[b] is
 * nonzero (prompt and decode rows): h' = round(h + beta * u) with the
 * arithmetic of the reference's one-row edit (src/kernels/cuda/
 * steering.cu:106-159), u = host_direction [D] (FP32).  No counterpart in the
 * reference, which edits one row once.  source_sequence < 0: beta = strength.
 * Otherwise beta = strength * ||h|| of sequence source_sequence's block
 * output at source_position before its edit (the one-row edit's norm law),
 * computed on the device during the prompt pass; the edit of that row then
 * equals the reference's one-row edit of it bit for bit.  Sequences prefilled
 * before the source may not be steered.  layer < 0 disables.  Applies from
 * the next prefill / decode call. */
DL_API dl_status dl_serve_set_steering(dl_serve* s, int layer, size_t first_position, float strength,
                                       const float* host_direction, const uint8_t* host_sequence_mask,
                                       int64_t source_sequence, size_t source_position);
/* The beta the steering edit used (host read). */
DL_API dl_status dl_serve_steering_strength(dl_serve* s, float* beta);
/* Decode step form: 1 (default) folds the split-K sums into the kernels that
 * consume them (the attention kernel builds its queries and appends the new
 * key/value from the qkv parts and merges its own splits; the o / down parts
 * go through residual add + RMSNorm, over NVLink peer memory under tensor
 * parallelism) and chains the kernels as programmatic dependent launches;
 * 0 runs every step as separate kernels.  Both give the same bits; the
 * switch exists to check that.  Takes effect at the next decode call. */
DL_API dl_status dl_serve_set_step_fusion(dl_serve* s, int on);

/* Split-K GEMM for few rows: Y = epilogue(X W^T) as dl_gemm_bf16, the K
 * extent cut in `parts` (0 = fill the SMs) whose FP32 partials
 * (dl_gemm_bf16_parts_workspace_bytes) are added in part order. */
DL_API size_t dl_gemm_bf16_parts_workspace_bytes(size_t M, size_t N, size_t K, size_t parts);
DL_API dl_status dl_gemm_bf16_parts(const void* x, size_t ldx, const void* w, void* y, size_t ldy, size_t M,
                                    size_t N, size_t K, int epilogue, size_t parts, void* workspace,
                                    void* stream);
/* Batched decode attention (head width 128): query [B][Hq][128]; sequence
 * b's keys 0..*position at kv + b*seq_stride + k_offset (values at
 * v_offset) + j*Hkv*128, elements; out [B][Hq*128] BF16; workspace of
 * dl_attention_decode_batched_workspace_bytes FP32. */
DL_API size_t dl_attention_decode_batched_workspace_bytes(size_t batch, size_t query_heads, size_t kv_heads,
                                                          size_t capacity);
/* The key ranges dl_attention_decode_batched (and the server's decode step)
 * cut each (sequence, KV head) into on a device of `sms` SMs: *splits even
 * ranges (*lead_q10 = 0), or two ranges whose first holds *lead_q10 / 1024
 * of the keys, rounded up to 64-key tiles.  Host arithmetic only. */
DL_API dl_status dl_attention_decode_batched_plan(size_t batch, size_t kv_heads, size_t capacity, int sms,
                                                  int* splits, int* lead_q10);
DL_API dl_status dl_attention_decode_batched(const void* query, const void* kv, size_t seq_stride,
                                             size_t k_offset, size_t v_offset, const int64_t* position,
                                             size_t batch, size_t query_heads, size_t kv_heads, size_t capacity,
                                             void* output, void* workspace, void* stream);

/* ------------------------------------------------------------------------ */
/* Device-side generation loop (DeviceSequence, src/inference/decoding/     */
/* device.h:84-139): dl_engine_start enqueues the prompt pass, the first    */
/* selection and ONE graph launch whose conditional WHILE node replays the  */
/* decode step on the device until a stop ID, a failed selection, a cancel  */
/* request or max_new selections; the host follows a journal of 32-byte     */
/* events in mapped host memory: event 0 = prompt consumed, event k = the   */
/* k-th selection, then one terminal event.                                 */
/* ------------------------------------------------------------------------ */
enum { DL_EVENT_NONE = 0, DL_EVENT_CONSUMED = 1, DL_EVENT_SELECTED = 2, DL_EVENT_TERMINAL = 3 };
enum { DL_REASON_LIMIT = 0, DL_REASON_EOS = 1, DL_REASON_CANCELLED = 2, DL_REASON_FAILURE = 3 };

typedef struct {
  uint8_t kind;      /* DL_EVENT_*; written last (0 until the event is complete) */
  uint8_t reason;    /* terminal events: DL_REASON_* */
  uint16_t reserved;
  uint32_t status;   /* selection status (0 ok) */
  uint64_t position; /* absolute position after the event */
  uint64_t count;    /* prompt tokens (consumed) or selections so far */
  uint32_t token;    /* selected token */
  float norm;        /* reserved (injection events) */
} dl_sequence_event;

/* Same arguments and validation as dl_engine_generate; returns at once. */
DL_API dl_status dl_engine_start(dl_engine* e, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                                 const dl_sampling* settings, uint64_t seed, const uint32_t* stop_ids,
                                 size_t n_stop, int prefill_mode);
/* Waits up to timeout_ms (< 0: no limit) for journal event `index`;
 * DL_NOT_READY if it did not arrive. */
DL_API dl_status dl_engine_collect(dl_engine* e, size_t index, int64_t timeout_ms, dl_sequence_event* out);
/* Asks the running loop to stop after its current step (terminal reason
 * DL_REASON_CANCELLED). */
DL_API dl_status dl_engine_request_stop(dl_engine* e);
/* Waits for the loop to finish; tokens_out (capacity max_new) receives the
 * selections, *n_out their count (a stop ID is included). */
DL_API dl_status dl_engine_drain(dl_engine* e, uint32_t* tokens_out, size_t* n_out, dl_generation_stats* stats);

#ifdef __cplusplus
}
#endif
#endif /* DOLITTLE_B200_H */
