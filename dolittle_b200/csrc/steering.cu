// Block-output steering edit, capture copy and verbalizer injection.
//
// intervene: src/kernels/cuda/steering.cu:106-159.  At absolute row `selected`
// (when it lies in this step's rows): 8 strided lane sums of fmul(v,v), a
// serial total of the 8, beta = strength * sqrt_rn(total), then
// h' = round(h + beta*u) with finiteness latches; state = {invalid, count},
// count making the edit one-shot (a second application is invalid).
// normalize: src/kernels/cuda/injection.cu:48-102, out = BF16((h/||h||)*scale).
// steer_rows / steer_beta: fixed-strength steering of every position from a
// first one (no reference counterpart; the reference edits one row once):
// beta = alpha * ||h_source|| by the intervene norm law, then the intervene
// update h' = round(h + beta*u) on every selected row, so at the source row
// it equals the one-row edit bit for bit.
// direction: src/kernels/cuda/steering.cu:68-98 (DeviceDirection::submit,
// :211-258).  delta_i = FP32(edited_i) - FP32(original_i); lane L of 8 sums
// fmul(delta, delta) serially over i = L + 8k; lane 0 adds the 8 lane sums in
// order; norm = sqrt_rn; status 1 (output untouched) on a zero or non-finite
// norm, else direction_i = delta_i / norm (div_rn), stored FP32.
#include "launch.h"
#include "steering.h"

namespace dl {
namespace {

constexpr int kLanes = 8;

__global__ void intervene_kernel(bf16* residual, const float* direction, const long long* position,
                                 unsigned* state, int width, long long selected, int rows,
                                 float strength) {
  allow_next();
  wait_prior();
  const long long first = *position;
  if (selected < first || selected - first >= rows) return;
  __shared__ float sums[kLanes];
  __shared__ float beta;
  __shared__ unsigned invalid;
  if (threadIdx.x == 0) {
    invalid = (state[0] || state[1] != 0) ? 1u : 0u;
    ++state[1];
  }
  __syncthreads();
  bf16* row = residual + size_t(selected - first) * width;
  if (threadIdx.x < kLanes) {
    float s = 0.f;
    for (int i = threadIdx.x; i < width; i += kLanes) {
      const float v = widen(row[i]);
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    sums[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < kLanes; ++i) s = __fadd_rn(s, sums[i]);
    beta = __fmul_rn(strength, __fsqrt_rn(s));
    if (!isfinite(beta)) invalid = 1;
  }
  __syncthreads();
  const bool valid = invalid == 0;
  __syncthreads();
  if (valid) {
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
      const float value = __fadd_rn(widen(row[i]), __fmul_rn(beta, direction[i]));
      const bf16 stored = narrow(value);
      if (!isfinite(value) || !isfinite(widen(stored))) atomicOr(&invalid, 1u);
      row[i] = stored;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) state[0] = invalid;
}

__global__ void copy_rows_kernel(const bf16* src, bf16* arena, const long long* position, int width, int rows) {
  allow_next();
  wait_prior();
  bf16* dst = arena + size_t(*position) * width;
  const size_t n = size_t(rows) * width;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

__global__ void normalize_kernel(const bf16* source, bf16* out, float* norm, unsigned* status, int width,
                                 float scale) {
  __shared__ float sums[kLanes];
  __shared__ unsigned invalid;
  if (threadIdx.x == 0) invalid = 0;
  __syncthreads();
  if (threadIdx.x < kLanes) {
    float s = 0.f;
    for (int i = threadIdx.x; i < width; i += kLanes) {
      const float v = widen(source[i]);
      if (!isfinite(v)) atomicOr(&invalid, 1u);
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    sums[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < kLanes; ++i) s = __fadd_rn(s, sums[i]);
    *norm = __fsqrt_rn(s);
    if (!isfinite(*norm) || *norm == 0.f) invalid = 1;
  }
  __syncthreads();
  const bool valid = invalid == 0;
  __syncthreads();
  if (valid) {
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
      const float value = __fmul_rn(__fdiv_rn(widen(source[i]), *norm), scale);
      const bf16 stored = narrow(value);
      if (!isfinite(value) || !isfinite(widen(stored))) atomicOr(&invalid, 1u);
      out[i] = stored;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *status = invalid;
}

// One CTA.  Only the 8 lane chains are serial (the law's order): every
// thread computes a tile of squared differences into shared memory first, and
// the chains then walk that tile with one shared load per step; the tile
// loop carries each lane's running sum.
template <typename T>
__global__ void direction_kernel(const T* original, const T* edited, float* out, unsigned* status, int width) {
  constexpr int kTile = 4096;
  __shared__ float sq[kTile];
  __shared__ float lane_sum[kLanes];
  __shared__ float norm_s;
  if (threadIdx.x < kLanes) lane_sum[threadIdx.x] = 0.f;
  for (int t0 = 0; t0 < width; t0 += kTile) {
    const int n = min(kTile, width - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float delta = __fsub_rn(float(edited[t0 + i]), float(original[t0 + i]));
      sq[i] = __fmul_rn(delta, delta);
    }
    __syncthreads();
    if (threadIdx.x < kLanes) {
      // kTile is a multiple of 8, so lane L's features in this tile are
      // t0 + L + 8k: the serial chain continues across tiles in order.
      float acc = lane_sum[threadIdx.x];
      for (int i = threadIdx.x; i < n; i += kLanes) acc = __fadd_rn(acc, sq[i]);
      lane_sum[threadIdx.x] = acc;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int i = 0; i < kLanes; ++i) total = __fadd_rn(total, lane_sum[i]);
    const float norm = __fsqrt_rn(total);
    norm_s = norm;
    *status = (!isfinite(norm) || norm == 0.f) ? 1u : 0u;
  }
  __syncthreads();
  const float norm = norm_s;
  if (!isfinite(norm) || norm == 0.f) return;
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    out[i] = __fdiv_rn(__fsub_rn(float(edited[i]), float(original[i])), norm);
}

// Steering strength from a row: beta = alpha * ||h|| with the intervene
// law's norm (8 strided lane sums of fmul(v, v), lanes added in order,
// sqrt_rn), so a fixed-strength edit of that row equals the one-row edit.
__global__ void steer_beta_kernel(const bf16* row, int width, float alpha, float* beta, unsigned* err) {
  __shared__ float sums[kLanes];
  if (threadIdx.x < kLanes) {
    float s = 0.f;
    for (int i = threadIdx.x; i < width; i += kLanes) {
      const float v = widen(row[i]);
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    sums[threadIdx.x] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < kLanes; ++i) s = __fadd_rn(s, sums[i]);
    const float b = __fmul_rn(alpha, __fsqrt_rn(s));
    *beta = b;
    if (!isfinite(b)) record_error(err, kErrSteer);
  }
}

// Fixed-strength steering of every row at a position >= first: one CTA per
// row, h' = round(h + fmul(beta, u)) (the intervene law's arithmetic).  Row r
// sits at position (pos ? *pos : base) + (per_sequence ? 0 : r) and belongs
// to sequence per_sequence ? r : 0 of `mask`.
__global__ void steer_rows_kernel(bf16* residual, int width, const long long* pos, long long base, int per_sequence,
                                  const unsigned char* mask, long long first, const float* beta,
                                  const float* direction, unsigned* err) {
  allow_next();
  wait_prior();
  const int r = blockIdx.x;
  const long long p = (pos ? *pos : base) + (per_sequence ? 0 : r);
  if (p < first || !mask[per_sequence ? r : 0]) return;
  const float b = *beta;
  bf16* row = residual + size_t(r) * width;
  bool bad = !isfinite(b);
  for (int i = threadIdx.x; i < width && !bad; i += blockDim.x) {
    const float value = __fadd_rn(widen(row[i]), __fmul_rn(b, direction[i]));
    const bf16 stored = narrow(value);
    if (!isfinite(value) || !isfinite(widen(stored))) bad = true;
    row[i] = stored;
  }
  if (bad) record_error(err, kErrSteer);
}

// arena[b][*position] = rows[b] for b < batch (block-output capture of a
// lockstep batch at the shared position).
__global__ void capture_batch_kernel(const bf16* rows, bf16* arena, size_t seq_stride, const long long* position,
                                     int width) {
  allow_next();
  wait_prior();
  const int b = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(rows + size_t(b) * width);
  uint4* dst = reinterpret_cast<uint4*>(arena + b * seq_stride + size_t(*position) * width);
  for (int i = threadIdx.x; i < width / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

cudaError_t launch_steer_beta(const bf16* row, int width, float alpha, float* beta, unsigned* err,
                              cudaStream_t stream) {
  steer_beta_kernel<<<1, 32, 0, stream>>>(row, width, alpha, beta, err);
  return cudaGetLastError();
}

cudaError_t launch_steer_rows(bf16* residual, int width, int rows, const long long* position, long long base,
                              bool per_sequence, const unsigned char* mask, long long first, const float* beta,
                              const float* direction, unsigned* err, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  steer_rows_kernel<<<rows, 256, 0, stream>>>(residual, width, position, base, per_sequence ? 1 : 0, mask, first,
                                              beta, direction, err);
  return cudaGetLastError();
}

cudaError_t launch_capture_batch(const bf16* rows, bf16* arena, size_t seq_stride, const long long* position,
                                 int width, int batch, cudaStream_t stream) {
  if (width % 8) return cudaErrorInvalidValue;
  capture_batch_kernel<<<batch, 128, 0, stream>>>(rows, arena, seq_stride, position, width);
  return cudaGetLastError();
}

cudaError_t launch_direction(bool bf16_input, const void* original, const void* edited, float* out,
                             unsigned* status, int width, cudaStream_t stream) {
  if (bf16_input)
    direction_kernel<<<1, 512, 0, stream>>>(static_cast<const bf16*>(original), static_cast<const bf16*>(edited),
                                            out, status, width);
  else
    direction_kernel<<<1, 512, 0, stream>>>(static_cast<const float*>(original), static_cast<const float*>(edited),
                                            out, status, width);
  return cudaGetLastError();
}

cudaError_t launch_intervene(bf16* residual, const float* direction, const long long* position, unsigned* state,
                             int width, long long selected, int rows, float strength, cudaStream_t stream,
                             bool pdl) {
  cudaLaunchConfig_t c = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.gridDim = dim3(1);
  c.blockDim = dim3(256);
  c.stream = stream;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&c, intervene_kernel, residual, direction, position, state, width, selected,
                            rows, strength);
}

cudaError_t launch_copy_rows(const bf16* src, bf16* arena, const long long* position, int width, int rows,
                             cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t c = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.gridDim = dim3(std::max(1, std::min(64, rows * width / 2048)));
  c.blockDim = dim3(256);
  c.stream = stream;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&c, copy_rows_kernel, src, arena, position, width, rows);
}

cudaError_t launch_normalize_injection(const bf16* source, bf16* out, float* norm, unsigned* status,
                                       int width, float scale, cudaStream_t stream) {
  normalize_kernel<<<1, 256, 0, stream>>>(source, out, norm, status, width, scale);
  return cudaGetLastError();
}

}  // namespace dl
