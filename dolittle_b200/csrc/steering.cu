// Block-output steering edit, capture copy and verbalizer injection.
//
// intervene: src/kernels/cuda/steering.cu:106-159.  At absolute row `selected`
// (when it lies in this step's rows): 8 strided lane sums of fmul(v,v), a
// serial total of the 8, beta = strength * sqrt_rn(total), then
// h' = round(h + beta*u) with finiteness latches; state = {invalid, count},
// count making the edit one-shot (a second application is invalid).
// normalize: src/kernels/cuda/injection.cu:48-102, out = BF16((h/||h||)*scale).
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

}  // namespace

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
