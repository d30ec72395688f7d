// ref_cuda_shim.cu -- TEST INFRASTRUCTURE ONLY (checker, never shipped).
//
// A C ABI over the reference's own CUDA kernels, compiled from the reference
// sources where they lie (oracle/Makefile) for compute_86 PTX only, exactly
// like the reference's Ampere build; on a B200 the driver JIT-compiles that
// PTX.  These entry points let GPU tests compare the product's sm_100a
// kernels bit-for-bit with the reference on identical device inputs, and let
// bench.py time the reference CUDA path as a reported baseline.
//
// Wrapped reference interfaces:
//   launch_* : src/kernels/cuda/launch.h:79-109
//   DeviceCategorical : src/inference/sampling/device.h:54-85
//   DeviceDirection : src/inference/steering/device.h:30-48
// ref_qwen3_forward composes the launch_* calls in the reference recipe
// order, src/models/qwen3/model.cpp:343-409.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <stdexcept>
#include <vector>

#include "gpu/cuda/device.h"
#include "inference/sampling/device.h"
#include "inference/steering/device.h"
#include "kernels/cuda/launch.h"
#include "tensors/representations/bf16.h"

namespace k = dolittle::kernels::cuda;
namespace sampling = dolittle::inference::sampling;
using dolittle::tensors::ElementType;

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
ElementType type_of(int bf16) {
  return bf16 ? ElementType::bfloat16 : ElementType::float32;
}
int launched() { return cudaGetLastError() == cudaSuccess ? 0 : 2; }
}  // namespace

REF_API int ref_projection(int bf16, const void* x, const void* w, void* y,
                           std::size_t rows, std::size_t in, std::size_t out,
                           void* stream, const std::size_t* output_position) {
  try {
    k::launch_projection(type_of(bf16), x, w, y, rows, in, out,
                         static_cast<cudaStream_t>(stream), output_position);
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_rms_norm(int bf16, const void* x, const void* w, void* y,
                         std::size_t rows, std::size_t width, float eps,
                         void* stream) {
  try {
    k::launch_rms_norm(type_of(bf16), x, w, y, rows, width, eps,
                       static_cast<cudaStream_t>(stream));
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_rotary(int bf16, const void* x, void* y, std::size_t positions,
                       std::size_t heads, std::size_t width,
                       std::size_t first_position, double theta, void* stream,
                       const std::size_t* device_position,
                       int positioned_output) {
  try {
    k::launch_rotary(type_of(bf16), x, y, positions, heads, width,
                     first_position, theta, static_cast<cudaStream_t>(stream),
                     device_position, positioned_output != 0);
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_attention_scale(float* out, std::size_t width, void* stream) {
  k::launch_attention_scale(out, width, static_cast<cudaStream_t>(stream));
  return launched();
}
REF_API int ref_attention(int bf16, const void* q, const void* kk,
                          const void* v, void* y, std::size_t positions,
                          std::size_t query_heads, std::size_t kv_heads,
                          std::size_t width, void* stream,
                          std::size_t first_position,
                          const std::size_t* device_position,
                          std::size_t capacity, const float* scale) {
  try {
    k::launch_attention(type_of(bf16), q, kk, v, y, positions, query_heads,
                        kv_heads, width, static_cast<cudaStream_t>(stream),
                        first_position, device_position, capacity, scale);
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_embedding(int bf16, const std::uint32_t* tokens, const void* w,
                          void* y, std::size_t rows, std::size_t width,
                          void* stream) {
  try {
    k::launch_embedding(type_of(bf16), tokens, w, y, rows, width,
                        static_cast<cudaStream_t>(stream));
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_add(int bf16, const void* a, const void* b, void* y,
                    std::size_t n, void* stream) {
  try {
    k::launch_add(type_of(bf16), a, b, y, n, static_cast<cudaStream_t>(stream));
  } catch (...) {
    return 1;
  }
  return launched();
}
REF_API int ref_silu_multiply(int bf16, const void* g, const void* u, void* y,
                              std::size_t n, void* stream) {
  try {
    k::launch_silu_multiply(type_of(bf16), g, u, y, n,
                            static_cast<cudaStream_t>(stream));
  } catch (...) {
    return 1;
  }
  return launched();
}

// ---------------------------------------------------------------------------
// Reference Qwen3 forward over raw device pointers (host-position variant of
// every launch; numerically identical to the device-position graph path).
// tensors: [0] embedding, [1] final norm, [2] lm_head, then 11 per block in
// the order in_norm, q, k, v, q_norm, k_norm, o, post_norm, gate, up, down.
// cache[2l] / cache[2l+1] = K / V [capacity][kv_heads][head_width].
// scratch: ref_qwen3_scratch_bytes(cfg, rows) bytes of device memory.
// ---------------------------------------------------------------------------
struct RefConfig {
  std::uint32_t hidden, query_heads, kv_heads, head_width, mlp_width,
      vocabulary, layers;
  float epsilon;
  double theta;
};

REF_API std::size_t ref_qwen3_scratch_bytes(const RefConfig* c,
                                            std::size_t rows) {
  const std::size_t D = c->hidden, Q = c->query_heads * c->head_width,
                    G = c->kv_heads * c->head_width, F = c->mlp_width;
  const std::size_t elems =
      rows * (2 * D + 3 * Q + 2 * G + 2 * F + D) + D + c->vocabulary;
  return 2 * elems + 256 + 64;
}

REF_API int ref_qwen3_forward(const RefConfig* c, const void* const* tensors,
                              void* const* cache, std::size_t capacity,
                              const std::uint32_t* device_tokens,
                              std::size_t rows, std::size_t first,
                              void* logits_last, int capture_layer,
                              void* capture_rows, void* scratch,
                              void* stream_handle) {
  const auto s = static_cast<cudaStream_t>(stream_handle);
  const auto bt = ElementType::bfloat16;
  const std::size_t D = c->hidden, H = c->query_heads, G = c->kv_heads,
                    d = c->head_width, F = c->mlp_width, V = c->vocabulary;
  auto* base = static_cast<std::uint16_t*>(scratch);
  auto* scale = reinterpret_cast<float*>(base);
  std::uint16_t* p = base + 128;
  auto take = [&](std::size_t n) {
    auto* r = p;
    p += n;
    return r;
  };
  auto* residual = take(rows * D);
  auto* normed = take(rows * D);
  auto* q = take(rows * H * d);
  auto* q2 = take(rows * H * d);
  auto* att = take(rows * H * d);
  auto* kraw = take(rows * G * d);
  auto* k2 = take(rows * G * d);
  auto* gate = take(rows * F);
  auto* up = take(rows * F);
  auto* proj = take(rows * D);
  auto* last = take(D);
  try {
    k::launch_attention_scale(scale, d, s);
    k::launch_embedding(bt, device_tokens, tensors[0], residual, rows, D, s);
    for (std::uint32_t l = 0; l < c->layers; ++l) {
      const void* const* w = tensors + 3 + 11 * l;
      auto* kc = static_cast<std::uint16_t*>(cache[2 * l]);
      auto* vc = static_cast<std::uint16_t*>(cache[2 * l + 1]);
      k::launch_rms_norm(bt, residual, w[0], normed, rows, D, c->epsilon, s);
      k::launch_projection(bt, normed, w[1], q, rows, D, H * d, s);
      k::launch_projection(bt, normed, w[2], kraw, rows, D, G * d, s);
      k::launch_projection(bt, normed, w[3], vc + first * G * d, rows, D,
                           G * d, s);
      k::launch_rms_norm(bt, q, w[4], q2, rows * H, d, c->epsilon, s);
      k::launch_rotary(bt, q2, q, rows, H, d, first, c->theta, s);
      k::launch_rms_norm(bt, kraw, w[5], k2, rows * G, d, c->epsilon, s);
      k::launch_rotary(bt, k2, kc + first * G * d, rows, G, d, first,
                       c->theta, s);
      k::launch_attention(bt, q, kc, vc, att, rows, H, G, d, s, first, nullptr,
                          capacity, scale);
      k::launch_projection(bt, att, w[6], proj, rows, H * d, D, s);
      k::launch_add(bt, residual, proj, residual, rows * D, s);
      k::launch_rms_norm(bt, residual, w[7], normed, rows, D, c->epsilon, s);
      k::launch_projection(bt, normed, w[8], gate, rows, D, F, s);
      k::launch_projection(bt, normed, w[9], up, rows, D, F, s);
      k::launch_silu_multiply(bt, gate, up, gate, rows * F, s);
      k::launch_projection(bt, gate, w[10], proj, rows, F, D, s);
      k::launch_add(bt, residual, proj, residual, rows * D, s);
      // capture_layer >= 0: that block's output rows; -2: every block's,
      // as [layers][rows][D].
      if (capture_rows && (capture_layer == static_cast<int>(l) || capture_layer == -2)) {
        auto* dst = static_cast<std::uint16_t*>(capture_rows) +
                    (capture_layer == -2 ? l * rows * D : 0);
        if (cudaMemcpyAsync(dst, residual, 2 * rows * D,
                            cudaMemcpyDeviceToDevice, s) != cudaSuccess)
          return 2;
      }
    }
    if (logits_last) {
      k::launch_rms_norm(bt, residual + (rows - 1) * D, tensors[1], last, 1, D,
                         c->epsilon, s);
      k::launch_projection(bt, last, tensors[2], logits_last, 1, D, V, s);
    }
  } catch (...) {
    return 1;
  }
  return launched();
}

// ---------------------------------------------------------------------------
// DeviceCategorical through the reference's own gpu::Device (device 0).
// ---------------------------------------------------------------------------
namespace {
struct SamplerHarness {
  std::unique_ptr<dolittle::gpu::Device> device;
  std::unique_ptr<dolittle::gpu::Queue> queue;
};
SamplerHarness& harness() {
  static SamplerHarness h;
  if (!h.device) {
    h.device = dolittle::gpu::cuda::open_device(0);
    h.queue = std::make_unique<dolittle::gpu::Queue>(h.device->create_queue());
  }
  return h;
}
void encode(const float* logits, std::size_t n, bool bf16,
            std::span<std::byte> bytes) {
  for (std::size_t i = 0; i < n; ++i) {
    if (bf16) {
      const auto b = dolittle::tensors::from_float(logits[i]).bits;
      std::memcpy(bytes.data() + 2 * i, &b, 2);
    } else {
      std::memcpy(bytes.data() + 4 * i, &logits[i], 4);
    }
  }
}
}  // namespace

// One diagnostic draw with explicit bits (DeviceCategorical::submit).
REF_API int ref_device_select(const float* logits, std::size_t n, int bf16,
                              int categorical, double temperature,
                              std::size_t top_k, double top_p,
                              std::uint64_t bits, std::uint32_t* result) {
  try {
    auto& h = harness();
    const std::size_t bytes = n * (bf16 ? 2 : 4);
    auto row = h.device->allocate({bytes, 256});
    auto staging = h.device->allocate_staging({bytes, 8});
    auto answer = h.device->allocate_staging({8, 8});
    encode(logits, n, bf16 != 0, staging.bytes());
    h.queue->upload({&row, 0, bytes}, {&staging, 0, bytes});
    sampling::DeviceCategorical selector(
        *h.device, *h.queue, n, bf16 ? ElementType::bfloat16 : ElementType::float32,
        sampling::DeviceCategorical::required_bytes(n));
    const sampling::Settings settings{
        categorical ? sampling::SelectionMode::categorical
                    : sampling::SelectionMode::greedy,
        temperature, top_k, top_p};
    const auto region = selector.submit({&row, 0, bytes}, {settings, bits});
    h.queue->download({&answer, 0, 8}, region);
    h.queue->drain();
    std::memcpy(result, answer.bytes().data(), 8);
    return 0;
  } catch (...) {
    return 1;
  }
}

// Device-owned MT19937-64 continuation (start + submit_next, draws times).
REF_API int ref_device_sequence(const float* logits, std::size_t n, int bf16,
                                double temperature, std::size_t top_k,
                                double top_p, std::uint64_t seed,
                                std::size_t draws, std::uint32_t* results) {
  try {
    auto& h = harness();
    const std::size_t bytes = n * (bf16 ? 2 : 4);
    auto row = h.device->allocate({bytes, 256});
    auto staging = h.device->allocate_staging({bytes, 8});
    auto answer = h.device->allocate_staging({8, 8});
    encode(logits, n, bf16 != 0, staging.bytes());
    h.queue->upload({&row, 0, bytes}, {&staging, 0, bytes});
    sampling::DeviceCategorical selector(
        *h.device, *h.queue, n, bf16 ? ElementType::bfloat16 : ElementType::float32,
        sampling::DeviceCategorical::required_bytes(n));
    const sampling::Settings settings{sampling::SelectionMode::categorical,
                                      temperature, top_k, top_p};
    selector.start(settings, seed, {});
    for (std::size_t i = 0; i < draws; ++i) {
      const auto region = selector.submit_next({&row, 0, bytes});
      h.queue->download({&answer, 0, 8}, region);
      h.queue->drain();
      std::memcpy(results + 2 * i, answer.bytes().data(), 8);
    }
    return 0;
  } catch (...) {
    return 1;
  }
}

// DeviceDirection over two reconstructions given as host bytes (BF16 bits or
// FP32): submit + finish through the reference's own gpu::Device.  status 1
// when finish rejects a zero or non-finite difference (the direction is then
// not read); otherwise the FP32 direction goes to `direction`.
REF_API int ref_direction(int bf16, const void* original, const void* edited,
                          std::size_t width, float* direction,
                          unsigned* status) {
  try {
    auto& h = harness();
    const std::size_t bytes = width * (bf16 ? 2 : 4);
    auto upload = [&](const void* src) {
      auto buffer = std::make_shared<dolittle::gpu::DeviceBuffer>(
          h.device->allocate({bytes, 256}));
      auto staging = h.device->allocate_staging({bytes, 8});
      std::memcpy(staging.bytes().data(), src, bytes);
      h.queue->upload({buffer.get(), 0, bytes}, {&staging, 0, bytes});
      h.queue->drain();
      return dolittle::inference::DeviceCapture{buffer, 0, bytes};
    };
    dolittle::inference::DeviceDirection dir(
        *h.device, *h.queue, upload(original), upload(edited),
        bf16 ? ElementType::bfloat16 : ElementType::float32, width);
    dir.submit();
    dolittle::inference::DeviceCapture out;
    try {
      out = dir.finish();
    } catch (const std::invalid_argument&) {
      *status = 1;
      return 0;
    }
    *status = 0;
    auto answer = h.device->allocate_staging({width * 4, 8});
    h.queue->download({&answer, 0, width * 4}, out.region());
    h.queue->drain();
    std::memcpy(direction, answer.bytes().data(), width * 4);
    return 0;
  } catch (...) {
    return 1;
  }
}
