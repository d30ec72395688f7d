// ref_host_shim.cpp -- TEST INFRASTRUCTURE ONLY (checker, never shipped).
//
// A C ABI over the reference's own host code, compiled from the reference
// sources where they lie (see oracle/Makefile) into oracle/_ref/:
//   - BF16 narrowing/widening: src/tensors/representations/bf16.cpp:43-60
//   - host selection law Categorical::select:
//     src/inference/sampling/categorical.cpp:146-201, with the std::mt19937_64
//     RandomStream of src/inference/sampling/sampler.h.
// Used by tests/ to pin oracle/dl_oracle.c against the reference itself.
#include <cstdint>
#include <random>
#include <span>
#include <stdexcept>

#include "inference/sampling/categorical.h"
#include "tensors/representations/bf16.h"

namespace sampling = dolittle::inference::sampling;

extern "C" {
__attribute__((visibility("default"))) std::uint16_t ref_bf16_from_float(
    float value) {
  return dolittle::tensors::from_float(value).bits;
}
__attribute__((visibility("default"))) float ref_bf16_to_float(
    std::uint16_t bits) {
  return dolittle::tensors::to_float(dolittle::tensors::BFloat16{bits});
}

// Opaque std::mt19937_64 streams so tests can check draw consumption.
__attribute__((visibility("default"))) void* ref_rng_create(
    std::uint64_t seed) {
  return new sampling::RandomStream(seed);
}
__attribute__((visibility("default"))) void ref_rng_destroy(void* rng) {
  delete static_cast<sampling::RandomStream*>(rng);
}
__attribute__((visibility("default"))) std::uint64_t ref_rng_next(void* rng) {
  return (*static_cast<sampling::RandomStream*>(rng))();
}
__attribute__((visibility("default"))) int ref_rng_equal(void* a, void* b) {
  return *static_cast<sampling::RandomStream*>(a) ==
         *static_cast<sampling::RandomStream*>(b);
}

// Returns 0 on success, 1 when the reference throws invalid_argument.
__attribute__((visibility("default"))) int ref_categorical_select(
    const float* logits, std::size_t n, int categorical, double temperature,
    std::size_t top_k, double top_p, void* rng, std::uint32_t* token) {
  try {
    sampling::Categorical selector(n);
    const sampling::Settings settings{
        categorical ? sampling::SelectionMode::categorical
                    : sampling::SelectionMode::greedy,
        temperature, top_k, top_p};
    *token = selector.select(std::span<const float>(logits, n), settings,
                             *static_cast<sampling::RandomStream*>(rng));
    return 0;
  } catch (const std::invalid_argument&) {
    return 1;
  }
}
}
