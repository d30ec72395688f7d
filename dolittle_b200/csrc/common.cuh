// Shared device helpers for the sm_100a kernels.
//
// Storage is BF16 with FP32 arithmetic.  The storage rounding (round to
// nearest even) and widening follow the reference's common.cuh:67-89; every
// kernel in this library keeps the reference's explicit rounding points and
// its FP32 operation order (the library is compiled with --fmad=false and
// uses explicit __fmaf_rn where the reference does).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace dl {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float widen(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 narrow(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float round_bf16(float v) { return widen(narrow(v)); }

// Two packed BF16 values (low half first) to FP32, exact.
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---------------------------------------------------------------------------
// Error word written by kernels whose bounded waits ran out.  Kernels never
// trap; they record a code and return, and the host reads the word.
// ---------------------------------------------------------------------------
enum : unsigned {
  kErrNone = 0,
  kErrWaitFull = 1,    // consumer gave up waiting for a weight stage
  kErrWaitEmpty = 2,   // producer gave up waiting for a free stage
  kErrBounds = 3,      // a device-side position/index check failed
  kErrGridSync = 4,    // a persistent kernel's grid barrier gave up waiting
  kErrSteer = 5,       // a steering strength or steered value was not finite
};

__device__ __forceinline__ void record_error(unsigned* err, unsigned code) {
  if (err) atomicCAS(err, 0u, code);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA engine, untiled) primitives.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase (try_wait may suspend the thread for a while).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2^32 SM cycles (about 2 s at 1.9 GHz) so a
// lost arrival cannot hang the GPU.  Returns false on timeout; the caller
// records an error word and unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - start > (1ll << 32)) return false;
  }
}

// L2 policy for streamed-once weights: evict first, keep KV/activations hot.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Global -> shared bulk copy completing on an mbarrier (transaction bytes).
// dst, src and bytes must be 16-byte aligned / a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  wait_prior() must precede every read
// of data written by the previous kernel in the stream; allow_next() lets the
// next kernel's CTAs start their independent prologue (weight streaming).
// Both are no-ops when the launch carries no PDL attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier for a subset of warps (id 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(unsigned id, unsigned threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p)));
  return v;
}
__device__ __forceinline__ float4 lds128f(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_addr(p)));
  return v;
}

// ---------------------------------------------------------------------------
// Reduction laws shared by several kernels.
// ---------------------------------------------------------------------------
// The reference's 32-lane tree: value += shfl_down(value, off), off = 1..16.
__device__ __forceinline__ float shuffle_down_tree32(float v) {
#pragma unroll
  for (unsigned off = 1; off < 32; off *= 2) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
  return v;
}

// The reference's RMSNorm inverse for one row held as FP32 in shared memory
// (normalization.cu:82-186): width <= 128 uses the warp law, larger widths
// the staged law.  Executed by one full warp; every lane returns the value.
__device__ __forceinline__ float rms_inverse_warp(const float* x, unsigned width, float eps) {
  const unsigned lane = threadIdx.x & 31u;
  float sum;
  if (width <= 128) {
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (unsigned c = 0; c < 4; ++c) {
      const unsigned col = lane + 32u * c;
      if (col < width) part[c] = __fmul_rn(x[col], x[col]);
    }
    sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  } else {
    // Staged law: component sums over columns t+128k for t = 4*lane + c,
    // then the four components of each lane in order.
    float part[4];
#pragma unroll
    for (unsigned c = 0; c < 4; ++c) {
      float p = 0.f;
      for (unsigned col = 4 * lane + c; col < width; col += 128) p = __fadd_rn(p, __fmul_rn(x[col], x[col]));
      part[c] = p;
    }
    sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
  }
  sum = shuffle_down_tree32(sum);
  const float total = __shfl_sync(0xffffffffu, sum, 0);
  const float mean = __fmul_rn(total, 1.0f / static_cast<float>(width));
  return rsqrtf(__fadd_rn(mean, eps));
}

// The staged-law inverse (width > 128) of one row held as FP32 in shared
// memory, computed by a whole CTA of at least 128 threads: thread t < 128
// runs component chain t (columns t, t + 128, ...), warp 0 adds each lane's
// four chains in order and runs the 32-lane tree; the same value as
// rms_inverse_warp.  Every thread of the CTA calls it and gets the value.
// `chains` is shared memory of 129 floats.
__device__ __forceinline__ float rms_inverse_block(const float* xs, int width, float eps, float* chains) {
  if (threadIdx.x < 128) {
    // Eight loads ahead of the chain's dependent adds (the same order).
    float chain = 0.f;
    int col = threadIdx.x;
    for (; col + 7 * 128 < width; col += 8 * 128) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = xs[col + k * 128];
#pragma unroll
      for (int k = 0; k < 8; ++k) chain = __fadd_rn(chain, __fmul_rn(v[k], v[k]));
    }
    for (; col < width; col += 128) chain = __fadd_rn(chain, __fmul_rn(xs[col], xs[col]));
    chains[threadIdx.x] = chain;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const float* c4 = chains + 4 * threadIdx.x;
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(c4[0], c4[1]), c4[2]), c4[3]);
    sum = shuffle_down_tree32(sum);
    const float total = __shfl_sync(0xffffffffu, sum, 0);
    if (threadIdx.x == 0) chains[128] = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / static_cast<float>(width)), eps));
  }
  __syncthreads();
  return chains[128];
}

}  // namespace dl
