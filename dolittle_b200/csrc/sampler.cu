// Device token selection under the reference device law
// (src/kernels/cuda/sampling.cu:106-376):
//  * greedy: maximum value, lowest ID on ties; NaN/+inf latch status 1; no
//    finite maximum gives status 2;
//  * categorical: candidates in stable order (value descending, ID
//    ascending; -0 == +0); keep = top_k or all; FP64 weights
//    exp((v - best)/T) (0 for non-finite v); inclusive serial prefix inside
//    fixed 256-entry tiles, serial exclusive scan of the tile totals; cutoff =
//    first i with cum/total >= top_p; selection = first i <= cutoff with
//    u < cum/retained; u = (word >> 11) * 2^-53;
//  * the device-owned stream is MT19937-64 (std::mt19937_64), one word per
//    categorical selection, latched after a stop ID or a failed selection;
//    or, when selected, Philox4x32-10 (Salmon et al., SC'11): draw k of row r
//    is the first two words of the block at counter {k lo, k hi, stream
//    0x5A4D504C, 0} under key seed + r, w = (word1 << 32) | word0, with the
//    same u = (w >> 11) * 2^-53.  The reference has only the MT19937-64
//    stream; the Philox stream is stateless per draw (no 312-word state).
// The stable order is produced by an LSD radix sort over the 32-bit keys.  For
// BF16 logits the low 16 key bits are a function of the sign, so sorting on
// the high 16 bits alone gives the same order (two passes instead of four).
#include <cstring>
#include <stdexcept>
#include <type_traits>
#include <vector>

#include "qknorm.cuh"
#include "sampler.h"

namespace dl {

struct SamplerState {
  uint64_t words[312];
  unsigned index, terminal;
  double draw;
  unsigned previous[2];
  unsigned engine;   // DL_RNG_MT19937_64 or DL_RNG_PHILOX4X32_10
  unsigned pad;
  uint64_t key;      // Philox key: seed + row
  uint64_t counter;  // Philox draws made
};

constexpr uint32_t kPhiloxSamplerStream = 0x5A4D504Cu;

namespace {

constexpr unsigned kW = 256;
constexpr unsigned kWarps = kW / 32;

struct ScanState {
  double total;
  unsigned cutoff, selected, ticket, pad;
};

struct Layout {
  uint2* keys_a;
  uint2* keys_b;
  double* prefix;
  unsigned* counts;
  unsigned* digit_totals;
  double* tile_totals;
  uint4* best;
  ScanState* scan;
  unsigned* result;
  SamplerState* state;
  unsigned char* stop_mask;
};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Layout layout(void* arena, size_t n) {
  const size_t blocks = (n + kW - 1) / kW;
  auto* b = static_cast<unsigned char*>(arena);
  size_t o = 0;
  Layout L;
  L.keys_a = reinterpret_cast<uint2*>(b + o); o = align_up(o + n * 8, 256);
  L.keys_b = reinterpret_cast<uint2*>(b + o); o = align_up(o + n * 8, 256);
  L.prefix = reinterpret_cast<double*>(b + o); o = align_up(o + n * 8, 256);
  L.counts = reinterpret_cast<unsigned*>(b + o); o = align_up(o + blocks * kW * 4, 256);
  L.digit_totals = reinterpret_cast<unsigned*>(b + o); o = align_up(o + kW * 4, 256);
  L.tile_totals = reinterpret_cast<double*>(b + o); o = align_up(o + blocks * 8, 256);
  L.best = reinterpret_cast<uint4*>(b + o); o = align_up(o + blocks * 16, 256);
  L.scan = reinterpret_cast<ScanState*>(b + o); o = align_up(o + sizeof(ScanState), 256);
  L.result = reinterpret_cast<unsigned*>(b + o); o = align_up(o + 8, 256);
  L.state = reinterpret_cast<SamplerState*>(b + o); o = align_up(o + sizeof(SamplerState), 256);
  L.stop_mask = b + o;
  return L;
}

// Row r of a batched sampler (blockIdx.y) owns the arena slice at r * stride
// bytes; its logits row sits at r * row_bytes past row 0.
template <class T>
__device__ __forceinline__ T* at_row(T* p, size_t stride) {
  using U = typename std::conditional<std::is_const<T>::value, const unsigned char, unsigned char>::type;
  return p ? reinterpret_cast<T*>(reinterpret_cast<U*>(p) + blockIdx.y * stride) : p;
}

__device__ __forceinline__ float load_logit(const void* row, unsigned i, bool bf16_in) {
  return bf16_in ? widen(static_cast<const bf16*>(row)[i]) : static_cast<const float*>(row)[i];
}

__device__ __forceinline__ unsigned descending_key(float v) {
  if (v == 0.0f) v = 0.0f;
  const unsigned bits = __float_as_uint(v);
  const unsigned mask = (0u - (bits >> 31)) | 0x80000000u;
  return ~(bits ^ mask);
}

// ---- MT19937-64 -----------------------------------------------------------
__global__ void seed_kernel(SamplerState* s, uint64_t seed, size_t stride, unsigned engine) {
  s = at_row(s, stride);
  seed += blockIdx.y;  // row r draws from the stream seeded with seed + r
  s->engine = engine;
  s->key = seed;
  s->counter = 0;
  s->words[0] = seed;
  for (unsigned i = 1; i < 312; ++i) {
    const uint64_t p = s->words[i - 1];
    s->words[i] = 6364136223846793005ULL * (p ^ (p >> 62)) + i;
  }
  s->index = 312;
  s->terminal = 0;
  s->draw = 0;
  s->previous[0] = s->previous[1] = 0;
}

__global__ void next_random_kernel(SamplerState* s, bool greedy, size_t stride) {
  s = at_row(s, stride);
  if (s->terminal || greedy) return;
  if (s->engine == DL_RNG_PHILOX4X32_10) {
    const uint64_t k = s->counter++;
    uint32_t c[4] = {uint32_t(k), uint32_t(k >> 32), kPhiloxSamplerStream, 0u};
    philox4x32_10(c, uint32_t(s->key), uint32_t(s->key >> 32));
    const uint64_t w = (uint64_t(c[1]) << 32) | c[0];
    s->draw = static_cast<double>(w >> 11) * 0x1.0p-53;
    return;
  }
  if (s->index == 312) {
    for (unsigned i = 0; i < 312; ++i) {
      const uint64_t x = (s->words[i] & 0xffffffff80000000ULL) | (s->words[(i + 1) % 312] & 0x7fffffffULL);
      s->words[i] = s->words[(i + 156) % 312] ^ (x >> 1) ^ ((x & 1) ? 0xb5026f5aa96619e9ULL : 0);
    }
    s->index = 0;
  }
  uint64_t x = s->words[s->index++];
  x ^= (x >> 29) & 0x5555555555555555ULL;
  x ^= (x << 17) & 0x71d67fffeda60000ULL;
  x ^= (x << 37) & 0xfff7eee000000000ULL;
  x ^= x >> 43;
  s->draw = static_cast<double>(x >> 11) * 0x1.0p-53;
}

__global__ void commit_kernel(SamplerState* s, unsigned* result, const unsigned char* stops, size_t stride) {
  s = at_row(s, stride);
  result = at_row(result, stride);
  stops = at_row(stops, stride);
  if (s->terminal) {
    result[0] = s->previous[0];
    result[1] = s->previous[1];
    return;
  }
  s->previous[0] = result[0];
  s->previous[1] = result[1];
  s->terminal = result[1] || stops[result[0]];
}

// ---- greedy ----------------------------------------------------------------
__device__ __forceinline__ bool better(float v, unsigned id, float bv, unsigned bid) {
  return v > bv || (v == bv && id < bid);
}

__global__ void greedy_kernel(const void* row, bool bf16_in, unsigned n, uint4* best, ScanState* scan,
                              unsigned* result, size_t stride, size_t row_bytes) {
  __shared__ uint4 warp_best[kWarps];
  __shared__ bool last;
  row = static_cast<const unsigned char*>(row) + blockIdx.y * row_bytes;
  best = at_row(best, stride);
  scan = at_row(scan, stride);
  result = at_row(result, stride);
  const unsigned i = blockIdx.x * kW + threadIdx.x;
  float v = -INFINITY;
  unsigned id = 0xffffffffu, flags = 0;
  if (i < n) {
    v = load_logit(row, i, bf16_in);
    if (isnan(v) || v == INFINITY) flags = 1;
    id = i;
    if (isnan(v)) v = -INFINITY;  // never selected; the status latch decides
  }
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const unsigned oid = __shfl_xor_sync(0xffffffffu, id, off);
    flags |= __shfl_xor_sync(0xffffffffu, flags, off);
    if (better(ov, oid, v, id)) { v = ov; id = oid; }
  }
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = make_uint4(__float_as_uint(v), id, flags, 0);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint4 b = warp_best[0];
    for (unsigned w = 1; w < kWarps; ++w) {
      const uint4 c = warp_best[w];
      if (better(__uint_as_float(c.x), c.y, __uint_as_float(b.x), b.y)) { b.x = c.x; b.y = c.y; }
      b.z |= c.z;
    }
    best[blockIdx.x] = b;
    __threadfence();
    last = atomicAdd(&scan->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  float bv = -INFINITY;
  unsigned bid = 0xffffffffu, fl = 0;
  for (unsigned b = 0; b < gridDim.x; ++b) {
    const uint4 c = __ldcg(&best[b]);
    fl |= c.z;
    if (better(__uint_as_float(c.x), c.y, bv, bid)) { bv = __uint_as_float(c.x); bid = c.y; }
  }
  scan->ticket = 0;
  result[1] = fl ? 1u : (isfinite(bv) ? 0u : 2u);
  result[0] = result[1] ? 0u : bid;
}

// result[0..1] of every row back to zero before a selection.
__global__ void clear_results_kernel(unsigned* result, size_t stride, unsigned rows) {
  const unsigned row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  unsigned* r = reinterpret_cast<unsigned*>(reinterpret_cast<unsigned char*>(result) + row * stride);
  r[0] = 0;
  r[1] = 0;
}

// ---- categorical -------------------------------------------------------------
__global__ void keys_kernel(const void* row, bool bf16_in, unsigned n, uint2* keys, unsigned* result, size_t stride,
                            size_t row_bytes) {
  row = static_cast<const unsigned char*>(row) + blockIdx.y * row_bytes;
  keys = at_row(keys, stride);
  result = at_row(result, stride);
  const unsigned i = blockIdx.x * kW + threadIdx.x;
  if (i >= n) return;
  const float v = load_logit(row, i, bf16_in);
  if (isnan(v) || v == INFINITY) atomicExch(&result[1], 1u);
  keys[i] = make_uint2(descending_key(v), i);
}

// Per-block digit counts, stable ranks inside a block come from warp match.
__device__ __forceinline__ void block_digit_ranks(unsigned digit, bool live, unsigned (*bins)[kW],
                                                  unsigned& peers) {
  const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (unsigned w = 0; w < kWarps; ++w) bins[w][threadIdx.x] = 0;
  __syncthreads();
  peers = __match_any_sync(0xffffffffu, live ? digit : 0x100u);
  if (live && lane == unsigned(__ffs(int(peers)) - 1)) bins[warp][digit] = __popc(peers);
  __syncthreads();
}

// Radix blocks of kRadixPer consecutive 256-key tiles: fewer, longer CTAs
// (and fewer per-block counts to scan) than one tile per CTA.
constexpr unsigned kRadixPer = 8;
constexpr unsigned kRadixBlock = kW * kRadixPer;
static_assert(kRadixPer == kWarps, "weights_kernel scans tile w with warp w");

__global__ void histogram_kernel(const uint2* keys, unsigned n, unsigned shift, unsigned* counts, size_t stride) {
  __shared__ unsigned bins[kW];
  keys = at_row(keys, stride);
  counts = at_row(counts, stride);
  const unsigned lane = threadIdx.x & 31;
  bins[threadIdx.x] = 0;
  __syncthreads();
#pragma unroll
  for (unsigned e = 0; e < kRadixPer; ++e) {
    const unsigned i = blockIdx.x * kRadixBlock + e * kW + threadIdx.x;
    const bool live = i < n;
    const unsigned digit = live ? (keys[i].x >> shift) & 0xffu : 0x100u;
    // One shared-memory add per distinct digit of the warp.
    const unsigned peers = __match_any_sync(0xffffffffu, digit);
    if (live && lane == unsigned(__ffs(int(peers)) - 1)) atomicAdd(&bins[digit], unsigned(__popc(peers)));
  }
  __syncthreads();
  counts[blockIdx.x * kW + threadIdx.x] = bins[threadIdx.x];
}

// Radix offsets, in two halves.  This kernel turns each digit column of the
// per-block counts into its exclusive prefix over the blocks, in place
// (counts[b][d] = keys with digit d in blocks b' < b), and writes the
// column's total to totals[d]; the scatter adds the exclusive scan of the
// totals over the digits.  Offsets are integer sums, so any order gives the
// same stable sort.  CTA g owns digits 32g .. 32g+31 (lane = digit, so a warp
// load is one 128-byte line of a block's counts) and warp w owns block segment
// w of kOffsetWarps, so the column walks run on kW / 32 CTAs side by side.
constexpr unsigned kOffsetWarps = 32;
__global__ void __launch_bounds__(32 * kOffsetWarps)
    digit_offsets_kernel(unsigned* counts, unsigned* totals, unsigned blocks, size_t stride) {
  __shared__ unsigned seg[kOffsetWarps][32];
  counts = at_row(counts, stride);
  totals = at_row(totals, stride);
  const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned d = blockIdx.x * 32 + lane;
  const unsigned per = (blocks + kOffsetWarps - 1) / kOffsetWarps;
  const unsigned b0 = min(blocks, w * per), b1 = min(blocks, b0 + per);
  unsigned sum = 0;
  for (unsigned b = b0; b < b1; b += 8) {
    unsigned c[8];
#pragma unroll
    for (unsigned k = 0; k < 8; ++k) c[k] = b + k < b1 ? counts[(b + k) * kW + d] : 0u;
#pragma unroll
    for (unsigned k = 0; k < 8; ++k) sum += c[k];
  }
  seg[w][lane] = sum;
  __syncthreads();
  unsigned run = 0;
  for (unsigned k = 0; k < w; ++k) run += seg[k][lane];
  if (w == kOffsetWarps - 1) totals[d] = run + sum;
  for (unsigned b = b0; b < b1; b += 8) {
    unsigned c[8];
#pragma unroll
    for (unsigned k = 0; k < 8; ++k) c[k] = b + k < b1 ? counts[(b + k) * kW + d] : 0u;
#pragma unroll
    for (unsigned k = 0; k < 8; ++k)
      if (b + k < b1) {
        counts[(b + k) * kW + d] = run;
        run += c[k];
      }
  }
}

__global__ void scatter_kernel(const uint2* in, uint2* out, unsigned n, unsigned shift, const unsigned* offsets,
                               const unsigned* totals, size_t stride) {
  __shared__ unsigned bins[kWarps][kW];
  __shared__ unsigned digit_base[kW];
  __shared__ unsigned warp_sum[kWarps];
  __shared__ unsigned running[kW], block_offset[kW];
  in = at_row(in, stride);
  out = at_row(out, stride);
  offsets = at_row(offsets, stride);
  totals = at_row(totals, stride);
  {
    // digit_base[d] = keys with a digit below d: exclusive scan of the
    // digit totals (thread = digit; warp scans, then the warp sums).
    const unsigned t = totals[threadIdx.x], ln = threadIdx.x & 31, wp = threadIdx.x >> 5;
    unsigned v = t;
    for (unsigned off = 1; off < 32; off <<= 1) {
      const unsigned o = __shfl_up_sync(0xffffffffu, v, off);
      if (ln >= off) v += o;
    }
    if (ln == 31) warp_sum[wp] = v;
    __syncthreads();
    unsigned before = 0;
    for (unsigned k = 0; k < wp; ++k) before += warp_sum[k];
    digit_base[threadIdx.x] = before + v - t;
  }
  // The block's tiles in key order; running[d] = keys with digit d in the
  // tiles before (block_digit_ranks starts with a CTA barrier, which
  // publishes digit_base and running).
  running[threadIdx.x] = 0;
  const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned base = offsets[blockIdx.x * kW + threadIdx.x];  // thread = digit
  block_offset[threadIdx.x] = base;
  for (unsigned e = 0; e < kRadixPer; ++e) {
    const unsigned i = blockIdx.x * kRadixBlock + e * kW + threadIdx.x;
    const bool live = i < n;
    const uint2 k = live ? in[i] : make_uint2(0, 0);
    const unsigned digit = (k.x >> shift) & 0xffu;
    unsigned peers;
    block_digit_ranks(digit, live, bins, peers);
    if (live) {
      unsigned rank = running[digit] + __popc(peers & ((1u << lane) - 1u));
      for (unsigned w = 0; w < warp; ++w) rank += bins[w][digit];
      out[digit_base[digit] + block_offset[digit] + rank] = k;
    }
    __syncthreads();  // ranks read running and bins
    unsigned add = 0;
    for (unsigned w = 0; w < kWarps; ++w) add += bins[w][threadIdx.x];
    running[threadIdx.x] += add;
    __syncthreads();  // running complete; bins free
  }
}

// kRadixPer tiles of 256 sorted keys per CTA: the weights of every key, then
// each tile's serial FP64 prefix (the law's order) by one lane per tile, the
// tiles side by side.
__global__ void weights_kernel(const void* row, bool bf16_in, const uint2* sorted, unsigned keep,
                               double temperature, double* prefix, double* tile_totals, size_t stride,
                               size_t row_bytes) {
  __shared__ double tile[kRadixPer][kW];
  row = static_cast<const unsigned char*>(row) + blockIdx.y * row_bytes;
  sorted = at_row(sorted, stride);
  prefix = at_row(prefix, stride);
  tile_totals = at_row(tile_totals, stride);
  const double best = static_cast<double>(load_logit(row, sorted[0].y, bf16_in));
#pragma unroll
  for (unsigned e = 0; e < kRadixPer; ++e) {
    const unsigned i = blockIdx.x * kRadixBlock + e * kW + threadIdx.x;
    double w = 0.0;
    if (i < keep) {
      const double v = static_cast<double>(load_logit(row, sorted[i].y, bf16_in));
      if (isfinite(v)) w = exp((v - best) / temperature);
    }
    tile[e][threadIdx.x] = w;
  }
  __syncthreads();
  const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;  // kWarps == kRadixPer
  const unsigned t = blockIdx.x * kRadixPer + warp;                // this warp's tile
  if (lane == 0 && t * kW < keep) {
    double sum = 0.0;
    for (unsigned j = 0; j < kW; ++j) {
      sum += tile[warp][j];
      tile[warp][j] = sum;
    }
    tile_totals[t] = sum;
  }
  __syncthreads();
#pragma unroll
  for (unsigned e = 0; e < kRadixPer; ++e) {
    const unsigned i = blockIdx.x * kRadixBlock + e * kW + threadIdx.x;
    if (i < keep) prefix[i] = tile[e][threadIdx.x];
  }
}

// Serial exclusive scan of the tile totals (the law's FP64 order), on a
// shared-memory copy so the serial loop does not wait on global loads.
__global__ void scan_tiles_kernel(double* tile_totals, unsigned keep, ScanState* scan, unsigned* result,
                                  size_t stride) {
  extern __shared__ double tiles_s[];
  tile_totals = at_row(tile_totals, stride);
  scan = at_row(scan, stride);
  result = at_row(result, stride);
  const unsigned tiles = (keep + kW - 1) / kW;
  for (unsigned b = threadIdx.x; b < tiles; b += blockDim.x) tiles_s[b] = tile_totals[b];
  __syncthreads();
  if (threadIdx.x == 0) {
    double total = 0.0;
    for (unsigned b = 0; b < tiles; ++b) {
      const double v = tiles_s[b];
      tiles_s[b] = total;
      total += v;
    }
    scan->total = total;
    scan->cutoff = keep - 1;
    scan->selected = keep - 1;
    if (!(total > 0.0)) result[1] = 2;
  }
  __syncthreads();
  for (unsigned b = threadIdx.x; b < tiles; b += blockDim.x) tile_totals[b] = tiles_s[b];
}

__device__ unsigned block_min(unsigned v) {
  __shared__ unsigned m[kWarps];
  for (int off = 16; off; off >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, off));
  if ((threadIdx.x & 31) == 0) m[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned r = m[0];
  for (unsigned w = 1; w < kWarps; ++w) r = min(r, m[w]);
  return r;
}

__global__ void cutoff_kernel(const double* prefix, const double* offsets, unsigned keep, double top_p,
                              ScanState* scan, size_t stride) {
  prefix = at_row(prefix, stride);
  offsets = at_row(offsets, stride);
  scan = at_row(scan, stride);
  unsigned c = 0xffffffffu;
  const double total = scan->total;
  for (unsigned e = 0; e < kRadixPer && c == 0xffffffffu; ++e) {
    const unsigned t = blockIdx.x * kRadixPer + e, i = t * kW + threadIdx.x;
    if (i < keep && (offsets[t] + prefix[i]) / total >= top_p) c = i;
  }
  const unsigned first = block_min(c);
  if (threadIdx.x == 0 && first != 0xffffffffu) atomicMin(&scan->cutoff, first);
}

__global__ void select_kernel(const double* prefix, const double* offsets, unsigned keep, double draw,
                              const SamplerState* state, ScanState* scan, size_t stride) {
  prefix = at_row(prefix, stride);
  offsets = at_row(offsets, stride);
  state = at_row(state, stride);
  scan = at_row(scan, stride);
  const unsigned last = scan->cutoff;
  const double retained = offsets[last / kW] + prefix[last];
  const double u = state ? state->draw : draw;
  unsigned c = 0xffffffffu;
  for (unsigned e = 0; e < kRadixPer && c == 0xffffffffu; ++e) {
    const unsigned t = blockIdx.x * kRadixPer + e, i = t * kW + threadIdx.x;
    if (i <= last && i < keep && u < (offsets[t] + prefix[i]) / retained) c = i;
  }
  const unsigned first = block_min(c);
  if (threadIdx.x == 0 && first != 0xffffffffu) atomicMin(&scan->selected, first);
}

__global__ void finish_kernel(const uint2* sorted, const ScanState* scan, unsigned* result, size_t stride) {
  sorted = at_row(sorted, stride);
  scan = at_row(scan, stride);
  result = at_row(result, stride);
  if (!result[1]) result[0] = sorted[min(scan->selected, scan->cutoff)].y;
}

// Row r: history row r (history_stride elements apart), step[r], residual
// row r; the shared position advances once (row 0).
__global__ void feed_kernel(const unsigned* result, unsigned* history, int* step, const bf16* embed,
                            bf16* residual, int width, long long* position, size_t stride, size_t history_stride) {
  const unsigned r = blockIdx.y;
  result = at_row(result, stride);
  if (history) history += r * history_stride;
  if (step) step += r;
  if (residual) residual += size_t(r) * width;
  if (r) position = nullptr;
  const unsigned token = result[0];
  if (threadIdx.x == 0) {
    if (history) history[step ? *step : 0] = token;
  }
  if (embed) {
    const bf16* src = embed + size_t(token) * width;
    for (int f = threadIdx.x; f < width; f += blockDim.x) residual[f] = src[f];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (step) ++*step;
    if (position) ++*position;
  }
}

}  // namespace

void validate_sampling(const dl_sampling& s, size_t vocabulary) {
  const bool finite_t = s.temperature == s.temperature && s.temperature < 1e308 && s.temperature > -1e308;
  const bool finite_p = s.top_p == s.top_p && s.top_p < 1e308 && s.top_p > -1e308;
  if ((s.mode != 0 && s.mode != 1) || !finite_t || s.temperature <= 0 || !finite_p || s.top_p <= 0 ||
      s.top_p > 1 || (s.mode == 0 && (s.temperature != 1 || s.top_k != 0 || s.top_p != 1)) ||
      s.top_k > vocabulary)
    throw std::invalid_argument("invalid sampling settings");
}

size_t sampler_required_bytes(size_t n) {
  const size_t blocks = (n + kW - 1) / kW;
  size_t o = 0;
  o = align_up(o + n * 8, 256);
  o = align_up(o + n * 8, 256);
  o = align_up(o + n * 8, 256);
  o = align_up(o + blocks * kW * 4, 256);
  o = align_up(o + kW * 4, 256);
  o = align_up(o + blocks * 8, 256);
  o = align_up(o + blocks * 16, 256);
  o = align_up(o + sizeof(ScanState), 256);
  o = align_up(o + 8, 256);
  o = align_up(o + sizeof(SamplerState), 256);
  return o + n;
}

cudaError_t sampler_init(Sampler& s, size_t vocabulary, bool bf16_input, unsigned rows) {
  s.vocabulary = vocabulary;
  s.bf16_input = bf16_input;
  s.rows = rows ? rows : 1;
  s.stride = align_up(sampler_required_bytes(vocabulary), 256);
  cudaError_t e = cudaMalloc(&s.arena, s.stride * s.rows);
  if (e != cudaSuccess) return e;
  e = cudaMemset(s.arena, 0, s.stride * s.rows);
  const Layout L = layout(s.arena, vocabulary);
  s.state = L.state;
  s.result = L.result;
  s.stop_mask = L.stop_mask;
  return e;
}

void sampler_free(Sampler& s) {
  if (s.arena) cudaFree(s.arena);
  s.arena = nullptr;
}

cudaError_t sampler_start(Sampler& s, const dl_sampling& settings, uint64_t seed, const uint32_t* stop_ids,
                          size_t n_stop, cudaStream_t stream) {
  std::vector<unsigned char> mask(s.vocabulary, 0);
  for (size_t i = 0; i < n_stop; ++i) mask[stop_ids[i]] = 1;
  cudaError_t e = cudaSuccess;
  for (unsigned r = 0; r < s.rows && e == cudaSuccess; ++r)
    e = cudaMemcpyAsync(s.stop_mask + r * s.stride, mask.data(), mask.size(), cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return e;
  seed_kernel<<<dim3(1, s.rows), 1, 0, stream>>>(s.state, seed, s.stride, s.engine);
  s.settings = settings;
  s.started = true;
  return cudaGetLastError();
}

cudaError_t sampler_submit(Sampler& s, const void* row, const dl_sampling& st, uint64_t bits, bool owned,
                           cudaStream_t stream, size_t row_stride) {
  const Layout L = layout(s.arena, s.vocabulary);
  const unsigned n = unsigned(s.vocabulary), blocks = (n + kW - 1) / kW, R = s.rows;
  const size_t S = s.stride, row_bytes = row_stride * (s.bf16_input ? 2 : 4);
  clear_results_kernel<<<(R + 255) / 256, 256, 0, stream>>>(L.result, S, R);
  const bool greedy = st.mode == 0;
  if (owned) next_random_kernel<<<dim3(1, R), 1, 0, stream>>>(L.state, greedy, S);
  if (greedy) {
    greedy_kernel<<<dim3(blocks, R), kW, 0, stream>>>(row, s.bf16_input, n, L.best, L.scan, L.result, S, row_bytes);
  } else {
    keys_kernel<<<dim3(blocks, R), kW, 0, stream>>>(row, s.bf16_input, n, L.keys_a, L.result, S, row_bytes);
    uint2* in = L.keys_a;
    uint2* out = L.keys_b;
    const unsigned radix_blocks = (n + kRadixBlock - 1) / kRadixBlock;
    for (unsigned shift = s.bf16_input ? 16 : 0; shift < 32; shift += 8) {
      histogram_kernel<<<dim3(radix_blocks, R), kW, 0, stream>>>(in, n, shift, L.counts, S);
      digit_offsets_kernel<<<dim3(kW / 32, R), 32 * kOffsetWarps, 0, stream>>>(L.counts, L.digit_totals,
                                                                                 radix_blocks, S);
      scatter_kernel<<<dim3(radix_blocks, R), kW, 0, stream>>>(in, out, n, shift, L.counts, L.digit_totals, S);
      uint2* t = in;
      in = out;
      out = t;
    }
    const unsigned keep = st.top_k ? unsigned(st.top_k) : n;
    const unsigned kept_tiles = (keep + kW - 1) / kW, kept_blocks = (keep + kRadixBlock - 1) / kRadixBlock;
    weights_kernel<<<dim3(kept_blocks, R), kW, 0, stream>>>(row, s.bf16_input, in, keep, st.temperature, L.prefix,
                                                            L.tile_totals, S, row_bytes);
    scan_tiles_kernel<<<dim3(1, R), kW, kept_tiles * sizeof(double), stream>>>(L.tile_totals, keep, L.scan, L.result,
                                                                                S);
    cutoff_kernel<<<dim3(kept_blocks, R), kW, 0, stream>>>(L.prefix, L.tile_totals, keep, st.top_p, L.scan, S);
    const double draw = static_cast<double>(bits >> 11) * 0x1.0p-53;
    select_kernel<<<dim3(kept_blocks, R), kW, 0, stream>>>(L.prefix, L.tile_totals, keep, draw,
                                                           owned ? L.state : nullptr, L.scan, S);
    finish_kernel<<<dim3(1, R), 1, 0, stream>>>(in, L.scan, L.result, S);
  }
  if (owned) commit_kernel<<<dim3(1, R), 1, 0, stream>>>(L.state, L.result, L.stop_mask, S);
  return cudaGetLastError();
}

int sampler_launch_count(const Sampler& s, const dl_sampling& st, bool owned) {
  const int radix_passes = s.bf16_input ? 2 : 4;
  const int body = st.mode == 0 ? 1 : 1 + 3 * radix_passes + 5;
  return 1 + body + (owned ? 2 : 0);  // the result clear, the selection, the draw and commit
}

unsigned* sampler_result(const Sampler& s, unsigned row) {
  return reinterpret_cast<unsigned*>(reinterpret_cast<unsigned char*>(s.result) + row * s.stride);
}

cudaError_t sampler_feed(Sampler& s, unsigned* history, int* step, const bf16* embed, bf16* residual, int width,
                         long long* position, cudaStream_t stream, size_t history_stride) {
  feed_kernel<<<dim3(1, s.rows), 256, 0, stream>>>(s.result, history, step, embed, residual, width, position,
                                                   s.stride, history_stride);
  return cudaGetLastError();
}

}  // namespace dl
