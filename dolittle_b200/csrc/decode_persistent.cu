// Persistent decode step kernel (see decode_persistent.h).
#include <algorithm>
#include <cmath>

#include "decode_persistent.h"
#include "gemv_device.cuh"
#include "launch.h"

namespace dl {
namespace {

using namespace gemv_dev;

constexpr int kConsumerWarps = kGemvConsumers / 32;
constexpr long long kSpinLimit = 1ll << 32;  // ~2 s of SM cycles
constexpr int kMaxInput8 = kPersistMaxInput / 8 / kGemvConsumers;  // 16-byte input loads per thread
constexpr int kMaxNorm8 = kPersistMaxNormInput / 8 / kGemvConsumers;
// Normed prologue: x row + norm weight (BF16) and the RMS law's 128 partials.
static_assert(4 * kPersistMaxNormInput + 128 * 4 <= kPersistUnionBytes, "prologue scratch");
// Score unit scratch: qs, ks, norm_vals (FP32), the raw q / k rows and the
// q / k norm weights (BF16).
constexpr int kScoreScratch = (8 * 128 + 128 + 8 * 128) * 4 + 8 * 128 * 2 + 2 * 128 * 2;

// Position of feature f of a 128-wide query row in the score unit's layout:
// lane l of the 8-lane dot product owns features 16l .. 16l+15 and reads them
// as four float4 at [k][l][4] (k = 0..3), so the 8 lanes of one key read 128
// contiguous bytes per load (no bank conflicts).
__device__ __forceinline__ int q_slot(int f) { return ((f & 15) >> 2) * 32 + (f >> 4) * 4 + (f & 3); }

// RMSNorm apply (two rounding points, normalization.cu:82-186) on 8 packed
// BF16 features.
__device__ __forceinline__ uint32_t norm_pair(uint32_t x2, uint32_t w2, float inv) {
  const bf16 lo = narrow(__fmul_rn(round_bf16(__fmul_rn(bf_lo(x2), inv)), bf_lo(w2)));
  const bf16 hi = narrow(__fmul_rn(round_bf16(__fmul_rn(bf_hi(x2), inv)), bf_hi(w2)));
  return uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
}
__device__ __forceinline__ uint4 normalize8(const uint4& x, const uint4& w, float inv) {
  return make_uint4(norm_pair(x.x, w.x, inv), norm_pair(x.y, w.y, inv), norm_pair(x.z, w.z, inv),
                    norm_pair(x.w, w.w, inv));
}

struct PHeader {
  uint64_t full[kPersistSlots];
  uint64_t empty[kPersistSlots];
  uint4 cta_best[kConsumerWarps];
  float wmax[8];
  float max_s[8];
  float den_s[8];
  float sums[8];
  float row_inv;
  float beta;
  unsigned invalid;
  unsigned abort_flag;     // any consumer warp gave up: stop issuing, unwind
  unsigned producer_done;
  unsigned issued;         // stages issued by the producer
  unsigned last_cta;
  unsigned chosen;
  unsigned sync_ok;
  unsigned pf_req;         // consumer-requested L2 prefetch bursts
  alignas(16) unsigned char desc[2][256];  // phase descriptors, fetched one phase ahead
  alignas(16) const bf16* attn[2][4];      // per block: q_norm, k_norm, k_cache, v_cache
  float rope[64][2];                       // RoPE cos, sin (storage-rounded) at this step's position
};
static_assert(sizeof(PHeader) <= kPersistHeaderBytes, "persistent header too large");
static_assert(sizeof(PGemv) <= 256 && sizeof(PGemv) % 16 == 0, "phase descriptor size");
static_assert(offsetof(PLayer, q_norm) % 16 == 0 && offsetof(PLayer, v_cache) == offsetof(PLayer, q_norm) + 24,
              "attention operands are copied as 32 contiguous bytes");

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ unsigned vload(const unsigned* p) { return *reinterpret_cast<const volatile unsigned*>(p); }
__device__ __forceinline__ void vstore(unsigned* p, unsigned v) { *reinterpret_cast<volatile unsigned*>(p) = v; }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier among the consumer threads of every CTA (all CTAs are
// co-resident: cooperative launch).  The CTA's writes are ordered before
// thread 0's release-add by the CTA barrier, and the acquire load that sees
// every arrival orders the other CTAs' writes before this CTA's later reads.
// (Publishing a generation flag from the last arrival instead measured
// slower here.)  The arrival counter only grows inside a launch; the last
// CTA to leave resets it.  Bounded: returns false when the other CTAs do not
// arrive within ~2 s, or when this CTA already aborted.
__device__ bool grid_sync(unsigned* counter, unsigned target, PHeader* h) {
  named_sync(1, kGemvConsumers);
  if (threadIdx.x == 0) {
    unsigned ok = vload(&h->abort_flag) ? 0u : 1u;
    if (ok) {
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
      if (ld_acquire(counter) < target) {
        const long long start = clock64();
        while (ld_acquire(counter) < target) {
          if (clock64() - start > kSpinLimit) {
            ok = 0;
            break;
          }
        }
      }
    }
    h->sync_ok = ok;
  }
  named_sync(1, kGemvConsumers);
  return h->sync_ok != 0;
}

// ---------------------------------------------------------------------------
// Producer (one lane): every projection phase's rows of this CTA, in the
// consumers' order, through the ring.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int find_segment(const PGemv& ph) {
  const int b = blockIdx.x;
  for (int i = 0; i < ph.nseg; ++i)
    if (b >= ph.seg[i].cta_begin && b < ph.seg[i].cta_begin + ph.seg[i].cta_count) return i;
  return -1;
}

// One stage = one 3D box {64 features, tile rows, feature blocks} at row y,
// feature block z (see encode_weight_map3d).
__device__ __forceinline__ void tma_load_stage(void* dst, const CUtensorMap* map, int y, int z, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_stage(const CUtensorMap* map, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(0), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ const PGemv& phase_ref(const PersistArgs& a, int l, int p) {
  if (l >= a.nlayers) return a.head;
  const PLayer& L = a.layers[l];
  return p == 0 ? L.qkv : p == 1 ? L.o : p == 2 ? L.gu : L.down;
}

// Position in this CTA's stage sequence: projection phase (block l,
// projection p; l == nlayers is the vocabulary head), tile t, k-step ks.
// Phases in which this CTA owns no rows are skipped, exactly as the
// consumers skip them.
struct Cursor {
  int l, p, t, ks;
  const CUtensorMap* map;
  int r0, tile_rows, ntiles, nk, nbox;
  bool valid;
};

__device__ __forceinline__ void cursor_seek(const PersistArgs& a, Cursor& c) {
  for (;;) {
    const PGemv& ph = phase_ref(a, c.l, c.p);
    const int si = find_segment(ph);
    if (si >= 0) {
      const PSeg& sg = ph.seg[si];
      const int local = blockIdx.x - sg.cta_begin;
      const int r0 = min(sg.rows, local * sg.rows_per_cta), r1 = min(sg.rows, r0 + sg.rows_per_cta);
      if (r1 > r0) {
        c.map = sg.map;
        c.r0 = r0;
        c.tile_rows = sg.tile_rows;
        c.ntiles = (r1 - r0 + sg.tile_rows - 1) / sg.tile_rows;
        c.nk = ph.in_width / sg.kc;
        c.nbox = sg.kc / kGemvBox;
        c.t = 0;
        c.ks = 0;
        c.valid = true;
        return;
      }
    }
    if (c.l >= a.nlayers) {
      c.valid = false;
      return;
    }
    if (++c.p == 4) {
      c.p = 0;
      ++c.l;
    }
  }
}

__device__ __forceinline__ void cursor_next(const PersistArgs& a, Cursor& c) {
  if (++c.ks < c.nk) return;
  c.ks = 0;
  if (++c.t < c.ntiles) return;
  if (c.l >= a.nlayers) {
    c.valid = false;
    return;
  }
  if (++c.p == 4) {
    c.p = 0;
    ++c.l;
  }
  cursor_seek(a, c);
}

// Two cursors over the same stage sequence.  The load cursor fills the
// shared-memory ring as slots free up.  The prefetch cursor serves bursts the
// consumers request when they enter a long stall (attention): while the
// producer waits for a free slot it pulls the next prefetch_stages stages past
// the load cursor into L2 with TMA prefetches, so HBM streams through the
// stall and the ring later refills from L2.
__device__ __forceinline__ void producer_main(const PersistArgs& a, unsigned char* ring, PHeader* h) {
  const uint64_t policy = evict_first_policy();
  Cursor ld{}, pf{};
  cursor_seek(a, ld);
  pf = ld;
  unsigned g = 0, pfc = 0, pf_seen = 0, burst_end = 0;
  bool ok = true;
  while (ld.valid && ok) {
    const int st = g % kPersistSlots;
    if (g >= kPersistSlots) {
      const unsigned parity = ((g / kPersistSlots) - 1) & 1;
      if (!mbar_try_wait(&h->empty[st], parity)) {
        const long long start = clock64();
        for (;;) {
          // Non-blocking test: the loop must stay awake to serve bursts.
          if (mbar_test_wait(&h->empty[st], parity)) break;
          const unsigned req = vload(&h->pf_req);
          if (req != pf_seen) {
            // A burst starts at the load cursor (the prefetch cursor jumps
            // there instead of walking the stages already loaded).
            pf_seen = req;
            pf = ld;
            pfc = g;
            burst_end = g + unsigned(a.prefetch_stages);
          }
          if (pf.valid && pfc < burst_end) {
            if (pfc >= g) tma_prefetch_stage(pf.map, pf.r0 + pf.t * pf.tile_rows, pf.ks * pf.nbox);
            cursor_next(a, pf);
            ++pfc;
            continue;
          }
          if (vload(&h->abort_flag) || clock64() - start > kSpinLimit) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
    }
    unsigned char* dst = ring + st * kPersistSlotBytes;
    const int tr0 = ld.r0 + ld.t * ld.tile_rows;
    mbar_arrive_expect_tx(&h->full[st], unsigned(ld.nbox) * ld.tile_rows * 128u);
    tma_load_stage(dst, ld.map, tr0, ld.ks * ld.nbox, &h->full[st], policy);
    ++g;
    vstore(&h->issued, g);
    cursor_next(a, ld);
  }
  vstore(&h->producer_done, 1u);
}

// ---------------------------------------------------------------------------
// Consumers: projection phases.
// ---------------------------------------------------------------------------
struct Best {
  float v = -INFINITY;
  unsigned id = 0xffffffffu, flags = 0;
};

// P = 16 law with 4 partials per thread (4 threads per row, 8 rows per warp:
// lane = 8 q + row offset): twice the warps of the 8-partial layout, which
// matters when a CTA owns only a few dozen rows.  Thread q holds partials
// 4q..4q+3 = features 16 m + 4 q + i; its 8-byte reads of a half-warp cover 8
// lines x 2 halves of one 16-byte chunk, conflict-free under the swizzle.
template <int KC>
__device__ __forceinline__ void stage_dense_q16(const unsigned char* stage, int tile_rows, int row, int q,
                                                const bf16* xs, int k0, float (&acc)[4]) {
#pragma unroll 4  // full unrolling of every instantiation overflows the instruction cache
  for (int m = 0; m < KC / 16; ++m) {
    const int b = (16 * m) >> 6;
    const int c = (((16 * m) & 63) >> 3) + (q >> 1);
    const int line = b * tile_rows + row;
    const uint2 w = sld8(stage + line * 128 + ((c ^ (line & 7)) << 4) + ((q & 1) << 3));
    const uint2 x = sld8(xs + k0 + 16 * m + 4 * q);
    fma_pair(acc[0], acc[1], x.x, w.x);
    fma_pair(acc[2], acc[3], x.y, w.y);
  }
}

// Halving tree of the P = 16 partials in the 4-partial layout: +8 (q, q^2),
// +4 (q, q^1), then +2 and +1 inside the thread.
__device__ __forceinline__ float reduce_q16(float (&acc)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 16));
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __shfl_xor_sync(0xffffffffu, acc[i], 8));
  acc[0] = __fadd_rn(acc[0], acc[2]);
  acc[1] = __fadd_rn(acc[1], acc[3]);
  return __fadd_rn(acc[0], acc[1]);
}

// Rows of one projection phase.  Q16 selects the 4-partial layout (P = 16
// only); otherwise the 8-partial layout of gemv_device.cuh.
template <int P, int KC, bool Q16>
__device__ void consume_rows(const PersistArgs& a, const PGemv& ph, const PSeg& sg, int r0, int r1,
                             const unsigned char* ring, PHeader* h, const bf16* xs, unsigned& g, bool& failed,
                             bf16* capture, Best& best) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = Q16 ? lane >> 3 : Layout<P>::slot(lane);
  const int my_row = Q16 ? warp * 8 + (lane & 7) : Layout<P>::row(warp, lane);
  const int I = ph.in_width;
  const int nk = I / KC;
  const int tile_rows = sg.tile_rows;
  const int ntiles = (r1 - r0 + tile_rows - 1) / tile_rows;
  const int epilogue = ph.epilogue;
  bf16* out = sg.out + (sg.out_row ? size_t(__ldcg(sg.out_row)) * sg.out_stride : 0);
  for (int t = 0; t < ntiles; ++t) {
    const int tr0 = r0 + t * tile_rows;
    const int trows = min(tile_rows, r1 - tr0);
    const bool active = my_row < trows;
    const int row = tr0 + my_row;
    // The residual value this thread will update, fetched before the stages.
    bf16 old = narrow(0.0f);
    if (epilogue == kEpilogueResidual && active && slot == 0) old = __ldcg(out + row);
    float acc[1][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[0][i] = 0.0f;
    for (int ks = 0; ks < nk; ++ks, ++g) {
      const int st = g % kPersistSlots;
      if (!failed && !mbar_wait(&h->full[st], (g / kPersistSlots) & 1)) {
        failed = true;
        vstore(&h->abort_flag, 1u);
        record_error(a.err, kErrWaitFull);
      }
      if (active && !failed) {
        if constexpr (Q16) {
          float(&a4)[4] = *reinterpret_cast<float(*)[4]>(&acc[0][0]);
          stage_dense_q16<KC>(ring + st * kPersistSlotBytes, tile_rows, my_row, slot, xs, ks * KC, a4);
        } else {
          stage_dense<1, P, KC>(ring + st * kPersistSlotBytes, tile_rows, my_row, slot, xs, I, ks * KC, acc);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&h->empty[st]);
    }
    float y;
    if constexpr (Q16) {
      float(&a4)[4] = *reinterpret_cast<float(*)[4]>(&acc[0][0]);
      y = reduce_q16(a4);
    } else {
      y = reduce_partials<P>(acc[0]);
    }
    if (epilogue == kEpilogueSwiGLU) {
      // Even row = gate o, odd row = up o; both rounded to storage first.
      const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
      if (active && slot == 0 && !failed && !(row & 1))
        out[row >> 1] = narrow(swiglu(round_bf16(y), round_bf16(partner)));
      continue;
    }
    if (!active || slot != 0 || failed) continue;
    const bf16 yb = narrow(y);
    if (epilogue == kEpilogueResidual) {
      const bf16 nv = narrow(__fadd_rn(widen(old), widen(yb)));
      out[row] = nv;
      if (capture) capture[row] = nv;
    } else {
      out[row] = yb;
      if (epilogue == kEpilogueArgmax) {
        const float v = widen(yb);
        if (isnan(v) || v == INFINITY) best.flags |= 1u;
        if (better(v, static_cast<unsigned>(row), best.v, best.id)) {
          best.v = v;
          best.id = static_cast<unsigned>(row);
        }
      }
    }
  }
}

// One projection phase: stage (and normalize) the input row, then this CTA's
// rows.  CTAs without rows in the phase only take part in the barrier.
__device__ void gemv_phase(const PersistArgs& a, const PGemv& ph, unsigned char* uni, const unsigned char* ring,
                           PHeader* h, unsigned& g, bool& failed, bf16* capture, Best& best) {
  const int si = find_segment(ph);
  if (si < 0) return;
  const PSeg& sg = ph.seg[si];
  const int local = blockIdx.x - sg.cta_begin;
  const int r0 = min(sg.rows, local * sg.rows_per_cta), r1 = min(sg.rows, r0 + sg.rows_per_cta);
  if (r1 <= r0) return;
  // Input row (and RMSNorm weight) by asynchronous 16-byte copies, all in
  // flight at once (L2 only: the row was written by other CTAs).
  const int I = ph.in_width;
  const uint4* xg = reinterpret_cast<const uint4*>(ph.x);
  const uint4* wg = reinterpret_cast<const uint4*>(ph.norm_w);
  const int n8 = I / 8;
  bf16* xs = reinterpret_cast<bf16*>(uni);
  uint4* xs4 = reinterpret_cast<uint4*>(uni);
  uint4* ws4 = xs4 + n8;  // norm weight (normed inputs are at most 4096 wide)
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < kMaxInput8; ++i) {
    const int q = threadIdx.x + i * kGemvConsumers;
    if (q < n8) cp_async16(xs4 + q, xg + q);
  }
  if (wg) {
#pragma unroll
    for (int i = 0; i < kMaxNorm8; ++i) {
      const int q = threadIdx.x + i * kGemvConsumers;
      if (q < n8) cp_async16(ws4 + q, wg + q);
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
  named_sync(1, kGemvConsumers);
  if (wg) {
    // The RMS law's partial c of lane L is the serial sum of squares of
    // x[4L + c + 128k], k = 0, 1, ...: 128 independent chains, one per
    // thread here (thread 4L + c reads x[t + 128k]).  Lane L of warp 0 then
    // adds its four partials in order and the shuffle-down tree finishes,
    // exactly as rms_inverse_smem does in one warp.
    float* parts = reinterpret_cast<float*>(uni + 4 * kPersistMaxNormInput);
    if (threadIdx.x < 128) {
      float p = 0.f;
#pragma unroll 8
      for (int col = threadIdx.x; col < I; col += 128) {
        const float v = widen(xs[col]);
        p = __fadd_rn(p, __fmul_rn(v, v));
      }
      parts[threadIdx.x] = p;
    }
    named_sync(1, kGemvConsumers);
    if (warp == 0) {
      const int lane = threadIdx.x & 31;
      float sum = __fadd_rn(__fadd_rn(__fadd_rn(parts[4 * lane], parts[4 * lane + 1]), parts[4 * lane + 2]),
                            parts[4 * lane + 3]);
      sum = shuffle_down_tree32(sum);
      const float total = __shfl_sync(0xffffffffu, sum, 0);
      const float inv = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / static_cast<float>(I)), a.eps));
      if (lane == 0) h->row_inv = inv;
    }
    named_sync(1, kGemvConsumers);
    const float inv = h->row_inv;
#pragma unroll
    for (int i = 0; i < kMaxNorm8; ++i) {
      const int q = threadIdx.x + i * kGemvConsumers;
      if (q < n8) xs4[q] = normalize8(xs4[q], ws4[q], inv);
    }
    named_sync(1, kGemvConsumers);
  }
  const bool p16 = sg.partials == 16;
  switch (sg.kc) {
#define DL_PERSIST_KC(K)                                                                         \
  case K:                                                                                        \
    if (p16)                                                                                     \
      consume_rows<16, K, true>(a, ph, sg, r0, r1, ring, h, xs, g, failed, capture, best);       \
    else                                                                                         \
      consume_rows<32, K, false>(a, ph, sg, r0, r1, ring, h, xs, g, failed, capture, best);      \
    break;
    DL_PERSIST_KC(64)
    DL_PERSIST_KC(128)
    DL_PERSIST_KC(256)
    DL_PERSIST_KC(512)
#undef DL_PERSIST_KC
    default:
      break;
  }
  // xs is rewritten by the next phase.
  named_sync(1, kGemvConsumers);
}

// ---------------------------------------------------------------------------
// Consumers: attention phases (same laws as attention_decode.cu).
// ---------------------------------------------------------------------------
// Scores of one (GQA group g, key slice) unit: QK-norm + RoPE of the group's
// query heads (warps 0..group-1) and the new key (warp 7), the new key into
// the K cache by the slice that holds it, then the scaled scores.
__device__ void score_unit(const PersistArgs& a, const bf16* const* ap, int g, int slice, int S, unsigned char* uni,
                           const PHeader* h) {
  float(*qs)[128] = reinterpret_cast<float(*)[128]>(uni);
  float* ks = reinterpret_cast<float*>(uni + 8 * 128 * 4);
  float(*norm_vals)[128] = reinterpret_cast<float(*)[128]>(uni + 8 * 128 * 4 + 128 * 4);
  bf16* raw = reinterpret_cast<bf16*>(uni + (8 * 128 + 128 + 8 * 128) * 4);  // [8][128]: q heads, key in row 7
  bf16* wnorm = raw + 8 * 128;                                                // [2][128]: q_norm, k_norm
  const bf16* q_norm = ap[0];
  const bf16* k_norm = ap[1];
  bf16* k_cache = const_cast<bf16*>(ap[2]);
  const int width = a.width, kv_heads = a.kv_heads, group = a.query_heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = S + 1;
  const int per = (count + a.score_slices - 1) / a.score_slices;
  const int j0 = slice * per, j1 = min(count, j0 + per);
  const bool owns_new_key = S >= j0 && S < j1;
  // One round of asynchronous copies: the group's raw q rows, the raw key and
  // the slice's cached keys (the new key S comes from ks).
  bf16* kslice = reinterpret_cast<bf16*>(uni + kScoreScratch);
  const int nkeys = max(0, j1 - j0);
  const bool staged = width % 8 == 0 && nkeys * width * 2 <= kPersistUnionBytes - kScoreScratch;
  const int chunks = width / 8;
  const bool raw_staged = width % 8 == 0;
  if (raw_staged) {
    for (int idx = threadIdx.x; idx < (group + 1) * chunks; idx += kGemvConsumers) {
      const int r = idx / chunks, q = idx % chunks;
      const bf16* src = r < group ? a.q_raw + size_t(g * group + r) * width : a.k_raw + size_t(g) * width;
      cp_async16(raw + (r < group ? r : 7) * 128 + 8 * q, src + 8 * q);
    }
    for (int idx = threadIdx.x; idx < 2 * chunks; idx += kGemvConsumers) {
      const int r = idx / chunks, q = idx % chunks;
      cp_async16(wnorm + r * 128 + 8 * q, (r == 0 ? q_norm : k_norm) + 8 * q);
    }
  }
  if (staged) {
    for (int idx = threadIdx.x; idx < nkeys * chunks; idx += kGemvConsumers) {
      const int j = idx / chunks, q = idx % chunks;
      if (j0 + j != S)
        cp_async16(kslice + size_t(j) * width + 8 * q, k_cache + (size_t(j0 + j) * kv_heads + g) * width + 8 * q);
    }
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
  // The PV phase reads every group's V rows of this key slice: pull them
  // into L2 now (one bulk prefetch of the contiguous rows j0 .. j1-1).
  if (threadIdx.x == 0 && g == 0 && nkeys > 0) {
    const bf16* v0 = ap[3] + size_t(j0) * kv_heads * width;
    const unsigned bytes = unsigned(nkeys) * kv_heads * width * 2;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(v0), "r"(bytes) : "memory");
  }
  named_sync(1, kGemvConsumers);
  if (warp < group || warp == 7) {
    const bool is_q = warp < group;
    const bf16* src = raw_staged ? raw + warp * 128
                                 : (is_q ? a.q_raw + size_t(g * group + warp) * width : a.k_raw + size_t(g) * width);
    const bf16* w = raw_staged ? wnorm + (is_q ? 0 : 128) : (is_q ? q_norm : k_norm);
    float x[4], part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = lane + 32 * c;
      x[c] = col < width ? widen(raw_staged ? src[col] : __ldcg(src + col)) : 0.f;
      if (col < width) part[c] = __fmul_rn(x[c], x[c]);
    }
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
    sum = shuffle_down_tree32(sum);
    const float total = __shfl_sync(0xffffffffu, sum, 0);
    const float inv = rsqrtf(__fadd_rn(__fmul_rn(total, 1.0f / static_cast<float>(width)), a.eps));
    float* nv = norm_vals[warp];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = lane + 32 * c;
      if (col < width) nv[col] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(x[c], inv)), widen(w[col])));
    }
    __syncwarp();
    const int half = width / 2;
    float* dst = is_q ? qs[warp] : ks;
    const bool permute = is_q && width == 128;
    for (int f = lane; f < half; f += 32) {
      const float co = h->rope[f][0], si = h->rope[f][1];
      const float va = nv[f], vb = nv[f + half];
      const float lo = round_bf16(__fsub_rn(round_bf16(__fmul_rn(va, co)), round_bf16(__fmul_rn(vb, si))));
      const float hi = round_bf16(__fadd_rn(round_bf16(__fmul_rn(vb, co)), round_bf16(__fmul_rn(va, si))));
      dst[permute ? q_slot(f) : f] = lo;
      dst[permute ? q_slot(f + half) : f + half] = hi;
      if (!is_q && owns_new_key) {
        bf16* kc = k_cache + (size_t(S) * kv_heads + g) * width;
        kc[f] = narrow(lo);
        kc[f + half] = narrow(hi);
      }
    }
  }
  named_sync(1, kGemvConsumers);
  const int lane8 = threadIdx.x & 7;
  const int span = width / 8 + (width % 8 != 0);
  const int begin = lane8 * span, end = min(begin + span, width);
  for (int base = j0; base < j1; base += kGemvConsumers / 8) {
    const int j = base + (threadIdx.x >> 3);
    const bool live = j < j1;
    float part[8];
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) part[hh] = 0.f;
    if (live && width == 128) {
      float kv[16];
      if (j == S) {
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = ks[begin + i];
      } else {
        uint4 w0, w1;
        if (staged) {
          const bf16* kr = kslice + size_t(j - j0) * width + begin;
          w0 = sld16(kr);
          w1 = sld16(kr + 8);
        } else {
          const uint4* kr = reinterpret_cast<const uint4*>(k_cache + (size_t(j) * kv_heads + g) * width + begin);
          w0 = __ldcg(kr);
          w1 = __ldcg(kr + 1);
        }
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 16; ++i) kv[i] = (i & 1) ? bf_hi(words[i >> 1]) : bf_lo(words[i >> 1]);
      }
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) {
        if (hh < group) {
          const float4* q4 = reinterpret_cast<const float4*>(qs[hh]) + lane8;
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 qv = q4[8 * k];
            acc = __fmaf_rn(qv.x, kv[4 * k], acc);
            acc = __fmaf_rn(qv.y, kv[4 * k + 1], acc);
            acc = __fmaf_rn(qv.z, kv[4 * k + 2], acc);
            acc = __fmaf_rn(qv.w, kv[4 * k + 3], acc);
          }
          part[hh] = acc;
        }
      }
    } else if (live) {
      const bf16* kr = k_cache + (size_t(j) * kv_heads + g) * width;
      const bf16* kl = kslice + size_t(j - j0) * width;
      for (int hh = 0; hh < group; ++hh) {
        float acc = 0.f;
        for (int f = begin; f < end; ++f)
          acc = __fmaf_rn(qs[hh][f], j == S ? ks[f] : widen(staged ? kl[f] : __ldcg(kr + f)), acc);
        part[hh] = acc;
      }
    }
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) {
      if (hh < group) {
        float v = part[hh];
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        part[hh] = v;
      }
    }
    if (live && lane8 == 0)
      for (int hh = 0; hh < group; ++hh)
        a.scores[size_t(g * group + hh) * a.score_stride + j] = __fmul_rn(part[hh], a.scale);
  }
  named_sync(1, kGemvConsumers);
}

// PV of one (GQA group g, feature slice [f0, f0+fpc)) unit.  Softmax law per
// query head: exact max, den = 32 strided serial partials of
// e = expf(s - max) + the shuffle-down tree, p = e / den.  The two
// contiguous key halves are serial chains per feature, added once.  Keys are
// staged in chunks (V slice and p) so any capacity fits the scratch.
__device__ void pv_unit(const PersistArgs& a, const bf16* const* ap, int g, int f0, int S, unsigned char* uni,
                        PHeader* h) {
  const int width = a.width, kv_heads = a.kv_heads, group = a.query_heads / kv_heads;
  const int fpc = a.pv_features;
  const int count = S + 1;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float* red = reinterpret_cast<float*>(uni);
  unsigned char* area = uni + kGemvConsumers * 4;
  const int area_bytes = kPersistUnionBytes - kGemvConsumers * 4 - 16;
  const int hq = warp >> 1, t64 = t & 63;
  const int half = t / (group * fpc);
  const int hh = (t / fpc) % group;
  const int fl = t % fpc;
  const int split = (count - 1) / 2 + 1;
  const bool live = half < 2;
  const int jb = half == 0 ? 0 : split, je = half == 0 ? split : count;
  const int vchunks = fpc / 8;
  const int c4 = (count + 3) & ~3;
  if (group * c4 * 4 + count * fpc * 2 <= area_bytes) {
    // Whole sequence in shared memory: the group's score rows and the V
    // slice arrive in one round of asynchronous copies, then max, den and
    // p = e / den run on shared memory and the chains read it.
    float* ss = reinterpret_cast<float*>(area);  // [group][c4]
    bf16* vs = reinterpret_cast<bf16*>(area + size_t(group) * c4 * 4);
    const int q4 = c4 / 4;
    for (int idx = t; idx < group * q4; idx += kGemvConsumers) {
      const int hx = idx / q4, q = idx % q4;
      cp_async16(ss + size_t(hx) * c4 + 4 * q, a.scores + size_t(g * group + hx) * a.score_stride + 4 * q);
    }
    for (int idx = t; idx < count * vchunks; idx += kGemvConsumers) {
      const int j = idx / vchunks, q = idx % vchunks;
      cp_async16(vs + size_t(j) * fpc + 8 * q, ap[3] + (size_t(j) * kv_heads + g) * width + f0 + 8 * q);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
    named_sync(1, kGemvConsumers);
    if (hq < group) {
      float* srow = ss + size_t(hq) * c4;
      float m = -INFINITY;
#pragma unroll 4
      for (int j = t64; j < count; j += 64) m = fmaxf(m, srow[j]);
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (lane == 0) h->wmax[warp] = m;
      named_sync(2 + hq, 64);
      const float maximum = fmaxf(h->wmax[2 * hq], h->wmax[2 * hq + 1]);
      // e = expf(s - max) once, by both warps; then the 32 strided serial
      // partials of the den law over the stored e; then p = e / den.
#pragma unroll 4
      for (int j = t64; j < count; j += 64) srow[j] = expf(srow[j] - maximum);
      named_sync(2 + hq, 64);
      if (warp == 2 * hq) {
        float acc = 0.f;
#pragma unroll 8
        for (int j = lane; j < count; j += 32) acc = __fadd_rn(acc, srow[j]);
#pragma unroll
        for (int off = 16; off; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
        if (lane == 0) h->den_s[hq] = acc;
      }
      named_sync(2 + hq, 64);
      const float den = h->den_s[hq];
#pragma unroll 4
      for (int j = t64; j < count; j += 64) srow[j] = srow[j] / den;
    }
    named_sync(1, kGemvConsumers);
    float acc = 0.f;
    if (live) {
      // Serial chain over this half's keys: p four keys at a time (one
      // aligned float4), unrolled so the loads run ahead of the FMAs.
      const float* ph = ss + size_t(hh) * c4;
      const bf16* col = vs + fl;
      int j = jb;
      for (; j < je && (j & 3); ++j) acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
      if (fpc == 8) {
#pragma unroll 4
        for (; j + 4 <= je; j += 4) {
          const float4 p4 = *reinterpret_cast<const float4*>(ph + j);
          acc = __fmaf_rn(p4.x, widen(col[8 * j]), acc);
          acc = __fmaf_rn(p4.y, widen(col[8 * j + 8]), acc);
          acc = __fmaf_rn(p4.z, widen(col[8 * j + 16]), acc);
          acc = __fmaf_rn(p4.w, widen(col[8 * j + 24]), acc);
        }
      }
      for (; j < je; ++j) acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
    }
    red[t] = acc;
    named_sync(1, kGemvConsumers);
    if (live && half == 0) {
      const float second = red[t + group * fpc];
      a.att[size_t(g * group + hh) * width + f0 + fl] = narrow(__fadd_rn(acc, second));
    }
    named_sync(1, kGemvConsumers);
    return;
  }
  const int chunk = (area_bytes / (2 * fpc + 4 * group)) / 8 * 8;
  bf16* vs = reinterpret_cast<bf16*>(area);
  float* p = reinterpret_cast<float*>(area + (size_t(chunk) * fpc * 2 + 15) / 16 * 16);
  // 1. max and den per query head: warps 2h and 2h+1.
  if (hq < group) {
    const float* srow = a.scores + size_t(g * group + hq) * a.score_stride;
    float m = -INFINITY;
    for (int j = t64; j < count; j += 64) m = fmaxf(m, __ldcg(srow + j));
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) h->wmax[warp] = m;
    named_sync(2 + hq, 64);
    const float maximum = fmaxf(h->wmax[2 * hq], h->wmax[2 * hq + 1]);
    if (warp == 2 * hq) {
      float acc = 0.f;
      for (int j = lane; j < count; j += 32) acc = __fadd_rn(acc, expf(__ldcg(srow + j) - maximum));
#pragma unroll
      for (int off = 16; off; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
      if (lane == 0) {
        h->den_s[hq] = acc;
        h->max_s[hq] = maximum;
      }
    }
  }
  named_sync(1, kGemvConsumers);
  // 2. Chunks of keys: stage V slice + p, then advance the chains.
  float acc = 0.f;
  for (int c0 = 0; c0 < count; c0 += chunk) {
    const int n = min(chunk, count - c0);
    for (int idx = t; idx < n * vchunks; idx += kGemvConsumers) {
      const int j = idx / vchunks, q = idx % vchunks;
      cp_async16(vs + size_t(j) * fpc + 8 * q, ap[3] + (size_t(c0 + j) * kv_heads + g) * width + f0 + 8 * q);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int idx = t; idx < group * n; idx += kGemvConsumers) {
      const int hx = idx / n, j = idx % n;
      const float s = __ldcg(a.scores + size_t(g * group + hx) * a.score_stride + c0 + j);
      p[size_t(hx) * chunk + j] = expf(s - h->max_s[hx]) / h->den_s[hx];
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    named_sync(1, kGemvConsumers);
    if (live) {
      const int lo = max(jb, c0), hi = min(je, c0 + n);
      const float* ph = p + size_t(hh) * chunk - c0;
      const bf16* col = vs + fl - size_t(c0) * fpc;
      int j = lo;
      for (; j + 4 <= hi; j += 4) {
        acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
        acc = __fmaf_rn(ph[j + 1], widen(col[size_t(j + 1) * fpc]), acc);
        acc = __fmaf_rn(ph[j + 2], widen(col[size_t(j + 2) * fpc]), acc);
        acc = __fmaf_rn(ph[j + 3], widen(col[size_t(j + 3) * fpc]), acc);
      }
      for (; j < hi; ++j) acc = __fmaf_rn(ph[j], widen(col[size_t(j) * fpc]), acc);
    }
    named_sync(1, kGemvConsumers);
  }
  red[t] = acc;
  named_sync(1, kGemvConsumers);
  if (live && half == 0) {
    const float second = red[t + group * fpc];
    a.att[size_t(g * group + hh) * width + f0 + fl] = narrow(__fadd_rn(acc, second));
  }
  named_sync(1, kGemvConsumers);
}

// One-shot steering edit of the selected row (src/kernels/cuda/steering.cu
// :106-159), by one CTA, then the block-output capture copy if requested.
__device__ void edit_phase(const PersistArgs& a, long long S, PHeader* h) {
  const int D = a.hidden;
  bf16* row = a.residual;
  if (a.edit_row == S) {
    unsigned* state = a.edit_state;
    if (threadIdx.x == 0) {
      h->invalid = (state[0] || state[1] != 0) ? 1u : 0u;
      ++state[1];
    }
    named_sync(1, kGemvConsumers);
    if (threadIdx.x < 8) {
      float s = 0.f;
      for (int i = threadIdx.x; i < D; i += 8) {
        const float v = widen(__ldcg(row + i));
        s = __fadd_rn(s, __fmul_rn(v, v));
      }
      h->sums[threadIdx.x] = s;
    }
    named_sync(1, kGemvConsumers);
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int i = 0; i < 8; ++i) s = __fadd_rn(s, h->sums[i]);
      h->beta = __fmul_rn(a.edit_strength, __fsqrt_rn(s));
      if (!isfinite(h->beta)) h->invalid = 1;
    }
    named_sync(1, kGemvConsumers);
    const bool valid = h->invalid == 0;
    named_sync(1, kGemvConsumers);
    if (valid) {
      const float beta = h->beta;
      for (int i = threadIdx.x; i < D; i += kGemvConsumers) {
        const float value = __fadd_rn(widen(__ldcg(row + i)), __fmul_rn(beta, a.edit_direction[i]));
        const bf16 stored = narrow(value);
        if (!isfinite(value) || !isfinite(widen(stored))) atomicOr(&h->invalid, 1u);
        row[i] = stored;
      }
    }
    named_sync(1, kGemvConsumers);
    if (threadIdx.x == 0) state[0] = h->invalid;
  }
  if (a.capture && a.capture_layer == a.edit_layer) {
    bf16* dst = a.capture + size_t(S) * D;
    for (int i = threadIdx.x; i < D; i += kGemvConsumers) dst[i] = __ldcg(row + i);
  }
  named_sync(1, kGemvConsumers);
}

// Greedy selection: per-CTA best -> partials; the last CTA reduces them,
// publishes {token, status}, records history / stop latch / position and
// writes the chosen token's embedding row as the next step's residual.
__device__ void head_select(const PersistArgs& a, PHeader* h, Best best) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best.v, off);
    const unsigned oid = __shfl_xor_sync(0xffffffffu, best.id, off);
    best.flags |= __shfl_xor_sync(0xffffffffu, best.flags, off);
    if (better(ov, oid, best.v, best.id)) {
      best.v = ov;
      best.id = oid;
    }
  }
  if (lane == 0) h->cta_best[warp] = make_uint4(__float_as_uint(best.v), best.id, best.flags, 0);
  named_sync(1, kGemvConsumers);
  if (threadIdx.x == 0) {
    uint4 b = h->cta_best[0];
    for (int w = 1; w < kConsumerWarps; ++w) {
      const uint4 c = h->cta_best[w];
      if (better(__uint_as_float(c.x), c.y, __uint_as_float(b.x), b.y)) {
        b.x = c.x;
        b.y = c.y;
      }
      b.z |= c.z;
    }
    a.partials[blockIdx.x] = b;
    __threadfence();
    h->last_cta = atomicAdd(a.ticket, 1u) == gridDim.x - 1;
  }
  named_sync(1, kGemvConsumers);
  if (!h->last_cta) return;
  __threadfence();
  float bv = -INFINITY;
  unsigned bid = 0xffffffffu, fl = 0;
  for (unsigned i = threadIdx.x; i < gridDim.x; i += kGemvConsumers) {
    const uint4 c = __ldcg(&a.partials[i]);
    fl |= c.z;
    if (better(__uint_as_float(c.x), c.y, bv, bid)) {
      bv = __uint_as_float(c.x);
      bid = c.y;
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const unsigned oid = __shfl_xor_sync(0xffffffffu, bid, off);
    fl |= __shfl_xor_sync(0xffffffffu, fl, off);
    if (better(ov, oid, bv, bid)) {
      bv = ov;
      bid = oid;
    }
  }
  if (lane == 0) h->cta_best[warp] = make_uint4(__float_as_uint(bv), bid, fl, 0);
  named_sync(1, kGemvConsumers);
  if (threadIdx.x == 0) {
    uint4 b = h->cta_best[0];
    for (int w = 1; w < kConsumerWarps; ++w) {
      const uint4 c = h->cta_best[w];
      if (better(__uint_as_float(c.x), c.y, __uint_as_float(b.x), b.y)) {
        b.x = c.x;
        b.y = c.y;
      }
      b.z |= c.z;
    }
    unsigned status = b.z ? 1u : 0u, token = 0;
    if (!status) {
      if (!isfinite(__uint_as_float(b.x)))
        status = 2;
      else
        token = b.y;
    }
    const SelectOutput& so = a.select;
    so.result[0] = token;
    so.result[1] = status;
    if (so.history) so.history[so.step ? *so.step : 0] = token;
    if (so.step) ++*so.step;
    if (so.terminal) *so.terminal |= (status != 0) || (so.stop_mask && so.stop_mask[token]);
    if (so.position) ++*so.position;
    *a.ticket = 0;
    h->chosen = token;
  }
  named_sync(1, kGemvConsumers);
  const SelectOutput& so = a.select;
  if (so.embed) {
    const bf16* src = so.embed + size_t(h->chosen) * so.width;
    for (int f = threadIdx.x; f < so.width; f += kGemvConsumers) so.residual[f] = src[f];
  }
}

__device__ __forceinline__ void consumer_main(const PersistArgs& a, unsigned char* uni, const unsigned char* ring, PHeader* h) {
  const long long S = __ldcg(a.position);
  const int score_units = a.kv_heads * a.score_slices;
  const int fslices = a.width / a.pv_features;
  const int pv_units = a.kv_heads * fslices;
  unsigned g = 0, target = 0;
  bool failed = false;  // this thread's ring wait gave up (sets abort_flag)
  bool aborted = false; // CTA-uniform: a barrier failed
  Best none;
  // Projection descriptor idx = 4 l + p (qkv, o, gu, down) into desc[idx & 1],
  // issued one projection ahead so its fields are in shared memory on entry.
  auto fetch_desc = [&](int idx) {
    const PLayer& Lx = a.layers[idx >> 2];
    const int p = idx & 3;
    const PGemv* src = p == 0 ? &Lx.qkv : p == 1 ? &Lx.o : p == 2 ? &Lx.gu : &Lx.down;
    if (threadIdx.x < int(sizeof(PGemv) / 16))
      cp_async16(h->desc[idx & 1] + 16 * threadIdx.x, reinterpret_cast<const unsigned char*>(src) + 16 * threadIdx.x);
    else if (p == 0 && threadIdx.x < int(sizeof(PGemv) / 16) + 2)
      cp_async16(reinterpret_cast<unsigned char*>(h->attn[(idx >> 2) & 1]) + 16 * (threadIdx.x - sizeof(PGemv) / 16),
                 reinterpret_cast<const unsigned char*>(&Lx.q_norm) + 16 * (threadIdx.x - sizeof(PGemv) / 16));
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int nproj = 4 * a.nlayers;
  auto desc = [&](int idx) -> const PGemv& {
    asm volatile("cp.async.wait_all;" ::: "memory");
    named_sync(1, kGemvConsumers);
    if (idx + 1 < nproj) fetch_desc(idx + 1);
    return *reinterpret_cast<const PGemv*>(h->desc[idx & 1]);
  };
  fetch_desc(0);
  // RoPE factors of this step's position, once per launch (rotary.cu:84-126).
  for (int f = threadIdx.x; f < a.width / 2; f += kGemvConsumers) {
    const float angle = __fmul_rn(static_cast<float>(S), a.inv_freq[f]);
    h->rope[f][0] = round_bf16(cosf(angle));
    h->rope[f][1] = round_bf16(sinf(angle));
  }
  auto sync = [&] {
    if (aborted) return;
    // Let the producer pull the next stages into L2 while this CTA waits.
    if (threadIdx.x == 0 && a.prefetch_stages > 0) vstore(&h->pf_req, vload(&h->pf_req) + 1);
    target += gridDim.x;
    if (!grid_sync(a.barrier, target, h)) {
      aborted = true;
      if (threadIdx.x == 0) {
        vstore(&h->abort_flag, 1u);
        record_error(a.err, kErrGridSync);
      }
    }
  };
  for (int l = 0; l < a.nlayers && !aborted; ++l) {
    gemv_phase(a, desc(4 * l), uni, ring, h, g, failed, nullptr, none);
    sync();
    if (aborted) break;
    for (int u = blockIdx.x; u < score_units; u += gridDim.x)
      score_unit(a, h->attn[l & 1], u % a.kv_heads, u / a.kv_heads, int(S), uni, h);
    sync();
    if (aborted) break;
    for (int u = blockIdx.x; u < pv_units; u += gridDim.x)
      pv_unit(a, h->attn[l & 1], u / fslices, (u % fslices) * a.pv_features, int(S), uni, h);
    sync();
    if (aborted) break;
    gemv_phase(a, desc(4 * l + 1), uni, ring, h, g, failed, nullptr, none);
    sync();
    if (aborted) break;
    gemv_phase(a, desc(4 * l + 2), uni, ring, h, g, failed, nullptr, none);
    sync();
    if (aborted) break;
    bf16* cap = (a.capture && a.capture_layer == l && a.edit_layer != l) ? a.capture + size_t(S) * a.hidden : nullptr;
    gemv_phase(a, desc(4 * l + 3), uni, ring, h, g, failed, cap, none);
    sync();
    if (aborted) break;
    if (a.edit_layer == l) {
      if (blockIdx.x == 0) edit_phase(a, S, h);
      sync();
    }
  }
  if (!aborted) {
    Best best;
    gemv_phase(a, a.head, uni, ring, h, g, failed, nullptr, best);
    named_sync(1, kGemvConsumers);
    if (vload(&h->abort_flag)) aborted = true;
    if (!aborted && a.head.epilogue == kEpilogueArgmax) head_select(a, h, best);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  named_sync(1, kGemvConsumers);
  if (!aborted) {
    if (threadIdx.x == 0 && atomicAdd(a.exit_ticket, 1u) == gridDim.x - 1) {
      *a.barrier = 0;
      *a.exit_ticket = 0;
    }
    return;
  }
  // Unwind: stop the producer, then wait (bounded) for its copies in flight.
  if (threadIdx.x == 0) {
    vstore(&h->abort_flag, 1u);
    const long long start = clock64();
    while (!vload(&h->producer_done) && clock64() - start < kSpinLimit) {
    }
    const unsigned issued = vload(&h->issued);
    for (unsigned j = issued > kPersistSlots ? issued - kPersistSlots : 0; j < issued; ++j)
      mbar_wait(&h->full[j % kPersistSlots], (j / kPersistSlots) & 1);
  }
}

__global__ void __launch_bounds__(kGemvThreads, 1) decode_persistent_kernel(const __grid_constant__ PersistArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  PHeader* h = reinterpret_cast<PHeader*>(smem);
  unsigned char* uni = smem + kPersistHeaderBytes;
  unsigned char* uend = uni + kPersistUnionBytes;
  const uint32_t ring_s = (smem_addr(uend) + 1023u) & ~1023u;
  unsigned char* ring = uend + (ring_s - smem_addr(uend));
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPersistSlots; ++s) {
      mbar_init(&h->full[s], 1);
      mbar_init(&h->empty[s], kConsumerWarps);
    }
    h->abort_flag = 0;
    h->pf_req = 0;
    h->producer_done = 0;
    h->issued = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x >> 5 == kConsumerWarps) {
    if ((threadIdx.x & 31) == 0) producer_main(a, ring, h);
    return;
  }
  consumer_main(a, uni, ring, h);
}

}  // namespace

bool plan_persist_gemv(PGemv& g, const PSegSpec* specs, int nseg, const bf16* x, const bf16* norm_w,
                       int in_width, int epilogue, int grid, CUtensorMap* maps) {
  const int I = in_width;
  if (nseg < 1 || nseg > kGemvMaxSegs || I <= 0 || I % kGemvBox || I > kPersistMaxInput ||
      (norm_w && I > kPersistMaxNormInput))
    return false;
  g = PGemv{};
  g.x = x;
  g.norm_w = norm_w;
  g.in_width = I;
  g.epilogue = epilogue;
  g.nseg = nseg;
  const bool pairs = epilogue == kEpilogueSwiGLU;
  long long total = 0;
  for (int i = 0; i < nseg; ++i) total += specs[i].rows;
  int assigned = 0;
  for (int i = 0; i < nseg; ++i) {
    const PSegSpec& sp = specs[i];
    PSeg& s = g.seg[i];
    if (sp.rows <= 0 || (pairs && sp.rows % 2) || (sp.partials != 16 && sp.partials != 32)) return false;
    int c = nseg == 1 ? grid : std::max(1, (int)std::llround((double)grid * sp.rows / total));
    if (i == nseg - 1) c = std::max(1, grid - assigned);
    c = std::min(c, sp.rows);
    int per = (sp.rows + c - 1) / c;
    if (pairs) per += per & 1;
    c = (sp.rows + per - 1) / per;
    // Threads per row: 4 for P = 16 (4-partial layout), P / 8 otherwise.
    const int maxr = kGemvConsumers / (sp.partials == 16 ? 4 : sp.partials / 8);
    const int nt = (per + maxr - 1) / maxr;
    int tr = (per + nt - 1) / nt;
    if (pairs) tr += tr & 1;
    int kc = 0;
    for (int cand : {512, 256, 128, 64})
      if (I % cand == 0 && (cand / kGemvBox) * tr * 128 <= kPersistSlotBytes) {
        kc = cand;
        break;
      }
    if (!kc || tr > maxr) return false;
    s.out = sp.out;
    s.out_row = sp.out_row;
    s.rows = sp.rows;
    s.partials = sp.partials;
    s.cta_begin = assigned;
    s.cta_count = c;
    s.rows_per_cta = per;
    s.tile_rows = tr;
    s.out_stride = sp.out_stride;
    s.kc = kc;
    if (!encode_weight_map3d(&maps[i], sp.w, uint64_t(sp.rows), uint64_t(I), uint32_t(tr), uint32_t(kc / kGemvBox)))
      return false;
    assigned += c;
  }
  return assigned <= grid;
}

bool decode_persistent_fits(int grid) {
  if (cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPersistSmem) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, kGemvThreads, kPersistSmem) !=
          cudaSuccess ||
      cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return per_sm >= 1 && grid <= per_sm * sms;
}

cudaError_t launch_decode_persistent(const PersistArgs& a, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = kPersistSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, a);
}

}  // namespace dl
