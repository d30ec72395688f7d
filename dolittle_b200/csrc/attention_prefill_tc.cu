// Causal GQA prompt attention on the 5th-generation tensor cores, for the
// fast prompt pass (tensor-core accumulation order, online softmax; checked
// against the reference-order path within tolerance like the tcgen05 GEMMs).
//
// One CTA (4 x kRowSplit warps) owns 128 query rows of one query head; query
// row r = TMEM lane r is shared by kRowSplit threads (warps w, w + 4, ...
// reach the same TMEM lane group), each owning 128 / kRowSplit columns.  Key blocks of 128, one pass:
//   S[kb] = Q K[kb]^T (tcgen05.mma, M = N = 128, K = 128 over the head width)
//           into one of two TMEM score buffers;
//   each thread reads its part of the row of S; the parts exchange their max
//   and sum through shared memory to update the row's running max m and sum
//   l of exp2(s - m) (masked beyond the row's position); each writes its
//   p = exp2(s - m) as FP16 into a 128-byte-swizzled K-major tile;
//   O[kb] = P V[kb] (A = P, B = V^T, both FP16) into TMEM; each thread rescales its
//   register copy of its 64 output columns by exp2(m_old - m_new) and adds
//   those of O[kb]; the output is O / l at the end.
// K and V^T blocks stream through two TMA stages, and the next block's score
// MMA is issued as soon as this block's P is written, so it overlaps the
// output update.  Scores carry the softmax scale times log2(e).  Q and K come
// in by TMA from the rotated queries and the K cache; V is read as V^T from a
// transposed copy (launch_vt_transpose) so both operands of both products are
// K-major.  The second product runs in FP16 (10-bit mantissa): p in [0, 1]
// rounded to FP16 carries 1/8 of the BF16 rounding error, and the BF16 values
// of V convert to FP16 exactly (the copy saturates at +-65504, far beyond any
// value a normed projection produces).  In BF16 the P rounding alone added as
// much error to the attention output as its final BF16 rounding.
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include <cmath>
#include <mutex>

#include "attention_prefill_tc.h"
#include "tcgen05.cuh"

namespace dl {
namespace {

using namespace tc;

constexpr int kTile = 128;                    // query rows per CTA, keys per block
constexpr int kRowSplit = 2;                  // threads per query row
constexpr int kThreads = kTile * kRowSplit;
constexpr int kRowChunks = 4 / kRowSplit;     // 32-column chunks of S / O per thread
constexpr int kAtomBytes = kTile * 64 * 2;    // [128 rows][64 BF16], one swizzle atom column
constexpr int kTileBytes = 2 * kAtomBytes;    // [128 rows][128 BF16]
constexpr int kSmem = 6 * kTileBytes + 1024;  // Q, 2 x K, 2 x V^T, P + alignment
constexpr uint32_t kTmemCols = 512;           // S0, S1, O (128 columns each)

struct alignas(64) AttnArgs {
  CUtensorMap map_q;   // {d, Hq, rows}: box {64, 1, 128}
  CUtensorMap map_k;   // {d, Hkv, C, 2L}: box {64, 1, 128, 1}; K of block l at index 2l
  CUtensorMap map_vt;  // {keys, d, Hkv}: box {64, 128, 1}
  bf16* out;           // [rows][Hq * d]
  int rows, layer, query_heads, kv_heads;
  long long first;     // absolute position of query row 0
  float scale_log2;    // softmax scale * log2(e)
  unsigned* err;
};

__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load4(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// 8 MMAs of K = 16 across the two swizzle atoms of a 128-wide K dimension;
// BF16 operands (S = Q K^T) or FP16 operands (O = P V).
template <bool F16>
__device__ __forceinline__ void mma_tile(uint32_t tmem_d, const unsigned char* a_tile, const unsigned char* b_tile,
                                         bool accumulate) {
  constexpr uint32_t idesc = F16 ? instr_desc_f16(kTile, kTile) : instr_desc_bf16(kTile, kTile);
  const uint32_t sa = smem_addr(a_tile), sb = smem_addr(b_tile);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t atom = uint32_t(kk >> 2) * kAtomBytes;
    const uint64_t off = uint64_t((kk & 3) * 2);
    mma_bf16(tmem_d, smem_desc_sw128(sa + atom) + off, smem_desc_sw128(sb + atom) + off, idesc,
             (accumulate || kk) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(kThreads, 1) attention_prefill_tc_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t q_bar, kv_bar[2], s_bar[2], o_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ float red_max[kRowSplit][kTile], red_sum[kRowSplit][kTile];  // the parts of each row
  const uint32_t base_s = (smem_addr(smem_raw) + 1023u) & ~1023u;
  unsigned char* sq = smem_raw + (base_s - smem_addr(smem_raw));
  // Stage st: K at sq + (1 + st) tiles, V^T at sq + (3 + st) tiles.
  auto sk = [&](int st) { return sq + (1 + st) * kTileBytes; };
  auto svt = [&](int st) { return sq + (3 + st) * kTileBytes; };
  unsigned char* sp = sq + 5 * kTileBytes;
  const int warp = threadIdx.x >> 5;
  const int hq = blockIdx.y;
  const int g = hq / (a.query_heads / a.kv_heads);
  const int q0 = blockIdx.x * kTile;
  const int r = threadIdx.x & (kTile - 1);  // row within the tile = TMEM lane
  const int h = threadIdx.x >> 7;           // columns [128 h / kRowSplit, 128 (h + 1) / kRowSplit)
  const int row = q0 + r;
  const bool live = row < a.rows;
  const long long pos = a.first + row;
  const long long last_pos = a.first + min(a.rows, q0 + kTile) - 1;
  const int nkb = int(last_pos / kTile) + 1;

  if (threadIdx.x == 0) {
    mbar_init(&q_bar, 1);
    mbar_init(&kv_bar[0], 1);
    mbar_init(&kv_bar[1], 1);
    mbar_init(&s_bar[0], 1);
    mbar_init(&s_bar[1], 1);
    mbar_init(&o_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;
  auto t_s = [&](int st) { return tmem + uint32_t(st * 128); };
  // Programmatic dependent launch: the prologue above overlaps the previous
  // kernel; nothing it wrote is read before this point.
  allow_next();
  wait_prior();
  const uint32_t t_o = tmem + 256;
  const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;

  // Thread 0 issues every TMA load and MMA.
  auto load_kv = [&](int kb) {
    const int st = kb & 1;
    mbar_arrive_expect_tx(&kv_bar[st], unsigned(2 * kTileBytes));
    tma_load4(sk(st), &a.map_k, 0, g, kb * kTile, 2 * a.layer, &kv_bar[st]);
    tma_load4(sk(st) + kAtomBytes, &a.map_k, 64, g, kb * kTile, 2 * a.layer, &kv_bar[st]);
    tma_load(svt(st), &a.map_vt, kb * kTile, 0, g, &kv_bar[st]);
    tma_load(svt(st) + kAtomBytes, &a.map_vt, kb * kTile + 64, 0, g, &kv_bar[st]);
  };
  auto fail = [&] {
    record_error(a.err, kErrWaitFull);
    abort_flag = 1;
  };
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&q_bar, unsigned(kTileBytes));
    tma_load(sq, &a.map_q, 0, hq, q0, &q_bar);
    tma_load(sq + kAtomBytes, &a.map_q, 64, hq, q0, &q_bar);
    load_kv(0);
    if (nkb > 1) load_kv(1);
    if (!mbar_wait(&q_bar, 0) || !mbar_wait(&kv_bar[0], 0)) {
      fail();
    } else {
      fence_after_sync();
      mma_tile<false>(t_s(0), sq, sk(0), false);
      mma_commit(&s_bar[0]);
    }
  }
  __syncthreads();

  float o[32 * kRowChunks];
#pragma unroll
  for (int i = 0; i < 32 * kRowChunks; ++i) o[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  unsigned o_phase = 0;
  for (int kb = 0; kb < nkb && !abort_flag; ++kb) {
    const int st = kb & 1;
    if (!mbar_wait(&s_bar[st], unsigned(kb >> 1) & 1)) fail();
    fence_after_sync();
    const int key0 = kb * kTile;
    // Block max over this row's visible keys (TMEM loads are warp-collective:
    // every lane loads, only the arithmetic is guarded).
    float bm = -INFINITY;
#pragma unroll 1
    for (int c = kRowChunks * h; c < kRowChunks * (h + 1); ++c) {
      uint32_t sv[32];
      tmem_ld32(t_s(st) + lane_base + uint32_t(c * 32), sv);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (key0 + c * 32 + i <= pos) bm = fmaxf(bm, __uint_as_float(sv[i]) * a.scale_log2);
    }
    red_max[h][r] = bm;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kRowSplit; ++j) bm = fmaxf(bm, red_max[j][r]);
    const float mn = fmaxf(m, bm);
    const bool use = live && mn != -INFINITY;
    const float alpha = (use && m != -INFINITY) ? exp2f(m - mn) : 0.f;
    float sum = 0.f;
#pragma unroll 1
    for (int c = kRowChunks * h; c < kRowChunks * (h + 1); ++c) {
      uint32_t sv[32];
      tmem_ld32(t_s(st) + lane_base + uint32_t(c * 32), sv);
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int k0 = key0 + c * 32 + i;
        const float p0 = (use && k0 <= pos) ? exp2f(__uint_as_float(sv[i]) * a.scale_log2 - mn) : 0.f;
        const float p1 = (use && k0 + 1 <= pos) ? exp2f(__uint_as_float(sv[i + 1]) * a.scale_log2 - mn) : 0.f;
        const __half2 h2 = __floats2half2_rn(p0, p1);
        sum += __low2float(h2) + __high2float(h2);  // l sums the FP16 weights the MMA sees
        packed[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      // Keys c*32 .. c*32+31 of the block: atom c / 2, chunks (c % 2) * 4 .. + 3.
      unsigned char* rowp = sp + (c >> 1) * kAtomBytes + r * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int chunk = (c & 1) * 4 + q;
        *reinterpret_cast<uint4*>(rowp + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      }
    }
    red_sum[h][r] = sum;
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();  // P complete; S[st] consumed
    if (use) {
      float total = red_sum[0][r];
#pragma unroll
      for (int j = 1; j < kRowSplit; ++j) total += red_sum[j][r];
      l = l * alpha + total;
      m = mn;
    }
    if (threadIdx.x == 0 && !abort_flag) {
      fence_after_sync();
      mma_tile<true>(t_o, sp, svt(st), false);
      mma_commit(&o_bar);
      if (kb + 1 < nkb) {
        // The next block's scores overlap this block's output update.
        if (!mbar_wait(&kv_bar[st ^ 1], unsigned((kb + 1) >> 1) & 1)) {
          fail();
        } else {
          fence_after_sync();
          mma_tile<false>(t_s(st ^ 1), sq, sk(st ^ 1), false);
          mma_commit(&s_bar[st ^ 1]);
        }
      }
    }
    if (!mbar_wait(&o_bar, o_phase)) fail();
    o_phase ^= 1;
    fence_after_sync();
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
      uint32_t ov[32];
      tmem_ld32(t_o + lane_base + uint32_t((kRowChunks * h + c) * 32), ov);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha, __uint_as_float(ov[i]));
    }
    fence_before_sync();
    __syncthreads();  // O and P free; stage st free once both MMAs of this block completed
    if (threadIdx.x == 0 && kb + 2 < nkb && !abort_flag) load_kv(kb + 2);
  }
  if (!abort_flag && live) {
    const float inv_l = l > 0.f ? 1.0f / l : 0.f;
    bf16* out = a.out + size_t(row) * (size_t(a.query_heads) * 128) + size_t(hq) * 128 + 32 * kRowChunks * h;
#pragma unroll
    for (int c = 0; c < 4 * kRowChunks; ++c) {
      uint32_t packed[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const __nv_bfloat162 h2 = __floats2bfloat162_rn(o[c * 8 + i] * inv_l, o[c * 8 + i + 1] * inv_l);
        packed[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      reinterpret_cast<uint4*>(out)[c] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// V^T of one block's cache in FP16: vt[g][f][j] = v[j][g][f] for j < keys
// (BF16 -> FP16 is exact in FP16's normal range; saturated beyond it).
__global__ void vt_transpose_kernel(const bf16* __restrict__ v, __half* __restrict__ vt, int keys, int kv_heads,
                                    int width, int vt_stride) {
  __shared__ __half tile[32][33];
  allow_next();
  wait_prior();
  const int g = blockIdx.z;
  const int j0 = blockIdx.x * 32, f0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int j = j0 + i, f = f0 + threadIdx.x;
    if (j < keys && f < width)
      tile[i][threadIdx.x] =
          __float2half_rn(fminf(fmaxf(__bfloat162float(v[(size_t(j) * kv_heads + g) * width + f]), -65504.f), 65504.f));
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int f = f0 + i, j = j0 + threadIdx.x;
    if (j < keys && f < width) vt[(size_t(g) * width + f) * vt_stride + j] = tile[threadIdx.x][i];
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
            const cuuint32_t* box, CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

struct AttnTcMaps {
  CUtensorMap q, k, vt;
};

bool attention_prefill_tc_supported(int query_heads, int kv_heads, int width) {
  return width == 128 && kv_heads > 0 && query_heads % kv_heads == 0;
}

AttnTcMaps* attention_prefill_tc_maps(const bf16* q, int max_rows, int query_heads, const bf16* kv_arena,
                                      size_t kv_block_bytes, int capacity, int layers, int kv_heads, int width,
                                      const bf16* vt, int vt_stride) {
  if (!attention_prefill_tc_supported(query_heads, kv_heads, width) || kv_block_bytes % 16 || vt_stride % 64)
    return nullptr;
  auto* m = new AttnTcMaps;
  const cuuint64_t qd[3] = {uint64_t(width), uint64_t(query_heads), uint64_t(max_rows)};
  const cuuint64_t qs[2] = {uint64_t(width) * 2, uint64_t(query_heads) * width * 2};
  const cuuint32_t qb[3] = {64, 1, 128};
  const cuuint64_t kd[4] = {uint64_t(width), uint64_t(kv_heads), uint64_t(capacity), uint64_t(2 * layers)};
  const cuuint64_t ks[3] = {uint64_t(width) * 2, uint64_t(kv_heads) * width * 2, kv_block_bytes};
  const cuuint32_t kb[4] = {64, 1, 128, 1};
  const cuuint64_t vd[3] = {uint64_t(vt_stride), uint64_t(width), uint64_t(kv_heads)};
  const cuuint64_t vs[2] = {uint64_t(vt_stride) * 2, uint64_t(width) * vt_stride * 2};
  const cuuint32_t vb[3] = {64, 128, 1};
  if (!encode(&m->q, q, 3, qd, qs, qb) || !encode(&m->k, kv_arena, 4, kd, ks, kb) ||
      !encode(&m->vt, vt, 3, vd, vs, vb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16)) {
    delete m;
    return nullptr;
  }
  return m;
}

void attention_prefill_tc_free(AttnTcMaps* m) { delete m; }

namespace {
cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, cudaLaunchAttribute* attr,
                              bool pdl) {
  cudaLaunchConfig_t c = {};
  c.gridDim = grid;
  c.blockDim = block;
  c.dynamicSmemBytes = smem;
  c.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}
}  // namespace

cudaError_t launch_vt_transpose(const bf16* v_cache, bf16* vt, int keys, int kv_heads, int width, int vt_stride,
                                cudaStream_t stream, bool pdl) {
  if (keys <= 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_config(dim3((keys + 31) / 32, (width + 31) / 32, kv_heads), dim3(32, 8), 0, stream, attr, pdl);
  return cudaLaunchKernelEx(&cfg, vt_transpose_kernel, v_cache, reinterpret_cast<__half*>(vt), keys, kv_heads, width,
                            vt_stride);
}

cudaError_t launch_attention_prefill_tc(const AttnTcMaps* maps, bf16* out, int rows, long long first, int layer,
                                        int query_heads, int kv_heads, float scale, unsigned* err,
                                        cudaStream_t stream, bool pdl) {
  if (!maps || rows <= 0) return cudaErrorInvalidValue;
  AttnArgs a = {};
  a.map_q = maps->q;
  a.map_k = maps->k;
  a.map_vt = maps->vt;
  a.out = out;
  a.rows = rows;
  a.first = first;
  a.layer = layer;
  a.query_heads = query_heads;
  a.kv_heads = kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(attention_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_config(dim3((rows + kTile - 1) / kTile, query_heads), dim3(kThreads), kSmem, stream, attr, pdl);
  return cudaLaunchKernelEx(&cfg, attention_prefill_tc_kernel, a);
}

}  // namespace dl
