// Causal GQA attention for callers that cannot allocate device memory.
//
// dl_attention needs a score workspace that its caller allocates.  Some
// callers cannot allocate device memory at all: a host that owns every device
// allocation through its own arena (the way Dolittle's executor plans all of
// its storage before generation and then guards against any further
// allocation), or a plugin loaded into a process whose allocator does not let
// outside code call cudaMalloc.  For them, dl_attention_fixed_scratch runs the
// same two kernels with the scores in a fixed array that lives in the
// library's own device memory, so it allocates nothing.
//
// Limits and sharing:
//  * the array holds kFixedScratchScores FP32 scores (4 MiB): positions *
//    query_heads * key capacity must not exceed that, or the call is rejected
//    with DL_INVALID_ARGUMENT before anything is launched;
//  * every GPU that loads the library keeps its 4 MiB copy until the process
//    exits;
//  * all calls on a device share the one array and it keeps whatever the last
//    call wrote; the score kernel writes every entry the softmax later reads,
//    so nothing has to start at zero.  Calls whose work overlaps on the GPU
//    (different streams, or host threads racing on one device) race on the
//    array: serialize them.
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current; make that first call
//    before any stream capture.  The address is kept for the life of the
//    process, so calls must not span a cudaDeviceReset (which unloads the
//    library's device module and may move the array).
#include <climits>
#include <mutex>
#include <string>

#include "../../include/dolittle_b200.h"
#include "launch.h"

namespace {

constexpr size_t kFixedScratchScores = DL_ATTENTION_FIXED_SCRATCH_SCORES;  // 4 MiB of FP32 scores
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, never a device address: the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_fixed_attention_scores[kFixedScratchScores];

std::mutex g_setup_mutex;
float* g_scratch_by_device[kMaxDevices] = {};

dl_status fixed_fail(dl_status s, const std::string& msg) {
  dl::set_last_error(msg);  // reported by dl_last_error()
  return s;
}

// Device address of the scratch on the current device (set up once per device).
dl_status scratch_for_current_device(float** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fixed_fail(DL_CUDA_ERROR, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (device < 0 || device >= kMaxDevices) return fixed_fail(DL_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_by_device[device]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fixed_attention_scores);
    if (e != cudaSuccess || !p)
      return fixed_fail(DL_CUDA_ERROR, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_scratch_by_device[device] = static_cast<float*>(p);
  }
  *out = g_scratch_by_device[device];
  return DL_OK;
}

}  // namespace

extern "C" {

DL_API dl_status dl_attention_fixed_scratch(dl_dtype type, const void* query, const void* key,
                                            const void* value, void* output, size_t positions,
                                            size_t query_heads, size_t kv_heads, size_t width, void* stream,
                                            size_t first_position, const size_t* device_position,
                                            size_t capacity) {
  if (type != DL_BF16) return fixed_fail(DL_UNSUPPORTED, "attention: only BF16 storage is supported");
  if (!query || !key || !value || !output || !positions || !query_heads || !kv_heads || !width)
    return fixed_fail(DL_INVALID_ARGUMENT, "attention: arguments");
  if (positions > INT_MAX || query_heads > INT_MAX)
    return fixed_fail(DL_INVALID_ARGUMENT, "attention: positions and query heads must fit an int");
  if (query_heads % kv_heads || query_heads / kv_heads > 8 || width > 128 || width % 8)
    return fixed_fail(DL_UNSUPPORTED, "attention: GQA group <= 8 and head width <= 128 (multiple of 8)");
  if (!device_position && first_position > 200 * 1024 / 4)
    return fixed_fail(DL_UNSUPPORTED, "attention: more than 51200 keys");
  const size_t cap = device_position ? capacity : first_position + positions;
  if (!cap) return fixed_fail(DL_INVALID_ARGUMENT, "attention: zero key capacity");
  if (cap * 4 > 200 * 1024) return fixed_fail(DL_UNSUPPORTED, "attention: more than 51200 keys");
  // positions * query_heads * cap > limit, checked without a product that could wrap.
  if (positions > kFixedScratchScores / query_heads / cap)
    return fixed_fail(DL_INVALID_ARGUMENT,
                      "attention: positions * query_heads * key capacity exceeds the fixed scratch of " +
                          std::to_string(kFixedScratchScores) + " scores (4 MiB)");
  float* scratch = nullptr;
  const dl_status s = scratch_for_current_device(&scratch);
  if (s != DL_OK) return s;
  const auto st = static_cast<cudaStream_t>(stream);
  const dl::RowPositions pos{reinterpret_cast<const long long*>(device_position), (long long)first_position};
  const int ctas = positions == 1 ? 16 : 8;
  cudaError_t e = dl::launch_attention_scores(static_cast<const dl::bf16*>(query), static_cast<const dl::bf16*>(key),
                                              scratch, pos, int(positions), int(query_heads), int(kv_heads),
                                              int(width), int(cap), dl::attention_scale(int(width)), ctas, st, false);
  if (e == cudaSuccess)
    e = dl::launch_attention_pv(scratch, static_cast<const dl::bf16*>(value), static_cast<dl::bf16*>(output), pos,
                                int(positions), int(query_heads), int(kv_heads), int(width), int(cap), st, false);
  if (e != cudaSuccess) return fixed_fail(DL_CUDA_ERROR, std::string("attention: ") + cudaGetErrorString(e));
  return DL_OK;
}

}  // extern "C"
