// Control kernels of the device-side generation loop (see sequence.h).
#include "sequence.h"

namespace dl {
namespace {

// Fields first, then (after a system-scope fence) the kind, which the host
// polls: an event is complete once its kind is nonzero.
__device__ void publish(dl_sequence_event* ev, unsigned kind, unsigned reason, unsigned status,
                        unsigned long long position, unsigned long long count, unsigned token) {
  volatile dl_sequence_event* v = ev;
  v->reason = static_cast<uint8_t>(reason);
  v->status = status;
  v->position = position;
  v->count = count;
  v->token = token;
  v->norm = 0.f;
  __threadfence_system();
  v->kind = static_cast<uint8_t>(kind);
  __threadfence_system();
}

__global__ void journal_consumed_kernel(dl_sequence_event* journal, unsigned long long count) {
  publish(journal, DL_EVENT_CONSUMED, 0, 0, count, count, 0);
}

__global__ void journal_selection_kernel(const int* step, const unsigned* result, const long long* position,
                                         const unsigned char* stop_mask, const unsigned* limit,
                                         const volatile unsigned* cancel, dl_sequence_event* journal,
                                         cudaGraphConditionalHandle loop, bool set_loop) {
  const unsigned k = unsigned(*step);
  const unsigned token = result[0], status = result[1];
  const unsigned long long pos = (unsigned long long)*position;
  publish(journal + k, DL_EVENT_SELECTED, 0, status, pos, k, token);
  unsigned reason = 0xffu;
  if (status) reason = DL_REASON_FAILURE;
  else if (stop_mask && stop_mask[token]) reason = DL_REASON_EOS;
  else if (*cancel) reason = DL_REASON_CANCELLED;
  else if (k >= *limit) reason = DL_REASON_LIMIT;
  if (reason != 0xffu) publish(journal + k + 1, DL_EVENT_TERMINAL, reason, status, pos, k, token);
  if (set_loop) cudaGraphSetConditional(loop, reason == 0xffu ? 1u : 0u);
}

}  // namespace

cudaError_t launch_journal_consumed(dl_sequence_event* journal, unsigned long long count, cudaStream_t stream) {
  journal_consumed_kernel<<<1, 1, 0, stream>>>(journal, count);
  return cudaGetLastError();
}

cudaError_t launch_journal_selection(const int* step, const unsigned* result, const long long* position,
                                     const unsigned char* stop_mask, const unsigned* limit,
                                     const volatile unsigned* cancel, dl_sequence_event* journal,
                                     cudaGraphConditionalHandle loop, bool set_loop, cudaStream_t stream) {
  journal_selection_kernel<<<1, 1, 0, stream>>>(step, result, position, stop_mask, limit, cancel, journal, loop,
                                                set_loop);
  return cudaGetLastError();
}

}  // namespace dl
