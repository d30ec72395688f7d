// Device-side generation loop (role of the reference's DeviceSequence,
// src/inference/decoding/device.h:84-139 and src/kernels/cuda/decode.cu:
// 68-230, 379-610): one CUDA graph whose conditional WHILE node replays the
// decode step until a stop ID, a failed selection, a cancel request or the
// token limit, journaling each consumed prompt and each selection as a
// 32-byte event in mapped host memory that the host polls.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/dolittle_b200.h"

namespace dl {

static_assert(sizeof(dl_sequence_event) == 32, "journal events are 32 bytes");

// Journal event 0: the prompt of `count` tokens was consumed.
cudaError_t launch_journal_consumed(dl_sequence_event* journal, unsigned long long count, cudaStream_t stream);

// After a selection (step = number of selections so far, read on the device):
// journal[step] = selected {token, status, position}; then if the sequence
// ends (status != 0 -> failure, stop_mask[token] -> eos, *cancel -> cancelled,
// step >= *limit -> limit) journal[step + 1] = terminal with the reason.  With
// set_loop, the WHILE node's condition becomes "continue".
cudaError_t launch_journal_selection(const int* step, const unsigned* result, const long long* position,
                                     const unsigned char* stop_mask, const unsigned* limit,
                                     const volatile unsigned* cancel, dl_sequence_event* journal,
                                     cudaGraphConditionalHandle loop, bool set_loop, cudaStream_t stream);

}  // namespace dl
