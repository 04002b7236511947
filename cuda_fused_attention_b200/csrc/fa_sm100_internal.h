// Library-internal helpers shared by the translation units of libfa_sm100.so.
// Not part of the C ABI: nothing here is exported (the library is built with
// -fvisibility=hidden and these carry no FA_API).
#pragma once

#include <cuda_runtime.h>

namespace fa_sm100_internal {

// fa_sm100_fwd without the causal key-range split, the one launch that takes workspace memory
// (from a stream-ordered pool): a launch that allocates nothing, for fa_sm100_fwd_host_static.
int forward_without_workspace(const void* q, const void* k, const void* v, void* o, int batch, int heads,
                              int seq_len, int head_dim, int causal, void* stream);

// Reads the device error word of the current device on `stream` (a copy ordered
// after the work already queued there, then a synchronisation of that stream)
// and clears it if it was set. Returns FA_STATUS_OK or FA_STATUS_DEVICE_TIMEOUT,
// or the cudaError_t of a failed copy. `word` (may be null) receives the raw
// value. Allocates nothing. The word is per device and shared by every launch
// on it, so a timeout of a launch that another caller made at the same time
// can be reported here instead of there.
int take_error_word(cudaStream_t stream, unsigned int* word);

}  // namespace fa_sm100_internal
