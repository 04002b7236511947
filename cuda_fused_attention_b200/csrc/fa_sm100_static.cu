// =============================================================================
// Host-buffer forward pass that allocates nothing: fa_sm100_fwd_host_static.
//
// fa_sm100_fwd_host stages Q/K/V/O through device buffers it obtains with
// cudaMalloc on first use. Some callers cannot allow that: code that must not
// allocate device memory after start-up (latency-critical or real-time paths,
// processes whose device memory is owned by a caching allocator or a fixed
// pool, integrations that forbid allocator calls while other work is
// running). For them this entry point stages through one file-scope
// __device__ array of fixed size instead. That array is part of the loaded
// module: every GPU that loads this library holds it until the process exits.
//
// Limits and behaviour:
//   * The array is kStaticStagingBytes = 32 MiB: four 8 MiB regions for Q, K, V
//     and O. Slabs (one batch*head each, seq_len*head_dim bf16 values) are
//     processed in chunks that fit a region, so one slab may be at most 8 MiB
//     (seq_len*head_dim <= 4,194,304 elements, e.g. N <= 32768 at D=128).
//     Larger slabs are rejected with FA_STATUS_STATIC_TOO_LARGE before any
//     CUDA call is made.
//   * No cudaMalloc, cudaFree, stream or event creation, and no allocating
//     library routine: copies, the kernel and the synchronisation all run on
//     the stream the caller passes (NULL = legacy default stream). The chunks
//     run one after another on that stream (no copy/compute overlap). Their
//     launches never use the causal key-range split, whose workspace would
//     come from a memory pool.
//   * Set-up: the first call on a device, with that device current, resolves
//     the array's device address once with cudaGetSymbolAddress (host code
//     cannot use the array's name as a device address). Make that first call
//     before any stream capture begins.
//   * Every call shares the one array and it keeps the last call's contents.
//     Nothing in it needs to start at zero: each chunk's Q/K/V are copied in
//     in full and a launch that completes writes every O element copied out.
//     A launch that gives up on a bounded device-side wait does not; the call
//     then returns FA_STATUS_DEVICE_TIMEOUT (it reads and clears the device
//     error word after its final synchronisation), and o_host must not be
//     used. Calls that overlap on the GPU (different streams or host threads
//     at once) race on the array; serialise them.
//   * Lazy module loading (CUDA's default) loads the module that holds the
//     array, and so allocates its 32 MiB, at the first call's
//     cudaGetSymbolAddress. A caller that forbids allocation after start-up
//     makes one call (any size) at start-up; later calls allocate nothing.
// =============================================================================
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "fa_sm100.h"
#include "fa_sm100_internal.h"

namespace {

constexpr size_t kStaticRegionBytes = 8ull << 20;                 // per tensor
constexpr size_t kStaticStagingBytes = 4 * kStaticRegionBytes;    // Q, K, V, O
constexpr int kMaxDevices = 64;

}  // namespace

// The staging array (device memory of the loaded module, one per device).
static __device__ __align__(256) unsigned char g_fa_static_staging[kStaticStagingBytes];

namespace {

struct StaticSlot {
    std::once_flag once;
    int status = FA_STATUS_OK;
    unsigned char* base = nullptr;   // device address of g_fa_static_staging on this device
};
StaticSlot g_static_slots[kMaxDevices];

// Resolve the array's device address on the current device, once.
int static_staging_base(int device, unsigned char** out)
{
    if (device < 0 || device >= kMaxDevices) return FA_STATUS_INVALID_ARGUMENT;
    StaticSlot& slot = g_static_slots[device];
    std::call_once(slot.once, [&]() {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_fa_static_staging);
        if (err != cudaSuccess) {
            slot.status = static_cast<int>(err);
            return;
        }
        slot.base = static_cast<unsigned char*>(ptr);
    });
    *out = slot.base;
    return slot.status;
}

}  // namespace

extern "C" {

size_t fa_sm100_static_staging_bytes(void) { return kStaticStagingBytes; }

int fa_sm100_fwd_host_static(const void* q_host, const void* k_host, const void* v_host, void* o_host, int batch,
                             int heads, int seq_len, int head_dim, int causal, void* stream)
{
    if (q_host == nullptr || k_host == nullptr || v_host == nullptr || o_host == nullptr) return FA_STATUS_INVALID_ARGUMENT;
    if (batch <= 0 || heads <= 0 || seq_len <= 0) return FA_STATUS_INVALID_ARGUMENT;
    if (!fa_sm100_supported(head_dim)) return FA_STATUS_UNSUPPORTED;
    const size_t slab_bytes = static_cast<size_t>(seq_len) * static_cast<size_t>(head_dim) * 2u;
    if (slab_bytes > kStaticRegionBytes) return FA_STATUS_STATIC_TOO_LARGE;

    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return static_cast<int>(err);
    unsigned char* base = nullptr;
    int status = static_staging_base(device, &base);
    if (status != FA_STATUS_OK) return status;

    void* dq = base;
    void* dk = base + kStaticRegionBytes;
    void* dv = base + 2 * kStaticRegionBytes;
    void* dout = base + 3 * kStaticRegionBytes;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    const long long slabs = static_cast<long long>(batch) * heads;
    const long long per_chunk = std::min<long long>(slabs, static_cast<long long>(kStaticRegionBytes / slab_bytes));
    const char* hq = static_cast<const char*>(q_host);
    const char* hk = static_cast<const char*>(k_host);
    const char* hv = static_cast<const char*>(v_host);
    char* ho = static_cast<char*>(o_host);

    for (long long first = 0; first < slabs; first += per_chunk) {
        const long long count = std::min(per_chunk, slabs - first);
        const size_t offset = static_cast<size_t>(first) * slab_bytes;
        const size_t bytes = static_cast<size_t>(count) * slab_bytes;
        if ((err = cudaMemcpyAsync(dq, hq + offset, bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(dk, hk + offset, bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(dv, hv + offset, bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess) break;
        status = fa_sm100_internal::forward_without_workspace(dq, dk, dv, dout, static_cast<int>(count), 1, seq_len,
                                                             head_dim, causal, stream);
        if (status != FA_STATUS_OK) break;
        if ((err = cudaMemcpyAsync(ho + offset, dout, bytes, cudaMemcpyDeviceToHost, s)) != cudaSuccess) break;
    }
    const cudaError_t sync = cudaStreamSynchronize(s);
    if (status != FA_STATUS_OK) return status;
    if (err != cudaSuccess) return static_cast<int>(err);
    if (sync != cudaSuccess) return static_cast<int>(sync);
    // A launch that gave up on a bounded wait did not write all of its O rows, so the
    // array's O region may still hold an earlier call's output: report the timeout instead
    // of returning that. Reading and clearing the word is two small copies, no allocation.
    return fa_sm100_internal::take_error_word(s, nullptr);
}

}  // extern "C"
