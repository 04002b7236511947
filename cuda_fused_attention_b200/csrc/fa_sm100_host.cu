// =============================================================================
// End-to-end entry with host buffers: fa_sm100_fwd_host (include/fa_sm100.h).
//
// The reference harness copies Q/K/V to the device, launches, and copies O
// back itself (benchmarks/bench_flash_attention.cu:545-560). This entry does
// the same work for a caller that holds host memory, pipelined so that PCIe
// traffic and tensor-core work overlap:
//
//   chunk c:   H2D q,k,v (copy-in stream)  -> forward (compute stream)
//              -> D2H o (copy-out stream)
//
// over chunks of whole (batch, head) slabs, double-buffered in device staging
// buffers that are allocated once per device and reused. With pinned host
// memory the copy engines run in both directions at once, so the call costs
// max(H2D, D2H, compute) plus one chunk of fill/drain, instead of the sum.
// =============================================================================
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "fa_sm100.h"
#include "fa_sm100_internal.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kChunkTargetBytes = 64ull << 20;   // per tensor per chunk
constexpr int kBuffers = 2;

struct Staging {
    std::mutex lock;
    size_t capacity = 0;                 // bytes per tensor per buffer
    void* q[kBuffers] = {};
    void* k[kBuffers] = {};
    void* v[kBuffers] = {};
    void* o[kBuffers] = {};
    cudaStream_t in = nullptr, compute = nullptr, out = nullptr;
    cudaEvent_t loaded[kBuffers] = {};   // H2D of buffer b finished
    cudaEvent_t computed[kBuffers] = {}; // forward on buffer b finished (q/k/v free)
    cudaEvent_t stored[kBuffers] = {};   // D2H of buffer b finished (o free)
    bool ready = false;
};

Staging g_staging[kMaxDevices];

void free_buffers(Staging& st)
{
    for (int b = 0; b < kBuffers; ++b) {
        cudaFree(st.q[b]); cudaFree(st.k[b]); cudaFree(st.v[b]); cudaFree(st.o[b]);
        st.q[b] = st.k[b] = st.v[b] = st.o[b] = nullptr;
    }
    st.capacity = 0;
}

// Streams and events that were created are destroyed again, so a failed set-up leaves
// nothing behind and the next call starts over cleanly.
void destroy_streams(Staging& st)
{
    for (cudaStream_t* s : {&st.in, &st.compute, &st.out}) {
        if (*s != nullptr) cudaStreamDestroy(*s);
        *s = nullptr;
    }
    for (int b = 0; b < kBuffers; ++b) {
        for (cudaEvent_t* e : {&st.loaded[b], &st.computed[b], &st.stored[b]}) {
            if (*e != nullptr) cudaEventDestroy(*e);
            *e = nullptr;
        }
    }
}

int ensure(Staging& st, size_t bytes)
{
    if (!st.ready) {
        bool created = cudaStreamCreateWithFlags(&st.in, cudaStreamNonBlocking) == cudaSuccess &&
                       cudaStreamCreateWithFlags(&st.compute, cudaStreamNonBlocking) == cudaSuccess &&
                       cudaStreamCreateWithFlags(&st.out, cudaStreamNonBlocking) == cudaSuccess;
        for (int b = 0; created && b < kBuffers; ++b) {
            created = cudaEventCreateWithFlags(&st.loaded[b], cudaEventDisableTiming) == cudaSuccess &&
                      cudaEventCreateWithFlags(&st.computed[b], cudaEventDisableTiming) == cudaSuccess &&
                      cudaEventCreateWithFlags(&st.stored[b], cudaEventDisableTiming) == cudaSuccess;
        }
        if (!created) {
            destroy_streams(st);
            cudaGetLastError();
            return FA_STATUS_HOST_ALLOC;
        }
        st.ready = true;
    }
    if (st.capacity >= bytes) return FA_STATUS_OK;
    free_buffers(st);
    for (int b = 0; b < kBuffers; ++b) {
        if (cudaMalloc(&st.q[b], bytes) != cudaSuccess || cudaMalloc(&st.k[b], bytes) != cudaSuccess ||
            cudaMalloc(&st.v[b], bytes) != cudaSuccess || cudaMalloc(&st.o[b], bytes) != cudaSuccess) {
            free_buffers(st);
            cudaGetLastError();
            return FA_STATUS_HOST_ALLOC;
        }
    }
    st.capacity = bytes;
    return FA_STATUS_OK;
}

}  // namespace

extern "C" {

int fa_sm100_fwd_host(const void* q_host, const void* k_host, const void* v_host, void* o_host, int batch,
                      int heads, int seq_len, int head_dim, int causal)
{
    if (q_host == nullptr || k_host == nullptr || v_host == nullptr || o_host == nullptr) return FA_STATUS_INVALID_ARGUMENT;
    if (batch <= 0 || heads <= 0 || seq_len <= 0) return FA_STATUS_INVALID_ARGUMENT;
    if (!fa_sm100_supported(head_dim)) return FA_STATUS_UNSUPPORTED;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return static_cast<int>(err);
    if (device < 0 || device >= kMaxDevices) return FA_STATUS_INVALID_ARGUMENT;

    const long long slabs = static_cast<long long>(batch) * heads;
    const size_t slab_bytes = static_cast<size_t>(seq_len) * head_dim * 2u;
    const long long per_chunk = std::max<long long>(1, std::min<long long>(slabs, kChunkTargetBytes / slab_bytes));
    const long long chunks = (slabs + per_chunk - 1) / per_chunk;

    Staging& st = g_staging[device];
    std::lock_guard<std::mutex> guard(st.lock);
    int status = ensure(st, static_cast<size_t>(per_chunk) * slab_bytes);
    if (status != FA_STATUS_OK) return status;

    const char* hq = static_cast<const char*>(q_host);
    const char* hk = static_cast<const char*>(k_host);
    const char* hv = static_cast<const char*>(v_host);
    char* ho = static_cast<char*>(o_host);

    for (long long c = 0; c < chunks; ++c) {
        const int b = static_cast<int>(c % kBuffers);
        const long long first = c * per_chunk;
        const long long count = std::min(per_chunk, slabs - first);
        const size_t offset = static_cast<size_t>(first) * slab_bytes;
        const size_t bytes = static_cast<size_t>(count) * slab_bytes;

        // q/k/v of buffer b are free once the forward two chunks back finished.
        if (c >= kBuffers && (err = cudaStreamWaitEvent(st.in, st.computed[b], 0)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(st.q[b], hq + offset, bytes, cudaMemcpyHostToDevice, st.in)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(st.k[b], hk + offset, bytes, cudaMemcpyHostToDevice, st.in)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(st.v[b], hv + offset, bytes, cudaMemcpyHostToDevice, st.in)) != cudaSuccess) break;
        if ((err = cudaEventRecord(st.loaded[b], st.in)) != cudaSuccess) break;

        // o of buffer b is free once its D2H two chunks back finished.
        if ((err = cudaStreamWaitEvent(st.compute, st.loaded[b], 0)) != cudaSuccess) break;
        if (c >= kBuffers && (err = cudaStreamWaitEvent(st.compute, st.stored[b], 0)) != cudaSuccess) break;
        // The chunk is a self-contained [count, 1, seq_len, head_dim] problem.
        status = fa_sm100_fwd(st.q[b], st.k[b], st.v[b], st.o[b], static_cast<int>(count), 1, seq_len, head_dim,
                              causal, st.compute);
        if (status != FA_STATUS_OK) break;
        if ((err = cudaEventRecord(st.computed[b], st.compute)) != cudaSuccess) break;

        if ((err = cudaStreamWaitEvent(st.out, st.computed[b], 0)) != cudaSuccess) break;
        if ((err = cudaMemcpyAsync(ho + offset, st.o[b], bytes, cudaMemcpyDeviceToHost, st.out)) != cudaSuccess) break;
        if ((err = cudaEventRecord(st.stored[b], st.out)) != cudaSuccess) break;
    }
    const cudaError_t sync_in = cudaStreamSynchronize(st.in);
    const cudaError_t sync_compute = cudaStreamSynchronize(st.compute);
    const cudaError_t sync_out = cudaStreamSynchronize(st.out);
    if (status != FA_STATUS_OK) return status;
    if (err != cudaSuccess) return static_cast<int>(err);
    if (sync_in != cudaSuccess) return static_cast<int>(sync_in);
    if (sync_compute != cudaSuccess) return static_cast<int>(sync_compute);
    if (sync_out != cudaSuccess) return static_cast<int>(sync_out);
    // A launch that gave up on a bounded wait left some of its O rows unwritten: report it
    // instead of returning those rows as a result.
    return fa_sm100_internal::take_error_word(st.compute, nullptr);
}

int fa_sm100_release_staging(void)
{
    int device = 0;
    const cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return static_cast<int>(err);
    if (device < 0 || device >= kMaxDevices) return FA_STATUS_INVALID_ARGUMENT;
    Staging& st = g_staging[device];
    std::lock_guard<std::mutex> guard(st.lock);
    cudaDeviceSynchronize();
    free_buffers(st);
    return FA_STATUS_OK;
}

}  // extern "C"
