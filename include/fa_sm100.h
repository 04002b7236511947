/*
 * fa_sm100.h -- C ABI of the Blackwell (sm_100a) fused attention forward pass.
 *
 * Plain C: pointers, ints and sizes only, no CUDA or torch types in the
 * signatures (a stream is passed as void* and is a cudaStream_t; NULL means the
 * legacy default stream, which is what the reference harness passes).
 *
 * The computation is the reference's hot path
 *     O = softmax(Q K^T / sqrt(D) + M) V
 * over contiguous BF16 tensors laid out [batch, heads, seq_len, head_dim] with
 * head_dim innermost, FP32 accumulation, M = 0 (dense) or the top-left aligned
 * causal mask key <= query. It replaces, one for one, the launch API declared in
 * the reference's include/flash_attention.h (namespace cuda_op_lab::flash_attention);
 * each entry point below names the reference symbol it stands in for.
 *
 * Status codes: 0 on success; a value in (0, 1000) is a cudaError_t returned by
 * the CUDA runtime; values >= 1000 are the FA_STATUS_* codes below.
 */
#ifndef FA_SM100_H
#define FA_SM100_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FA_STATUS_OK                 0
#define FA_STATUS_INVALID_ARGUMENT   1001 /* null pointer, non-positive dimension, size overflow */
#define FA_STATUS_UNSUPPORTED        1002 /* head_dim not in {64, 128} */
#define FA_STATUS_MISALIGNED         1003 /* a tensor base is not 16-byte aligned */
#define FA_STATUS_NO_SM100           1004 /* current device is not compute capability 10.x */
#define FA_STATUS_DRIVER_ENTRY       1005 /* cuTensorMapEncodeTiled could not be resolved */
#define FA_STATUS_TENSOR_MAP         1006 /* cuTensorMapEncodeTiled rejected a tensor */
#define FA_STATUS_DEVICE_TIMEOUT     1007 /* a device-side bounded wait ran out (see fa_sm100_device_status) */
#define FA_STATUS_HOST_ALLOC         1008 /* pinned/device staging memory could not be obtained */
#define FA_STATUS_BUILD_MISMATCH     1009 /* kernel registers at launch cannot cover its warpgroup split */
#define FA_STATUS_STATIC_TOO_LARGE   1010 /* a slab exceeds the fixed staging of fa_sm100_fwd_host_static */

/* Resource report; same fields and meaning as the reference's FusedTilingInfo
 * (include/flash_attention.h:60-72). */
typedef struct FaTilingInfo {
    int supported;
    int block_size;
    int tile_kv;
    int rows_per_block;
    int shared_bytes_per_block;
    int registers_per_thread;
    int local_bytes_per_thread;
    int max_blocks_per_sm;
    int device_shared_bytes_per_sm;
    int shared_limited_blocks_per_sm;
} FaTilingInfo;

/* Forward pass on the current device, asynchronous on `stream`.
 * Replaces launch_attention_tensorcore_v3 (include/flash_attention.h:92,
 * kernels/v3/v3_tensorcore.cu:722-750). q, k, v, o: device pointers, 16-byte
 * aligned, each batch*heads*seq_len*head_dim bf16 elements. Every element of o
 * is written. o may be q (O written over Q) and k may be v. A causal launch with few (batch, head) slabs and long rows may
 * split the key range of its heaviest row pairs across several CTAs; such a
 * launch takes its workspace (partials of the split rows) from a memory pool
 * of the library, allocated and freed in order on `stream` (stream-ordered
 * allocation, so concurrent launches on other streams never share it). */
FA_API int fa_sm100_fwd(const void* q, const void* k, const void* v, void* o,
                 int batch, int heads, int seq_len, int head_dim, int causal, void* stream);

/* Same as fa_sm100_fwd over the slab range [slab_begin, slab_end) of the
 * flattened batch*heads axis: the per-GPU shard of a multi-GPU call. Pointers
 * are the bases of the full tensors. No reference counterpart (the reference
 * is single-GPU); it is the unit the multi-GPU driver partitions. */
FA_API int fa_sm100_fwd_slabs(const void* q, const void* k, const void* v, void* o,
                       int batch, int heads, int seq_len, int head_dim, int causal,
                       long long slab_begin, long long slab_end, void* stream);

/* Replaces tensorcore_v3_supported (include/flash_attention.h:90). 1 or 0. */
FA_API int fa_sm100_supported(int head_dim);

/* Replaces query_tensorcore_v3 (include/flash_attention.h:94). Returns a status. */
FA_API int fa_sm100_query(int head_dim, FaTilingInfo* info);

/* Replaces tensorcore_v3_hbm_bytes (include/flash_attention.h:96): algorithmic
 * DRAM traffic model with the same accounting (Q read once, O written once, a
 * K and a V tile per CTA per key tile it visits). */
FA_API double fa_sm100_hbm_bytes(int batch, int heads, int seq_len, int head_dim, int causal);

/* Minimum DRAM traffic of the operation: Q, K, V read once and O written once. */
FA_API double fa_sm100_min_bytes(int batch, int heads, int seq_len, int head_dim);

/* attention_flops (include/flash_attention.h:27, kernels/v0_unfused.cu:118-126):
 * 4*B*H*D*pairs with pairs = N^2 dense, N(N+1)/2 causal. */
FA_API double fa_attention_flops(int batch, int heads, int seq_len, int head_dim, int causal);

/* default_scale (include/flash_attention.h:21-24): 1/sqrt(head_dim) in float. */
FA_API float fa_default_scale(int head_dim);

/* Reads and clears the device-side error word of the current device after a
 * device synchronisation. FA_STATUS_OK, FA_STATUS_DEVICE_TIMEOUT, or a
 * cudaError_t from the synchronisation. `detail` (may be NULL) receives the raw
 * word: bit 0 set by any timeout, bits 8..15 the id of the wait that gave up.
 * There is one word per device, shared by every launch, stream and host thread
 * on it: with concurrent callers, a timeout is reported to whichever caller
 * reads the word first (this call, or fa_sm100_fwd_host /
 * fa_sm100_fwd_host_static, which read and clear it after their own work). */
FA_API int fa_sm100_device_status(unsigned int* detail);

/* Debug builds only (libfa_sm100_debug.so, compiled with FA_SM100_DEBUG_DUMP; the
 * counterpart of the reference's FA_V3_DEBUG_DUMP option, kernels/v3/v3_tensorcore.cu:
 * 101, :189-204, :680-709): CTA 0 of each launch writes what its first Q tile sees at
 * each stage of the tcgen05 path, and this call copies the last launch's dump to `out`
 * (FA_SM100_DEBUG_FLOATS floats, row major):
 *   [FA_SM100_DEBUG_S + 128*r + k]  QK^T of query row r of the tile and key k of key tile 0,
 *                                   as loaded from TMEM, before scale and mask
 *   [FA_SM100_DEBUG_P + 128*r + k]  P of the same element as the PV MMA reads it (bf16 -> f32)
 *   [FA_SM100_DEBUG_O + 128*r + d]  O after the last PV, before the 1/l scaling
 *   [FA_SM100_DEBUG_L + r]          row sum l;  [FA_SM100_DEBUG_M + r] final row max
 *   [FA_SM100_DEBUG_INFO + 0..7]    slab, first query row of the tile, seq_len, head_dim,
 *                                   causal, one-tile kernel (0/1), key tiles, 1
 * The product library returns FA_STATUS_UNSUPPORTED. */
#define FA_SM100_DEBUG_S      0
#define FA_SM100_DEBUG_P      16384
#define FA_SM100_DEBUG_O      32768
#define FA_SM100_DEBUG_L      49152
#define FA_SM100_DEBUG_M      49280
#define FA_SM100_DEBUG_INFO   49408
#define FA_SM100_DEBUG_FLOATS 49416
FA_API int fa_sm100_debug_read(float* out, size_t floats);

/* Human-readable text for a status code. */
FA_API const char* fa_sm100_status_string(int status);

/* Test-only entry: the forward pass with a stall injected into the MMA warp
 * (it waits on a barrier that nothing arrives on) and the bounded-wait limit
 * set to timeout_ns. The kernel must give up, report FA_STATUS_DEVICE_TIMEOUT
 * through fa_sm100_device_status, release its tensor memory and return.
 * No reference counterpart. */
FA_API int fa_sm100_fwd_inject_stall(const void* q, const void* k, const void* v, void* o,
                              int batch, int heads, int seq_len, int head_dim, int causal,
                              unsigned long long timeout_ns, void* stream);

/* Test-only: arms a stall (as in fa_sm100_fwd_inject_stall, with limit
 * timeout_ns, at most one second) for the next forward launch that this host
 * thread makes through any entry point, so that tests can check how the
 * host-buffer entries report a device-side timeout. One-shot. No reference
 * counterpart. */
FA_API int fa_sm100_test_arm_stall(unsigned long long timeout_ns);

/* Test-only: which kernel instantiation this host thread's launches use -- 0 the
 * launcher's own choice (the default), 1 one 128-row Q tile per CTA, 2 a row pair
 * (two Q tiles) per CTA -- so that tests can run both on the same shapes. Stays set
 * until changed. No reference counterpart. */
FA_API int fa_sm100_test_force_kernel(int kind);

/* Test-only: the causal key-range split for this host thread's launches of the row-pair
 * kernel -- -1 the launcher's own choice (the default), 0 never, L > 0 every row pair with
 * more than L key tiles is processed by several CTAs of at most L key tiles each, whose
 * partial results the last of them merges (L is raised where a pair would need more than
 * 64 chunks). Stays set until changed. No reference counterpart. */
FA_API int fa_sm100_test_force_split(int split_len);

/* End-to-end call with HOST buffers (pageable or pinned): copies Q/K/V in,
 * runs the forward pass and copies O out, pipelined over slab chunks on two
 * streams of the current device, then synchronises. Uses staging buffers that
 * the library allocates on first use and keeps (see fa_sm100_release_staging).
 * If a launch gave up on a bounded device-side wait, the call returns
 * FA_STATUS_DEVICE_TIMEOUT (it reads and clears the device error word) and
 * o_host is incomplete.
 * No reference counterpart: the reference harness does these copies itself
 * (benchmarks/bench_flash_attention.cu:545-560). */
FA_API int fa_sm100_fwd_host(const void* q_host, const void* k_host, const void* v_host, void* o_host,
                      int batch, int heads, int seq_len, int head_dim, int causal);

/* Frees the staging buffers of fa_sm100_fwd_host on the current device. */
FA_API int fa_sm100_release_staging(void);

/* Host-buffer forward pass that allocates nothing, for callers that cannot
 * allocate device memory (no cudaMalloc/cudaFree, no stream or event creation,
 * no allocating library routine). No counterpart in the reference. Same result
 * as fa_sm100_fwd_host; Q/K/V/O are staged through one fixed 32 MiB file-scope
 * __device__ array (fa_sm100_static_staging_bytes()) that every GPU loading the
 * library holds until exit, one slab (seq_len*head_dim bf16) at most 8 MiB,
 * else FA_STATUS_STATIC_TOO_LARGE. Runs on `stream` (NULL = legacy default)
 * and synchronises it. The first call on a device resolves the array's device
 * address (cudaGetSymbolAddress) with that device current: make it before any
 * stream capture. Under lazy module loading (CUDA's default) that first call
 * is also when the module holding the array is loaded, which allocates its
 * 32 MiB: a caller that forbids allocation after start-up makes one call at
 * start-up. A device-side timeout is returned as FA_STATUS_DEVICE_TIMEOUT
 * (o_host is then not a result). All calls share the array: calls that
 * overlap on the GPU race, so serialise them. */
FA_API int fa_sm100_fwd_host_static(const void* q_host, const void* k_host, const void* v_host, void* o_host,
                                    int batch, int heads, int seq_len, int head_dim, int causal, void* stream);

/* Size in bytes of the fixed staging array used by fa_sm100_fwd_host_static. */
FA_API size_t fa_sm100_static_staging_bytes(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* FA_SM100_H */
