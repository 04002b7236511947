// flash_attention_sm100.h -- C++ launch API of the sm_100a fused attention
// forward pass, in the reference's namespace and with the reference's shapes.
//
// It adds one variant to the API of the reference's include/flash_attention.h
// (namespace cuda_op_lab::flash_attention), with the same four-function pattern
// as its tensor-core kernel (include/flash_attention.h:90-96):
//
//   sm100_supported         <-> tensorcore_v3_supported
//   launch_attention_sm100  <-> launch_attention_tensorcore_v3
//   query_sm100             <-> query_tensorcore_v3
//   sm100_hbm_bytes         <-> tensorcore_v3_hbm_bytes
//
// Built inside the reference tree (its include/ on the include path), the
// reference's own AttentionShape / FusedTilingInfo / default_scale /
// attention_flops are used. Built standalone, layout-identical definitions
// are provided below so that either way the structs are the same bytes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "fa_sm100.h"

#if __has_include("flash_attention.h") && !defined(FA_SM100_STANDALONE)
#include "flash_attention.h"
#else
namespace cuda_op_lab::flash_attention {

struct AttentionShape
{
    int batch;
    int heads;
    int seq_len;   // query and key/value length (self-attention)
    int head_dim;  // 64 or 128
};

inline float default_scale(int head_dim) { return 1.0f / std::sqrt(static_cast<float>(head_dim)); }

inline double attention_flops(const AttentionShape& shape, bool causal)
{
    return fa_attention_flops(shape.batch, shape.heads, shape.seq_len, shape.head_dim, causal ? 1 : 0);
}

struct FusedTilingInfo
{
    bool supported;
    int block_size;
    int tile_kv;
    int rows_per_block;
    int shared_bytes_per_block;
    int registers_per_thread;
    int local_bytes_per_thread;
    int max_blocks_per_sm;
    int device_shared_bytes_per_sm;
    int shared_limited_blocks_per_sm;
};

}  // namespace cuda_op_lab::flash_attention
#endif

namespace cuda_op_lab::flash_attention {

// head_dim 64 or 128.
FA_API bool sm100_supported(int head_dim);

// Asynchronous on `stream`, like every reference launcher. Unsupported head_dim
// returns without launching (as launch_attention_tensorcore_v3 does). Any other
// rejected argument also launches nothing; its FA_STATUS_* code is kept in
// sm100_last_status() for the calling thread. Launch errors are reported there
// as well (the library links its own CUDA runtime, so its launch errors are not
// visible to the caller's cudaGetLastError()).
FA_API void launch_attention_sm100(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                                   __nv_bfloat16* o, const AttentionShape& shape, bool causal,
                                   cudaStream_t stream = nullptr);

// Status of the calling thread's last launch_attention_sm100 (0 = ok).
FA_API int sm100_last_status();

FA_API FusedTilingInfo query_sm100(int head_dim);

FA_API double sm100_hbm_bytes(const AttentionShape& shape, bool causal);

}  // namespace cuda_op_lab::flash_attention
