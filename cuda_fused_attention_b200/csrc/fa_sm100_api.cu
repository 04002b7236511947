// C++ launch API (include/flash_attention_sm100.h) over the C ABI (include/fa_sm100.h).
// Mirrors the reference's four-function pattern for a kernel variant
// (include/flash_attention.h:90-96, kernels/v3/v3_tensorcore.cu:717-818).
#define FA_SM100_STANDALONE 1
#include "flash_attention_sm100.h"

namespace cuda_op_lab::flash_attention {

namespace {
thread_local int t_last_status = FA_STATUS_OK;
}

bool sm100_supported(int head_dim) { return fa_sm100_supported(head_dim) != 0; }

void launch_attention_sm100(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                            __nv_bfloat16* o, const AttentionShape& shape, bool causal, cudaStream_t stream)
{
    if (!sm100_supported(shape.head_dim)) {
        t_last_status = FA_STATUS_UNSUPPORTED;
        return;
    }
    t_last_status = fa_sm100_fwd(q, k, v, o, shape.batch, shape.heads, shape.seq_len, shape.head_dim,
                                 causal ? 1 : 0, static_cast<void*>(stream));
}

int sm100_last_status() { return t_last_status; }

FusedTilingInfo query_sm100(int head_dim)
{
    FaTilingInfo raw{};
    FusedTilingInfo info{};
    if (fa_sm100_query(head_dim, &raw) != FA_STATUS_OK) return info;
    info.supported = raw.supported != 0;
    info.block_size = raw.block_size;
    info.tile_kv = raw.tile_kv;
    info.rows_per_block = raw.rows_per_block;
    info.shared_bytes_per_block = raw.shared_bytes_per_block;
    info.registers_per_thread = raw.registers_per_thread;
    info.local_bytes_per_thread = raw.local_bytes_per_thread;
    info.max_blocks_per_sm = raw.max_blocks_per_sm;
    info.device_shared_bytes_per_sm = raw.device_shared_bytes_per_sm;
    info.shared_limited_blocks_per_sm = raw.shared_limited_blocks_per_sm;
    return info;
}

double sm100_hbm_bytes(const AttentionShape& shape, bool causal)
{
    return fa_sm100_hbm_bytes(shape.batch, shape.heads, shape.seq_len, shape.head_dim, causal ? 1 : 0);
}

}  // namespace cuda_op_lab::flash_attention
