// =============================================================================
// Reference shim -- TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, never shipped).
//
// The reference keeps its CPU FP64 oracle, its generator and its comparison in
// an anonymous namespace inside the benchmark executable's translation unit
// (benchmarks/bench_flash_attention.cu:20-389). To call those functions
// unmodified, this shim compiles that translation unit in place (from the
// reference tree, -I<reference root>) with its main() renamed, and exports
// C wrappers around the functions. It also exports the reference's own
// tensor-core kernel (kernels/v3/v3_tensorcore.cu:722) and its unfused kernel
// (kernels/v0_unfused.cu:140) built for sm_100a, as GPU second opinions.
//
// oracle/Makefile is the recipe; nothing from the reference is copied here.
// =============================================================================

#define main fa_reference_benchmark_main
#include "benchmarks/bench_flash_attention.cu"
#undef main

#include <cstdint>
#include <cstring>
#include <vector>

namespace {

std::vector<__nv_bfloat16> to_bf16_vector(const uint16_t* bits, size_t count)
{
    std::vector<__nv_bfloat16> out(count);
    std::memcpy(out.data(), bits, count * sizeof(uint16_t));
    return out;
}

}  // namespace

extern "C" {

void ref_fill_normal(uint16_t* out, size_t count, unsigned seed)
{
    std::vector<__nv_bfloat16> host(count);
    fill_normal(host, seed);
    std::memcpy(out, host.data(), count * sizeof(uint16_t));
}

float ref_bf16_ulp(float value) { return bf16_ulp(value); }

void ref_reference_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                             int batch, int heads, int seq_len, int head_dim, int causal)
{
    const size_t count = static_cast<size_t>(batch) * heads * seq_len * head_dim;
    const auto hq = to_bf16_vector(q, count);
    const auto hk = to_bf16_vector(k, count);
    const auto hv = to_bf16_vector(v, count);
    std::vector<double> reference(count);
    reference_attention(hq, hk, hv, reference, AttentionShape{batch, heads, seq_len, head_dim}, causal != 0);
    std::memcpy(out, reference.data(), count * sizeof(double));
}

// Returns the reference's Accuracy fields in a plain array:
// {vs_double, row_scaled, max_abs, ulp, out_nan, out_inf, ref_nan, ref_inf, passed}
void ref_compare(const uint16_t* device_out, const double* reference_values,
                 int batch, int heads, int seq_len, int head_dim, double* fields)
{
    const size_t count = static_cast<size_t>(batch) * heads * seq_len * head_dim;
    const auto got = to_bf16_vector(device_out, count);
    const std::vector<double> want(reference_values, reference_values + count);
    const Accuracy accuracy = compare(got, want, AttentionShape{batch, heads, seq_len, head_dim});
    fields[0] = accuracy.vs_double;
    fields[1] = accuracy.row_scaled;
    fields[2] = accuracy.max_abs;
    fields[3] = accuracy.ulp;
    fields[4] = static_cast<double>(accuracy.output_nan);
    fields[5] = static_cast<double>(accuracy.output_inf);
    fields[6] = static_cast<double>(accuracy.reference_nan);
    fields[7] = static_cast<double>(accuracy.reference_inf);
    fields[8] = accuracy.passed() ? 1.0 : 0.0;
}

double ref_attention_flops(int batch, int heads, int seq_len, int head_dim, int causal)
{
    return attention_flops(AttentionShape{batch, heads, seq_len, head_dim}, causal != 0);
}

double ref_tensorcore_v3_hbm_bytes(int batch, int heads, int seq_len, int head_dim, int causal)
{
    return tensorcore_v3_hbm_bytes(AttentionShape{batch, heads, seq_len, head_dim}, causal != 0);
}

int ref_tensorcore_v3_supported(int head_dim) { return tensorcore_v3_supported(head_dim) ? 1 : 0; }

// The reference's launchers return void; the caller polls cudaGetLastError.
int ref_launch_tensorcore_v3(const void* q, const void* k, const void* v, void* o,
                             int batch, int heads, int seq_len, int head_dim, int causal, void* stream)
{
    launch_attention_tensorcore_v3(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                                   static_cast<const __nv_bfloat16*>(v), static_cast<__nv_bfloat16*>(o),
                                   AttentionShape{batch, heads, seq_len, head_dim}, causal != 0,
                                   static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

size_t ref_unfused_workspace_bytes(int batch, int heads, int seq_len, int head_dim)
{
    return unfused_workspace_bytes(AttentionShape{batch, heads, seq_len, head_dim});
}

int ref_launch_unfused(const void* q, const void* k, const void* v, void* o, void* workspace,
                       int batch, int heads, int seq_len, int head_dim, int causal, void* stream)
{
    launch_attention_unfused(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                             static_cast<const __nv_bfloat16*>(v), static_cast<__nv_bfloat16*>(o),
                             static_cast<float*>(workspace), AttentionShape{batch, heads, seq_len, head_dim},
                             causal != 0, static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
