// =============================================================================
// CPU FP64 attention oracle -- TEST INFRASTRUCTURE ONLY.
//
// This file is the checker for the sm_100a kernel in cuda_fused_attention_b200/.
// It is never linked into the product library and the product never calls it.
// Only tests/, __graft_entry__.smoke() and the cpu_baseline / reference legs of
// bench.py load it.
//
// It restates, in plain C++, the correctness machinery that the reference
// (RichterWang/cuda_fused_attention) keeps inside its benchmark executable:
//
//   fill_normal          benchmarks/bench_flash_attention.cu:86-92
//   bf16_ulp             benchmarks/bench_flash_attention.cu:95-102
//   reference_attention  benchmarks/bench_flash_attention.cu:105-145
//   compare / Accuracy   benchmarks/bench_flash_attention.cu:148-218
//   attention_flops      kernels/v0_unfused.cu:118-126
//   input families       kernels/ablation/experiments.cu:283-289
//
// The arithmetic has to be alike for the restatement to be bit-exact: bf16
// inputs are widened to double, the dot product accumulates in double in key
// order, the scale is double(float(1/sqrt(D))), the row max starts at -1e300,
// the exponentials are std::exp of the max-subtracted scores, and the output is
// (sum_k p_k v_k) / (sum_k p_k) accumulated in key order. The inputs come from
// std::mt19937 + std::normal_distribution<float>, rounded to bf16 with the
// CUDA host conversion, exactly like the reference generator.
//
// Pinning: tests/golden/golden.json holds SHA-256 digests of the inputs and of
// the FP64 outputs produced by the reference's own functions (compiled from the
// reference sources into oracle/_ref by oracle/Makefile). tests/test_oracle.py
// recomputes them here and requires bit equality.
// =============================================================================

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <thread>
#include <vector>

namespace {

inline float bf16_bits_to_float(uint16_t bits)
{
    __nv_bfloat16_raw raw;
    raw.x = bits;
    return __bfloat162float(__nv_bfloat16(raw));
}

inline uint16_t float_to_bf16_bits(float value)
{
    const __nv_bfloat16_raw raw = static_cast<__nv_bfloat16_raw>(__float2bfloat16(value));
    return raw.x;
}

// One (batch*head) slab, query rows [row_begin, row_end). out points at the
// slab's first output row (row_begin's output goes to out + row_begin * d).
// Follows bench_flash_attention.cu:113-143 statement for statement.
void attention_slab_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                         int n, int d, bool causal, double scale, int row_begin, int row_end,
                         std::vector<double>& scores)
{
    for (int query = row_begin; query < row_end; ++query)
    {
        const int limit = causal ? query + 1 : n;

        double row_max = -1.0e300;
        for (int key = 0; key < limit; ++key)
        {
            double dot = 0.0;
            const uint16_t* q_row = q + static_cast<size_t>(query) * d;
            const uint16_t* k_row = k + static_cast<size_t>(key) * d;
            for (int dim = 0; dim < d; ++dim)
                dot += static_cast<double>(bf16_bits_to_float(q_row[dim])) *
                       static_cast<double>(bf16_bits_to_float(k_row[dim]));
            scores[key] = dot * scale;
            row_max = std::max(row_max, scores[key]);
        }

        double sum = 0.0;
        for (int key = 0; key < limit; ++key)
        {
            scores[key] = std::exp(scores[key] - row_max);
            sum += scores[key];
        }

        for (int dim = 0; dim < d; ++dim)
        {
            double accumulator = 0.0;
            for (int key = 0; key < limit; ++key)
                accumulator += scores[key] * static_cast<double>(bf16_bits_to_float(v[static_cast<size_t>(key) * d + dim]));
            out[static_cast<size_t>(query) * d + dim] = accumulator / sum;
        }
    }
}

// default_scale (include/flash_attention.h:21-24) widened to double the way
// the oracle does it (bench_flash_attention.cu:109).
inline double oracle_scale(int d)
{
    return static_cast<double>(1.0f / std::sqrt(static_cast<float>(d)));
}

}  // namespace

extern "C" {

// Per-kernel accuracy summary; the fields and their meaning follow the
// reference's Accuracy struct (bench_flash_attention.cu:148-164).
struct FaOracleAccuracy
{
    double vs_double;
    double row_scaled;
    double max_abs;
    double ulp;
    double mean_abs;
    double mean_ulp;
    uint64_t output_nan;
    uint64_t output_inf;
    uint64_t reference_nan;
    uint64_t reference_inf;
    int passed;
};

float fa_oracle_bf16_to_float(uint16_t bits) { return bf16_bits_to_float(bits); }
uint16_t fa_oracle_float_to_bf16(float value) { return float_to_bf16_bits(value); }

// bench_flash_attention.cu:86-92
void fa_oracle_fill_normal(uint16_t* out, size_t count, unsigned seed)
{
    std::mt19937 engine(seed);
    std::normal_distribution<float> dist(0.0f, 1.0f);
    for (size_t i = 0; i < count; ++i) out[i] = float_to_bf16_bits(dist(engine));
}

// Input families of kernels/ablation/experiments.cu:283-289, applied in place to
// q/k/v that were filled with seeds 11/22/33:
//   0 random N(0,1); 1 all zero; 2 all one; 3 V = (i mod d) - d/2;
//   4 Q and K multiplied by 4 (large logits).
// Family 5 is BASELINE config 3: only Q multiplied by 4.
void fa_oracle_apply_family(uint16_t* q, uint16_t* k, uint16_t* v, size_t count, int head_dim, int family)
{
    for (size_t i = 0; i < count; ++i)
    {
        switch (family)
        {
            case 1: q[i] = k[i] = v[i] = float_to_bf16_bits(0.0f); break;
            case 2: q[i] = k[i] = v[i] = float_to_bf16_bits(1.0f); break;
            case 3: v[i] = float_to_bf16_bits(static_cast<float>(static_cast<int>(i % head_dim) - head_dim / 2)); break;
            case 4:
                q[i] = float_to_bf16_bits(bf16_bits_to_float(q[i]) * 4.0f);
                k[i] = float_to_bf16_bits(bf16_bits_to_float(k[i]) * 4.0f);
                break;
            case 5: q[i] = float_to_bf16_bits(bf16_bits_to_float(q[i]) * 4.0f); break;
            default: break;
        }
    }
}

// bench_flash_attention.cu:95-102 (with the 2^-133 floor of the main harness)
float fa_oracle_bf16_ulp(float value)
{
    if (value == 0.0f || !std::isfinite(value)) return std::ldexp(1.0f, -126 - 7);
    int exponent = 0;
    std::frexp(std::abs(value), &exponent);
    return std::ldexp(1.0f, std::max(exponent - 8, -133));
}

// kernels/v0_unfused.cu:118-126
double fa_oracle_attention_flops(int batch, int heads, int seq_len, int head_dim, int causal)
{
    const double n = static_cast<double>(seq_len);
    const double pairs = causal ? n * (n + 1.0) / 2.0 : n * n;
    return 4.0 * pairs * static_cast<double>(head_dim) * static_cast<double>(batch) * static_cast<double>(heads);
}

// Whole-tensor oracle, single thread: bench_flash_attention.cu:105-145.
void fa_oracle_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                         int batch, int heads, int seq_len, int head_dim, int causal)
{
    const int n = seq_len;
    const int d = head_dim;
    const double scale = oracle_scale(d);
    std::vector<double> scores(static_cast<size_t>(n));
    for (int bh = 0; bh < batch * heads; ++bh)
    {
        const size_t slab = static_cast<size_t>(bh) * n * d;
        attention_slab_rows(q + slab, k + slab, v + slab, out + slab, n, d, causal != 0, scale, 0, n, scores);
    }
}

// Query rows [row_begin, row_end) of one slab; out receives (row_end-row_begin)*d
// values. Same arithmetic as above; used to sample rows at large configs.
void fa_oracle_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                              int seq_len, int head_dim, int causal, long long slab,
                              int row_begin, int row_end)
{
    const int n = seq_len;
    const int d = head_dim;
    const size_t base = static_cast<size_t>(slab) * n * d;
    std::vector<double> scores(static_cast<size_t>(n));
    std::vector<double> rows(static_cast<size_t>(n) * d);
    attention_slab_rows(q + base, k + base, v + base, rows.data(), n, d, causal != 0,
                        oracle_scale(d), row_begin, row_end, scores);
    std::memcpy(out, rows.data() + static_cast<size_t>(row_begin) * d,
                sizeof(double) * static_cast<size_t>(row_end - row_begin) * d);
}

// Slab-parallel oracle over `threads` host threads: slabs [slab_begin, slab_end)
// are dealt round-robin. Every slab costs the same, so this scales with cores.
void fa_oracle_attention_parallel(const uint16_t* q, const uint16_t* k, const uint16_t* v, double* out,
                                  int seq_len, int head_dim, int causal,
                                  long long slab_begin, long long slab_end, int threads)
{
    const int n = seq_len;
    const int d = head_dim;
    const double scale = oracle_scale(d);
    threads = std::max(1, threads);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
    {
        pool.emplace_back([=]() {
            std::vector<double> scores(static_cast<size_t>(n));
            for (long long bh = slab_begin + t; bh < slab_end; bh += threads)
            {
                const size_t slab = static_cast<size_t>(bh) * n * d;
                attention_slab_rows(q + slab, k + slab, v + slab, out + slab, n, d, causal != 0, scale, 0, n, scores);
            }
        });
    }
    for (auto& worker : pool) worker.join();
}

// bench_flash_attention.cu:167-218 over `rows` rows of width head_dim. The mean
// columns are additions for the multi-row summaries the bench reports.
void fa_oracle_compare(const uint16_t* device_out, const double* reference, long long rows, int head_dim,
                       double ulp_tolerance, FaOracleAccuracy* result_out)
{
    FaOracleAccuracy result{};
    const int d = head_dim;
    double sum_abs = 0.0;
    double sum_ulp = 0.0;
    size_t finite_count = 0;

    for (long long row = 0; row < rows; ++row)
    {
        const size_t base = static_cast<size_t>(row) * d;

        double row_scale = 0.0;
        for (int dim = 0; dim < d; ++dim)
            if (std::isfinite(reference[base + dim]))
                row_scale = std::max(row_scale, std::abs(reference[base + dim]));

        const float scale_ulp = fa_oracle_bf16_ulp(static_cast<float>(row_scale));

        for (int dim = 0; dim < d; ++dim)
        {
            const float got = bf16_bits_to_float(device_out[base + dim]);
            const double want = reference[base + dim];

            result.output_nan += std::isnan(got);
            result.output_inf += std::isinf(got);
            result.reference_nan += std::isnan(want);
            result.reference_inf += std::isinf(want);
            if (!std::isfinite(got) || !std::isfinite(want))
            {
                result.vs_double = result.row_scaled = result.max_abs = result.ulp =
                    std::numeric_limits<double>::infinity();
                continue;
            }

            const double abs_error = std::abs(static_cast<double>(got) - want);
            const double denominator = std::max(std::abs(want), 1.0e-6);
            result.vs_double = std::max(result.vs_double, abs_error / denominator);
            result.max_abs = std::max(result.max_abs, abs_error);
            result.row_scaled = std::max(result.row_scaled, abs_error / std::max(row_scale, 1.0e-6));

            const float rounded = bf16_bits_to_float(float_to_bf16_bits(static_cast<float>(want)));
            const double ulp = std::abs(static_cast<double>(got) - rounded) / scale_ulp;
            result.ulp = std::max(result.ulp, ulp);
            sum_abs += abs_error;
            sum_ulp += ulp;
            ++finite_count;
        }
    }

    result.mean_abs = finite_count ? sum_abs / static_cast<double>(finite_count) : 0.0;
    result.mean_ulp = finite_count ? sum_ulp / static_cast<double>(finite_count) : 0.0;
    result.passed = result.output_nan == 0 && result.output_inf == 0 && result.reference_nan == 0 &&
                    result.reference_inf == 0 && std::isfinite(result.ulp) && result.ulp <= ulp_tolerance;
    *result_out = result;
}

}  // extern "C"
