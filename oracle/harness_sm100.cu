// =============================================================================
// The reference harness with the sm_100a kernel as one more Entry -- TEST
// INFRASTRUCTURE ONLY (built into oracle/_ref/, never shipped).
//
// A maintainer adopts the kernel by adding a runner and an Entry to the
// reference's benchmarks/bench_flash_attention.cu (runners :342-370, Entry and
// kEntries :372-387) and linking the library. This program does exactly that
// without editing the reference: it compiles that translation unit in place
// (from the reference tree, -I<reference root>) with its main() renamed,
// defines the runner and the Entry the way the file defines its own, and runs
// the file's two procedures over the selected entries:
//   * the accuracy suite (:507-586): shape (1, 2, 256, D), D in {64, 128},
//     dense and causal, inputs fill_normal(11/22/33), output NaN-poisoned,
//     compare() against reference_attention() with the 2.0-ULP row-scale gate;
//   * the performance loop (:588-700): for each case, fill_normal inputs,
//     time_iterations() (5 warm-ups, 30 event-timed launches, median and IQR),
//     NaN/Inf count of the output, speed-up against v0 as the harness reports it.
// flash_attention_sm100.h sees the reference's include/ here and so takes the
// reference's own AttentionShape and FusedTilingInfo: the program links and
// runs only if the library's C++ API is ABI-compatible with those types.
//
// usage: harness_sm100 --host-only
//            host functions through the reference types; no CUDA call.
//        harness_sm100 [--entries name,name,...] [--cases grid | B,H,N,D,causal[;...]]
//            entries default to every reference entry plus sm100_tcgen05; cases
//            default to the harness's own grid (kCases, :75-84).
// One JSON object per line on stdout. Exit status 0 only if every accuracy
// check passed, every timed output was finite and every sm100 launch returned 0.
// =============================================================================

#define main fa_reference_harness_main
#include "benchmarks/bench_flash_attention.cu"
#undef main

#include "flash_attention_sm100.h"

#include <cstring>
#include <sstream>
#include <string>
#include <vector>

namespace {

using cuda_op_lab::flash_attention::launch_attention_sm100;
using cuda_op_lab::flash_attention::query_sm100;
using cuda_op_lab::flash_attention::sm100_hbm_bytes;
using cuda_op_lab::flash_attention::sm100_last_status;
using cuda_op_lab::flash_attention::sm100_supported;

// The runner a maintainer adds beside run_tensorcore_v3 (:366-370).
void run_sm100(void* context)
{
    Buffers& buffers = *static_cast<Buffers*>(context);
    launch_attention_sm100(buffers.q, buffers.k, buffers.v, buffers.o, buffers.shape, buffers.causal, nullptr);
}

constexpr const char* kSm100Name = "sm100_tcgen05";

// kEntries (:379-387) plus the new row.
std::vector<Entry> all_entries()
{
    std::vector<Entry> entries(std::begin(kEntries), std::end(kEntries));
    entries.push_back({kSm100Name, run_sm100, sm100_supported});
    return entries;
}

bool is_sm100(const Entry& entry) { return std::strcmp(entry.name, kSm100Name) == 0; }

// The harness's algorithmic traffic column (:643-650) for the two tensor-core
// entries; the others report none here.
double traffic_gb(const Entry& entry, const AttentionShape& shape, bool causal)
{
    if (is_sm100(entry)) return sm100_hbm_bytes(shape, causal) / 1.0e9;
    if (std::strcmp(entry.name, "v3_tensorcore") == 0) return tensorcore_v3_hbm_bytes(shape, causal) / 1.0e9;
    return -1.0;
}

std::string shape_json(const AttentionShape& shape, bool causal)
{
    std::ostringstream out;
    out << "\"batch\": " << shape.batch << ", \"heads\": " << shape.heads << ", \"seq_len\": " << shape.seq_len
        << ", \"head_dim\": " << shape.head_dim << ", \"causal\": " << (causal ? 1 : 0);
    return out.str();
}

// After a run: the launch status the library keeps for the calling thread
// (launch errors of a library with its own CUDA runtime do not reach the
// caller's cudaGetLastError) and its device-side error word.
int sm100_status_after_sync()
{
    const int launch = sm100_last_status();
    if (launch != FA_STATUS_OK) return launch;
    return fa_sm100_device_status(nullptr);
}

int host_only()
{
    std::printf("{\"host_only\": true, \"sm100_supported\": [%d, %d, %d, %d], \"v3_supported\": [%d, %d, %d, %d]}\n",
                sm100_supported(32), sm100_supported(64), sm100_supported(96), sm100_supported(128),
                tensorcore_v3_supported(32), tensorcore_v3_supported(64), tensorcore_v3_supported(96),
                tensorcore_v3_supported(128));
    const AttentionShape shapes[] = {{1, 2, 128, 64}, {2, 8, 2048, 64}, {4, 16, 4096, 128},
                                     {1, 32, 16384, 128}, {16, 32, 8192, 128}, {1, 3, 1000, 128}};
    for (const AttentionShape& shape : shapes) {
        for (bool causal : {false, true}) {
            std::printf("{%s, \"attention_flops\": %.17g, \"fa_attention_flops\": %.17g, "
                        "\"sm100_hbm_bytes\": %.17g, \"fa_sm100_hbm_bytes\": %.17g, \"v3_hbm_bytes\": %.17g}\n",
                        shape_json(shape, causal).c_str(), attention_flops(shape, causal),
                        fa_attention_flops(shape.batch, shape.heads, shape.seq_len, shape.head_dim, causal),
                        sm100_hbm_bytes(shape, causal),
                        fa_sm100_hbm_bytes(shape.batch, shape.heads, shape.seq_len, shape.head_dim, causal),
                        tensorcore_v3_hbm_bytes(shape, causal));
        }
    }
    return 0;
}

bool accuracy_suite(const std::vector<Entry>& entries)
{
    bool all_passed = true;
    for (int head_dim : {64, 128}) {
        for (bool causal : {false, true}) {
            const AttentionShape shape{kAccuracyBatch, kAccuracyHeads, kAccuracySeq, head_dim};
            const size_t count = static_cast<size_t>(shape.batch) * shape.heads * shape.seq_len * shape.head_dim;
            const size_t bytes = count * sizeof(__nv_bfloat16);
            std::vector<__nv_bfloat16> host_q(count), host_k(count), host_v(count), host_o(count);
            std::vector<double> reference(count);
            fill_normal(host_q, 11u);
            fill_normal(host_k, 22u);
            fill_normal(host_v, 33u);
            reference_attention(host_q, host_k, host_v, reference, shape, causal);

            __nv_bfloat16 *device_q = nullptr, *device_k = nullptr, *device_v = nullptr, *device_o = nullptr;
            float* workspace = nullptr;
            CUDA_CHECK(cudaMalloc(&device_q, bytes));
            CUDA_CHECK(cudaMalloc(&device_k, bytes));
            CUDA_CHECK(cudaMalloc(&device_v, bytes));
            CUDA_CHECK(cudaMalloc(&device_o, bytes));
            CUDA_CHECK(cudaMalloc(&workspace, unfused_workspace_bytes(shape)));
            CUDA_CHECK(cudaMemcpy(device_q, host_q.data(), bytes, cudaMemcpyHostToDevice));
            CUDA_CHECK(cudaMemcpy(device_k, host_k.data(), bytes, cudaMemcpyHostToDevice));
            CUDA_CHECK(cudaMemcpy(device_v, host_v.data(), bytes, cudaMemcpyHostToDevice));
            Buffers buffers{device_q, device_k, device_v, device_o, workspace, shape, causal};

            for (const Entry& entry : entries) {
                if (!entry.supported(head_dim)) continue;
                CUDA_CHECK(cudaMemset(device_o, 0xff, bytes));   // bf16 0xffff is NaN
                entry.func(&buffers);
                CUDA_CHECK(cudaGetLastError());
                CUDA_CHECK(cudaDeviceSynchronize());
                const int status = is_sm100(entry) ? sm100_status_after_sync() : 0;
                CUDA_CHECK(cudaMemcpy(host_o.data(), device_o, bytes, cudaMemcpyDeviceToHost));
                const Accuracy accuracy = compare(host_o, reference, shape);
                const bool passed = accuracy.passed() && status == 0;
                all_passed = all_passed && passed;
                std::printf("{\"suite\": \"accuracy\", \"kernel\": \"%s\", %s, \"vs_double\": %.6e, "
                            "\"row_scaled_error\": %.6e, \"max_abs_error\": %.6e, \"row_scale_ulp\": %.4f, "
                            "\"output_nan\": %zu, \"output_inf\": %zu, \"reference_nan\": %zu, "
                            "\"reference_inf\": %zu, \"status\": %d, \"passed\": %s}\n",
                            entry.name, shape_json(shape, causal).c_str(), accuracy.vs_double, accuracy.row_scaled,
                            accuracy.max_abs, accuracy.ulp, accuracy.output_nan, accuracy.output_inf,
                            accuracy.reference_nan, accuracy.reference_inf, status, passed ? "true" : "false");
                std::fflush(stdout);
            }
            CUDA_CHECK(cudaFree(device_q));
            CUDA_CHECK(cudaFree(device_k));
            CUDA_CHECK(cudaFree(device_v));
            CUDA_CHECK(cudaFree(device_o));
            CUDA_CHECK(cudaFree(workspace));
        }
    }
    return all_passed;
}

bool performance_case(const std::vector<Entry>& entries, const Case& item)
{
    const AttentionShape& shape = item.shape;
    const size_t count = static_cast<size_t>(shape.batch) * shape.heads * shape.seq_len * shape.head_dim;
    const size_t bytes = count * sizeof(__nv_bfloat16);
    std::vector<__nv_bfloat16> host(count);
    __nv_bfloat16 *device_q = nullptr, *device_k = nullptr, *device_v = nullptr, *device_o = nullptr;
    CUDA_CHECK(cudaMalloc(&device_q, bytes));
    CUDA_CHECK(cudaMalloc(&device_k, bytes));
    CUDA_CHECK(cudaMalloc(&device_v, bytes));
    CUDA_CHECK(cudaMalloc(&device_o, bytes));
    fill_normal(host, 11u);
    CUDA_CHECK(cudaMemcpy(device_q, host.data(), bytes, cudaMemcpyHostToDevice));
    fill_normal(host, 22u);
    CUDA_CHECK(cudaMemcpy(device_k, host.data(), bytes, cudaMemcpyHostToDevice));
    fill_normal(host, 33u);
    CUDA_CHECK(cudaMemcpy(device_v, host.data(), bytes, cudaMemcpyHostToDevice));

    // v0's workspace, tried as the harness tries it (:614-629); only v0 needs it.
    bool wants_v0 = false;
    for (const Entry& entry : entries) wants_v0 = wants_v0 || std::strcmp(entry.name, "v0_unfused") == 0;
    float* workspace = nullptr;
    bool run_v0 = false;
    if (wants_v0) {
        const cudaError_t workspace_status = cudaMalloc(&workspace, unfused_workspace_bytes(shape));
        run_v0 = workspace_status == cudaSuccess;
        if (workspace_status == cudaErrorMemoryAllocation) cudaGetLastError();
        else CUDA_CHECK(workspace_status);
    }
    Buffers buffers{device_q, device_k, device_v, device_o, workspace, shape, item.causal};
    const double flops = attention_flops(shape, item.causal);

    bool all_ok = true;
    double baseline_ms = 0.0;
    for (const Entry& entry : entries) {
        const bool v0 = std::strcmp(entry.name, "v0_unfused") == 0;
        const char* skip = !entry.supported(shape.head_dim) ? "unsupported"
                                                            : (v0 && !run_v0 ? "workspace_allocation_failed" : nullptr);
        if (skip != nullptr) {
            std::printf("{\"suite\": \"performance\", \"kernel\": \"%s\", %s, \"status\": \"%s\"}\n", entry.name,
                        shape_json(shape, item.causal).c_str(), skip);
            continue;
        }
        CUDA_CHECK(cudaMemset(device_o, 0xff, bytes));
        const Timing timing = time_iterations(entry.func, &buffers);
        const int launch_status = is_sm100(entry) ? sm100_status_after_sync() : 0;
        CUDA_CHECK(cudaMemcpy(host.data(), device_o, bytes, cudaMemcpyDeviceToHost));
        size_t output_nan = 0, output_inf = 0;
        for (const auto value : host) {
            const float output = __bfloat162float(value);
            output_nan += std::isnan(output);
            output_inf += std::isinf(output);
        }
        const bool finite = output_nan == 0 && output_inf == 0;
        const bool ok = finite && launch_status == 0;
        all_ok = all_ok && ok;
        if (v0 && finite) baseline_ms = timing.median_ms;
        const double speedup = (baseline_ms > 0.0 && finite) ? baseline_ms / timing.median_ms : -1.0;
        const double tflops = flops / (timing.median_ms / 1.0e3) / 1.0e12;
        std::printf("{\"suite\": \"performance\", \"kernel\": \"%s\", %s, \"status\": \"%s\", "
                    "\"warmup_iters\": %d, \"timed_iters\": %d, \"median_ms\": %.6f, \"q1_ms\": %.6f, "
                    "\"q3_ms\": %.6f, \"iqr_ms\": %.6f, \"speedup_vs_v0\": %.4f, \"tflops\": %.3f, "
                    "\"algorithmic_hbm_gb\": %.6f, \"output_nan\": %zu, \"output_inf\": %zu, \"launch_status\": %d}\n",
                    entry.name, shape_json(shape, item.causal).c_str(), finite ? "ok" : "nonfinite_output",
                    kWarmupIters, kTimedIters, timing.median_ms, timing.q1_ms, timing.q3_ms, timing.iqr_ms, speedup,
                    tflops, traffic_gb(entry, shape, item.causal), output_nan, output_inf, launch_status);
        std::fflush(stdout);
    }
    CUDA_CHECK(cudaFree(device_q));
    CUDA_CHECK(cudaFree(device_k));
    CUDA_CHECK(cudaFree(device_v));
    CUDA_CHECK(cudaFree(device_o));
    if (workspace != nullptr) CUDA_CHECK(cudaFree(workspace));
    return all_ok;
}

std::vector<std::string> split(const std::string& text, char separator)
{
    std::vector<std::string> parts;
    std::string part;
    std::istringstream in(text);
    while (std::getline(in, part, separator))
        if (!part.empty()) parts.push_back(part);
    return parts;
}

int usage(const char* program)
{
    std::fprintf(stderr, "usage: %s --host-only | [--entries name,...] [--cases grid|B,H,N,D,causal[;...]]\n",
                 program);
    return 2;
}

}  // namespace

int main(int argc, char** argv)
{
    std::vector<Entry> entries = all_entries();
    std::vector<Case> cases = kCases;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--host-only") return host_only();
        if (i + 1 >= argc) return usage(argv[0]);
        const std::string value = argv[++i];
        if (arg == "--entries") {
            std::vector<Entry> chosen;
            for (const std::string& name : split(value, ','))
                for (const Entry& entry : all_entries())
                    if (name == entry.name) chosen.push_back(entry);
            if (chosen.size() != split(value, ',').size()) return usage(argv[0]);
            entries = chosen;
        } else if (arg == "--cases") {
            if (value == "grid") continue;
            cases.clear();
            for (const std::string& item : split(value, ';')) {
                const std::vector<std::string> fields = split(item, ',');
                if (fields.size() != 5) return usage(argv[0]);
                cases.push_back({{std::stoi(fields[0]), std::stoi(fields[1]), std::stoi(fields[2]),
                                  std::stoi(fields[3])},
                                 std::stoi(fields[4]) != 0, "command line"});
            }
        } else {
            return usage(argv[0]);
        }
    }

    int device = 0;
    CUDA_CHECK(cudaGetDevice(&device));
    cudaDeviceProp props{};
    CUDA_CHECK(cudaGetDeviceProperties(&props, device));
    std::printf("{\"device\": \"%s\", \"sm\": \"%d%d\"}\n", props.name, props.major, props.minor);
    for (int head_dim : {64, 128}) {
        const FusedTilingInfo info = query_sm100(head_dim);
        std::printf("{\"tiling\": \"%s\", \"head_dim\": %d, \"supported\": %s, \"block_size\": %d, \"tile_kv\": %d, "
                    "\"rows_per_block\": %d, \"shared_bytes_per_block\": %d, \"registers_per_thread\": %d, "
                    "\"local_bytes_per_thread\": %d, \"max_blocks_per_sm\": %d}\n",
                    kSm100Name, head_dim, info.supported ? "true" : "false", info.block_size, info.tile_kv,
                    info.rows_per_block, info.shared_bytes_per_block, info.registers_per_thread,
                    info.local_bytes_per_thread, info.max_blocks_per_sm);
    }
    std::fflush(stdout);

    bool ok = accuracy_suite(entries);
    for (const Case& item : cases) ok = performance_case(entries, item) && ok;
    return ok ? 0 : 1;
}
