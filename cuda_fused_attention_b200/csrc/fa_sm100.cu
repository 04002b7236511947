// =============================================================================
// Blackwell (sm_100a) fused attention forward:  O = softmax(Q K^T / sqrt(D) + M) V
//
// The hot path of RichterWang/cuda_fused_attention, re-designed for B200. The
// reference computes it with launch_attention_tensorcore_v3
// (kernels/v3/v3_tensorcore.cu:418-750): 64 query rows per CTA, Q in
// registers, cp.async double buffering and warp-level mma.sync. Here:
//
//   * One CTA owns 256 query rows of one (batch, head) slab, as two 128-row Q
//     tiles that ping-pong between two softmax warpgroups. When a grid of such
//     CTAs would fill less than half the GPU (dense), or the row pairs fit in one
//     wave (causal), each CTA takes a single Q tile (the second warpgroup idles)
//     with S double-buffered in tensor memory, so that the next key tile's QK^T
//     runs during the softmax. Causal launches with very long rows and few slabs
//     split each row pair's key range across CTAs and merge the partial results.
//   * QK^T and PV are tcgen05.mma (kind::f16, M=128, N=128 / N=D, BF16 in,
//     FP32 accumulate) issued by one thread of the MMA warp. S and O live in
//     tensor memory: S0 | S1 | O0 | O1 = 512 columns at D=128.
//   * P (bf16) is written back over S in tensor memory and fed to the PV MMA as
//     its A operand straight from TMEM; P never touches shared memory.
//   * Q, K and V stream in with TMA (3-D tensor maps over [slabs, N, D], 128-byte
//     swizzle, zero fill past N) into a K/V ring of mbarrier-guarded stages.
//   * Softmax is one thread per row: a thread loads its whole S row from TMEM,
//     so the row max and row sum need no shuffles. exp is ex2 with log2(e)
//     folded into the scale. A row's exponent base moves (and O is rescaled in
//     TMEM) only when one of its scores exceeds the base by a factor 2^16.
//   * Causal: key tiles above the diagonal are never loaded or computed; only
//     the diagonal tile(s) and a ragged tail tile take the element mask. Blocks
//     run in groups of slabs sized to L2, heaviest units first across a group.
//   * Epilogue: O from TMEM, times 1/l, to bf16, into the (now free) Q tile of
//     shared memory in the swizzled layout, then one TMA store per 64 columns.
//
// Every mbarrier wait is bounded (default one second): on expiry the kernel
// records the wait site in a device error word, raises a CTA-wide abort flag,
// drains its own TMA loads and MMAs, frees tensor memory and returns.
//
// Warp roles (384 threads = 3 warpgroups):
//   warps 0-3   softmax + correction + epilogue for Q tile 0 (TMEM lanes 0-127)
//   warps 4-7   the same for Q tile 1
//   warp  8     TMEM allocator and MMA issuer (lane 0)
//   warp  9     TMA producer (lane 0)
//   warps 10-11 idle (they complete the third warpgroup for the register split)
// Registers: launched at 168 per thread; the softmax warpgroups grow to 216 and the
// third warpgroup shrinks to 72 (setmaxnreg), 2*128*216 + 128*72 = 384*168.
// =============================================================================

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstddef>
#include <cstring>
#include <mutex>

#include "fa_sm100.h"
#include "fa_sm100_internal.h"
#include "fa_sm100_ptx.cuh"

namespace fa_sm100 {

constexpr int kBlockM = 128;    // query rows per Q tile == TMEM lanes
constexpr int kBlockN = 128;    // keys per K/V tile
constexpr int kQTiles = 2;      // Q tiles per CTA (a row pair); small grids use one
constexpr int kRowsPerCta = kBlockM * kQTiles;
constexpr int kThreads = 384;
constexpr int kMmaWarp = 8;
constexpr int kLoadWarp = 9;
constexpr uint32_t kRegsLaunch = 168;    // ptxas's allocation at 384 threads, 1 CTA/SM
constexpr uint32_t kRegsSoftmax = 216;
constexpr uint32_t kRegsOther = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kThreads * kRegsLaunch,
              "the warpgroup register split must fit in the registers the CTA launches with");
// Lazy correction: a row keeps its exponent base until one of its scores exceeds it by
// more than 16 in the exp2 domain, so p <= 2^16 meanwhile; the final 1/l makes that exact.
// P is bf16 (relative precision independent of magnitude) and O and l accumulate in fp32,
// where N * 2^16 * |v| stays far from overflow for every accepted N (<= 2^30). A warp
// moves its base (O correction + redo of 64 exponentials) when any of its 32 rows needs
// it; with a threshold of 8 instead, peaky rows (Q scaled by 4, config 3) made that
// happen often enough to cost ~30 %.
constexpr float kRescaleThreshold = 16.0f;
constexpr uint32_t kTmemCols = 512;      // row pairs: S0 | S1 | O0 | O1; one tile: S(even j) | S(odd j) | O0

constexpr int kSubBytes = kBlockM * 128;    // one 128-row x 64-element bf16 swizzle block (16 KB)
constexpr int kMaxChunks = 64;              // key-range split: chunks per unit at most

// Wait-site ids recorded in the error word (bits 8..15).
enum WaitSite : uint32_t {
    kSiteMmaQ = 1, kSiteMmaK = 2, kSiteMmaV = 3, kSiteMmaP0 = 4, kSiteMmaP1 = 5,
    kSiteLoadEmpty = 6, kSiteSoftS = 7, kSiteSoftO = 8, kSiteEpilogue = 9, kSiteInjected = 10,
    kSiteDrain = 11, kSitePartial = 12,
};

template <int D>
struct Cfg {
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    // A split partial of one Q tile: O as [D/4 column groups][128 rows] of float4 (a warp's 32
    // rows of one column group are 512 contiguous bytes), then the 128 row maxima and sums.
    static constexpr int kPartTileFloats = D * kBlockM + 2 * kBlockM;
    static constexpr int kSub = D / 64;                       // swizzle blocks per row
    static constexpr int kTileBytes = kSub * kSubBytes;       // one Q, K or V tile
    static constexpr int kStages = (D == 128) ? 4 : 8;        // K/V ring slots
    static constexpr int kQOff = 0;
    static constexpr int kRingOff = kQTiles * kTileBytes;
    static constexpr int kBarOff = kRingOff + kStages * kTileBytes;
    // q_full[2] kv_full[S] kv_empty[S] s_full[2] p_half[2] p_full[2] pv_half_done[2] o_full[2]
    // epi[2] drain never
    static constexpr int kBarQFull = 0;
    static constexpr int kBarKvFull = 2;
    static constexpr int kBarKvEmpty = 2 + kStages;
    static constexpr int kBarSFull = 2 + 2 * kStages;
    static constexpr int kBarPHalf = kBarSFull + 2;       // first 64 keys of P written
    static constexpr int kBarPFull = kBarPHalf + 2;       // all of P written (and O corrected)
    static constexpr int kBarPvHalf = kBarPFull + 2;      // first-half PV MMAs completed
    static constexpr int kBarOFull = kBarPvHalf + 2;
    static constexpr int kBarEpi = kBarOFull + 2;
    static constexpr int kBarDrain = kBarEpi + 2;
    static constexpr int kBarNever = kBarDrain + 1;
    static constexpr int kBarPart = kBarNever + 1;        // split: all softmax threads wrote their partial rows
    static constexpr int kBarPartDone = kBarPart + 1;     // split: this chunk has counted itself in
    static constexpr int kNumBars = kBarPartDone + 1;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;   // tmem base, abort flag, last-chunk flag (u32)
    static constexpr int kItemOff = kMiscOff + 16;            // the CTA's work item (WorkItem), for the epilogue
    static constexpr int kSmemUsed = kItemOff + 32;
    static constexpr int kSmemBytes = kSmemUsed + 1024;       // slack for 1024-byte alignment
    static constexpr uint32_t kColS0 = 0;
    static constexpr uint32_t kColS1 = kBlockN;
    static constexpr uint32_t kColO0 = 2 * kBlockN;
    static constexpr uint32_t kColO1 = 2 * kBlockN + D;
    static constexpr uint32_t kIdescQK = make_idesc_bf16(kBlockM, kBlockN, false);
    static constexpr uint32_t kIdescPV = make_idesc_bf16(kBlockM, D, true);
    static_assert(kColO1 + D <= kTmemCols, "TMEM budget");
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// A CTA's work item as decoded at kernel start; kept in shared memory so that the values only
// the epilogue needs do not occupy registers through the main loop.
struct WorkItem {
    int slab_local;     // slab within this launch
    int unit;           // row pair (or Q tile in the one-tile kernel) of the slab
    int chunk;          // chunk of the unit's key range
    int nchunks;        // chunks the unit's key range is split into (1 = not split)
    int reserved0;      // (unused: with the key-tile range at this offset ptxas allocates the
                        //  row-pair kernel without a spill)
    int kv_begin;       // first key tile of this CTA
    int n_kv;           // key tiles of this CTA
    int reserved1;
};

struct Params {
    int seq_len;
    int num_units;              // CTAs per slab: ceil(seq_len / 256), or / 128 for the one-tile kernel
    long long slab_begin;       // first slab of this launch in the full tensor
    float scale_log2;           // default_scale(D) * log2(e)
    int causal;
    int inject_stall;           // test only: the MMA warp waits on a barrier nothing arrives on
    unsigned long long timeout_ns;
    long long num_slabs;        // slabs in this launch
    int chunk;                  // causal block order: slabs per group (see the kernel's work item)
    // Causal key-range split (0 = none): a unit with more than split_len key tiles is processed
    // by ceil(tiles / split_len) CTAs ("chunks"), each over a contiguous range of its key tiles;
    // the last chunk of a unit to finish merges the others' partials into the output.
    int split_len;
    int items;                  // work items per slab: units, or chunks when split
    int max_chunks;             // chunks of the heaviest unit (the stride of the per-unit arrays)
    unsigned long long epoch;   // this launch's tag (48 bits) in the arrival counters and flags
    unsigned long long* arrive; // [slabs * num_units]: epoch << 16 | chunks counted in
    unsigned long long* flags;  // [slabs * num_units * max_chunks]: epoch once that chunk's partial is written
    float* partial;             // [slabs * num_units * max_chunks][Q tiles][Cfg::kPartTileFloats]
};

// Device error word of this module instance (one per device). Bit 0: some wait
// timed out; bits 8..15: the site of the first recorded timeout.
__device__ unsigned int g_fa_error_word;

#ifdef FA_SM100_DEBUG_DUMP
// Layout check of the tcgen05 data path (debug builds only, libfa_sm100_debug.so): CTA 0
// writes what its Q tile 0 sees at each stage, so a test can check the stages one by one.
// Float offsets (FA_SM100_DEBUG_* in fa_sm100.h):
//   S [128][128]  QK^T of Q tile 0 and key tile 0 as loaded from TMEM (before scale and mask)
//   P [128][128]  P of that tile as the PV MMA reads it from TMEM (bf16 widened to f32)
//   O [128][128]  O of Q tile 0 after its last PV, before the 1/l scaling (D columns used)
//   L [128]       row sum l;  M [128] final exponent base (running row max of raw scores)
//   I [8]         slab, first query row, seq_len, head_dim, causal, one-tile kernel, key tiles, 1
constexpr int kDbgS = 0;
constexpr int kDbgP = kDbgS + 128 * 128;
constexpr int kDbgO = kDbgP + 128 * 128;
constexpr int kDbgL = kDbgO + 128 * 128;
constexpr int kDbgM = kDbgL + 128;
constexpr int kDbgInfo = kDbgM + 128;
constexpr int kDbgFloats = kDbgInfo + 8;
static_assert(kDbgFloats == FA_SM100_DEBUG_FLOATS, "debug dump layout");
__device__ float g_fa_debug[kDbgFloats];

// P columns [col0, col0 + 16 * chunks) of a row, read back from TMEM (packed bf16 pairs).
__device__ __forceinline__ void debug_dump_p(uint32_t t_p, int row, int key0, int chunks32)
{
    for (int c = 0; c < chunks32; ++c) {
        uint32_t w[32];
        tmem_ld32(t_p + static_cast<uint32_t>(c * 32), w);
        tmem_wait_ld();
        reg_fence32(w);
        for (int i = 0; i < 32; ++i) {
            g_fa_debug[kDbgP + row * 128 + key0 + 64 * c + 2 * i] = __uint_as_float(w[i] << 16);
            g_fa_debug[kDbgP + row * 128 + key0 + 64 * c + 2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
}
#endif

__device__ __forceinline__ void record_timeout(volatile uint32_t* abort_flag, uint32_t site)
{
    *abort_flag = 1u;
    atomicCAS(&g_fa_error_word, 0u, 1u | (site << 8));
    atomicOr(&g_fa_error_word, 1u);
}

// Bounded wait on an mbarrier phase. Returns false when the CTA is aborting or
// the wait ran past timeout_ns (which raises the abort itself).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                             unsigned long long timeout_ns, uint32_t site)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 7u) == 0u) {
            if (*abort_flag) return false;
            if (global_timer_ns() - start > timeout_ns) {
                record_timeout(abort_flag, site);
                return false;
            }
        }
    }
}

// Bounded wait used on the abort path: ignores the abort flag, still gives up
// after timeout_ns.
__device__ __forceinline__ bool wait_drain(uint32_t bar, uint32_t parity, unsigned long long timeout_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 7u) == 0u && global_timer_ns() - start > timeout_ns) {
            atomicOr(&g_fa_error_word, 1u);
            return false;
        }
    }
}

// The exponent-base arithmetic, with every rounding explicit (never contracted into an
// FMA, whatever the surrounding code lets the compiler fuse), so that both kernel
// instantiations round a row identically. A row keeps its base until a half-tile maximum
// exceeds it by kRescaleThreshold.
__device__ __forceinline__ bool rebase_needed(float half_max, float row_max, float sl2)
{
    return __fmul_rn(__fsub_rn(half_max, row_max), sl2) > kRescaleThreshold;
}

__device__ __forceinline__ float rebase_alpha(float row_max, float m_new, float sl2)
{
    return ex2_approx(__fsub_rn(__fmul_rn(row_max, sl2), __fmul_rn(m_new, sl2)));
}

__device__ __forceinline__ float exp_base(float row_max, float sl2)
{
    return row_max == -INFINITY ? 0.0f : __fmul_rn(row_max, sl2);
}

// QK^T for one Q tile against one K tile: D/16 MMAs of M=128, N=128, K=16.
// Both operands K-major in 128-byte swizzled 64-element blocks; the K step
// advances 32 bytes inside a block, then moves to the next block.
template <int D>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_saddr, uint32_t k_saddr)
{
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = static_cast<uint32_t>((kk >> 2) * kSubBytes + (kk & 3) * 32);
        const uint64_t a = make_smem_desc(q_saddr + off, 16, 1024);
        const uint64_t b = make_smem_desc(k_saddr + off, 16, 1024);
        umma_ss(d_tmem, a, b, Cfg<D>::kIdescQK, kk > 0 ? 1u : 0u);
    }
}

// O (+)= P V over key steps [kFirst, kLast) of 16 keys (8 in a tile): MMAs of
// M=128, N=D, K=16. P comes from TMEM (16 keys =
// 8 columns of packed bf16 pairs); V is MN-major: 64-column blocks kSubBytes
// apart (LBO), 8-key row groups 1024 bytes apart (SBO).
template <int D, int kFirst, int kLast>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_saddr, bool accumulate)
{
#pragma unroll
    for (int kk = kFirst; kk < kLast; ++kk) {
        const uint64_t b = make_smem_desc(v_saddr + static_cast<uint32_t>(kk * 16 * 128), kSubBytes, 1024);
        umma_ts(d_tmem, p_tmem + static_cast<uint32_t>(kk * 8), b, Cfg<D>::kIdescPV,
                (accumulate || kk > 0) ? 1u : 0u);
    }
}

// kOneTile = false: a CTA per row pair (two Q tiles). kOneTile = true: a CTA per 128-row
// Q tile, for grids too small to fill the GPU with pairs; warpgroup 1 then idles.
// kSplit = true (row pairs only): the causal key-range split (Params::split_len). Separate
// instantiations, so that the row-pair kernel carries no code of the other two: the split's
// epilogue alone, compiled into it, made its main loop 2-17 % slower.
template <int D, bool kOneTile, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
              const Params p)
{
    using C = Cfg<D>;
    static_assert(!(kSplit && kOneTile), "the key-range split is a row-pair kernel feature");
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment: the 128-byte swizzle pattern repeats every 8 rows.
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_addr);

    const uint32_t sq = base + C::kQOff;
    const uint32_t ring = base + C::kRingOff;
    const uint32_t bars = base + C::kBarOff;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kMiscOff + 4);
    volatile uint32_t* last_flag = reinterpret_cast<volatile uint32_t*>(smem + C::kMiscOff + 8);
    auto bar = [&](int index) -> uint32_t { return bars + static_cast<uint32_t>(index) * 8u; };

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    // Tensor memory: S0 | S1 | O0 | O1. The one-tile kernel uses S0 and S1 as a double buffer
    // (key tile j in S_(j & 1)), so that QK^T of the next key tile runs during the softmax.
    constexpr uint32_t kCols = kTmemCols;
    constexpr uint32_t kColO0 = C::kColO0;

    // ---- work item ---------------------------------------------------------------
    // A unit is a row pair (256 rows, two Q tiles) of one slab, or in the one-tile kernel a
    // single 128-row Q tile.
    // Dense: slab-major (the CTAs of a slab run together and share its K/V through L2).
    // Causal: slabs in groups of p.chunk; within a group the units go heaviest first,
    // each unit for every slab of the group, so the longest CTAs of the last slabs do not
    // start late and stretch the tail, while the K/V of only one group (sized on the host
    // to a fraction of L2) is being read at a time.
    constexpr bool two = !kOneTile;                      // a second Q tile in this CTA
    const int n = p.seq_len;
    const int kv_tiles_all = (n + kBlockN - 1) / kBlockN;
    // Key tiles a unit attends to, and the chunks its key range is split into.
    auto unit_tiles = [&](int u) -> int {
        const int t0 = u * (two ? kQTiles : 1);
        return p.causal ? min(kv_tiles_all, t0 + (two ? 2 : 1)) : kv_tiles_all;
    };
    auto unit_chunks = [&](int u) -> int {
        return p.split_len > 0 ? (unit_tiles(u) + p.split_len - 1) / p.split_len : 1;
    };
    const long long block = blockIdx.x;
    long long slab_local;
    int unit;
    int chunk = 0, nchunks = 1;
    if (p.causal) {
        const long long per_group = static_cast<long long>(p.chunk) * p.items;
        const long long group = block / per_group;
        const long long first = group * p.chunk;
        const long long in_group = min(static_cast<long long>(p.chunk), p.num_slabs - first);
        const long long within = block - group * per_group;
        const long long level = within / in_group;
        slab_local = first + (within - level * in_group);
        if (kSplit && p.split_len > 0) {
            // Items of a slab: units heaviest first, each unit's chunks in key order.
            int item = static_cast<int>(level);
            unit = 0;
            for (int u = p.num_units - 1; u >= 0; --u) {
                const int ncu = unit_chunks(u);
                if (item < ncu || u == 0) {
                    unit = u;
                    nchunks = ncu;
                    chunk = min(item, ncu - 1);
                    break;
                }
                item -= ncu;
            }
        } else {
            unit = p.num_units - 1 - static_cast<int>(level);
        }
    } else {
        slab_local = block / p.num_units;
        unit = static_cast<int>(block - slab_local * p.num_units);
    }
    const int slab = static_cast<int>(p.slab_begin + slab_local);
    const int tile0 = unit * (two ? kQTiles : 1);        // first 128-row Q tile of this CTA
    // Fields of the work item in shared memory, read through their 32-bit shared addresses.
    auto item_field = [&](int offset) -> int {
        int value;
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(value) : "r"(base + C::kItemOff + static_cast<uint32_t>(offset)));
        return value;
    };
    const int q_row0 = tile0 * kBlockM;
    const int tiles = unit_tiles(unit);
    // Chunk c of a unit covers key tiles [c * tiles / nchunks, (c + 1) * tiles / nchunks) (32-bit: the
    // host splits only units with at most kMaxChunks chunks, so c * tiles < 2^31).
    const int kv_begin_0 = chunk * tiles / nchunks;
    const int n_kv_0 = (chunk + 1) * tiles / nchunks - kv_begin_0;
    if (kSplit && threadIdx.x == 0) {
        WorkItem* item_smem = reinterpret_cast<WorkItem*>(smem + C::kItemOff);
        item_smem->slab_local = static_cast<int>(slab_local);
        item_smem->unit = unit;
        item_smem->chunk = chunk;
        item_smem->nchunks = nchunks;
        item_smem->kv_begin = kv_begin_0;
        item_smem->n_kv = n_kv_0;
    }

    // ---- set-up ---------------------------------------------------------------
    // Barrier set-up, one barrier per lane of warp 0: p_half, p_full and epi count the 128
    // threads of a softmax warpgroup, every other barrier a single arrival (an expect_tx, a
    // tcgen05.commit or the inject-stall barrier nobody arrives on).
    if (warp == 0) {
        for (int b = lane; b < C::kNumBars; b += 32) {
            const bool per_thread = (b >= C::kBarPHalf && b < C::kBarPvHalf) || (b >= C::kBarEpi && b < C::kBarDrain);
            const uint32_t count = b == C::kBarPart ? (kOneTile ? kBlockM : kRowsPerCta) : (per_thread ? kBlockM : 1);
            mbar_init(bar(b), count);
        }
        if (lane == 0) *abort_flag = 0u;
        fence_mbarrier_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Key tiles of this CTA: [kv_begin, kv_begin + n_kv) (loaded where each role starts).
    const int kv_begin = kSplit ? item_field(offsetof(WorkItem, kv_begin)) : 0;
    const int n_kv = kSplit ? item_field(offsetof(WorkItem, n_kv)) : n_kv_0;
    const unsigned long long timeout = p.timeout_ns;

    if (warp == kLoadWarp) {
        // ======================= TMA producer ==================================
        regs_decrease<kRegsOther>();
        if (lane == 0) {
            tma_prefetch_map(&tm_q);
            tma_prefetch_map(&tm_k);
            tma_prefetch_map(&tm_v);
            tma_prefetch_map(&tm_o);
            for (int t = 0; t < (two ? 2 : 1); ++t) {
                mbar_arrive_expect_tx(bar(C::kBarQFull + t), C::kTileBytes);
#pragma unroll
                for (int s = 0; s < C::kSub; ++s)
                    tma_load_3d(sq + t * C::kTileBytes + s * kSubBytes, &tm_q, bar(C::kBarQFull + t), s * 64,
                                q_row0 + t * kBlockM, slab);
            }
            bool ok = true;
            int issued = 0;
            for (int i = 0; i < 2 * n_kv; ++i) {
                const int slot = i % C::kStages;
                const int use = i / C::kStages;
                if (use > 0 && !wait_bounded(bar(C::kBarKvEmpty + slot), (use - 1) & 1, abort_flag, timeout,
                                             kSiteLoadEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(bar(C::kBarKvFull + slot), C::kTileBytes);
                const CUtensorMap* map = (i & 1) ? &tm_v : &tm_k;
                const int key0 = (kv_begin + (i >> 1)) * kBlockN;
#pragma unroll
                for (int s = 0; s < C::kSub; ++s)
                    tma_load_3d(ring + slot * C::kTileBytes + s * kSubBytes, map, bar(C::kBarKvFull + slot),
                                s * 64, key0, slab);
                ++issued;
            }
            if (!ok) {
                // Abort: let every copy this CTA started land before shared memory goes away.
                wait_drain(bar(C::kBarQFull + 0), 0, timeout);
                if (two) wait_drain(bar(C::kBarQFull + 1), 0, timeout);
                for (int i = max(0, issued - C::kStages); i < issued; ++i)
                    wait_drain(bar(C::kBarKvFull + i % C::kStages), (i / C::kStages) & 1, timeout);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ======================= MMA issuer ====================================
        regs_decrease<kRegsOther>();
        if (lane == 0) {
            const uint32_t t_s0 = tmem_base + C::kColS0;
            const uint32_t t_s1 = tmem_base + C::kColS1;
            const uint32_t t_o0 = tmem_base + kColO0;
            const uint32_t t_o1 = tmem_base + C::kColO1;
            const uint32_t sq0 = sq;
            const uint32_t sq1 = sq + C::kTileBytes;
            auto slot_addr = [&](int i) -> uint32_t { return ring + (i % C::kStages) * C::kTileBytes; };
            auto full_bar = [&](int i) -> uint32_t { return bar(C::kBarKvFull + i % C::kStages); };
            auto empty_bar = [&](int i) -> uint32_t { return bar(C::kBarKvEmpty + i % C::kStages); };
            auto full_par = [&](int i) -> uint32_t { return static_cast<uint32_t>((i / C::kStages) & 1); };

            bool ok = wait_bounded(bar(C::kBarQFull + 0), 0, abort_flag, timeout, kSiteMmaQ) &&
                      (!two || wait_bounded(bar(C::kBarQFull + 1), 0, abort_flag, timeout, kSiteMmaQ));
            if (ok && p.inject_stall) ok = wait_bounded(bar(C::kBarNever), 0, abort_flag, timeout, kSiteInjected);
            if (ok) ok = wait_bounded(full_bar(0), full_par(0), abort_flag, timeout, kSiteMmaK);
            if constexpr (two) {
                if (ok) {
                    tc_fence_after();
                    issue_qk<D>(t_s0, sq0, slot_addr(0));
                    umma_commit(bar(C::kBarSFull + 0));
                    issue_qk<D>(t_s1, sq1, slot_addr(0));
                    umma_commit(bar(C::kBarSFull + 1));
                    umma_commit(empty_bar(0));
                }
                for (int j = 0; ok && j < n_kv; ++j) {
                    const int vi = 2 * j + 1;      // ring index of V_j
                    const int ki = 2 * j + 2;      // ring index of K_{j+1}
                    const bool more = j + 1 < n_kv;
                    const bool last = !more;
                    const uint32_t par = static_cast<uint32_t>(j & 1);
                    if (!wait_bounded(full_bar(vi), full_par(vi), abort_flag, timeout, kSiteMmaV)) { ok = false; break; }
                    // Tile 0: PV over the first 64 keys as soon as that half of P is in TMEM.
                    if (!wait_bounded(bar(C::kBarPHalf + 0), par, abort_flag, timeout, kSiteMmaP0)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 0, 4>(t_o0, t_s0, slot_addr(vi), j > 0);
                    umma_commit(bar(C::kBarPvHalf + 0));
                    if (!wait_bounded(bar(C::kBarPFull + 0), par, abort_flag, timeout, kSiteMmaP0)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 4, 8>(t_o0, t_s0, slot_addr(vi), true);
                    if (last) umma_commit(bar(C::kBarOFull + 0));
                    if (more) {
                        if (!wait_bounded(full_bar(ki), full_par(ki), abort_flag, timeout, kSiteMmaK)) { ok = false; break; }
                        tc_fence_after();
                        issue_qk<D>(t_s0, sq0, slot_addr(ki));
                        umma_commit(bar(C::kBarSFull + 0));
                    }
                    // Tile 1, same pattern.
                    if (!wait_bounded(bar(C::kBarPHalf + 1), par, abort_flag, timeout, kSiteMmaP1)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 0, 4>(t_o1, t_s1, slot_addr(vi), j > 0);
                    umma_commit(bar(C::kBarPvHalf + 1));
                    if (!wait_bounded(bar(C::kBarPFull + 1), par, abort_flag, timeout, kSiteMmaP1)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 4, 8>(t_o1, t_s1, slot_addr(vi), true);
                    umma_commit(empty_bar(vi));
                    if (last) umma_commit(bar(C::kBarOFull + 1));
                    if (more) {
                        issue_qk<D>(t_s1, sq1, slot_addr(ki));
                        umma_commit(bar(C::kBarSFull + 1));
                        umma_commit(empty_bar(ki));
                    }
                }
            } else {
                // One Q tile, S double-buffered: key tile j in S_(j & 1). QK^T(j+1) is issued before
                // the PV of tile j waits for its P, so it runs while the softmax works on tile j. The
                // P barriers are per buffer (kBarPHalf/kBarPFull + b, phase (j >> 1) & 1): the softmax
                // can finish tile j + 1 before this thread waits for tile j's P, never tile j + 2,
                // whose S is issued only after that wait. kBarPvHalf + 1 completes when tile j's PV
                // has: the softmax waits on it before it rescales O for tile j + 1.
                if (ok) {
                    tc_fence_after();
                    issue_qk<D>(t_s0, sq0, slot_addr(0));
                    umma_commit(bar(C::kBarSFull + 0));
                    umma_commit(empty_bar(0));
                }
                uint32_t t_sj = t_s0;                 // S of key tile j; the other buffer is t_sj ^ kBlockN
                for (int j = 0; ok && j < n_kv; ++j) {
                    const int vi = 2 * j + 1;
                    if (j + 1 < n_kv) {
                        const int ki = vi + 1;
                        if (!wait_bounded(full_bar(ki), full_par(ki), abort_flag, timeout, kSiteMmaK)) { ok = false; break; }
                        tc_fence_after();
                        issue_qk<D>(t_sj ^ kBlockN, sq0, slot_addr(ki));
                        umma_commit(bar(C::kBarSFull + ((j + 1) & 1)));
                        umma_commit(empty_bar(ki));
                    }
                    if (!wait_bounded(full_bar(vi), full_par(vi), abort_flag, timeout, kSiteMmaV)) { ok = false; break; }
                    if (!wait_bounded(bar(C::kBarPHalf + (j & 1)), (j >> 1) & 1, abort_flag, timeout, kSiteMmaP0)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 0, 4>(t_o0, t_sj, slot_addr(vi), j > 0);
                    umma_commit(bar(C::kBarPvHalf + 0));
                    if (!wait_bounded(bar(C::kBarPFull + (j & 1)), (j >> 1) & 1, abort_flag, timeout, kSiteMmaP0)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv<D, 4, 8>(t_o0, t_sj, slot_addr(vi), true);
                    umma_commit(empty_bar(vi));
                    umma_commit(bar(C::kBarPvHalf + 1));
                    if (j + 1 == n_kv) umma_commit(bar(C::kBarOFull + 0));
                    t_sj ^= kBlockN;
                }
            }
            // Every MMA issued above must finish before tensor memory is released.
            umma_commit(bar(C::kBarDrain));
            wait_drain(bar(C::kBarDrain), 0, timeout);
        }
        __syncwarp();
    } else if (warp < 4 || (warp < kMmaWarp && two)) {
        // ======================= softmax / correction / epilogue ================
        regs_increase<kRegsSoftmax>();
        const int t = warp / 4;                    // Q tile of this warpgroup
        const int quarter = warp % 4;              // TMEM lane quarter of this warp
        const int r = quarter * 32 + lane;         // row within the Q tile == TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        // S of the current key tile: the Q tile's own buffer (row pairs), or S_(j & 1) in the
        // one-tile kernel, which flips between S0 and S1 after every key tile.
        uint32_t t_s = lane_base + (t == 0 ? C::kColS0 : C::kColS1);
        static_assert((C::kColS0 ^ C::kColS1) == kBlockN && C::kColS0 == 0, "S buffers at columns 0 and 128");
        const uint32_t t_o = lane_base + (t == 0 ? kColO0 : C::kColO1);
        const int row = q_row0 + t * kBlockM + r;            // query index in the slab
        const int limit = p.causal ? min(row, n - 1) : n - 1;  // last key this row attends to
        // Local key-tile indices from which a tile needs the element mask: the causal diagonal,
        // and the first tile that reaches past N.
        const int diag_local = tile0 + t - kv_begin;
        const int tail_local = n / kBlockN - kv_begin;
        const float sl2 = p.scale_log2;

        float row_max = -INFINITY;   // running max of raw scores
        float row_sum = 0.0f;        // running sum of exp2((s - max) * sl2), fp32 before rounding
        bool ok = true;

        float m_base = 0.0f;         // row_max * sl2, the exp2 offset in use (0 while row_max = -inf)
        const uint64_t c2 = f2_pack(sl2, sl2);

        // O *= scale (per row) in TMEM; warp-collective.
        auto rescale_o = [&](float scale) {
            const uint64_t a2 = f2_pack(scale, scale);
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(t_o + static_cast<uint32_t>(c * 32), o);
                tmem_wait_ld();
                reg_fence32(o);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float o0, o1;
                    f2_unpack(fmul2(f2_pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), a2), o0, o1);
                    o[2 * i] = __float_as_uint(o0);
                    o[2 * i + 1] = __float_as_uint(o1);
                }
                tmem_st32(t_o + static_cast<uint32_t>(c * 32), o);
            }
        };

        // Exponentiate 64 scores (two 32-column chunks) against base `mb`, pack P to bf16
        // pairs and accumulate the fp32 sum; also return the raw max of the 64 scores. The
        // max and the exponentials are independent instruction streams.
        auto exp_half = [&](const uint32_t (&lo)[32], const uint32_t (&hi)[32], float mb,
                            uint32_t (&out)[32], float& half_sum, float& half_max, uint32_t p_tmem) {
            const uint64_t nb2 = f2_pack(-mb, -mb);
            uint64_t sum_a = f2_pack(0.0f, 0.0f), sum_b = f2_pack(0.0f, 0.0f);
            float ma = __uint_as_float(lo[0]), mb_ = __uint_as_float(hi[0]);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t (&src)[32] = (i < 16) ? lo : hi;
                const int k = (i & 15) * 2;
                if (k > 0 || i >= 16) {
                    if (i < 16) ma = max3f(ma, __uint_as_float(src[k]), __uint_as_float(src[k + 1]));
                    else mb_ = max3f(mb_, __uint_as_float(src[k]), __uint_as_float(src[k + 1]));
                } else {
                    ma = fmaxf(ma, __uint_as_float(src[1]));
                }
                const uint64_t x = ffma2(f2_pack(__uint_as_float(src[k]), __uint_as_float(src[k + 1])), c2, nb2);
                float x0, x1;
                f2_unpack(x, x0, x1);
                const uint64_t pr = f2_pack(ex2_approx(x0), ex2_approx(x1));
                if (i & 1) sum_b = fadd2(sum_b, pr);
                else sum_a = fadd2(sum_a, pr);
                float p0, p1;
                f2_unpack(pr, p0, p1);
                out[i] = pack_bf16x2(p0, p1);
                // Each 16 packed pairs go to TMEM as soon as they are complete, so that little
                // store latency is left to wait for before P is handed to the MMA.
                if (i == 15) tmem_st16(p_tmem, *reinterpret_cast<uint32_t (*)[16]>(&out[0]));
                if (i == 31) tmem_st16(p_tmem + 16, *reinterpret_cast<uint32_t (*)[16]>(&out[16]));
            }
            float sa0, sa1, sb0, sb1;
            f2_unpack(sum_a, sa0, sa1);
            f2_unpack(sum_b, sb0, sb1);
            half_sum = (sa0 + sa1) + (sb0 + sb1);
            half_max = fmaxf(ma, mb_);
        };

        for (int j = 0; j < n_kv; ++j) {
            // Barrier set of this key tile's S buffer: the Q tile's own (row pairs), or that of
            // S_(j & 1) (one tile; those barriers complete once per two key tiles).
            ok = __all_sync(0xffffffffu, wait_bounded(bar(C::kBarSFull + (kOneTile ? (j & 1) : t)),
                                                      static_cast<uint32_t>(kOneTile ? (j >> 1) & 1 : j & 1),
                                                      abort_flag, timeout, kSiteSoftS));
            if (!ok) break;
            tc_fence_after();

            uint32_t s[4][32];
            tmem_ld32(t_s + 0, s[0]);
            tmem_ld32(t_s + 32, s[1]);
            tmem_ld32(t_s + 64, s[2]);
            tmem_ld32(t_s + 96, s[3]);
            tmem_wait_ld();
            reg_fence32(s[0]);
            reg_fence32(s[1]);
            reg_fence32(s[2]);
            reg_fence32(s[3]);
#ifdef FA_SM100_DEBUG_DUMP
            if (blockIdx.x == 0 && j == 0 && t == 0)
                for (int i = 0; i < 128; ++i) g_fa_debug[kDbgS + r * 128 + i] = __uint_as_float(s[i / 32][i % 32]);
#endif

            const bool mask_tile = (p.causal && j >= diag_local) || j >= tail_local;
            if (mask_tile) {
                const int key0 = ((kSplit ? item_field(offsetof(WorkItem, kv_begin)) : 0) + j) * kBlockN;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (key0 + c * 32 + i > limit) s[c][i] = __float_as_uint(-INFINITY);
            }

            if (j == 0) {
                // First tile: the base is the tile's row max (no exponent to keep yet).
                float mx[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float a = __uint_as_float(s[c][0]), b = __uint_as_float(s[c][1]);
#pragma unroll
                    for (int i = 2; i < 32; i += 4) {
                        a = max3f(a, __uint_as_float(s[c][i]), __uint_as_float(s[c][i + 1]));
                        b = max3f(b, __uint_as_float(s[c][i + 2]), __uint_as_float(s[c][i + 3]));
                    }
                    mx[c] = fmaxf(a, b);
                }
                row_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
                m_base = exp_base(row_max, sl2);
            }

            float o_scale = 1.0f;    // O correction owed before the first PV of this tile reads O
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t packed[32];
                float hsum, hmax;
                exp_half(s[2 * h], s[2 * h + 1], m_base, packed, hsum, hmax,
                         t_s + static_cast<uint32_t>(32 * h));
                // Optimistic: the exponentials used the current base. If any score of this half
                // exceeds it by more than the threshold (rare after the first tile), move the
                // base, correct what was accumulated on the old one, and redo this half.
                const bool need = rebase_needed(hmax, row_max, sl2);
                if (__any_sync(0xffffffffu, need)) {
                    const float m_new = need ? hmax : row_max;
                    const float alpha = need ? rebase_alpha(row_max, m_new, sl2) : 1.0f;
                    row_sum = __fmul_rn(row_sum, alpha);
                    row_max = m_new;
                    m_base = exp_base(row_max, sl2);
                    if (h == 0) {
                        o_scale *= alpha;
                    } else {
                        // The first-half PV of this tile may be running on the old base: let it
                        // finish, then correct O (including its contribution) now.
                        ok = __all_sync(0xffffffffu, wait_bounded(bar(C::kBarPvHalf + t), j & 1, abort_flag,
                                                                  timeout, kSiteSoftO));
                        if (!ok) break;
                        tc_fence_after();
                        rescale_o(alpha);
                    }
                    exp_half(s[2 * h], s[2 * h + 1], m_base, packed, hsum, hmax,
                         t_s + static_cast<uint32_t>(32 * h));
                }
                row_sum = __fadd_rn(row_sum, hsum);
                // P of this half is in TMEM (stored by exp_half; a redo above stored it again).
                if (h == 0) {
                    // Keys 0-63 of P are final: correct O first (the PV is the next reader of O;
                    // at j = 0 it overwrites O), then hand the first half to the MMA.
                    if (j > 0 && __any_sync(0xffffffffu, o_scale != 1.0f)) {
                        if constexpr (kOneTile) {
                            // This tile's S can be ready before the previous tile's PV has
                            // finished accumulating into O: wait for that PV first.
                            ok = __all_sync(0xffffffffu, wait_bounded(bar(C::kBarPvHalf + 1),
                                                                      static_cast<uint32_t>((j - 1) & 1), abort_flag,
                                                                      timeout, kSiteSoftO));
                            if (!ok) break;
                            tc_fence_after();
                        }
                        rescale_o(o_scale);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(bar(C::kBarPHalf + (kOneTile ? (j & 1) : t)));
                }
            }
            if (!ok) break;
            tmem_wait_st();
#ifdef FA_SM100_DEBUG_DUMP
            if (blockIdx.x == 0 && j == 0 && t == 0) debug_dump_p(t_s, r, 0, 2);
#endif
            tc_fence_before();
            mbar_arrive(bar(C::kBarPFull + (kOneTile ? (j & 1) : t)));
            if constexpr (kOneTile) t_s ^= kBlockN;
        }

        // ---- epilogue ---------------------------------------------------------
        if (ok) ok = __all_sync(0xffffffffu, wait_bounded(bar(C::kBarOFull + t), 0, abort_flag, timeout, kSiteSoftO));
        // The last QK MMA of this tile has completed, so its Q tile is free: final values are
        // staged there in the 128-byte swizzled layout the store map expects.
        const uint32_t stage = sq + static_cast<uint32_t>(t * C::kTileBytes);
        auto stage32 = [&](int c, const float (&v)[32]) {
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) packed[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
            const int sub = (c * 32) / 64;
            const int chunk0 = ((c * 32) % 64) / 8;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int phys = (chunk0 + q) ^ (r & 7);
                const uint32_t addr = stage + static_cast<uint32_t>(sub * kSubBytes + r * 128 + phys * 16);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
                             :: "r"(addr), "r"(packed[4 * q]), "r"(packed[4 * q + 1]),
                                "r"(packed[4 * q + 2]), "r"(packed[4 * q + 3]) : "memory");
            }
        };
        auto store_tile = [&]() {
            fence_proxy_async_smem();
            mbar_arrive(bar(C::kBarEpi + t));
            if (r == 0) {
                if (wait_bounded(bar(C::kBarEpi + t), 0, abort_flag, timeout, kSiteEpilogue)) {
#pragma unroll
                    for (int s = 0; s < C::kSub; ++s)
                        tma_store_3d(&tm_o, stage + static_cast<uint32_t>(s * kSubBytes), s * 64,
                                     q_row0 + t * kBlockM, slab);
                    tma_store_commit();
                    tma_store_wait_read_all();
                }
            }
        };
        const int e_nchunks = kSplit ? item_field(offsetof(WorkItem, nchunks)) : 1;
        if (kSplit && e_nchunks > 1) {
            // ---- a chunk of a split unit. Thread 0 counts the chunk in on the unit's arrival
            // counter (tagged with this launch's epoch, so it needs no zeroing). A chunk that is
            // not the last writes its partial -- O on its own base, the raw row maxima and the
            // row sums -- and publishes it with an epoch flag. The last chunk waits (bounded) for
            // those flags -- every chunk it waits for has already counted in, so it is running and
            // waits for nothing -- and merges all chunks in chunk order, its own O straight from
            // tensor memory, so the result does not depend on the order of arrival.
            const int nchunks = e_nchunks;
            const int chunk = item_field(offsetof(WorkItem, chunk));
            const long long unit_index = static_cast<long long>(item_field(offsetof(WorkItem, slab_local))) *
                                         p.num_units + item_field(offsetof(WorkItem, unit));
            constexpr int kTilesPerCta = two ? kQTiles : 1;
            const size_t chunk_stride = static_cast<size_t>(kTilesPerCta) * C::kPartTileFloats;
            // This tile's partial in chunk 0 of the unit; chunk cc is chunk_stride floats further.
            float* unit_tile = p.partial + static_cast<size_t>(unit_index) * p.max_chunks * chunk_stride +
                               static_cast<size_t>(t) * C::kPartTileFloats;
            unsigned long long* unit_flags = p.flags + unit_index * p.max_chunks;
            if (threadIdx.x == 0) {
                uint32_t role = 2u;     // gave up
                if (ok) {
                    unsigned long long* counter = p.arrive + unit_index;
                    unsigned long long seen = *reinterpret_cast<volatile unsigned long long*>(counter);
                    unsigned int arrival = 0;
                    for (int attempt = 0; attempt < 1024; ++attempt) {
                        const bool current = (seen >> 16) == p.epoch;
                        const unsigned long long next = current ? seen + 1 : ((p.epoch << 16) | 1ull);
                        const unsigned long long prev = atomicCAS(counter, seen, next);
                        if (prev == seen) {
                            arrival = current ? static_cast<unsigned int>(seen & 0xFFFFu) : 0u;
                            role = arrival == static_cast<unsigned int>(nchunks - 1) ? 1u : 0u;
                            break;
                        }
                        seen = prev;
                    }
                    if (role == 2u) record_timeout(abort_flag, kSitePartial);
                }
                *last_flag = role;
                mbar_arrive(bar(C::kBarPartDone));
            }
            if (ok) ok = __all_sync(0xffffffffu, wait_bounded(bar(C::kBarPartDone), 0, abort_flag, timeout, kSitePartial));
            const uint32_t role = ok ? *last_flag : 2u;
            if (role == 0u) {
                tc_fence_after();
                float* mine = unit_tile + static_cast<size_t>(chunk) * chunk_stride;
                float4* cols = reinterpret_cast<float4*>(mine);
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tmem_ld32(t_o + static_cast<uint32_t>(c * 32), o);
                    tmem_wait_ld();
                    reg_fence32(o);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        cols[(c * 8 + q) * kBlockM + r] =
                            make_float4(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]),
                                        __uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3]));
                }
                mine[D * kBlockM + r] = row_max;
                mine[D * kBlockM + kBlockM + r] = row_sum;
                __threadfence();
                mbar_arrive(bar(C::kBarPart));
                if (threadIdx.x == 0 && wait_bounded(bar(C::kBarPart), 0, abort_flag, timeout, kSitePartial)) {
                    __threadfence();
                    st_release_gpu(unit_flags + chunk, p.epoch);
                }
            } else if (role == 1u) {
                // Wait until every other chunk's partial is published (each thread polls; bounded).
                bool ready = true;
                for (int cc = 0; cc < nchunks && ready; ++cc) {
                    if (cc == chunk) continue;
                    if (ld_acquire_gpu(unit_flags + cc) == p.epoch) continue;
                    const uint64_t begin = global_timer_ns();
                    while (ld_acquire_gpu(unit_flags + cc) != p.epoch) {
                        if (*abort_flag) { ready = false; break; }
                        if (global_timer_ns() - begin > timeout) {
                            record_timeout(abort_flag, kSitePartial);
                            ready = false;
                            break;
                        }
                    }
                }
                ok = __all_sync(0xffffffffu, ready);
            }
            if (role == 1u && ok) {
                tc_fence_after();
                auto chunk_max = [&](int cc) { return cc == chunk ? row_max : __ldcg(unit_tile + cc * chunk_stride + D * kBlockM + r); };
                auto chunk_sum = [&](int cc) {
                    return cc == chunk ? row_sum : __ldcg(unit_tile + cc * chunk_stride + D * kBlockM + kBlockM + r);
                };
                float top = -INFINITY;
                for (int cc = 0; cc < nchunks; ++cc) top = fmaxf(top, chunk_max(cc));
                const float top_base = exp_base(top, sl2);
                auto weight = [&](float m) { return m == -INFINITY ? 0.0f : ex2_approx(exp_base(m, sl2) - top_base); };
                float total = 0.0f;
                for (int cc = 0; cc < nchunks; ++cc) total = __fadd_rn(total, __fmul_rn(weight(chunk_max(cc)), chunk_sum(cc)));
                const float inv = total > 0.0f ? 1.0f / total : 0.0f;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    float acc[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
                    for (int cc = 0; cc < nchunks; ++cc) {
                        const float w = weight(chunk_max(cc));
                        if (cc == chunk) {
                            uint32_t o[32];
                            tmem_ld32(t_o + static_cast<uint32_t>(c * 32), o);
                            tmem_wait_ld();
                            reg_fence32(o);
#pragma unroll
                            for (int i = 0; i < 32; ++i) acc[i] = fmaf(w, __uint_as_float(o[i]), acc[i]);
                        } else {
                            const float4* cols = reinterpret_cast<const float4*>(unit_tile + cc * chunk_stride);
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const float4 v4 = __ldcg(cols + (c * 8 + q) * kBlockM + r);
                                acc[4 * q] = fmaf(w, v4.x, acc[4 * q]);
                                acc[4 * q + 1] = fmaf(w, v4.y, acc[4 * q + 1]);
                                acc[4 * q + 2] = fmaf(w, v4.z, acc[4 * q + 2]);
                                acc[4 * q + 3] = fmaf(w, v4.w, acc[4 * q + 3]);
                            }
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[i] *= inv;
                    stage32(c, acc);
                }
                store_tile();
            }
        } else if (ok) {
            tc_fence_after();
            const float inv = row_sum > 0.0f ? 1.0f / row_sum : 0.0f;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(t_o + static_cast<uint32_t>(c * 32), o);
                tmem_wait_ld();
                reg_fence32(o);
#ifdef FA_SM100_DEBUG_DUMP
                if (blockIdx.x == 0 && t == 0) {
                    for (int i = 0; i < 32; ++i) g_fa_debug[kDbgO + r * 128 + c * 32 + i] = __uint_as_float(o[i]);
                    if (c == 0) {
                        g_fa_debug[kDbgL + r] = row_sum;
                        g_fa_debug[kDbgM + r] = row_max;
                    }
                    if (c == 0 && r == 0) {
                        const float info[8] = {static_cast<float>(slab), static_cast<float>(q_row0),
                                               static_cast<float>(n), static_cast<float>(D),
                                               static_cast<float>(p.causal), kOneTile ? 1.0f : 0.0f,
                                               static_cast<float>(n_kv), 1.0f};
                        for (int i = 0; i < 8; ++i) g_fa_debug[kDbgInfo + i] = info[i];
                    }
                }
#endif
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
                stage32(c, v);
            }
            store_tile();
        }
        tc_fence_before();
    } else {
        // Warps 10-11 (idle members of the third warpgroup), and warpgroup 1 when the CTA has
        // no second Q tile.
        regs_decrease<kRegsOther>();
    }

    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kCols);
    }
}

}  // namespace fa_sm100

// =============================================================================
// Host side
// =============================================================================
namespace {

using namespace fa_sm100;

constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;   // one second

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult query{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// Per-device one-time state: architecture check and the shared-memory opt-in.
struct DeviceState {
    std::once_flag once;
    int status = FA_STATUS_OK;
    int sm_count = 0;
};
DeviceState g_devices[kMaxDevices];

int prepare_device(int device)
{
    if (device < 0 || device >= kMaxDevices) return FA_STATUS_INVALID_ARGUMENT;
    DeviceState& state = g_devices[device];
    std::call_once(state.once, [&]() {
        int major = 0;
        cudaError_t err = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
        if (err != cudaSuccess) { state.status = static_cast<int>(err); return; }
        if (major != 10) { state.status = FA_STATUS_NO_SM100; return; }
        err = cudaDeviceGetAttribute(&state.sm_count, cudaDevAttrMultiProcessorCount, device);
        if (err != cudaSuccess) { state.status = static_cast<int>(err); return; }
        const void* const kernels[] = {
            reinterpret_cast<const void*>(fa_fwd_kernel<64, false, false>),
            reinterpret_cast<const void*>(fa_fwd_kernel<64, true, false>),
            reinterpret_cast<const void*>(fa_fwd_kernel<64, false, true>),
            reinterpret_cast<const void*>(fa_fwd_kernel<128, false, false>),
            reinterpret_cast<const void*>(fa_fwd_kernel<128, true, false>),
            reinterpret_cast<const void*>(fa_fwd_kernel<128, false, true>)};
        for (int i = 0; i < 6 && err == cudaSuccess; ++i)
            err = cudaFuncSetAttribute(kernels[i], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       i < 3 ? Cfg<64>::kSmemBytes : Cfg<128>::kSmemBytes);
        if (err != cudaSuccess) { state.status = static_cast<int>(err); return; }
        // The warpgroup register split (setmaxnreg) waits forever if the CTA launched with
        // fewer registers than it hands out: refuse to launch such a build.
        for (const void* func : kernels) {
            cudaFuncAttributes attributes{};
            err = cudaFuncGetAttributes(&attributes, func);
            if (err != cudaSuccess) { state.status = static_cast<int>(err); return; }
            if (static_cast<uint32_t>(attributes.numRegs) * kThreads <
                2u * 128u * kRegsSoftmax + 128u * kRegsOther) {
                state.status = FA_STATUS_BUILD_MISMATCH;
                return;
            }
        }
    });
    return state.status;
}

// 3-D view [slabs, seq_len, head_dim] of a contiguous bf16 tensor; box = 64
// columns (128 bytes, the swizzle span) x 128 rows x 1 slab; rows past seq_len
// read as zero and are clipped on store.
int make_map(CUtensorMap* map, const void* ptr, long long slabs, int seq_len, int head_dim)
{
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return FA_STATUS_DRIVER_ENTRY;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(seq_len),
                                static_cast<cuuint64_t>(slabs)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * 2u,
                                   static_cast<cuuint64_t>(seq_len) * static_cast<cuuint64_t>(head_dim) * 2u};
    const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(kBlockM), 1u};
    const cuuint32_t elem_strides[3] = {1u, 1u, 1u};
    const CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                            elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return res == CUDA_SUCCESS ? FA_STATUS_OK : FA_STATUS_TENSOR_MAP;
}

// The four tensor maps of a call depend only on the base pointers and the shape, so a
// caller that launches on the same buffers again (a timing loop, a serving step) reuses
// them instead of encoding them on every call. Per host thread, a few entries, replaced
// round-robin; a pointer freed and reallocated keeps a valid map (same address, same shape).
struct MapSet {
    CUtensorMap q, k, v, o;
    const void* ptr[4];
    long long slabs;
    int seq_len;
    int head_dim;
    bool valid;
};
constexpr int kMapCacheEntries = 4;
thread_local MapSet t_maps[kMapCacheEntries];
thread_local int t_maps_next = 0;

int lookup_maps(const void* q, const void* k, const void* v, const void* o, long long slabs, int seq_len,
                int head_dim, const MapSet** out)
{
    for (const MapSet& set : t_maps) {
        if (set.valid && set.ptr[0] == q && set.ptr[1] == k && set.ptr[2] == v && set.ptr[3] == o &&
            set.slabs == slabs && set.seq_len == seq_len && set.head_dim == head_dim) {
            *out = &set;
            return FA_STATUS_OK;
        }
    }
    MapSet& set = t_maps[t_maps_next];
    t_maps_next = (t_maps_next + 1) % kMapCacheEntries;
    set.valid = false;
    int status;
    if ((status = make_map(&set.q, q, slabs, seq_len, head_dim)) != FA_STATUS_OK) return status;
    if ((status = make_map(&set.k, k, slabs, seq_len, head_dim)) != FA_STATUS_OK) return status;
    if ((status = make_map(&set.v, v, slabs, seq_len, head_dim)) != FA_STATUS_OK) return status;
    if ((status = make_map(&set.o, o, slabs, seq_len, head_dim)) != FA_STATUS_OK) return status;
    set.ptr[0] = q;
    set.ptr[1] = k;
    set.ptr[2] = v;
    set.ptr[3] = o;
    set.slabs = slabs;
    set.seq_len = seq_len;
    set.head_dim = head_dim;
    set.valid = true;
    *out = &set;
    return FA_STATUS_OK;
}

int validate(const void* q, const void* k, const void* v, const void* o, int batch, int heads, int seq_len,
             int head_dim, long long slab_begin, long long slab_end)
{
    if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return FA_STATUS_INVALID_ARGUMENT;
    if (batch <= 0 || heads <= 0 || seq_len <= 0) return FA_STATUS_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return FA_STATUS_UNSUPPORTED;
    const long long slabs = static_cast<long long>(batch) * heads;
    if (slabs > INT_MAX) return FA_STATUS_INVALID_ARGUMENT;
    if (seq_len > (1 << 30)) return FA_STATUS_INVALID_ARGUMENT;
    if (slab_begin < 0 || slab_end > slabs || slab_begin > slab_end) return FA_STATUS_INVALID_ARGUMENT;
    const uintptr_t any = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                          reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o);
    if (any & 15u) return FA_STATUS_MISALIGNED;
    return FA_STATUS_OK;
}

template <int D>
int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
           const Params& params, bool one_tile, long long slabs, cudaStream_t stream)
{
    const bool split = !one_tile && params.split_len > 0;
    const long long blocks = slabs * params.items;
    if (blocks <= 0) return FA_STATUS_OK;
    if (blocks > INT_MAX) return FA_STATUS_INVALID_ARGUMENT;
    const unsigned grid = static_cast<unsigned>(blocks);
    if (one_tile)
        fa_fwd_kernel<D, true, false><<<grid, kThreads, Cfg<D>::kSmemBytes, stream>>>(mq, mk, mv, mo, params);
    else if (split)
        fa_fwd_kernel<D, false, true><<<grid, kThreads, Cfg<D>::kSmemBytes, stream>>>(mq, mk, mv, mo, params);
    else
        fa_fwd_kernel<D, false, false><<<grid, kThreads, Cfg<D>::kSmemBytes, stream>>>(mq, mk, mv, mo, params);
    return static_cast<int>(cudaGetLastError());
}

// Test-only: a stall armed by fa_sm100_test_arm_stall for the next launch this host thread
// makes, whichever entry point makes it (0 = none armed).
thread_local unsigned long long t_armed_stall_ns = 0;
// Test-only: the kernel instantiation for this host thread's launches (fa_sm100_test_force_kernel):
// 0 = the launcher's choice, 1 = one Q tile per CTA, 2 = row pairs.
thread_local int t_forced_kernel = 0;
// Test-only: the causal key-range split for this host thread's launches
// (fa_sm100_test_force_split): -1 = the launcher's choice, 0 = none, L > 0 = chunks of L key tiles.
thread_local int t_forced_split = -1;

// Workspace of split launches (arrival counters, flags, partials): stream-ordered allocations from
// a per-device pool (cudaMallocFromPoolAsync / cudaFreeAsync on the launch stream), so that
// concurrent launches on different streams never share a workspace; the pool keeps its memory
// between launches (release threshold at its maximum).
struct SplitPool {
    std::once_flag once;
    int status = FA_STATUS_OK;
    cudaMemPool_t pool = nullptr;
};
SplitPool g_split_pools[kMaxDevices];

int split_pool(int device, cudaMemPool_t* out)
{
    SplitPool& sp = g_split_pools[device];
    std::call_once(sp.once, [&]() {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        cudaError_t err = cudaMemPoolCreate(&sp.pool, &props);
        if (err == cudaSuccess) {
            uint64_t keep = UINT64_MAX;
            err = cudaMemPoolSetAttribute(sp.pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
        if (err != cudaSuccess) {
            sp.status = static_cast<int>(err);
            cudaGetLastError();
        }
    });
    *out = sp.pool;
    return sp.status;
}

// Key tiles of unit u (a row pair) of a causal launch, and the chunks of a split.
inline int pair_tiles(int u, int kv_all) { return std::min(kv_all, 2 * u + 2); }
inline int split_items(int units, int kv_all, int split_len)
{
    int items = 0;
    for (int u = 0; u < units; ++u) items += (pair_tiles(u, kv_all) + split_len - 1) / split_len;
    return items;
}

int forward(const void* q, const void* k, const void* v, void* o, int batch, int heads, int seq_len, int head_dim,
            int causal, long long slab_begin, long long slab_end, void* stream, int inject_stall,
            unsigned long long timeout_ns, bool allow_workspace = true)
{
    int status = validate(q, k, v, o, batch, heads, seq_len, head_dim, slab_begin, slab_end);
    if (status != FA_STATUS_OK) return status;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return static_cast<int>(err);
    status = prepare_device(device);
    if (status != FA_STATUS_OK) return status;
    if (slab_end == slab_begin) return FA_STATUS_OK;

    const long long slabs = static_cast<long long>(batch) * heads;
    const MapSet* maps = nullptr;
    if ((status = lookup_maps(q, k, v, o, slabs, seq_len, head_dim, &maps)) != FA_STATUS_OK) return status;

    if (inject_stall == 0 && t_armed_stall_ns != 0) {
        inject_stall = 1;
        timeout_ns = t_armed_stall_ns;
        t_armed_stall_ns = 0;
    }
    const long long count = slab_end - slab_begin;
    const int sms = g_devices[device].sm_count;
    Params params{};
    params.seq_len = seq_len;
    // Kernel choice. A CTA normally takes a row pair (two Q tiles whose softmax phases overlap
    // on one SM). Dense: when even one CTA per Q tile would leave SMs idle, each Q tile gets its
    // own CTA instead (twice the CTAs, each with a shorter critical path). Causal: when the row
    // pairs fit in one wave, the longest CTA sets the time, and one Q tile per CTA (S double-
    // buffered, so its QK^T overlaps its softmax) shortens it: 0.60-0.76x the row-pair time at
    // (1,8,2048,D), (2,8,2048,D), (1,4,8192,D) and (1,2,16384,128) (B200, CUDA-graph replay).
    const int pairs = (seq_len + kRowsPerCta - 1) / kRowsPerCta;
    const int kv_all = (seq_len + kBlockN - 1) / kBlockN;
    bool single = causal ? count * pairs <= sms : count * pairs * kQTiles <= sms;
    // Causal key-range split (row-pair kernel only): chunks of split_len key tiles. Against one Q
    // tile per CTA it pays only for very long rows in a grid whose row pairs fit in one wave:
    // (1,1,32768,128) 296.1 -> 265.5 us in chunks of a sixth of the key tiles (halves: 295.6 us).
    // At D = 64, and up to 128 key tiles at D = 128, the one-tile kernel was faster than every
    // chunk length measured: (1,1,32768,64) 244.9 us against 266.1, (1,8,2048,D) 19.6 / 22.6
    // against 22.2 / 26.9, (1,4,8192,D) 64.4 / 74.8 against 86.3 / 89.4, (1,2,16384,128) 147.2
    // against 153.5.
    int split_len = 0;
    if (causal && head_dim == 128 && count * pairs <= sms && kv_all >= 256) {
        split_len = (kv_all + 5) / 6;
        single = false;
    }
    if (t_forced_split >= 0) split_len = t_forced_split;
    if (t_forced_kernel != 0) single = t_forced_kernel == 1;
    if (single || !causal || !allow_workspace) split_len = 0;
    if (split_len > 0) {
        split_len = std::max(split_len, (kv_all + kMaxChunks - 1) / kMaxChunks);
        if (split_len >= kv_all) split_len = 0;         // no unit would be split
    }
    params.num_units = single ? (seq_len + kBlockM - 1) / kBlockM : pairs;
    params.split_len = split_len;
    params.items = split_len > 0 ? split_items(pairs, kv_all, split_len) : params.num_units;
    params.slab_begin = slab_begin;
    params.scale_log2 = fa_default_scale(head_dim) * 1.4426950408889634f;
    params.causal = causal ? 1 : 0;
    params.inject_stall = inject_stall;
    params.timeout_ns = timeout_ns;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    params.num_slabs = count;
    {
        // Causal groups: as many slabs as keep the group's K and V within 32 MB of L2.
        const long long kv_bytes = 4LL * seq_len * head_dim;
        const long long by_l2 = kv_bytes > 0 ? (32LL << 20) / kv_bytes : count;
        params.chunk = static_cast<int>(std::max(1LL, std::min(count, by_l2)));
    }
    void* workspace = nullptr;
    if (split_len > 0) {
        // [arrival counters: slabs * units u64][flags: slabs * units * max_chunks u64]
        // [partials: slabs * units * max_chunks * 2 tiles * (D + 2) * 128 floats]. Nothing needs
        // zeroing: counters and flags carry this launch's epoch.
        params.max_chunks = (kv_all + split_len - 1) / split_len;
        const size_t units = static_cast<size_t>(count) * pairs;
        const size_t arrive_bytes = units * 8u;
        const size_t flag_bytes = units * params.max_chunks * 8u;
        const size_t partial_bytes = units * params.max_chunks * kQTiles * static_cast<size_t>(head_dim + 2) * kBlockM *
                                     sizeof(float);
        cudaMemPool_t pool = nullptr;
        int pool_status = split_pool(device, &pool);
        if (pool_status == FA_STATUS_OK &&
            cudaMallocFromPoolAsync(&workspace, arrive_bytes + flag_bytes + partial_bytes, pool, s) == cudaSuccess) {
            static std::atomic<unsigned long long> epochs{0};
            unsigned long long epoch = 0;
            while (epoch == 0) epoch = (epochs.fetch_add(1) + 1) & ((1ull << 48) - 1);
            params.epoch = epoch;
            params.arrive = static_cast<unsigned long long*>(workspace);
            params.flags = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + arrive_bytes);
            params.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + arrive_bytes + flag_bytes);
        } else {
            // No workspace: the unsplit launch computes the same result.
            cudaGetLastError();
            if (workspace != nullptr) cudaFreeAsync(workspace, s);
            workspace = nullptr;
            params.split_len = 0;
            params.items = params.num_units;
        }
    }
    const int launched = head_dim == 64 ? launch<64>(maps->q, maps->k, maps->v, maps->o, params, single, count, s)
                                        : launch<128>(maps->q, maps->k, maps->v, maps->o, params, single, count, s);
    if (workspace != nullptr) {
        const cudaError_t freed = cudaFreeAsync(workspace, s);
        if (launched == FA_STATUS_OK && freed != cudaSuccess) return static_cast<int>(freed);
    }
    return launched;
}

}  // namespace

namespace fa_sm100_internal {

int forward_without_workspace(const void* q, const void* k, const void* v, void* o, int batch, int heads,
                              int seq_len, int head_dim, int causal, void* stream)
{
    const long long slabs = (batch > 0 && heads > 0) ? static_cast<long long>(batch) * heads : 0;
    return forward(q, k, v, o, batch, heads, seq_len, head_dim, causal, 0, slabs, stream, 0, kDefaultTimeoutNs,
                   false);
}

int take_error_word(cudaStream_t stream, unsigned int* word)
{
    unsigned int value = 0;
    cudaError_t err = cudaMemcpyFromSymbolAsync(&value, g_fa_error_word, sizeof(value), 0, cudaMemcpyDeviceToHost,
                                                stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return static_cast<int>(err);
    if (word != nullptr) *word = value;
    if (value == 0) return FA_STATUS_OK;
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbolAsync(g_fa_error_word, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return static_cast<int>(err);
    return FA_STATUS_DEVICE_TIMEOUT;
}

}  // namespace fa_sm100_internal

extern "C" {

int fa_sm100_fwd(const void* q, const void* k, const void* v, void* o, int batch, int heads, int seq_len,
                 int head_dim, int causal, void* stream)
{
    const long long slabs = (batch > 0 && heads > 0) ? static_cast<long long>(batch) * heads : 0;
    return forward(q, k, v, o, batch, heads, seq_len, head_dim, causal, 0, slabs, stream, 0, kDefaultTimeoutNs);
}

int fa_sm100_fwd_slabs(const void* q, const void* k, const void* v, void* o, int batch, int heads, int seq_len,
                       int head_dim, int causal, long long slab_begin, long long slab_end, void* stream)
{
    return forward(q, k, v, o, batch, heads, seq_len, head_dim, causal, slab_begin, slab_end, stream, 0,
                   kDefaultTimeoutNs);
}

int fa_sm100_fwd_inject_stall(const void* q, const void* k, const void* v, void* o, int batch, int heads,
                              int seq_len, int head_dim, int causal, unsigned long long timeout_ns, void* stream)
{
    if (timeout_ns == 0 || timeout_ns > kDefaultTimeoutNs) return FA_STATUS_INVALID_ARGUMENT;
    const long long slabs = (batch > 0 && heads > 0) ? static_cast<long long>(batch) * heads : 0;
    return forward(q, k, v, o, batch, heads, seq_len, head_dim, causal, 0, slabs, stream, 1, timeout_ns);
}

int fa_sm100_test_arm_stall(unsigned long long timeout_ns)
{
    if (timeout_ns == 0 || timeout_ns > kDefaultTimeoutNs) return FA_STATUS_INVALID_ARGUMENT;
    t_armed_stall_ns = timeout_ns;
    return FA_STATUS_OK;
}

int fa_sm100_test_force_split(int split_len)
{
    if (split_len < -1) return FA_STATUS_INVALID_ARGUMENT;
    t_forced_split = split_len;
    return FA_STATUS_OK;
}

int fa_sm100_test_force_kernel(int kind)
{
    if (kind < 0 || kind > 2) return FA_STATUS_INVALID_ARGUMENT;
    t_forced_kernel = kind;
    return FA_STATUS_OK;
}

int fa_sm100_supported(int head_dim) { return (head_dim == 64 || head_dim == 128) ? 1 : 0; }

float fa_default_scale(int head_dim) { return 1.0f / std::sqrt(static_cast<float>(head_dim)); }

double fa_attention_flops(int batch, int heads, int seq_len, int head_dim, int causal)
{
    const double n = static_cast<double>(seq_len);
    const double pairs = causal ? n * (n + 1.0) / 2.0 : n * n;
    return 4.0 * pairs * static_cast<double>(head_dim) * static_cast<double>(batch) * static_cast<double>(heads);
}

double fa_sm100_min_bytes(int batch, int heads, int seq_len, int head_dim)
{
    return 4.0 * static_cast<double>(batch) * heads * seq_len * head_dim * 2.0;
}

// Traffic model of the row-pair kernel. The one-tile kernel, which only small grids use,
// fetches each K/V tile once per 128-row Q tile instead of once per pair.
double fa_sm100_hbm_bytes(int batch, int heads, int seq_len, int head_dim, int causal)
{
    const double element = 2.0;
    const double slabs = static_cast<double>(batch) * heads;
    double bytes = 2.0 * slabs * seq_len * head_dim * element;     // Q read once, O written once
    const int pairs = (seq_len + kRowsPerCta - 1) / kRowsPerCta;
    const int kv_all = (seq_len + kBlockN - 1) / kBlockN;
    double kv_tiles = 0.0;
    for (int pair = 0; pair < pairs; ++pair)
        kv_tiles += causal ? (2 * pair + 2 < kv_all ? 2 * pair + 2 : kv_all) : kv_all;
    bytes += 2.0 * slabs * kv_tiles * kBlockN * head_dim * element;   // a K and a V tile per visit
    return bytes;
}

int fa_sm100_query(int head_dim, FaTilingInfo* info)
{
    if (info == nullptr) return FA_STATUS_INVALID_ARGUMENT;
    std::memset(info, 0, sizeof(*info));
    info->supported = fa_sm100_supported(head_dim);
    if (!info->supported) return FA_STATUS_OK;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return static_cast<int>(err);
    const int status = prepare_device(device);
    if (status != FA_STATUS_OK) return status;
    const void* func = head_dim == 64 ? reinterpret_cast<const void*>(fa_fwd_kernel<64, false, false>)
                                      : reinterpret_cast<const void*>(fa_fwd_kernel<128, false, false>);
    const int dynamic_bytes = head_dim == 64 ? Cfg<64>::kSmemBytes : Cfg<128>::kSmemBytes;
    cudaFuncAttributes attributes{};
    if ((err = cudaFuncGetAttributes(&attributes, func)) != cudaSuccess) return static_cast<int>(err);
    info->block_size = kThreads;
    info->tile_kv = kBlockN;
    info->rows_per_block = kRowsPerCta;
    info->shared_bytes_per_block = static_cast<int>(attributes.sharedSizeBytes) + dynamic_bytes;
    info->registers_per_thread = attributes.numRegs;
    info->local_bytes_per_thread = static_cast<int>(attributes.localSizeBytes);
    int blocks = 0;
    if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, func, kThreads, dynamic_bytes)) != cudaSuccess)
        return static_cast<int>(err);
    info->max_blocks_per_sm = blocks;
    int shared_per_sm = 0;
    cudaDeviceGetAttribute(&shared_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
    info->device_shared_bytes_per_sm = shared_per_sm;
    info->shared_limited_blocks_per_sm =
        info->shared_bytes_per_block > 0 ? shared_per_sm / info->shared_bytes_per_block : 0;
    return FA_STATUS_OK;
}

int fa_sm100_device_status(unsigned int* detail)
{
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return static_cast<int>(err);
    unsigned int word = 0;
    err = cudaMemcpyFromSymbol(&word, g_fa_error_word, sizeof(word));
    if (err != cudaSuccess) return static_cast<int>(err);
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_fa_error_word, &zero, sizeof(zero));
    if (err != cudaSuccess) return static_cast<int>(err);
    if (detail != nullptr) *detail = word;
    return word ? FA_STATUS_DEVICE_TIMEOUT : FA_STATUS_OK;
}

int fa_sm100_debug_read(float* out, size_t floats)
{
#ifdef FA_SM100_DEBUG_DUMP
    if (out == nullptr || floats < static_cast<size_t>(kDbgFloats)) return FA_STATUS_INVALID_ARGUMENT;
    cudaError_t err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpyFromSymbol(out, g_fa_debug, sizeof(float) * kDbgFloats);
    return static_cast<int>(err);
#else
    (void)out;
    (void)floats;
    return FA_STATUS_UNSUPPORTED;
#endif
}

const char* fa_sm100_status_string(int status)
{
    switch (status) {
        case FA_STATUS_OK: return "ok";
        case FA_STATUS_INVALID_ARGUMENT: return "invalid argument";
        case FA_STATUS_UNSUPPORTED: return "unsupported head_dim (64 or 128)";
        case FA_STATUS_MISALIGNED: return "tensor base not 16-byte aligned";
        case FA_STATUS_NO_SM100: return "device is not sm_100 (B200)";
        case FA_STATUS_DRIVER_ENTRY: return "cuTensorMapEncodeTiled unavailable";
        case FA_STATUS_TENSOR_MAP: return "tensor map encoding failed";
        case FA_STATUS_DEVICE_TIMEOUT: return "device-side wait timed out";
        case FA_STATUS_HOST_ALLOC: return "staging allocation failed";
        case FA_STATUS_BUILD_MISMATCH: return "kernel built with fewer registers than its warpgroup split needs";
        case FA_STATUS_STATIC_TOO_LARGE: return "slab larger than the fixed staging of fa_sm100_fwd_host_static";
        default: break;
    }
    if (status > 0 && status < 1000) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

}  // extern "C"
