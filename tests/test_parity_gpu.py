"""Parity of the sm_100a kernel with the CPU FP64 oracle, through the C ABI.

Gate (bench_flash_attention.cu:52, :159-163): finite output
and max |O - bf16(O_ref)| <= 2.0 BF16 ULP of the row's output scale
(max_d |O_ref|), the reference's row-scale metric. Small shapes compare every
element; BASELINE configs 3-5 compare a deterministic sample of rows (first,
last, diagonal-adjacent rows of the first and last slab, plus a strided set)
and check the size-independent all-ones identity over the whole output.
Outputs are NaN-poisoned (bf16 0xFFFF) before each launch, as the reference
harness does (bench_flash_attention.cu:555-556), so unwritten elements fail.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2.0   # row-scale BF16 ULP


def _to_dev(bits, device):
    import torch
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def _to_host_bits(t):
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16).ravel()


def _poisoned_like(t):
    import torch
    o = torch.empty_like(t)
    o.view(torch.int16).fill_(-1)     # 0xFFFF = bf16 NaN
    return o


def run_kernel(q, k, v, shape, causal, device, stream=None):
    import torch
    from cuda_fused_attention_b200 import launch_attention_sm100
    dq, dk, dv = _to_dev(q, device), _to_dev(k, device), _to_dev(v, device)
    do = _poisoned_like(dq)
    launch_attention_sm100(dq, dk, dv, do, shape, causal, stream)
    torch.cuda.synchronize()
    return _to_host_bits(do)


def check_device_clean():
    from cuda_fused_attention_b200 import device_status
    status, word = device_status()
    assert status == 0 and word == 0, (status, hex(word))


def assert_parity(got, ref, d, what):
    acc = __import__("fa_oracle").compare(got, ref, d, TOL)
    assert acc["output_nan"] == 0 and acc["output_inf"] == 0, (what, acc)
    assert acc["passed"], (what, acc)
    return acc


def _full_case(oracle, cuda_device, b, h, n, d, causal, family=0):
    from cuda_fused_attention_b200 import AttentionShape
    q, k, v = oracle.make_inputs(b, h, n, d, family)
    ref = oracle.attention(q, k, v, b, h, n, d, causal)
    got = run_kernel(q, k, v, AttentionShape(b, h, n, d), causal, cuda_device)
    return assert_parity(got, ref, d, (b, h, n, d, causal, family))


def test_config1_plumbing(oracle, cuda_device):
    """(1,2,128,64) dense, every element."""
    acc = _full_case(oracle, cuda_device, 1, 2, 128, 64, 0)
    assert acc["ulp"] <= TOL
    check_device_clean()


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
def test_accuracy_shapes(oracle, cuda_device, d, causal):
    """The reference's accuracy suite shape (1,2,256,D) x mask (bench_flash_attention.cu:514-530)."""
    _full_case(oracle, cuda_device, 1, 2, 256, d, causal)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
def test_boundary_lengths(oracle, cuda_device, d, causal):
    """Lengths around the 128-key tile and 256-row CTA boundaries, plus the lite sweep's set."""
    for n in (1, 7, 63, 64, 65, 127, 128, 129, 255, 256, 257, 383, 511, 513):
        _full_case(oracle, cuda_device, 1, 2, n, d, causal)


def _single_tile_dispatch(slabs, n, causal=False):
    """The launcher's small-grid rule: one 128-row Q tile per CTA when a CTA per Q tile would
    still leave SMs idle (dense: slabs * row pairs * 2 <= SM count), or when the row pairs fit
    in one wave (causal: slabs * row pairs <= SM count); else a row pair per CTA."""
    import torch
    sm_count = torch.cuda.get_device_properties(0).multi_processor_count
    pairs = slabs * ((n + 255) // 256)
    return (pairs if causal else pairs * 2) <= sm_count


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
def test_boundary_lengths_row_pairs(oracle, cuda_device, d, causal):
    """The same boundaries on a grid large enough for row-pair CTAs, including pairs whose
    second Q tile has no valid row (N = 128, 257, 300, 383, 513): that tile is computed on
    zero-filled rows and its store is clipped."""
    from cuda_fused_attention_b200 import _lib
    lib = _lib.load()
    b, h = 3, 25
    try:
        assert lib.fa_sm100_test_force_kernel(2) == 0      # row pairs, whatever the grid
        for n in (1, 65, 128, 129, 255, 256, 257, 300, 383, 513):
            _full_case(oracle, cuda_device, b, h, n, d, causal)
    finally:
        lib.fa_sm100_test_force_kernel(0)
    assert not _single_tile_dispatch(b * h, 513, causal)
    assert _single_tile_dispatch(2, 513, causal)   # the (1, 2, N) cases above ran one tile per CTA
    check_device_clean()


@pytest.mark.parametrize("family", [1, 2, 3, 4])
def test_input_families(oracle, cuda_device, family):
    """kernels/ablation/experiments.cu:283-289: zeros, ones, structured V, Q,K x4."""
    for d in (64, 128):
        for causal in (0, 1):
            for n in (1, 33, 129, 300):
                _full_case(oracle, cuda_device, 1, 2, n, d, causal, family)


@pytest.mark.parametrize("causal", [0, 1])
def test_config2_full(oracle, cuda_device, causal):
    """(2,8,2048,64), every element."""
    _full_case(oracle, cuda_device, 2, 8, 2048, 64, causal)


def _sampled_rows(n, slabs):
    rows = {0, 1, 127, 128, 255, 256, n // 2, n - 2, n - 1}
    rows |= set(range(0, n, max(1, n // 48)))
    picks = []
    for slab in sorted({0, slabs // 2, slabs - 1}):
        for r in sorted(x for x in rows if 0 <= x < n):
            picks.append((slab, r))
    return picks


# The reference generator's inputs of the last sampled shape: config 5 has 1.6e9 values (tens of
# seconds on the host), generated once for its dense and its causal test.
_REFERENCE_INPUTS = {}


def _reference_inputs(oracle, b, h, n, d, family):
    key = (b, h, n, d, family)
    if key not in _REFERENCE_INPUTS:
        _REFERENCE_INPUTS.clear()
        _REFERENCE_INPUTS[key] = oracle.make_inputs(b, h, n, d, family)
    return _REFERENCE_INPUTS[key]


def _sampled_case(oracle, cuda_device, b, h, n, d, causal, family, generator):
    import torch
    from cuda_fused_attention_b200 import AttentionShape
    shape = AttentionShape(b, h, n, d)
    if generator == "reference":
        q, k, v = _reference_inputs(oracle, b, h, n, d, family)
        dq, dk, dv = _to_dev(q, cuda_device), _to_dev(k, cuda_device), _to_dev(v, cuda_device)
    else:   # seeded torch N(0,1) -> bf16 on the device (configs too large for the CPU generator)
        g = torch.Generator(device=cuda_device)
        ts = []
        for seed in (11, 22, 33):
            g.manual_seed(seed)
            ts.append(torch.randn(shape.numel, generator=g, device=cuda_device).to(torch.bfloat16))
        dq, dk, dv = ts
        if family == 5:
            dq = (dq.float() * 4).to(torch.bfloat16)
    do = _poisoned_like(dq)
    from cuda_fused_attention_b200 import launch_attention_sm100
    launch_attention_sm100(dq, dk, dv, do, shape, causal)
    torch.cuda.synchronize()
    check_device_clean()
    # No element left unwritten anywhere.
    assert not torch.isnan(do.float()).any().item()
    picks = _sampled_rows(n, b * h)
    slab_elems = n * d
    worst = None
    for slab in sorted({s for s, _ in picks}):
        rows = [r for s, r in picks if s == slab]
        sl = slice(slab * slab_elems, (slab + 1) * slab_elems)
        q = _to_host_bits(dq[sl]); k = _to_host_bits(dk[sl]); v = _to_host_bits(dv[sl])
        o = _to_host_bits(do[sl]).reshape(n, d)
        for r in rows:
            ref = oracle.attention_rows(q, k, v, n, d, causal, 0, r, r + 1)
            acc = assert_parity(o[r], ref, d, (b, h, n, d, causal, slab, r))
            worst = acc if worst is None or acc["ulp"] > worst["ulp"] else worst
    return worst


def test_config3_sampled(oracle, cuda_device):
    """(4,16,4096,128) causal, Q x 4 (peaky rows)."""
    _sampled_case(oracle, cuda_device, 4, 16, 4096, 128, 1, 5, "reference")


def test_config4_sampled(oracle, cuda_device):
    """(1,32,16384,128) causal, long context."""
    _sampled_case(oracle, cuda_device, 1, 32, 16384, 128, 1, 0, "reference")


@pytest.mark.parametrize("causal", [0, 1])
def test_config5_sampled(oracle, cuda_device, causal):
    """(16,32,8192,128) dense and causal."""
    _sampled_case(oracle, cuda_device, 16, 32, 8192, 128, causal, 0, "reference")


@pytest.mark.parametrize("causal", [0, 1])
def test_config5_all_ones_identity(cuda_device, causal):
    """Size-independent property over the whole config-5 output: Q=K=V=1 gives O=1 exactly."""
    import torch
    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100
    shape = AttentionShape(16, 32, 8192, 128)
    ones = torch.ones(shape.numel, dtype=torch.bfloat16, device=cuda_device)
    o = _poisoned_like(ones)
    launch_attention_sm100(ones, ones, ones, o, shape, causal)
    torch.cuda.synchronize()
    assert torch.equal(o, ones)
    check_device_clean()


def test_deterministic_and_stream(oracle, cuda_device):
    """Bit-identical across launches and on a non-default stream."""
    import torch
    from cuda_fused_attention_b200 import AttentionShape
    b, h, n, d = 2, 4, 1000, 128
    q, k, v = oracle.make_inputs(b, h, n, d)
    first = run_kernel(q, k, v, AttentionShape(b, h, n, d), 1, cuda_device)
    s = torch.cuda.Stream(device=cuda_device)
    second = run_kernel(q, k, v, AttentionShape(b, h, n, d), 1, cuda_device, stream=s)
    assert np.array_equal(first, second)


def test_cached_tensor_maps_follow_pointers_and_shape(oracle, cuda_device):
    """The launcher reuses encoded tensor maps per (pointers, shape). Six buffer sets (more than
    the per-thread cache holds), launched twice in turn, and one set of allocations launched
    as three different shapes and then the first again, must each match the oracle."""
    import torch
    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100
    count = 2 * 200 * 64
    sets = []
    for i in range(6):
        q, k, v = (oracle.fill_normal(count, 100 + 3 * i + j) for j in range(3))
        dq, dk, dv = (_to_dev(x, cuda_device) for x in (q, k, v))
        sets.append(((q, k, v), (dq, dk, dv, _poisoned_like(dq))))

    def launch_and_check(host, dev, b, h, n, d, causal):
        q, k, v = host
        dq, dk, dv, do = dev
        do.view(torch.int16).fill_(-1)
        launch_attention_sm100(dq, dk, dv, do, AttentionShape(b, h, n, d), causal)
        torch.cuda.synchronize()
        ref = oracle.attention(q, k, v, b, h, n, d, causal)
        assert_parity(_to_host_bits(do), ref, d, ("cached maps", b, h, n, d, causal))

    for _ in range(2):
        for host, dev in sets:
            launch_and_check(host, dev, 1, 2, 200, 64, 1)
    host, dev = sets[0]
    for b, h, n, d in [(1, 4, 100, 64), (1, 1, 200, 128), (2, 2, 50, 128), (1, 2, 200, 64)]:
        launch_and_check(host, dev, b, h, n, d, 0)
    check_device_clean()


def test_slab_range_writes_only_its_slabs(oracle, cuda_device):
    import torch
    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100_slabs
    b, h, n, d = 2, 3, 300, 64
    shape = AttentionShape(b, h, n, d)
    q, k, v = oracle.make_inputs(b, h, n, d)
    ref = oracle.attention(q, k, v, b, h, n, d, 0)
    dq, dk, dv = _to_dev(q, cuda_device), _to_dev(k, cuda_device), _to_dev(v, cuda_device)
    do = _poisoned_like(dq)
    launch_attention_sm100_slabs(dq, dk, dv, do, shape, False, 2, 5)
    torch.cuda.synchronize()
    got = _to_host_bits(do).reshape(b * h, n * d)
    assert np.all(got[:2] == 0xFFFF) and np.all(got[5:] == 0xFFFF)
    assert_parity(got[2:5].ravel(), ref.reshape(b * h, n * d)[2:5].ravel(), d, "slabs 2..5")


def test_host_entry_matches_device_entry(oracle, cuda_device):
    """fa_sm100_fwd_host (H2D + forward + D2H, chunk-pipelined) equals the device entry bit for bit."""
    import torch
    from cuda_fused_attention_b200 import AttentionShape, attention_forward_host
    b, h, n, d = 3, 20, 2048, 128          # 60 slabs: several 64 MB chunks
    shape = AttentionShape(b, h, n, d)
    q, k, v = oracle.make_inputs(b, h, n, d)
    for causal in (0, 1):
        want = run_kernel(q, k, v, shape, causal, cuda_device)
        hq, hk, hv = (torch.from_numpy(x.view(np.int16)).pin_memory() for x in (q, k, v))
        ho = torch.empty_like(hq).pin_memory()
        ho.fill_(-1)
        attention_forward_host(hq, hk, hv, ho, shape, causal)
        assert np.array_equal(ho.numpy().view(np.uint16), want)
        po = np.full_like(q, 0xFFFF)           # pageable host memory works too
        attention_forward_host(q, k, v, po, shape, causal)
        assert np.array_equal(po, want)


def test_against_reference_v3_built_for_sm100(oracle, cuda_device):
    """The reference's own v3 kernel (kernels/v3/v3_tensorcore.cu) built for sm_100a, run on the
    same inputs, as a second opinion. Ours must pass the gate on every shape. v3's error is
    reported, not asserted: built for sm_100a it exceeds the gate and is not run-to-run
    deterministic on B200 (two launches on the same inputs can differ), even at its own accuracy
    shape (1,2,256,D) which it passes on the reference's sm_86 GPU."""
    import torch
    ref_lib = oracle.load_reference()
    if ref_lib is None:
        pytest.skip("oracle/_ref/libfa_ref.so was not built (needs the reference tree at build time)")
    from cuda_fused_attention_b200 import AttentionShape
    report = []
    for (b, h, n, d, causal) in [(1, 2, 256, 64, 0), (1, 2, 256, 64, 1), (1, 2, 256, 128, 0), (1, 2, 256, 128, 1),
                                 (1, 2, 512, 64, 1), (1, 2, 1024, 128, 1), (2, 8, 2048, 64, 0),
                                 (2, 8, 2048, 64, 1), (1, 4, 1000, 128, 0)]:
        q, k, v = oracle.make_inputs(b, h, n, d)
        ref = oracle.attention(q, k, v, b, h, n, d, causal)
        mine = run_kernel(q, k, v, AttentionShape(b, h, n, d), causal, cuda_device)
        mine_again = run_kernel(q, k, v, AttentionShape(b, h, n, d), causal, cuda_device)
        a_mine = assert_parity(mine, ref, d, "sm100")
        assert np.array_equal(mine, mine_again)
        dq, dk, dv = _to_dev(q, cuda_device), _to_dev(k, cuda_device), _to_dev(v, cuda_device)
        runs = []
        for _ in range(2):
            do = _poisoned_like(dq)
            torch.cuda.synchronize()
            rc = ref_lib.ref_launch_tensorcore_v3(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(),
                                                  b, h, n, d, causal, None)
            assert rc == 0
            torch.cuda.synchronize()
            runs.append(_to_host_bits(do))
        theirs = oracle.compare(runs[0], ref, d, TOL)
        report.append(f"({b},{h},{n},{d}) causal={causal}: sm100 {a_mine['ulp']:.2f} ulp (deterministic), "
                      f"v3@sm_100a {theirs['ulp']:.2f} ulp, v3 run-to-run identical: "
                      f"{bool(np.array_equal(runs[0], runs[1]))}")
    print("\n".join(report))


def test_config1_against_reference_unfused(oracle, cuda_device):
    """BASELINE config 1 names v0_unfused as the plumbing second opinion (kernels/v0_unfused.cu:140)."""
    import torch
    ref_lib = oracle.load_reference()
    if ref_lib is None:
        pytest.skip("oracle/_ref/libfa_ref.so was not built")
    from cuda_fused_attention_b200 import AttentionShape
    b, h, n, d = 1, 2, 128, 64
    q, k, v = oracle.make_inputs(b, h, n, d)
    ref = oracle.attention(q, k, v, b, h, n, d, 0)
    mine = run_kernel(q, k, v, AttentionShape(b, h, n, d), 0, cuda_device)
    dq, dk, dv = _to_dev(q, cuda_device), _to_dev(k, cuda_device), _to_dev(v, cuda_device)
    do = _poisoned_like(dq)
    ws = torch.empty(int(ref_lib.ref_unfused_workspace_bytes(b, h, n, d)) // 4, dtype=torch.float32,
                     device=cuda_device)
    assert ref_lib.ref_launch_unfused(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), ws.data_ptr(),
                                      b, h, n, d, 0, None) == 0
    torch.cuda.synchronize()
    assert_parity(_to_host_bits(do), ref, d, "v0")
    assert_parity(mine, ref, d, "sm100")


def test_query_reports_resources(cuda_device):
    from cuda_fused_attention_b200 import query_sm100
    for d in (64, 128):
        info = query_sm100(d)
        assert info["supported"] == 1 and info["block_size"] == 384 and info["tile_kv"] == 128
        assert info["rows_per_block"] == 256 and info["max_blocks_per_sm"] == 1
        assert info["local_bytes_per_thread"] < 64
    assert query_sm100(96)["supported"] == 0


def test_one_tile_kernel_equals_row_pair_kernel(oracle, cuda_device):
    """The two instantiations give the same bits for every row, whatever the launcher picks:
    the one-tile kernel spreads a row over two threads but keeps the row-pair kernel's
    arithmetic (same base decisions, same summation order). Forced on the same shapes,
    including the x4 families, whose peaky rows move the exponent base on either half of a
    tile. (Launches the launcher splits by key range sum in another order: within tolerance
    of these, tests/test_split_gpu.py.)"""
    import torch
    from cuda_fused_attention_b200 import AttentionShape, _lib
    lib = _lib.load()
    assert lib.fa_sm100_test_force_split(0) == 0      # the key-range split sums differently
    try:
        for (b, h, n, d) in [(2, 5, 1500, 64), (3, 4, 1000, 128), (1, 3, 4096, 128), (2, 2, 300, 64)]:
            for family in (0, 4, 5):
                q, k, v = oracle.make_inputs(b, h, n, d, family)
                for causal in (0, 1):
                    outs = []
                    for kind in (1, 2):
                        assert lib.fa_sm100_test_force_kernel(kind) == 0
                        outs.append(run_kernel(q, k, v, AttentionShape(b, h, n, d), causal, cuda_device))
                    assert np.array_equal(outs[0], outs[1]), (b, h, n, d, family, causal)
        check_device_clean()
    finally:
        lib.fa_sm100_test_force_kernel(0)
        lib.fa_sm100_test_force_split(-1)


@pytest.mark.parametrize("b, h, n, d, causal", [(1, 1, 32768, 128, 1), (1, 1, 32768, 64, 1), (1, 2, 16384, 128, 1),
                                                (1, 1, 32768, 128, 0)])
def test_long_rows_sampled(oracle, cuda_device, b, h, n, d, causal):
    """Long rows in a grid of few slabs, where the launcher's choice differs: (1,1,32768,128)
    causal splits each row pair's 256 key tiles into chunks of a sixth (partials merged in chunk
    order); (1,1,32768,64) and (1,2,16384,128) causal run one Q tile per CTA through 256 and 128
    key tiles (S double-buffered); (1,1,32768,128) dense runs 128 row-pair CTAs. Sampled rows
    against the FP64 oracle, the reference's own generator."""
    _sampled_case(oracle, cuda_device, b, h, n, d, causal, 0, "reference")


@pytest.mark.parametrize("kernel, split, b, h, n, causal", [(1, 0, 1, 2, 700, 1), (2, 0, 2, 3, 700, 0),
                                                             (2, 3, 1, 2, 2048, 1)])
def test_in_place_output_and_shared_k_v(oracle, cuda_device, kernel, split, b, h, n, causal):
    """O written over Q (each Q tile is read by one CTA, before it writes the same rows of O; with
    the key-range split the merging chunk stores only after every other chunk of its rows has
    published), and one tensor passed as both K and V: the same bits as separate buffers, for
    one Q tile per CTA, row pairs, and row pairs with the key range split."""
    import torch
    from cuda_fused_attention_b200 import AttentionShape, _lib, launch_attention_sm100
    lib = _lib.load()
    d = 128
    q, k, _ = oracle.make_inputs(b, h, n, d)
    shape = AttentionShape(b, h, n, d)
    assert lib.fa_sm100_test_force_kernel(kernel) == 0 and lib.fa_sm100_test_force_split(split) == 0
    try:
        dq, dk = _to_dev(q, cuda_device), _to_dev(k, cuda_device)
        dkv = dk.clone()                        # V = K, as its own buffer
        separate = _poisoned_like(dq)
        launch_attention_sm100(dq, dk, dkv, separate, shape, causal)
        shared = _poisoned_like(dq)
        launch_attention_sm100(dq, dk, dk, shared, shape, causal)          # K and V: one tensor
        in_place = dq.clone()
        launch_attention_sm100(in_place, dk, dk, in_place, shape, causal)  # O over Q
        torch.cuda.synchronize()
    finally:
        lib.fa_sm100_test_force_split(-1)
        lib.fa_sm100_test_force_kernel(0)
    check_device_clean()
    want = _to_host_bits(separate)
    assert np.array_equal(_to_host_bits(shared), want)
    assert np.array_equal(_to_host_bits(in_place), want)
    ref = oracle.attention(q, k, k, b, h, n, d, causal)
    assert oracle.compare(want, ref, d, 2.0)["passed"]


@pytest.mark.parametrize("causal", [0, 1])
def test_tensors_past_2_31_elements(oracle, cuda_device, causal):
    """(65,32,8192,128): 2.18e9 elements per tensor (4.4 GB each). The last slab starts past 2^31
    elements, so a 32-bit index or offset anywhere on the path (tensor maps, slab coordinates,
    work-item decode) would show as a wrong or unwritten last slab. Sampled rows of the first,
    middle and last slab against the FP64 oracle; no element left unwritten (seeded torch inputs
    on the device)."""
    import torch
    free, _ = torch.cuda.mem_get_info()
    if free < 24 << 30:
        pytest.skip("needs 24 GiB of free device memory")
    _sampled_case(oracle, cuda_device, 65, 32, 8192, 128, causal, 0, "torch")
