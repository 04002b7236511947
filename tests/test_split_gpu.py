"""The causal key-range split of the row-pair kernel, through the C ABI.

A causal grid that fits in one wave is as slow as its heaviest row pair, which sees every key
tile up to the diagonal. The launcher can split such pairs: a pair with more than L key tiles
is processed by several CTAs ("chunks") of at most L key tiles each; every chunk writes its
unnormalised O with its row maxima and sums to a workspace and counts itself in, and the chunk
that completes the pair merges all partials in chunk order and stores the output.

These tests force the split (fa_sm100_test_force_split) on shapes the launcher would not split,
so that every chunk length from one key tile up is covered: L = 1 gives Q tile 0 of each pair a
chunk that is entirely masked (an empty partial). Gate: the reference's 2-ULP row-scale BF16
tolerance against the FP64 oracle; and the result is deterministic (the merge order does not
depend on which chunk finishes last).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2.0


def _run(lib, q, k, v, shape, causal, device, split, kernel=2):
    import torch
    from cuda_fused_attention_b200 import launch_attention_sm100
    dq, dk, dv = (torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(device) for x in (q, k, v))
    do = torch.empty_like(dq)
    do.view(torch.int16).fill_(-1)
    assert lib.fa_sm100_test_force_kernel(kernel) == 0
    assert lib.fa_sm100_test_force_split(split) == 0
    try:
        launch_attention_sm100(dq, dk, dv, do, shape, causal)
        torch.cuda.synchronize()
    finally:
        lib.fa_sm100_test_force_split(-1)
        lib.fa_sm100_test_force_kernel(0)
    return do.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("d", [64, 128])
def test_split_matches_oracle_for_every_chunk_length(oracle, cuda_device, d):
    from cuda_fused_attention_b200 import AttentionShape, _lib, device_status
    lib = _lib.load()
    for (b, h, n) in [(2, 3, 1000), (1, 4, 2048), (3, 2, 300)]:
        for family in (0, 4, 5):
            q, k, v = oracle.make_inputs(b, h, n, d, family)
            ref = oracle.attention(q, k, v, b, h, n, d, 1)
            for split in (1, 2, 3, 5):
                got = _run(lib, q, k, v, AttentionShape(b, h, n, d), 1, cuda_device, split)
                acc = oracle.compare(got, ref, d, TOL)
                assert acc["output_nan"] == 0 and acc["output_inf"] == 0, (b, h, n, d, family, split, acc)
                assert acc["passed"], (b, h, n, d, family, split, acc)
    assert device_status() == (0, 0)


def test_split_is_deterministic_and_close_to_unsplit(oracle, cuda_device):
    from cuda_fused_attention_b200 import AttentionShape, _lib
    lib = _lib.load()
    b, h, n, d = 16, 4, 1024, 64          # 64 slabs: counters and partials of many pairs at once
    q, k, v = oracle.make_inputs(b, h, n, d)
    shape = AttentionShape(b, h, n, d)
    first = _run(lib, q, k, v, shape, 1, cuda_device, 2)
    second = _run(lib, q, k, v, shape, 1, cuda_device, 2)
    assert np.array_equal(first, second)
    unsplit = _run(lib, q, k, v, shape, 1, cuda_device, 0)
    ref = oracle.attention(q, k, v, b, h, n, d, 1)
    for got in (first, unsplit):
        assert oracle.compare(got, ref, d, TOL)["passed"]


def test_split_is_ignored_where_it_does_not_apply(oracle, cuda_device):
    """Dense launches and the one-tile kernel never split; a forced split there is a no-op."""
    from cuda_fused_attention_b200 import AttentionShape, _lib
    lib = _lib.load()
    b, h, n, d = 1, 2, 700, 128
    q, k, v = oracle.make_inputs(b, h, n, d)
    shape = AttentionShape(b, h, n, d)
    for causal, kernel in ((0, 2), (1, 1)):
        plain = _run(lib, q, k, v, shape, causal, cuda_device, 0, kernel)
        forced = _run(lib, q, k, v, shape, causal, cuda_device, 1, kernel)
        assert np.array_equal(plain, forced)
