"""The CPU oracle (oracle/fa_oracle.cpp) pinned against the reference's own functions.

tests/golden/golden.json was produced by tests/golden/make_golden.py from the
reference's generator, FP64 oracle and comparison compiled from its sources
(benchmarks/bench_flash_attention.cu:86-218, kernels/v0_unfused.cu:118-126).
Every case here must reproduce it bit for bit.
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.json")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as fh:
        return json.load(fh)


def _bf16_round(values):
    f = values.astype(np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def test_golden_cases_bit_exact(oracle, golden):
    assert len(golden["cases"]) >= 90
    for case in golden["cases"]:
        b, h, n, d = case["shape"]
        q, k, v = oracle.make_inputs(b, h, n, d, case["family"])
        assert _sha(q) == case["q_sha256"], case
        assert _sha(k) == case["k_sha256"], case
        assert _sha(v) == case["v_sha256"], case
        out = oracle.attention(q, k, v, b, h, n, d, case["causal"])
        assert _sha(out) == case["out_sha256"], case
        assert [float(x) for x in out[:4]] == case["out_head"]


def test_golden_compare_metric(oracle, golden):
    """The comparison restatement gives the reference's Accuracy fields exactly."""
    for case in golden["cases"][:60]:
        b, h, n, d = case["shape"]
        q, k, v = oracle.make_inputs(b, h, n, d, case["family"])
        ref = oracle.attention(q, k, v, b, h, n, d, case["causal"])
        got = _bf16_round(ref)
        got[::7] = got[::7] + np.uint16(1)
        acc = oracle.compare(got, ref, d)
        want = case["perturbed_compare"]
        mine = [acc["vs_double"], acc["row_scaled"], acc["max_abs"], acc["ulp"], acc["output_nan"],
                acc["output_inf"], acc["reference_nan"], acc["reference_inf"], float(acc["passed"])]
        for a, w in zip(mine, want):
            assert (a == w) or (math.isinf(a) and math.isinf(w)), (case["shape"], mine, want)


def test_golden_ulp_and_flops(oracle, golden):
    for arg, want in golden["bf16_ulp"]:
        value = float("inf") if arg == "inf" else arg
        assert oracle.bf16_ulp(value) == want
    for cfg, causal, want in golden["attention_flops"]:
        assert oracle.attention_flops(*cfg, causal) == want


def test_rows_variant_matches_full(oracle):
    b, h, n, d = 1, 3, 200, 64
    q, k, v = oracle.make_inputs(b, h, n, d)
    for causal in (0, 1):
        full = oracle.attention(q, k, v, b, h, n, d, causal).reshape(b * h, n, d)
        part = oracle.attention_rows(q, k, v, n, d, causal, 2, 37, 150).reshape(-1, d)
        assert np.array_equal(part, full[2, 37:150])


def test_parallel_matches_serial(oracle):
    b, h, n, d = 2, 3, 130, 128
    q, k, v = oracle.make_inputs(b, h, n, d)
    serial = oracle.attention(q, k, v, b, h, n, d, 1, threads=1)
    parallel = oracle.attention(q, k, v, b, h, n, d, 1, threads=4)
    assert np.array_equal(serial, parallel)


def test_hand_computable_cases(oracle):
    """N=1 returns V[0]; all-ones returns exactly 1 (the SURVEY's golden self-tests)."""
    for d in (64, 128):
        q, k, v = oracle.make_inputs(1, 2, 1, d)
        out = oracle.attention(q, k, v, 1, 2, 1, d, 0)
        vf = (v.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        assert np.array_equal(out, vf)
        q, k, v = oracle.make_inputs(1, 2, 65, d, family=2)
        out = oracle.attention(q, k, v, 1, 2, 65, d, 1)
        assert np.all(out == 1.0)


def test_live_against_reference_build(oracle):
    """Where oracle/_ref was built (reference tree present), compare on fresh shapes."""
    ref = oracle.load_reference()
    if ref is None:
        pytest.skip("oracle/_ref/libfa_ref.so not built here (reference tree absent)")
    import ctypes
    for (b, h, n, d, c) in [(1, 1, 77, 64, 1), (2, 1, 190, 128, 0)]:
        q, k, v = oracle.make_inputs(b, h, n, d)
        mine = oracle.attention(q, k, v, b, h, n, d, c)
        theirs = np.empty_like(mine)
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        ref.ref_reference_attention(p(q), p(k), p(v), p(theirs), b, h, n, d, c)
        assert np.array_equal(mine.view(np.uint64), theirs.view(np.uint64))
