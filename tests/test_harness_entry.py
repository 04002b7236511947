"""The kernel registered as one more Entry of the reference's own benchmark harness.

oracle/_ref/harness_sm100 (built from oracle/harness_sm100.cu where the reference tree
exists) compiles the reference's benchmarks/bench_flash_attention.cu unmodified, adds the
runner and Entry a maintainer would add (:366-387) and runs the file's accuracy suite
(:507-586) and performance loop (:588-700). It includes include/flash_attention_sm100.h
next to the reference's include/flash_attention.h, so it only links if the C++ API is
ABI-compatible with the reference's AttentionShape and FusedTilingInfo.

The CPU test runs its host-only mode; the GPU test runs both procedures over the
harness's own 60-case grid (kCases, :75-84) for v0 (the harness's speed-up baseline),
the reference's v3 built for sm_100a, and this kernel.
"""
import json
import math
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "harness_sm100")


def _harness_or_skip():
    if not os.path.exists(HARNESS):
        pytest.skip("oracle/_ref/harness_sm100 not built (needs the reference tree at build time)")
    return HARNESS


def _run(args, timeout):
    run = subprocess.run([_harness_or_skip(), *args], capture_output=True, text=True, timeout=timeout)
    lines = [json.loads(line) for line in run.stdout.splitlines() if line.startswith("{")]
    return run, lines


def test_host_functions_through_reference_types():
    run, lines = _run(["--host-only"], timeout=120)
    assert run.returncode == 0, run.stderr
    head, rows = lines[0], lines[1:]
    assert head["sm100_supported"] == [0, 1, 0, 1]
    assert head["sm100_supported"] == head["v3_supported"]   # same supported domain as v3
    assert len(rows) == 12
    for row in rows:
        # The reference's attention_flops on its own AttentionShape equals the C ABI's.
        assert row["attention_flops"] == row["fa_attention_flops"]
        # sm100_hbm_bytes receives the reference's AttentionShape by reference: the same
        # value as the plain-int C entry point means the layouts agree.
        assert row["sm100_hbm_bytes"] == row["fa_sm100_hbm_bytes"]
        assert row["sm100_hbm_bytes"] < row["v3_hbm_bytes"]   # 256-row CTAs re-read K/V less


def test_rejects_unknown_arguments():
    run, _ = _run(["--entries", "no_such_kernel"], timeout=60)
    assert run.returncode == 2
    run, _ = _run(["--cases", "1,2,3"], timeout=60)
    assert run.returncode == 2


@pytest.mark.gpu
def test_reference_harness_with_sm100_entry():
    run, lines = _run(["--entries", "v0_unfused,v3_tensorcore,sm100_tcgen05", "--cases", "grid"], timeout=1200)
    assert run.returncode == 0, run.stderr[-2000:]
    device = lines[0]
    assert device["sm"].startswith("10")
    tiling = [line for line in lines if "tiling" in line]
    assert [t["head_dim"] for t in tiling] == [64, 128] and all(t["supported"] for t in tiling)
    assert all(t["local_bytes_per_thread"] == 0 for t in tiling)

    accuracy = [line for line in lines if line.get("suite") == "accuracy" and line["kernel"] == "sm100_tcgen05"]
    assert len(accuracy) == 4
    for line in accuracy:
        assert line["passed"] and line["status"] == 0
        assert line["output_nan"] == 0 and line["output_inf"] == 0
        assert line["row_scale_ulp"] <= 2.0

    performance = [line for line in lines if line.get("suite") == "performance"]
    ours = {(l["batch"], l["seq_len"], l["head_dim"], l["causal"]): l
            for l in performance if l["kernel"] == "sm100_tcgen05"}
    v3 = {(l["batch"], l["seq_len"], l["head_dim"], l["causal"]): l
          for l in performance if l["kernel"] == "v3_tensorcore"}
    assert len(ours) == 60 and len(v3) == 60
    for key, line in ours.items():
        assert line["status"] == "ok" and line["launch_status"] == 0, (key, line)
        assert line["output_nan"] == 0 and line["output_inf"] == 0
    ratios = {key: v3[key]["median_ms"] / ours[key]["median_ms"] for key in ours}
    geomean = math.exp(sum(math.log(r) for r in ratios.values()) / len(ratios))
    print(f"\nreference harness grid, speed-up over v3 (sm_100a build): geomean {geomean:.2f}x, "
          f"min {min(ratios.values()):.2f}x, max {max(ratios.values()):.2f}x")
    for key in sorted(ours):
        b, n, d, c = key
        print(f"  B={b} H=8 N={n:5d} D={d:3d} causal={c}: sm100 {ours[key]['median_ms']:.4f} ms "
              f"({ours[key]['tflops']:.1f} TFLOP/s)  v3 {v3[key]['median_ms']:.4f} ms  x{ratios[key]:.2f}")
    assert geomean > 1.0
