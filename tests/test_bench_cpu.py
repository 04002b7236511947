"""Host logic of bench.py that needs no GPU: the result line, the clock/power summary, the
slab partition and the roofline inputs it reads from files."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def test_stdout_carries_only_the_result_line():
    # A child that writes to file descriptor 1 from below Python (as NCCL does) after the
    # bench has taken stdout for its result: only the JSON line may reach stdout.
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench\n"
        "bench._keep_stdout_for_result()\n"
        "os.write(1, b'NCCL version banner\\n')\n"
        "print('a library print')\n"
        "bench.emit({'metric': 'm', 'value': 1.0})\n" % ROOT)
    run = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    lines = run.stdout.splitlines()
    assert len(lines) == 1 and json.loads(lines[0]) == {"metric": "m", "value": 1.0}
    assert "NCCL version banner" in run.stderr and "a library print" in run.stderr


def test_clock_summary_parses_samples():
    bench = _bench()
    sampler = bench.ClockSampler(0)
    sampler.lines = [(float(i), line) for i, line in enumerate([
        "1965, 1965, 420.5, Not Active, Not Active, Not Active, Not Active",
        "1605, 1965, 995.1, Not Active, Not Active, Not Active, Active",
        "1590, 1965, 1002.3, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ])]
    summary = sampler.summary()
    assert summary["samples"] == 3
    assert summary["sm_mhz"] == 1605 and summary["sm_max_mhz"] == 1965
    assert summary["reasons"] == ["sw_power_cap"]
    assert summary["power_w"] == 995.1 and summary["power_max_w"] == 1002.3
    assert bench.ClockSampler(0).summary()["samples"] == 0
    # A window that starts at the second sample drops the idle first one.
    late = sampler.summary(since=1.0)
    assert late["samples"] == 2 and late["sm_mhz"] == (1605 + 1590) / 2
    # Round trip through the fixed-length form the ranks all-gather.
    back = bench.clock_summary_from_fields(bench.clock_fields(summary))
    assert back["sm_mhz"] == 1605 and back["reasons"] == ["sw_power_cap"] and back["samples"] == 3


def test_cpu_step_gives_every_thread_a_whole_slab_of_one_mask():
    """A reference-arm step: every host thread one whole slab with the same mask (so no thread
    idles while another finishes); flops counted with the reference's FLOP formula; the
    reference's own function when oracle/_ref is built."""
    bench = _bench()
    import fa_oracle
    for causal in (0, 1):
        flops, seconds, kind = bench.cpu_slab_step(3, 256, 64, causal)
        assert flops == 3 * fa_oracle.attention_flops(1, 1, 256, 64, causal)
        assert seconds > 0
        assert kind == ("reference" if fa_oracle.load_reference() is not None else "port")
    sample = bench.cpu_sample(2, 3, 128, 64)
    assert sample["flops"] == 2 * (2 * fa_oracle.attention_flops(1, 1, 128, 64, 0) +
                                   fa_oracle.attention_flops(1, 1, 128, 64, 1))
    assert set(sample["per_mask"]) == {"dense", "causal"}


def test_slab_ranges_cover_every_slab_once():
    bench = _bench()
    for total in (1, 7, 512):
        for world in (1, 2, 3, 8):
            ranges = [bench.slab_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - b for b, e in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_roofline_inputs():
    bench = _bench()
    peak, source = bench.measured_peak()
    assert peak > 0 and source
    traffic = bench.profile_traffic()
    assert traffic is not None and traffic["bytes_per_launch"] > 0
    # At least Q, K and V of a config-5 launch are read once, and O is written (partly still in L2).
    minimum = 3 * 16 * 32 * 8192 * 128 * 2
    assert traffic["bytes_per_launch"] >= minimum


def test_cpu_extrapolation_is_exact_by_flops():
    bench = _bench()
    from cuda_fused_attention_b200 import AttentionShape, attention_flops
    full = AttentionShape(16, 32, 8192, 128)
    want = attention_flops(full, False) + attention_flops(full, True)
    e = bench.cpu_extrapolation(0.02)
    assert e["step_flops"] == want
    assert abs(e["step_s"] - want / 0.02e12) < 1e-9 * e["step_s"]
    assert "not measured" in e["note"]
