"""The C-ABI library loads and exports every entry point include/*.h declares.

CPU-only: no call here reaches a GPU. Argument validation happens on the host
before any CUDA call, so rejected arguments are checked here too.
"""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_c_symbols():
    names = []
    for fname in sorted(os.listdir(os.path.join(ROOT, "include"))):
        text = open(os.path.join(ROOT, "include", fname)).read()
        names += re.findall(r"FA_API\s+[\w\s\*]*?\b(fa_\w+)\s*\(", text)
    return sorted(set(names))


def _declared_cpp_symbols():
    text = open(os.path.join(ROOT, "include", "flash_attention_sm100.h")).read()
    return sorted(set(re.findall(r"FA_API\s+[\w:\s\*]*?\b(sm100_\w+|launch_attention_sm100|query_sm100)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from cuda_fused_attention_b200 import _lib
    return _lib.load()


def test_every_declared_c_symbol_is_exported(lib):
    from cuda_fused_attention_b200 import _lib
    declared = _declared_c_symbols()
    assert len(declared) >= 13
    assert set(declared) == set(_lib.SIGNATURES), "binding table out of sync with include/fa_sm100.h"
    for name in declared:
        assert hasattr(lib, name), name


def test_cpp_api_symbols_exported(lib):
    path = lib._name
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", path], capture_output=True, text=True, check=True).stdout
    for name in _declared_cpp_symbols():
        assert re.search(r"cuda_op_lab::flash_attention::" + name + r"\(", out), name


def test_no_library_internals_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib._name], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    plain_c = {s for s in exported if s.startswith("fa_")}
    assert plain_c == set(_declared_c_symbols())


def test_host_only_functions(lib):
    from cuda_fused_attention_b200 import AttentionShape, attention_flops, default_scale, sm100_hbm_bytes, \
        sm100_min_bytes, sm100_supported
    assert sm100_supported(64) and sm100_supported(128)
    assert not sm100_supported(96) and not sm100_supported(256)
    import numpy as np
    assert default_scale(128) == float(np.float32(1.0) / np.sqrt(np.float32(128)))
    assert default_scale(64) == 0.125
    cfg5 = AttentionShape(16, 32, 8192, 128)
    assert attention_flops(cfg5, False) == 4.0 * 8192 * 8192 * 128 * 16 * 32
    assert attention_flops(cfg5, True) == 4.0 * 8192 * 8193 / 2 * 128 * 16 * 32
    assert sm100_min_bytes(cfg5) == 4 * 16 * 32 * 8192 * 128 * 2
    # Traffic model: Q+O once, plus a K and a V tile per 256-row CTA per key tile.
    assert sm100_hbm_bytes(cfg5, False) == 2 * 16 * 32 * 8192 * 128 * 2 + 2.0 * 512 * 32 * 64 * 128 * 128 * 2
    assert sm100_hbm_bytes(cfg5, True) < sm100_hbm_bytes(cfg5, False)


def test_flops_match_oracle(oracle):
    from cuda_fused_attention_b200 import AttentionShape, attention_flops
    for cfg in [(1, 2, 128, 64), (2, 8, 2048, 64), (4, 16, 4096, 128), (1, 32, 16384, 128), (16, 32, 8192, 128)]:
        for c in (0, 1):
            assert attention_flops(AttentionShape(*cfg), c) == oracle.attention_flops(*cfg, c)


def test_rejected_arguments_without_gpu(lib):
    fake = ctypes.c_void_p(0x10000)
    odd = ctypes.c_void_p(0x10008)
    cases = [
        ((None, fake, fake, fake, 1, 2, 128, 64, 0, None), 1001),
        ((fake, fake, fake, fake, 0, 2, 128, 64, 0, None), 1001),
        ((fake, fake, fake, fake, 1, 2, -5, 64, 0, None), 1001),
        ((fake, fake, fake, fake, 1, 2, 128, 96, 0, None), 1002),
        ((fake, fake, odd, fake, 1, 2, 128, 64, 0, None), 1003),
    ]
    for args, want in cases:
        assert lib.fa_sm100_fwd(*args) == want
    assert lib.fa_sm100_fwd_slabs(fake, fake, fake, fake, 1, 2, 128, 64, 0, 1, 3, None) == 1001
    assert lib.fa_sm100_fwd_slabs(fake, fake, fake, fake, 1, 2, 128, 64, 0, 2, 1, None) == 1001
    assert lib.fa_sm100_fwd_inject_stall(fake, fake, fake, fake, 1, 2, 128, 64, 0, 0, None) == 1001
    assert lib.fa_sm100_fwd_host(None, fake, fake, fake, 1, 2, 128, 64, 0) == 1001
    assert lib.fa_sm100_fwd_host(fake, fake, fake, fake, 1, 2, 128, 80, 0) == 1002
    assert lib.fa_sm100_test_arm_stall(0) == 1001
    assert lib.fa_sm100_test_arm_stall(2_000_000_000) == 1001
    assert lib.fa_sm100_test_force_kernel(3) == 1001
    assert lib.fa_sm100_test_force_kernel(0) == 0


def test_status_strings(lib):
    for code in (0, 1001, 1002, 1003, 1004, 1005, 1006, 1007, 1008, 1009, 1010):
        assert lib.fa_sm100_status_string(code)
    assert b"unknown" in lib.fa_sm100_status_string(123456)


def test_python_wrapper_rejects_bad_tensors():
    import torch
    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100
    shape = AttentionShape(1, 1, 8, 64)
    t = torch.zeros(8 * 64, dtype=torch.float32)
    with pytest.raises(TypeError):
        launch_attention_sm100(t, t, t, t, shape)
    b = torch.zeros(8 * 64, dtype=torch.bfloat16)
    with pytest.raises(TypeError):   # CPU tensor: no silent CPU path
        launch_attention_sm100(b, b, b, b, shape)


def test_python_wrapper_requires_one_device():
    """The C entry points launch on the current device: the Python wrapper makes the tensors'
    device current, and rejects arguments spread over two devices before any CUDA call."""
    import torch
    from cuda_fused_attention_b200 import _device_of

    class Fake:
        def __init__(self, device):
            self.device = torch.device(device)

    assert _device_of(Fake("cuda:1"), Fake("cuda:1"), 1234, Fake("cuda:1")) == torch.device("cuda:1")
    assert _device_of(1, 2, 3, 4) is None
    with pytest.raises(ValueError, match="one device"):
        _device_of(Fake("cuda:0"), Fake("cuda:1"), Fake("cuda:0"), Fake("cuda:0"))
