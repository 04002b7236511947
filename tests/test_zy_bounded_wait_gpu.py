"""Failure detection on the GPU without a fault: a wait that runs out.

fa_sm100_fwd_inject_stall (or a stall armed with fa_sm100_test_arm_stall for the
next launch of any entry point) makes the MMA warp wait on an mbarrier that
nothing arrives on, with a 20 ms limit. The kernel must give up, record the wait site
in the device error word, drain its own copies, free its tensor memory and
return; the host reads FA_STATUS_DEVICE_TIMEOUT, and the same context then runs
a normal forward correctly (tensor memory was released, nothing is stuck).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


# (1, 2, 256, 64) launches one 128-row Q tile per CTA (small grid); (3, 25, 256, 64) launches
# row-pair CTAs (75 slabs x 1 pair x 2 tiles > 148 SMs).
@pytest.mark.parametrize("b, h", [(1, 2), (3, 25)])
def test_injected_stall_times_out_and_context_survives(oracle, cuda_device, b, h):
    import torch
    from cuda_fused_attention_b200 import STATUS_DEVICE_TIMEOUT, AttentionShape, device_status, \
        launch_attention_sm100
    from cuda_fused_attention_b200 import _lib
    lib = _lib.load()
    n, d = 256, 64
    q, k, v = oracle.make_inputs(b, h, n, d)
    dev = [torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device) for x in (q, k, v)]
    o = torch.empty_like(dev[0])
    assert device_status() == (0, 0)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    rc = lib.fa_sm100_fwd_inject_stall(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), o.data_ptr(),
                                       b, h, n, d, 0, 20_000_000, stream)
    assert rc == 0
    status, word = device_status()
    assert status == STATUS_DEVICE_TIMEOUT
    assert word & 1 and (word >> 8) & 0xFF == 10      # site 10: the injected wait
    assert device_status() == (0, 0)                   # read-and-clear
    # The context is intact: a normal launch right after is correct.
    ref = oracle.attention(q, k, v, b, h, n, d, 1)
    o.view(torch.int16).fill_(-1)
    launch_attention_sm100(dev[0], dev[1], dev[2], o, AttentionShape(b, h, n, d), True)
    torch.cuda.synchronize()
    acc = oracle.compare(o.view(torch.int16).cpu().numpy().view(np.uint16), ref, d)
    assert acc["passed"], acc
    assert device_status() == (0, 0)


def test_host_entry_reports_device_timeout(oracle, cuda_device):
    """fa_sm100_fwd_host reads the error word after its own work: a launch that gave up (armed
    stall, 20 ms) surfaces as FA_STATUS_DEVICE_TIMEOUT from the call itself, the word is
    cleared, and the next call is correct."""
    from cuda_fused_attention_b200 import STATUS_DEVICE_TIMEOUT, device_status
    from cuda_fused_attention_b200 import _lib
    lib = _lib.load()
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    b, h, n, d = 1, 2, 256, 64
    q, k, v = oracle.make_inputs(b, h, n, d)
    ref = oracle.attention(q, k, v, b, h, n, d, 0)
    got = np.full_like(q, 0xFFFF)
    assert device_status() == (0, 0)
    assert lib.fa_sm100_test_arm_stall(20_000_000) == 0
    assert lib.fa_sm100_fwd_host(P(q), P(k), P(v), P(got), b, h, n, d, 0) == STATUS_DEVICE_TIMEOUT
    assert device_status() == (0, 0)
    assert lib.fa_sm100_fwd_host(P(q), P(k), P(v), P(got), b, h, n, d, 0) == 0
    assert oracle.compare(got, ref, d)["passed"]
