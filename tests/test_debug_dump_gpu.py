"""Stage-by-stage check of the tcgen05 data path with the debug build of the library.

libfa_sm100_debug.so is the product sources compiled with FA_SM100_DEBUG_DUMP (the
counterpart of the reference's FA_V3_DEBUG_DUMP, kernels/v3/v3_tensorcore.cu:189-204,
:680-709). CTA 0 of a launch dumps, for its first 128-row Q tile: S of key tile 0 as the
softmax loads it from TMEM, P as the PV MMA reads it back, O after the last PV before 1/l,
and the row sums and maxima. Each stage is checked on its own, so a layout or descriptor
error shows where it enters:

* S against Q K^T from the bf16 inputs (catches Q/K shared-memory descriptors, swizzle,
  instruction descriptor, TMEM lane/column mapping of the accumulator);
* P against 2^((S - m) * log2(e)/sqrt(D)) of the dumped S with the tile's row max m, and 0
  where masked (catches the softmax's column mapping, masking, packing of bf16 pairs);
* the final output against bf16(O_dump / l) bit for bit, and l against the sum of the
  exponentials of the whole row (catches the PV operand layouts and the epilogue).

Both kernel instantiations are covered: (1, 2, N) runs one Q tile per CTA, (3, 25, N) runs
row pairs. N = 300 makes key tile 2 a ragged tail.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLOATS, S_OFF, P_OFF, O_OFF, L_OFF, M_OFF, INFO_OFF = 49416, 0, 16384, 32768, 49152, 49280, 49408
LOG2E = 1.4426950408889634


def _debug_lib():
    from cuda_fused_attention_b200.build import DEBUG_LIB_PATH
    lib = ctypes.CDLL(DEBUG_LIB_PATH)
    lib.fa_sm100_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    lib.fa_sm100_debug_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    return lib


def _bf16_to_f64(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _f32_to_bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_product_library_has_no_dump():
    from cuda_fused_attention_b200 import _lib
    buf = np.zeros(FLOATS, np.float32)
    assert _lib.load().fa_sm100_debug_read(buf.ctypes.data_as(ctypes.c_void_p), FLOATS) == 1002


@pytest.mark.parametrize("b, h, one_tile", [(1, 2, 1), (3, 25, 0)])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [0, 1])
def test_each_stage_of_the_first_tile(oracle, cuda_device, b, h, one_tile, d, causal):
    import torch
    n = 300
    lib = _debug_lib()
    q, k, v = oracle.make_inputs(b, h, n, d)
    dev = [torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device) for x in (q, k, v)]
    o = torch.empty_like(dev[0])
    assert lib.fa_sm100_fwd(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), o.data_ptr(),
                            b, h, n, d, causal, None) == 0
    dump = np.zeros(FLOATS, np.float32)
    assert lib.fa_sm100_debug_read(dump.ctypes.data_as(ctypes.c_void_p), FLOATS) == 0
    slab, row0, seq, dim, msk, one, n_kv, valid = (int(x) for x in dump[INFO_OFF:INFO_OFF + 8])
    assert (seq, dim, msk, one, valid) == (n, d, causal, one_tile, 1)
    out = o.view(torch.int16).cpu().numpy().view(np.uint16).reshape(b * h, n, d)

    qs = _bf16_to_f64(q.reshape(b * h, n, d)[slab])
    ks = _bf16_to_f64(k.reshape(b * h, n, d)[slab])
    vs = _bf16_to_f64(v.reshape(b * h, n, d)[slab])
    rows = np.arange(row0, row0 + 128)
    qt = np.zeros((128, d))
    live = rows < n
    qt[live] = qs[rows[live]]                       # rows past N are zero-filled by TMA

    # Stage 1: S = Q K^T of key tile 0 (fp32 accumulation of bf16 products).
    s_dump = dump[S_OFF:S_OFF + 128 * 128].reshape(128, 128).astype(np.float64)
    s_ref = qt @ ks[:128].T
    bound = np.abs(qt) @ np.abs(ks[:128]).T
    assert np.all(np.abs(s_dump - s_ref) <= 1e-5 * bound + 1e-30), "S differs from Q K^T"

    # Stage 2: P of key tile 0 on the tile's row max (the first tile sets the exponent base).
    c = float(np.float32(np.float32(1.0 / np.sqrt(np.float32(d))) * np.float32(LOG2E)))
    limit = np.where(causal, np.minimum(rows, n - 1), n - 1)
    keys = np.arange(128)
    allowed = keys[None, :] <= limit[:, None]
    m0 = np.where(allowed, s_dump, -np.inf).max(axis=1)
    p_ref = np.where(allowed, np.exp2((s_dump - m0[:, None]) * c), 0.0)
    p_dump = dump[P_OFF:P_OFF + 128 * 128].reshape(128, 128).astype(np.float64)
    assert np.all(p_dump[~allowed] == 0.0), "masked P not zero"
    assert np.all(np.abs(p_dump - p_ref) <= 2.0 ** -8 * p_ref + 1e-30), "P differs from exp2 of S"

    # Stage 3: the output is bf16(O / l) of the dumped O and l, bit for bit; l is the sum of the
    # row's exponentials on the final base M.
    o_dump = dump[O_OFF:O_OFF + 128 * 128].reshape(128, 128)[:, :d]
    l_dump = dump[L_OFF:L_OFF + 128]
    m_dump = dump[M_OFF:M_OFF + 128].astype(np.float64)
    inv = (np.float32(1.0) / l_dump).astype(np.float32)
    want = _f32_to_bf16_bits(o_dump * inv[:, None])
    assert np.array_equal(out[slab, rows[live]], want[live]), "output is not bf16(O / l)"
    s_all = qt @ ks.T
    allowed_all = np.arange(n)[None, :] <= limit[:, None]
    l_ref = np.where(allowed_all, np.exp2((s_all - m_dump[:, None]) * c), 0.0).sum(axis=1)
    assert np.allclose(l_dump[live], l_ref[live], rtol=2e-4), "row sum differs"
    # And O itself: P V accumulated over all keys on the base M (P rounded to bf16 in the MMA).
    p_all = np.where(allowed_all, np.exp2((s_all - m_dump[:, None]) * c), 0.0)
    o_ref = p_all @ vs
    scale = np.abs(p_all) @ np.abs(vs)
    assert np.all(np.abs(o_dump[live] - o_ref[live]) <= 2.0 ** -7 * scale[live] + 1e-30), "O differs from P V"
    assert n_kv == (3 if not causal else min(3, row0 // 128 + (1 if one_tile else 2)))   # the CTA's key tiles
