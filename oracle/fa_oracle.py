"""numpy front end of the CPU FP64 oracle -- TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (the C++ restatement in fa_oracle.cpp of the
reference's oracle, generator and comparison) and, where it was built,
oracle/_ref/libfa_ref.so (the reference's own functions and kernels compiled
from its sources). Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs use this module; the product never imports it.
"""
import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libfa_ref.so")
SEEDS = (11, 22, 33)   # Q, K, V seeds of benchmarks/bench_flash_attention.cu:528-530
ULP_TOLERANCE = 2.0    # benchmarks/bench_flash_attention.cu:52

_VP = ctypes.c_void_p
_lock = threading.Lock()
_lib = None
_ref = None


class Accuracy(ctypes.Structure):
    _fields_ = [("vs_double", ctypes.c_double), ("row_scaled", ctypes.c_double),
                ("max_abs", ctypes.c_double), ("ulp", ctypes.c_double),
                ("mean_abs", ctypes.c_double), ("mean_ulp", ctypes.c_double),
                ("output_nan", ctypes.c_uint64), ("output_inf", ctypes.c_uint64),
                ("reference_nan", ctypes.c_uint64), ("reference_inf", ctypes.c_uint64),
                ("passed", ctypes.c_int)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


def reference_tree():
    """The reference source tree used to build oracle/_ref: the REFERENCE environment variable,
    else a `reference` directory beside the repository; None where neither exists (as on a
    machine that only runs the prebuilt files)."""
    candidates = [os.environ.get("REFERENCE"), os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")]
    for path in candidates:
        if path and os.path.isfile(os.path.join(path, "benchmarks", "bench_flash_attention.cu")):
            return os.path.abspath(path)
    return None


def build():
    """Compile liboracle.so (and the reference shim where the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    tree = reference_tree()
    if tree is not None:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REFERENCE={tree}"], check=True)


def load():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB):
                subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
            lib = ctypes.CDLL(LIB)
            lib.fa_oracle_bf16_ulp.restype = ctypes.c_float
            lib.fa_oracle_bf16_ulp.argtypes = [ctypes.c_float]
            lib.fa_oracle_attention_flops.restype = ctypes.c_double
            lib.fa_oracle_fill_normal.argtypes = [_VP, ctypes.c_size_t, ctypes.c_uint]
            lib.fa_oracle_apply_family.argtypes = [_VP, _VP, _VP, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
            lib.fa_oracle_attention.argtypes = [_VP, _VP, _VP, _VP] + [ctypes.c_int] * 5
            lib.fa_oracle_attention_rows.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_longlong, ctypes.c_int, ctypes.c_int]
            lib.fa_oracle_attention_parallel.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int,
                                                         ctypes.c_int, ctypes.c_longlong, ctypes.c_longlong,
                                                         ctypes.c_int]
            lib.fa_oracle_compare.argtypes = [_VP, _VP, ctypes.c_longlong, ctypes.c_int, ctypes.c_double,
                                              ctypes.POINTER(Accuracy)]
            _lib = lib
        return _lib


def load_reference():
    """The reference's own functions (oracle/_ref/libfa_ref.so), or None if not built."""
    global _ref
    with _lock:
        if _ref is None and os.path.exists(REF_LIB):
            ref = ctypes.CDLL(REF_LIB)
            ref.ref_bf16_ulp.restype = ctypes.c_float
            ref.ref_bf16_ulp.argtypes = [ctypes.c_float]
            ref.ref_attention_flops.restype = ctypes.c_double
            ref.ref_tensorcore_v3_hbm_bytes.restype = ctypes.c_double
            ref.ref_unfused_workspace_bytes.restype = ctypes.c_size_t
            ref.ref_launch_tensorcore_v3.argtypes = [_VP, _VP, _VP, _VP] + [ctypes.c_int] * 5 + [_VP]
            ref.ref_launch_unfused.argtypes = [_VP, _VP, _VP, _VP, _VP] + [ctypes.c_int] * 5 + [_VP]
            ref.ref_reference_attention.argtypes = [_VP, _VP, _VP, _VP] + [ctypes.c_int] * 5
            _ref = ref
        return _ref


def _p(a):
    return a.ctypes.data_as(_VP)


def fill_normal(count, seed):
    out = np.empty(count, np.uint16)
    load().fa_oracle_fill_normal(_p(out), count, seed)
    return out


def make_inputs(batch, heads, seq_len, head_dim, family=0):
    """Seeded Q, K, V (bf16 bits) in [B, H, N, D] order, input family applied."""
    count = batch * heads * seq_len * head_dim
    q, k, v = (fill_normal(count, s) for s in SEEDS)
    if family:
        load().fa_oracle_apply_family(_p(q), _p(k), _p(v), count, head_dim, family)
    return q, k, v


def attention(q, k, v, batch, heads, seq_len, head_dim, causal, threads=None):
    """FP64 output [B*H*N*D]; slab-parallel across `threads` host threads."""
    out = np.empty(batch * heads * seq_len * head_dim, np.float64)
    slabs = batch * heads
    threads = threads or min(slabs, os.cpu_count() or 1)
    if threads <= 1:
        load().fa_oracle_attention(_p(q), _p(k), _p(v), _p(out), batch, heads, seq_len, head_dim, int(causal))
    else:
        load().fa_oracle_attention_parallel(_p(q), _p(k), _p(v), _p(out), seq_len, head_dim, int(causal),
                                            0, slabs, threads)
    return out


def attention_rows(q, k, v, seq_len, head_dim, causal, slab, row_begin, row_end):
    out = np.empty((row_end - row_begin) * head_dim, np.float64)
    load().fa_oracle_attention_rows(_p(q), _p(k), _p(v), _p(out), seq_len, head_dim, int(causal), slab,
                                    row_begin, row_end)
    return out


def compare(got_bits, reference, head_dim, tolerance=ULP_TOLERANCE):
    """Row-scale BF16 ULP metric of bench_flash_attention.cu:167-218 (+ means)."""
    got_bits = np.ascontiguousarray(got_bits, dtype=np.uint16)
    reference = np.ascontiguousarray(reference, dtype=np.float64)
    rows = reference.size // head_dim
    acc = Accuracy()
    load().fa_oracle_compare(_p(got_bits), _p(reference), rows, head_dim, tolerance, ctypes.byref(acc))
    return acc.as_dict()


def bf16_ulp(value):
    return float(load().fa_oracle_bf16_ulp(value))


def attention_flops(batch, heads, seq_len, head_dim, causal):
    return float(load().fa_oracle_attention_flops(batch, heads, seq_len, head_dim, int(causal)))
