"""Generate tests/golden/golden.json from the reference's OWN functions.

Run in a container that holds the reference tree (it is compiled from its own
sources into oracle/_ref/libfa_ref.so by `make -C oracle ref`). The JSON pins:

* the seeded generator (SHA-256 of the bf16 bytes of Q, K and V),
* the CPU FP64 oracle (SHA-256 of the float64 output bytes, plus a few values),
* the comparison metric (the reference's Accuracy fields on a perturbed output),
* bf16_ulp and attention_flops on fixed arguments,

for the case matrix the reference's own tests use (bench_flash_attention.cu:514-530,
bench_flash_attention_lite.cu:48, kernels/ablation/experiments.cu:283-289) plus the
128-row tile boundaries of the new kernel and the BASELINE configs 1 and 2.

tests/test_oracle.py recomputes every entry with oracle/liboracle.so (the
restatement) and requires bit equality. Usage: python tests/golden/make_golden.py
"""
import ctypes
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
OUT = os.path.join(ROOT, "tests", "golden", "golden.json")
VP = ctypes.c_void_p


def load_reference():
    path = os.path.join(ROOT, "oracle", "_ref", "libfa_ref.so")
    if not os.path.exists(path):
        sys.exit("oracle/_ref/libfa_ref.so is missing: run `make -C oracle ref` where the reference tree exists")
    lib = ctypes.CDLL(path)
    lib.ref_bf16_ulp.restype = ctypes.c_float
    lib.ref_bf16_ulp.argtypes = [ctypes.c_float]
    lib.ref_attention_flops.restype = ctypes.c_double
    lib.ref_tensorcore_v3_hbm_bytes.restype = ctypes.c_double
    return lib


def sha(array):
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def fill(lib, count, seed):
    out = np.empty(count, np.uint16)
    lib.ref_fill_normal(out.ctypes.data_as(VP), ctypes.c_size_t(count), ctypes.c_uint(seed))
    return out


def bf16_round(values):
    """float64 -> bf16 bits (round to nearest even), for building perturbed outputs."""
    f = values.astype(np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def apply_family(q, k, v, head_dim, family):
    """kernels/ablation/experiments.cu:283-289, family 5 = BASELINE config 3 (Q x 4)."""
    def to_f(bits):
        return (bits.astype(np.uint32) << 16).view(np.float32)

    idx = np.arange(q.size)
    if family == 1:
        q[:] = k[:] = v[:] = 0
    elif family == 2:
        q[:] = k[:] = v[:] = bf16_round(np.ones(q.size))
    elif family == 3:
        v[:] = bf16_round(((idx % head_dim).astype(np.int64) - head_dim // 2).astype(np.float64))
    elif family == 4:
        q[:] = bf16_round(to_f(q).astype(np.float64) * 4.0)
        k[:] = bf16_round(to_f(k).astype(np.float64) * 4.0)
    elif family == 5:
        q[:] = bf16_round(to_f(q).astype(np.float64) * 4.0)


def cases():
    out = []
    out.append((1, 2, 128, 64, 0, 0))
    for d in (64, 128):                                      # accuracy shapes
        for c in (0, 1):
            out.append((1, 2, 256, d, c, 0))
    for d in (64, 128):                                      # tile boundaries
        for c in (0, 1):
            for n in (1, 7, 63, 64, 65, 127, 128, 129, 255, 257):
                out.append((1, 2, n, d, c, 0))
    for family in (1, 2, 3, 4):                              # input families
        for d in (64, 128):
            for c in (0, 1):
                for n in (1, 65, 129):
                    out.append((1, 2, n, d, c, family))
    out.append((1, 2, 256, 128, 1, 5))                       # config 3 distribution
    out.append((2, 8, 2048, 64, 0, 0))
    out.append((2, 8, 2048, 64, 1, 0))
    return out


def main():
    lib = load_reference()
    records = []
    for (b, h, n, d, c, family) in cases():
        count = b * h * n * d
        q, k, v = fill(lib, count, 11), fill(lib, count, 22), fill(lib, count, 33)
        apply_family(q, k, v, d, family)
        ref = np.empty(count, np.float64)
        lib.ref_reference_attention(q.ctypes.data_as(VP), k.ctypes.data_as(VP), v.ctypes.data_as(VP),
                                    ref.ctypes.data_as(VP), b, h, n, d, c)
        # A perturbed "device" output: bf16(ref) with every 7th element moved by one bf16 step.
        got = bf16_round(ref)
        got[::7] = got[::7] + np.uint16(1)
        fields = np.zeros(9, np.float64)
        lib.ref_compare(got.ctypes.data_as(VP), ref.ctypes.data_as(VP), b, h, n, d, fields.ctypes.data_as(VP))
        records.append({
            "shape": [b, h, n, d], "causal": c, "family": family,
            "q_sha256": sha(q), "k_sha256": sha(k), "v_sha256": sha(v),
            "out_sha256": sha(ref),
            "out_head": [float(x) for x in ref[:4]],
            "out_sum": float(ref.sum()),
            "perturbed_compare": [float(x) for x in fields],
        })
        print(f"case {b},{h},{n},{d} causal={c} family={family}")
    ulp_args = [0.0, 1.0e-30, 1.5e-38, 0.0625, 0.1, 0.5, 0.99, 1.0, 1.5, 3.0, 100.0, -2.5, float("inf")]
    ulps = [float(lib.ref_bf16_ulp(x)) for x in ulp_args]
    configs = [(1, 2, 128, 64), (2, 8, 2048, 64), (4, 16, 4096, 128), (1, 32, 16384, 128), (16, 32, 8192, 128)]
    flops = [[list(cfg), c, float(lib.ref_attention_flops(*cfg, c))] for cfg in configs for c in (0, 1)]
    v3_bytes = [[list(cfg), c, float(lib.ref_tensorcore_v3_hbm_bytes(*cfg, c))] for cfg in configs for c in (0, 1)]
    doc = {
        "generator": "tests/golden/make_golden.py using oracle/_ref/libfa_ref.so (reference sources)",
        "seeds": {"q": 11, "k": 22, "v": 33},
        "cases": records,
        "bf16_ulp": [[a if np.isfinite(a) else "inf", u] for a, u in zip(ulp_args, ulps)],
        "attention_flops": flops,
        "tensorcore_v3_hbm_bytes": v3_bytes,
    }
    with open(OUT, "w") as fh:
        json.dump(doc, fh, indent=1)
    print("wrote", OUT, len(records), "cases")


if __name__ == "__main__":
    main()
