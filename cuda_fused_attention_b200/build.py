"""Build recipe for the sm_100a extension library (in-tree, no JIT cache).

    python -m cuda_fused_attention_b200.build

compiles cuda_fused_attention_b200/csrc/*.cu with nvcc for sm_100a only into
cuda_fused_attention_b200/lib/libfa_sm100.so. The library exports the C ABI of
include/fa_sm100.h and the C++ API of include/flash_attention_sm100.h; the CUDA
runtime is linked statically and the driver is reached only through
cudaGetDriverEntryPoint, so the .so needs nothing but libc/libstdc++ and the
NVIDIA driver at run time.

The same sources compiled with FA_SM100_DEBUG_DUMP give lib/libfa_sm100_debug.so,
whose kernel also dumps its intermediate tiles for layout checks
(fa_sm100_debug_read); only tests load it.
"""
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libfa_sm100.so")
DEBUG_LIB_PATH = os.path.join(LIB_DIR, "libfa_sm100_debug.so")
SOURCES = ["fa_sm100.cu", "fa_sm100_host.cu", "fa_sm100_api.cu", "fa_sm100_static.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = os.path.join(cuda_home, "bin", "nvcc")
    return candidate if os.path.exists(candidate) else (shutil.which("nvcc") or "nvcc")


def compile_command(output=LIB_PATH, extra=()):
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    return [nvcc_path(), "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS,
            "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
            "-I", os.path.join(ROOT, "include"), "-I", CSRC,
            *extra, *srcs, "-o", output]


def needs_build():
    if not os.path.exists(LIB_PATH) or not os.path.exists(DEBUG_LIB_PATH):
        return True
    lib_time = min(os.path.getmtime(LIB_PATH), os.path.getmtime(DEBUG_LIB_PATH))
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    return any(os.path.getmtime(d) > lib_time for d in deps)


def build(force=False, verbose=True, ptxas_verbose=False):
    """Compile the library if a source is newer than it; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    cmds = [compile_command(extra=extra),
            compile_command(output=DEBUG_LIB_PATH, extra=["-DFA_SM100_DEBUG_DUMP"])]
    procs = []
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    failed = 0
    for proc in procs:
        out, err = proc.communicate()
        if verbose or proc.returncode != 0:
            sys.stdout.write(out)
            sys.stderr.write(err)
        failed = failed or proc.returncode
    if failed:
        raise RuntimeError(f"nvcc failed with exit code {failed}")
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, ptxas_verbose="-v" in sys.argv)
