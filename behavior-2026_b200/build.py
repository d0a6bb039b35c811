"""Build the engine library behavior-2026_b200/libpi05.so for sm_100a (B200) with nvcc.

Cross-compiles without a GPU.  The CUDA runtime is linked statically, as the reference engine did
(docs/archive/windows/π05_네이티브엔진.md:109), so the library does not clash with another runtime
loaded in the same process.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libpi05.so")
SOURCES = ["engine.cu", "static_scratch.cu", "preprocess.cu", "tokenizer.cpp"]
DEPS = SOURCES + ["common.cuh", "attention_bwd_tc.cuh", "gemm_tc.cuh", "attention.cuh", "kernels.cuh", "pi05_model.h", "train.cuh",
                  "train_kernels.cuh", "attention_bwd.cuh", "attention_tc.cuh", "denoise_mega.cuh", "attention_sig.cuh", "gemm_wide.cuh", "gemm_pair.cuh", "attention_bwd_dq_pipe.cuh", "resize.cuh", "dp_nccl.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-shared",
]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(HERE, "..", "include", "pi05.h")]
    return any(os.path.getmtime(d) > t for d in deps)


SERVER = os.path.join(HERE, "pi05_server")
SERVER_SRC = [os.path.join(HERE, "server", f) for f in ("pi05_server.cpp", "wire.h")]


def build_server(verbose=False):
    """the policy server binary (host C++ over libpi05.so, found next to it at run time)"""
    if os.path.exists(SERVER) and all(os.path.getmtime(SERVER) >= os.path.getmtime(p)
                                      for p in SERVER_SRC + [LIB, os.path.join(HERE, "..", "include", "pi05.h")]):
        return SERVER
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-o", SERVER, SERVER_SRC[0], "-L" + HERE, "-lpi05",
           "-Wl,-rpath,$ORIGIN", "-lpthread"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("g++ failed building pi05_server")
    return SERVER


def build(force=False, verbose=False):
    if force or stale():
        cmd = [nvcc()] + NVCC_FLAGS + ["-o", LIB] + [os.path.join(CSRC, s) for s in SOURCES]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed building libpi05.so")
    build_server(verbose)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
