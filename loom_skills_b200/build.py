"""Build liblk.so in-tree with nvcc for sm_100a (no torch extension machinery: the library is a plain C ABI)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "liblk.so")
SOURCES = ["lk_api.cu", "lk_dequant.cu", "lk_mv.cu", "lk_mvq8.cu","lk_gemm.cu", "lk_mxfp4.cu", "lk_moe.cu", "lk_peer.cu",
           "lk_noalloc.cu", "lk_mvmx.cu", "lk_mvg.cu", "lk_moeq8.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(HERE, "..", "include", "lk.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, jobs=None):
    """Compile every .cu under csrc/ to an object, then link liblk.so. Objects go to csrc/_build (git-ignored)."""
    if not force and not _stale():
        return LIB
    bdir = os.path.join(CSRC, "_build")
    os.makedirs(bdir, exist_ok=True)
    procs = []
    objs = []
    for src in SOURCES:
        obj = os.path.join(bdir, src.replace(".cu", ".o"))
        objs.append(obj)
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stdout.write(out)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for " + ", ".join(failed))
    tmp = LIB + ".tmp"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp, "-lcudart"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
