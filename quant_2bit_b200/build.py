"""Build libbcjr_b200.so in-tree with nvcc for sm_100a.

    python -m quant_2bit_b200.build          # or quant_2bit_b200.build.build()

The library is a plain C-ABI shared object (include/bcjr_b200.h); it links
the CUDA runtime statically and has no torch dependency.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbcjr_b200.so")
SOURCES = ["bcjr_capi.cu", "bcjr_generic.cu", "bcjr_l16.cu", "bcjr_b4.cu", "bcjr_noalloc.cu", "bcjr_rht.cu",
           "bcjr_viterbi.cu", "bcjr_vit_b4.cu", "bcjr_vit_b2.cu", "bcjr_codes.cu", "bcjr_l16_cl4.cu", "bcjr_probe.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "bcjr_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, ptxas_info=False):
    """Compile every source into one shared library (skipped when up to date)."""
    if not force and not _stale():
        return LIB
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    cmds, objs = [], []
    for s in srcs:
        obj = os.path.join(CSRC, s.replace(".cu", ".o"))
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", os.path.join(CSRC, s), "-o", obj]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
        objs.append(obj)
    # the translation units are independent: compile them side by side
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as ex:
        for f in [ex.submit(subprocess.run, c, check=True) for c in cmds]:
            f.result()
    cmd = [_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
