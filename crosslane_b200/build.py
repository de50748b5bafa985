"""Build the CUDA expert lane into crosslane_b200/libcrosslane_b200.so (sm_100a).

    python crosslane_b200/build.py          # incremental
    python crosslane_b200/build.py --force  # rebuild everything
    python crosslane_b200/build.py --trace  # the phase-trace build, libcrosslane_b200_trace.so

(Run as a file, not `-m`: importing the package loads the library being rebuilt.)

Plain nvcc, one object per .cu, linked into an in-tree shared library with the
static CUDA runtime; the library's interface is include/crosslane_b200.h.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcrosslane_b200.so")
# The phase-trace build (-DCLB_FLOW_TRACE: %globaltimer stamps at the stack kernel's phase
# boundaries, read back with clb_stack_trace_read); load it with CROSSLANE_B200_LIB.
BUILD_TRACE = os.path.join(HERE, "_build_trace")
LIB_TRACE = os.path.join(HERE, "libcrosslane_b200_trace.so")
SOURCES = ["clb_kernels.cu", "clb_bank.cu", "clb_noalloc.cu", "clb_stack.cu", "clb_prefill.cu",
           "clb_pack_io.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
                "--expt-relaxed-constexpr"]


def _deps():
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "crosslane_b200.h"))
    return max(os.path.getmtime(h) for h in headers)


def _compile(src, force, build_dir=BUILD, extra=()):
    obj = os.path.join(build_dir, src.replace(".cu", ".o"))
    path = os.path.join(CSRC, src)
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), _deps()):
        return obj, False
    cmd = [NVCC] + FLAGS + list(extra) + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, True


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    build_dir, lib, extra = (BUILD_TRACE, LIB_TRACE, ["-DCLB_FLOW_TRACE"]) if trace else (BUILD, LIB, [])
    os.makedirs(build_dir, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, build_dir, extra), SOURCES))
    objs = [o for o, _ in results]
    rebuilt = any(r for _, r in results)
    if rebuilt or force or not os.path.exists(lib) or os.path.getmtime(lib) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", lib] + objs + ["-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("built", lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--trace", action="store_true", help="the phase-trace build (libcrosslane_b200_trace.so)")
    a = ap.parse_args()
    try:
        build(a.force, verbose=True, trace=a.trace)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
