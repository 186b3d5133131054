"""Build libfa_sm100.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python fused-attention_b200/build.py            # incremental build
    python fused-attention_b200/build.py --force    # rebuild everything
    python fused-attention_b200/build.py --verbose  # also print ptxas register/smem usage

The shared library lands next to the Python package (attention/libfa_sm100.so), so it travels
with the source tree.  Objects go to _build/ (not committed).

build_stall_test() compiles the same sources into _build/libfa_sm100_stalltest.so for the
failure-detection GPU test only: every kernel's UMMA issuer waits at pipeline step 1 on an
mbarrier that nothing arrives at, with a 20 ms pipeline-wait limit (teardown waits keep their 2 s
limit), so the kernels' bounded-wait abort path runs on a normal input.  The product library
never contains that wait.
"""
import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "attention", "libfa_sm100.so")
STALL_OUT = os.path.join(BUILD, "libfa_sm100_stalltest.so")
STALL_FLAGS = ["-DFA_TEST_STALL_STEP=1", "-DFA_WAIT_TIMEOUT_NS=20000000ull"]
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
SOURCES = ["fa_api.cu", "fa_fwd.cu", "fa_bwd.cu", "fa_noalloc.cu", "fa_unfused.cu"]
HEADERS = ["fa_sm100.cuh", "fa_internal.h"]

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def _newer(src_list, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in src_list)


def build(force=False, verbose=False, out=OUT, extra_flags=(), obj_dir=BUILD):
    os.makedirs(obj_dir, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "fa_sm100.h")]
    jobs = []
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(obj_dir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer([s] + headers, o):
            cmd = [NVCC, *ARCH, *FLAGS, *extra_flags, "-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append((src, cmd))

    def run(job):
        name, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return name, r

    failed = False
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for name, r in ex.map(run, jobs):
            if r.returncode != 0 or verbose:
                sys.stderr.write(f"--- nvcc {name}\n{r.stdout}{r.stderr}")
            failed |= r.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed")
    if force or jobs or _newer(objs, out):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", out, *objs, "-lcudart_static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return out


def build_stall_test(force=False, verbose=False):
    """The failure-detection test library (see the module docstring)."""
    return build(force, verbose, out=STALL_OUT, extra_flags=STALL_FLAGS,
                 obj_dir=os.path.join(BUILD, "stalltest"))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_stall_test(force=a.force))
