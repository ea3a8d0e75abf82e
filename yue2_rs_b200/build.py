"""Builds libyue2cuda.so (sm_100a) in-tree with nvcc.

    python -m yue2_rs_b200.build            # incremental
    python -m yue2_rs_b200.build --force    # rebuild everything

Objects go to yue2_rs_b200/_build/ (git-ignored); the shared library lands next to
this file so that it travels with the source tree.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libyue2cuda.so")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["kernels_layer.cu", "kernels_gemv.cu", "kernels_sample.cu", "gemm_rows.cu", "kernels_gemm_tc.cu", "kernels_gemm_skinny.cu", "kernels_prefill_attn.cu", "kernels_prefill_attn_tc.cu", "engine.cu", "engine_sample.cu", "checkpoint.cu", "dropin.cu", "dropin_f32.cu", "noalloc.cu", "synthesize.cu", "tp.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off,-O2",
                "-I" + CSRC, "-I" + INCLUDE]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps(src):
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INCLUDE, "yue2_cuda.h"))
    return [src] + headers


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj):
    cmd = [nvcc()] + FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force=False, verbose=True):
    os.makedirs(BUILD, exist_ok=True)
    objs, jobs = [], []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, _deps(src)):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for f in [ex.submit(_compile, s, o) for s, o in jobs]:
                o = f.result()
                if verbose:
                    print("compiled", os.path.relpath(o, HERE), flush=True)
    if force or jobs or _stale(OUT, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", OUT + ".tmp"] + objs + ["-lcuda", "-lcublasLt",
                                                           "-Xlinker", "-rpath=/usr/local/cuda/lib64", "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(OUT + ".tmp", OUT)
        if verbose:
            print("linked", OUT, flush=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
