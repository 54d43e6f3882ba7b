"""Builds libvkllm_b200.so (the C-ABI library) for sm_100a with nvcc.

Every source under csrc/ is compiled to an object in _build/ (skipped when the object is newer
than the source and every header), then linked with the static CUDA runtime into lib/.
Usage: python vkllm.c_b200/build.py [-j N] [--verbose]
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libvkllm_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    out = []
    for d, _, files in os.walk(CSRC):
        for f in sorted(files):
            if f.endswith((".cu", ".cpp")):
                out.append(os.path.join(d, f))
    return sorted(out)


def headers():
    hs = []
    for base in (CSRC, os.path.join(ROOT, "include")):
        for d, _, files in os.walk(base):
            hs += [os.path.join(d, f) for f in files if f.endswith((".h", ".cuh", ".hpp"))]
    return hs


def flags():
    return [
        "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
        "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "--expt-relaxed-constexpr",
        "-Xptxas", "-warn-spills",
    ] + ARCH


def compile_one(src, verbose):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    obj = os.path.join(BUILD, rel + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, ""
    cmd = [nvcc()] + flags() + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc()] + flags() + ["-x", "cu", "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(jobs=8, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = sources()
    objs, logs = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, log in ex.map(lambda s: compile_one(s, verbose), srcs):
            objs.append(obj)
            if log.strip():
                logs.append(log)
    newest_obj = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest_obj:
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl", "-lpthread", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    for l in logs:
        sys.stderr.write(l)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=os.cpu_count() or 8)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.verbose))
