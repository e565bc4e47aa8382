"""Build the provider library libfyodor_b200.so for sm_100a with nvcc.

Usage: python fyodor_b200/build.py (the package import would load the library).
The library is written next to this file so it travels with the source
tree; it links the CUDA runtime statically and NCCL dynamically.
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(HERE, "libfyodor_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-I" + os.path.join(ROOT, "include")]
COMMON += os.environ.get("FYB_NVCC_FLAGS", "").split()  # extra flags for experimental builds


def _nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else (shutil.which("nvcc") or "nvcc")


# Sources compiled once per variant (object suffix, extra flags): each
# instantiation of the persistent decode kernel is its own compilation, so
# they run in parallel.
VARIANTS = {
    "decode_inst.cu": [("%d_%d" % (hd, g), ["-DFYB_DK_HD=%d" % hd, "-DFYB_DK_G=%d" % g])
                       for hd in (128, 64) for g in (1, 2, 4, 8)],
}


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def units():
    """(source, object suffix, extra flags) of every compilation."""
    out = []
    for src in sources():
        out += [(src, suffix, flags) for suffix, flags in VARIANTS.get(src, [("", [])])]
    return out


def _compile(unit, verbose):
    src, suffix, flags = unit
    obj = os.path.join(OBJ, src + ("." + suffix if suffix else "") + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    deps += [os.path.join(ROOT, "include", h) for h in os.listdir(os.path.join(ROOT, "include"))]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [_nvcc()] + ARCH + COMMON + flags + ["-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [_nvcc(), "-x", "cu"] + ARCH + COMMON + flags + ["-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s %s:\n%s\n%s" % (src, suffix, r.stdout, r.stderr))
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    todo = units()
    # the longest compilations first
    todo.sort(key=lambda u: u[0] != "decode_inst.cu")
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(os.cpu_count() or 8, len(todo))) as ex:
        objs = list(ex.map(lambda u: _compile(u, verbose), todo))
    newest = max(os.path.getmtime(o) for o in objs)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    cmd = [_nvcc()] + ARCH + ["-shared", "-o", LIB + ".tmp"] + objs + [
        "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
