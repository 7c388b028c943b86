"""Build the ltx25 CUDA library for sm_100a, in-tree.

    python vpipe-ltx-2.5_b200/build.py [--jobs N] [--force]

Compiles every source under csrc/ and host/ with nvcc
(-gencode arch=compute_100a,code=sm_100a) and links
vpipe-ltx-2.5_b200/lib/libltx25_cuda.so.  Incremental: an object is rebuilt
when its source or any header in the package is newer.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "lib")
OBJ_DIR = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(OUT_DIR, "libltx25_cuda.so")
# the plugin entry (plugin/ltx25-plugin-cuda.cc against the in-repo vpipe
# stub headers), linked against LIB
PLUGIN = os.path.join(OUT_DIR, "vpipe-ltx-2.5-b200.so")
PLUGIN_SRC = os.path.join(HERE, "plugin", "ltx25-plugin-cuda.cc")
CXX = os.environ.get("CXX", "g++")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-I" + os.path.join(REPO, "include")]


def sources():
    srcs = sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))
    srcs += sorted(glob.glob(os.path.join(HERE, "host", "*.cc")))
    return srcs


def headers():
    hs = glob.glob(os.path.join(HERE, "csrc", "*.h")) + \
        glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + \
        glob.glob(os.path.join(HERE, "host", "*.h")) + \
        glob.glob(os.path.join(REPO, "include", "*.h"))
    return hs


def obj_for(src):
    rel = os.path.relpath(src, HERE).replace(os.sep, "_")
    return os.path.join(OBJ_DIR, rel + ".o")


def compile_one(src, force, verbose):
    obj = obj_for(src)
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj, None
    cmd = [NVCC] + ARCH + FLAGS + ["-x", "cu", "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"FAILED {src}\n{' '.join(cmd)}\n{r.stdout}{r.stderr}"
    return obj, (r.stdout + r.stderr) if verbose else None


def build(force=False, jobs=8, verbose=False):
    os.makedirs(OBJ_DIR, exist_ok=True)
    objs = []
    errors = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, msg in ex.map(lambda s: compile_one(s, force, verbose), sources()):
            objs.append(obj)
            if msg and msg.startswith("FAILED"):
                errors.append(msg)
            elif msg:
                print(msg)
    if errors:
        raise RuntimeError("\n".join(errors))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            # libcuda.so is resolved at run time on the GPU box; link with the
            # driver stub when the build box has no driver.
            cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
                "-L/usr/local/cuda/lib64/stubs", "-lcuda"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    build_plugin(force)
    build_diag(force)
    return LIB


def build_diag(force=False):
    """Measurement tools under diag/ (not linked into the library)."""
    for src in sorted(glob.glob(os.path.join(HERE, "diag", "*.cu"))):
        out = os.path.join(OUT_DIR, "diag_" + os.path.splitext(os.path.basename(src))[0])
        deps = [src] + headers()
        if not force and os.path.exists(out) and \
                os.path.getmtime(out) >= max(os.path.getmtime(d) for d in deps):
            continue
        cmd = [NVCC] + ARCH + ["-O3", "-std=c++17", src, "-o", out]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"diag build failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")


def build_plugin(force=False):
    """The plugin shim: host C++ only, warnings as errors, rpath to LIB."""
    deps = [PLUGIN_SRC, LIB] + glob.glob(os.path.join(HERE, "plugin", "stub", "plugin", "*.h")) \
        + glob.glob(os.path.join(REPO, "include", "*.h*"))
    if not force and os.path.exists(PLUGIN) and \
            os.path.getmtime(PLUGIN) >= max(os.path.getmtime(d) for d in deps):
        return PLUGIN
    cmd = [CXX, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-Werror",
           "-fvisibility=hidden", "-I" + os.path.join(REPO, "include"),
           "-I" + os.path.join(HERE, "plugin", "stub"), PLUGIN_SRC, "-o", PLUGIN,
           "-L" + OUT_DIR, "-lltx25_cuda", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"plugin build failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")
    return PLUGIN


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true", help="ptxas -v")
    a = ap.parse_args()
    try:
        print(build(a.force, a.jobs, a.verbose))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
