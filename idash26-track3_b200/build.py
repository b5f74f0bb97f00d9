"""Build libddg.so in-tree for sm_100a (nvcc, no JIT cache).

Each csrc/*.cu / *.cpp is compiled to _build/<name>.o (rebuilt when it or any
header in csrc/ or include/ is newer), then linked into ./libddg.so next to
this file, the command-line drop-in cli/ddg_inference.cpp into
./ddg_inference against it, and the offline tools cli/ddg_share.cpp and
cli/ddg_export_weights.cpp (plain C++) into ./ddg_share and
./ddg_export_weights.  NCCL comes from the pip-installed nvidia-nccl package torch ships
with, with the system copy as a fallback.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libddg.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def nccl_paths():
    cands = []
    try:
        import nvidia.nccl as _n  # type: ignore

        root = list(_n.__path__)[0]
        cands.append((os.path.join(root, "include"), os.path.join(root, "lib")))
    except Exception:
        pass
    cands.append(("/usr/include", "/usr/lib/x86_64-linux-gnu"))
    for inc, lib in cands:
        if os.path.exists(os.path.join(inc, "nccl.h")) and glob.glob(os.path.join(lib, "libnccl.so*")):
            return inc, lib
    return None, None


def _flags(extra_verbose=False):
    f = ARCH + ["-rdc=true", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
                "-I" + os.path.join(REPO, "include"), "-I" + CSRC]
    inc, _ = nccl_paths()
    if inc:
        f += ["-I" + inc, "-DDDG_HAVE_NCCL=1"]
    if extra_verbose:
        f += ["-Xptxas", "-v"]
    return f


def _headers_mtime():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) + \
        glob.glob(os.path.join(REPO, "include", "*.h"))
    return max([os.path.getmtime(h) for h in hs] + [0])


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    hmt = _headers_mtime()
    flags = _flags(ptxas_v)

    def obj(src):
        return os.path.join(BUILD, os.path.basename(src) + ".o")

    def need(src):
        o = obj(src)
        return force or ptxas_v or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(src), hmt)

    def compile_one(src):
        cmd = [nvcc] + flags + ["-c", src, "-o", obj(src)]
        if src.endswith(".cpp"):
            cmd = [nvcc] + flags + ["-x", "cu", "-c", src, "-o", obj(src)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        return r.stderr

    todo = [s for s in srcs if need(s)]
    if todo:
        with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
            for src, log in zip(todo, ex.map(compile_one, todo)):
                if verbose or ptxas_v:
                    sys.stderr.write(f"== {os.path.basename(src)}\n{log}")
    if todo or not os.path.exists(LIB):
        link = [nvcc] + ARCH + ["-rdc=true", "-shared", "-o", LIB] + [obj(s) for s in srcs]
        _, libdir = nccl_paths()
        if libdir:
            link += ["-L" + libdir, "-lnccl", "-Xlinker", "-rpath=" + libdir]
        link += ["-lpthread"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    build_cli(force)
    build_tools(force)
    return LIB


def build_cli(force: bool = False) -> str:
    """The command-line drop-in (cli/ddg_inference.cpp), linked against the
    in-tree libddg.so with an $ORIGIN run path."""
    src = os.path.join(HERE, "cli", "ddg_inference.cpp")
    out = os.path.join(HERE, "ddg_inference")
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(src),
                                                                        os.path.getmtime(LIB), _headers_mtime()):
        return out
    cmd = [_nvcc(), "-O2", "-std=c++17", "-I" + os.path.join(REPO, "include"), src, "-o", out,
           "-L" + HERE, "-lddg", "-Xlinker", "-rpath=$ORIGIN", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("ddg_inference build failed:\n" + r.stderr)
    return out


TOOLS = ("ddg_share", "ddg_export_weights")


def build_tools(force: bool = False) -> list:
    """The offline tools (cli/ddg_share.cpp, cli/ddg_export_weights.cpp): plain
    C++17, no CUDA, built next to libddg.so."""
    cxx = shutil.which("g++") or "g++"
    outs = []
    for name in TOOLS:
        src = os.path.join(HERE, "cli", name + ".cpp")
        out = os.path.join(HERE, name)
        outs.append(out)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
            continue
        r = subprocess.run([cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", src, "-o", out], capture_output=True,
                           text=True)
        if r.returncode != 0:
            raise RuntimeError(f"{name} build failed:\n" + r.stderr)
    return outs


if __name__ == "__main__":
    print(build(verbose=True, ptxas_v="-v" in sys.argv, force="-f" in sys.argv))
