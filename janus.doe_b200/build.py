"""Build recipe for the B200 engine: libjdgpu.so (CUDA kernels + C ABI + host model code)
and the `m` command-line front end, both compiled in place for sm_100a.

    python janus.doe_b200/build.py [--force]
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INC = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libjdgpu.so")
CLI = os.path.join(HERE, "m")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-diag-suppress", "177"]
CU_SOURCES = ["jdg_engine.cu", "jdg_host.cu", "jdg_noalloc.cu"]
C_SOURCES = ["jd_model.c"]


def _nvcc():
    for p in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if p and os.path.exists(p):
            return p
    raise RuntimeError("nvcc not found")


def _nccl_root():
    """The NCCL that ships with the Python environment (the one PyTorch loads), so that the
    engine and torch.distributed share one libnccl in a process."""
    try:
        import nvidia.nccl
        root = list(nvidia.nccl.__path__)[0]
        if os.path.exists(os.path.join(root, "lib", "libnccl.so.2")):
            return root
    except ImportError:
        pass
    return None


def _nccl_flags():
    root = _nccl_root()
    if root:
        d = os.path.join(root, "lib")
        return ["-L" + d, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + d]
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/local/lib", "/usr/lib64"):
        if os.path.exists(os.path.join(d, "libnccl.so")) or os.path.exists(os.path.join(d, "libnccl.so.2")):
            name = "nccl" if os.path.exists(os.path.join(d, "libnccl.so")) else ":libnccl.so.2"
            return ["-L" + d, "-l" + name, "-Xlinker", "-rpath=" + d]
    raise RuntimeError("libnccl not found")


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r


def build_lib(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in sorted(os.listdir(CSRC)) if h.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INC, "jdgpu.h"))
    objs = []
    nvcc = _nvcc()
    for s in CU_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        if force or _newer(obj, [src] + headers):
            root = _nccl_root()
            inc = ["-I" + os.path.join(root, "include")] if root else []
            _run([nvcc] + ARCH + NVCC_FLAGS + inc + ["-I" + INC, "-c", src, "-o", obj])
            if verbose:
                print("compiled", s)
        objs.append(obj)
    for s in C_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        if force or _newer(obj, [src] + headers):
            _run(["gcc", "-O3", "-std=gnu11", "-fPIC", "-fvisibility=hidden", "-I" + INC, "-c", src, "-o", obj])
            if verbose:
                print("compiled", s)
        objs.append(obj)
    if force or _newer(LIB, objs):
        _run([nvcc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + _nccl_flags() + ["-lpthread", "-lm"])
        if verbose:
            print("linked", LIB)
    return LIB


def build_cli(force=False):
    src = os.path.join(CSRC, "m_cli.c")
    if not os.path.exists(src):
        return None
    if force or _newer(CLI, [src, LIB, os.path.join(INC, "jdgpu.h")]):
        _run(["gcc", "-O2", "-std=gnu11", "-I" + INC, src, "-o", CLI, "-L" + HERE, "-ljdgpu",
              "-Wl,-rpath,$ORIGIN", "-lm"])
    return CLI


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_cli(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print("ok")
