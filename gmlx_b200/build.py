"""Build libkq_cuda.so (sm_100a) in-tree with nvcc.

The library is a plain C-ABI shared object (``include/kq_cuda.h``); Python
loads it with ctypes (``gmlx_b200/_lib.py``).  The grid and value-table header is
generated first from the installed gguf-py package (``csrc/gen_tables.py``).
Objects are compiled in parallel and relinked only when a source changed;
each flag set (normal / ``KQ_DEVELOPMENT``) keeps its own object directory, and
the library is relinked whenever it was last linked from the other set.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
DEV = bool(os.environ.get("KQ_DEVELOPMENT"))
BUILD = os.path.join(HERE, "_build", "dev" if DEV else "release")
STAMP = os.path.join(HERE, "_build", "linked_config")
LIB = os.path.join(HERE, "libkq_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
SOURCES = ["kq_dequant.cu", "kq_gemv.cu", "kq_moe.cu", "kq_capi.cu", "kq_noalloc.cu", "kq_gemm_sm100.cu", "kq_chain.cu", "kq_allreduce.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]
if DEV:  # development switches (GEMV debug word, timestamps)
    FLAGS.append("-DKQ_DEVELOPMENT")


def _deps():
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(HERE, "..", "include", "kq_cuda.h"))
    hdrs.append(os.path.join(CSRC, "_gen", "kq_tables.h"))
    return max(os.path.getmtime(h) for h in hdrs if os.path.exists(h))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    s = os.path.join(CSRC, src)
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(s), _deps()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    sys.path.insert(0, CSRC)
    try:
        import gen_tables
    finally:
        sys.path.pop(0)
    gen_tables.write(os.path.join(CSRC, "_gen"))
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    config = " ".join(FLAGS)
    linked = open(STAMP).read() if os.path.exists(STAMP) else None
    if (not os.path.exists(LIB) or linked != config
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        with open(STAMP, "w") as f:
            f.write(config)
    return LIB


EXT_DIR = os.path.join(HERE, "_ext")
EXT_SO = os.path.join(EXT_DIR, "kq_torch.so")


def build_torch_ext(verbose: bool = False) -> str:
    """Compile the torch C++ fast path of the decode ops (csrc/kq_torch.cpp)
    in-tree into _ext/kq_torch.so (rebuilt only when its source changed)."""
    import torch.utils.cpp_extension as ce
    os.makedirs(EXT_DIR, exist_ok=True)
    ce.load(name="kq_torch", sources=[os.path.join(CSRC, "kq_torch.cpp")], build_directory=EXT_DIR,
            extra_cflags=["-O3"], with_cuda=True, verbose=verbose)
    return EXT_SO


def load_torch_ext():
    """Import the prebuilt _ext/kq_torch.so (None when it was not built)."""
    if not os.path.exists(EXT_SO):
        return None
    import importlib.util
    import torch  # noqa: F401  (the extension links against the loaded torch libraries)
    spec = importlib.util.spec_from_file_location("kq_torch", EXT_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_torch_ext(verbose="-v" in sys.argv))
