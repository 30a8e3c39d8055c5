"""Build the Q6W sm_100a shared library in-tree.

    python build.py            # -> q6w_b200/libq6w_b200.so

The library is plain nvcc output with an ``extern "C"`` ABI (see
include/q6w_b200.h); it links only the CUDA runtime, no torch.
"""

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = ["csrc/codec.cu", "csrc/linear.cu", "csrc/model.cu"]
OUT = HERE / "q6w_b200" / "libq6w_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def build(verbose=False, jobs=None):
    inc = ["-I", str(ROOT / "include"), "-I", str(HERE / "csrc")]
    objs = []
    procs = []
    tmp = HERE / "_build"
    tmp.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = tmp / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, *inc, "-c", str(HERE / src), "-o", str(obj)]
        procs.append((src, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    logs = []
    for src, obj, p in procs:
        out, _ = p.communicate()
        logs.append(f"== {src}\n{out}")
        if p.returncode != 0:
            sys.stderr.write(out)
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(str(obj))
    link = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *objs, "-lcudart"]
    subprocess.run(link, check=True)
    (tmp / "ptxas.log").write_text("\n".join(logs))
    if verbose:
        print("\n".join(logs))
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
