"""Build ``libnested_ssm.so`` (the C-ABI library) in-tree for sm_100a with nvcc.

The library has no torch dependency: plain ``extern "C"`` entry points over
device pointers (``include/nested_ssm.h``).  ``python -m nested_ssm_b200.build``
rebuilds it; ``--ptxas`` also prints the per-kernel register / spill report.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libnested_ssm.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = ["nssm_abi.cu", "nssm_pb16.cu", "nssm_pb32.cu", "nssm_pb64.cu", "nssm_static.cu", "nssm_scan.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _deps() -> list[str]:
    out = [os.path.join(INCLUDE, "nested_ssm.h")]
    for f in os.listdir(CSRC):
        if f.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(CSRC, f))
    return out


def is_stale(lib: str = LIB_PATH) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(d) > t for d in _deps())


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False,
          out: str | None = None, defines: list[str] | None = None) -> str:
    """Compile the library if it is missing or older than its sources; return its path.
    ``out`` / ``defines`` build a variant elsewhere (e.g. ``["NSSM_STEP_MINB=3"]``)."""
    target = out or LIB_PATH
    if not force and out is None and not is_stale():
        return LIB_PATH
    common = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC]
    for d in defines or []:
        common.append("-D" + d)
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    objdir = target + ".objs"
    os.makedirs(objdir, exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc_path(), *common, "-c", os.path.join(CSRC, src), "-o", obj]
        if not quiet:
            print("[nested_ssm_b200] " + " ".join(cmd), file=sys.stderr)
        procs.append((obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    objs, errs = [], []
    for obj, pr in procs:
        out, err = pr.communicate()
        if pr.returncode != 0:
            errs.append(f"{obj}: nvcc failed ({pr.returncode}):\n{out}\n{err}")
        elif ptxas_verbose:
            print(err, file=sys.stderr)
        objs.append(obj)
    if errs:
        raise RuntimeError("\n".join(errs))
    link = [nvcc_path(), *ARCH_FLAGS, "--shared", "-o", target + ".tmp", *objs]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    shutil.rmtree(objdir, ignore_errors=True)
    os.replace(target + ".tmp", target)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/spill report")
    ap.add_argument("--out", default=None, help="build a variant library at this path")
    ap.add_argument("-D", dest="defines", action="append", default=[], help="extra preprocessor define")
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas, ptxas_verbose=a.ptxas, out=a.out, defines=a.defines))
