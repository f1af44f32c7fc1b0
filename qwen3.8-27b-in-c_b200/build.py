"""Build recipe for the in-tree shared libraries of this package.

    python qwen3.8-27b-in-c_b200/build.py [--verbose]

Produces, next to this file:
  libqwenb200.so  CUDA engine + C ABI (include/qwen_b200.h), sm_100a only
  libqbsynth.so   seeded synthetic GGUF writer (host C)
and, when the reference sources are present, the parity checker
oracle/_ref/libqwenref.so (oracle/Makefile).
"""
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")

CU_SOURCES = ["qb_quant.cu", "qb_qmv_tc.cu", "qb_layers.cu", "qb_sample.cu", "qb_engine.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
    "--expt-relaxed-constexpr",
    "-I", CSRC, "-I", INCLUDE,
]


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_engine(verbose=False, force=False, extra_flags=(), out=None, objdir=None):
    nvcc = _nvcc()
    out = out or os.path.join(PKG, "libqwenb200.so")
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INCLUDE, "qwen_b200.h"))
    objs = []
    objdir = objdir or os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            _run([nvcc, *NVCC_FLAGS, *extra_flags, "-c", s, "-o", o], verbose)
    if force or _stale(out, objs):
        _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", out, *objs,
              "-Xlinker", "-Bsymbolic"], verbose)
    return out


def build_synth(verbose=False, force=False):
    out = os.path.join(PKG, "libqbsynth.so")
    src = os.path.join(CSRC, "synth_gguf.c")
    if force or _stale(out, [src, os.path.join(CSRC, "synth_gguf.h")]):
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-o", out, src, "-lm", "-lpthread"], verbose)
    return out


def reference_dir():
    """Where the reference checkout lies: $QB_REFERENCE_DIR, else a directory
    named "reference" beside this repository.  None when neither has the
    reference sources (the parity checker is then not built here)."""
    ref = os.environ.get("QB_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
    return ref if os.path.isfile(os.path.join(ref, "src", "model.c")) else None


def build_oracle(verbose=False, clis=False):
    """The checker: compiled only where the reference sources exist.  With clis, also
    the reference CLI on the reference engine and relinked against libqwenb200 (the
    end-to-end CLI test; the library must be built first)."""
    ref = reference_dir()
    if ref is None:
        return None
    targets = ["all", "reference-cli", "relink-cli"] if clis else ["all"]
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={ref}", *targets], verbose)
    return os.path.join(ROOT, "oracle", "_ref", "libqwenref.so")


def build_all(verbose=False, force=False):
    build_synth(verbose, force)
    out = build_engine(verbose, force)
    build_oracle(verbose, clis=True)
    return out


if __name__ == "__main__":
    v = "--verbose" in sys.argv or "-v" in sys.argv
    f = "--force" in sys.argv
    print(build_all(verbose=v, force=f))
