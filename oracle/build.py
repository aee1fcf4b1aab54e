"""Build recipe for the CPU oracle (test infrastructure: the checker, never the product path).

Compiles rope_kv_oracle.c into oracle/liboracle_rope_kv.so. -ffp-contract=off keeps every
multiply and add separately rounded, as PyTorch's eager elementwise kernels are. OpenMP lets the
CPU baseline use every host core; a compiler without libgomp gets a single-threaded build.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "rope_kv_oracle.c")
OUT = os.path.join(HERE, "liboracle_rope_kv.so")
BASE_FLAGS = ["-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-Wall"]


def _compilers():
    seen = []
    for cand in ("gcc", "/usr/bin/gcc", os.environ.get("CC")):
        path = shutil.which(cand) if cand else None
        if path and path not in seen:
            seen.append(path)
    return seen


def build(force=False, verbose=False):
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= os.path.getmtime(SRC)):
        return OUT
    errors = []
    for openmp in (True, False):
        for cc in _compilers():
            cmd = [cc] + BASE_FLAGS + (["-fopenmp"] if openmp else []) + [SRC, "-o", OUT]
            proc = subprocess.run(cmd, capture_output=True, text=True)
            if verbose:
                print(" ".join(cmd), proc.stdout, proc.stderr, file=sys.stderr)
            if proc.returncode == 0:
                return OUT
            errors.append(f"{' '.join(cmd)}: {proc.stderr.strip()[-300:]}")
    raise RuntimeError("could not build the CPU oracle:\n" + "\n".join(errors))


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
