"""Installs the reference project, unmodified, into baseline/_ref (git-ignored; it travels to
the GPU machines with the working tree).

  python baseline/build_ref.py [--reference /path/to/reference/checkout]

1. The offline pip install of the reference checkout, from a copy in a temporary directory
   (the build writes into its source tree), with TORCH_CUDA_ARCH_LIST=10.0a so that the
   reference's own setup.py -- which pins sm_120 by default and lets the environment override
   it (its setup.py:11,45) -- builds its CUDA extension decode_kernels.cuda._ext for sm_100a.
   The reference's setup() declares no Python packages, so this installs the compiled module
   alone.
2. The reference's sources beside it, as its checkout lays them out: decode_kernels/ (its cuda
   wrapper and its PyTorch oracle, decode_kernels/reference), the benchmarks/ harness, tests/,
   conftest.py, and setup.py with csrc/ (its build-contract tests import setup.py and list
   csrc/).

What uses it: bench.py's reference_gpu measurement (the reference's kernels, rebuilt for
sm_100a, on the same GPU) and cpu_baseline_torch (the reference's PyTorch oracle on the host
cores), and tests/test_reference_suite_gpu.py, which runs the reference's own kernel tests
through the drop-in shim. Nothing in the product imports it.

The checkout is found from --reference or DECODE_REFERENCE_ROOT; nothing is copied into the
tracked tree.
"""
import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
PY_TREES = ("decode_kernels", "benchmarks", "tests", "csrc")
PY_FILES = ("conftest.py", "setup.py")


def install(reference, jobs):
    if os.path.isdir(TARGET):
        shutil.rmtree(TARGET)
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "reference")
        shutil.copytree(reference, src, ignore=shutil.ignore_patterns("results", "__pycache__",
                                                                      "*.so", "build"))
        env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a", MAX_JOBS=str(jobs))
        log = os.path.join(HERE, "_ref_build.log")
        with open(log, "w") as f:
            subprocess.run([sys.executable, "-m", "pip", "install", "-v", "--no-index",
                            "--no-build-isolation", "--find-links", "/opt/wheelhouse",
                            "--target", TARGET, src], check=True, env=env, stdout=f,
                           stderr=subprocess.STDOUT)
        with open(log) as f:
            text = f.read()
        if "arch=compute_100a,code=sm_100a" not in text:
            raise SystemExit(f"the reference extension was not built for sm_100a; see {log}")
        for name in PY_TREES:
            dst = os.path.join(TARGET, name)
            shutil.copytree(os.path.join(src, name), dst, dirs_exist_ok=True,
                            ignore=shutil.ignore_patterns("__pycache__"))
        for name in PY_FILES:
            shutil.copy2(os.path.join(src, name), os.path.join(TARGET, name))
    ext = [f for f in os.listdir(os.path.join(TARGET, "decode_kernels", "cuda"))
           if f.startswith("_ext") and f.endswith(".so")]
    if not ext:
        raise SystemExit("the install produced no decode_kernels/cuda/_ext*.so")
    print(f"reference installed in {TARGET} ({ext[0]}, built for sm_100a)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DECODE_REFERENCE_ROOT"))
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(a.reference):
        raise SystemExit("pass --reference or set DECODE_REFERENCE_ROOT to the reference checkout")
    install(os.path.abspath(a.reference), a.jobs)


if __name__ == "__main__":
    main()
