"""Build recipe for the CPU oracle (test infrastructure): g++ -> _build/liboracle.so.

The flags keep IEEE single-precision semantics (no FMA contraction, no
fast-math) so the oracle's fp32 steps round exactly like the CUDA kernels'.
x86-64-v3 (AVX2/FMA) runs on any current server CPU, so the .so built here
also runs on the GPU box's host.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "fmoe_oracle.cpp")
OUT = os.path.join(HERE, "_build", "liboracle.so")
CXX = os.environ.get("FMOE_ORACLE_CXX", "g++")  # the system g++ (ships libgomp)
FLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c++17", "-ffp-contract=off",
         "-fno-fast-math"]


def build(force=False):
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    if force or not os.path.exists(OUT) or os.path.getmtime(OUT) < os.path.getmtime(SRC):
        r = subprocess.run([CXX, *FLAGS, SRC, "-o", OUT], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force="-f" in sys.argv))
