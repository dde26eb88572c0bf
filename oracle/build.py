"""Build recipe for the CPU oracle (test infrastructure, not a product path).

Compiles oracle/xsg_oracle.cpp (render path), oracle/xsg_oracle_smpl.cpp
(SMPL skinning), oracle/xsg_oracle_nodes.cpp (scene assembly) and
oracle/xsg_oracle_camgrad.cpp (camera-parameter gradients) with g++
into oracle/_build/libxsg_oracle.so.
-ffp-contract=off and no -march flag keep every float operation rounded as
written, so the oracle is the plain scalar restatement of the reference's
arithmetic.  OpenMP parallelises over pixels/Gaussians for the timed CPU
baseline.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRCS = [os.path.join(HERE, f) for f in ("xsg_oracle.cpp", "xsg_oracle_smpl.cpp", "xsg_oracle_nodes.cpp",
                                             "xsg_oracle_camgrad.cpp")]
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "libxsg_oracle.so")


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(s) for s in SRCS)):
        return OUT
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp",
           "-ffp-contract=off", "-fno-fast-math", *SRCS, "-o", OUT + ".tmp"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
