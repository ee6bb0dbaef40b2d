"""Build the C restatement of the oracle (test infrastructure only):

    python oracle/build_oracle.py

Compiles ``oracle/ckpt_scan.c`` with gcc -O3 -fopenmp into
``oracle/libmrorc.so`` (git-ignored; it travels to the GPU box with the tree).
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ckpt_scan.c")
OUT = os.path.join(HERE, "libmrorc.so")


def build(force=False):
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-o", OUT, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
