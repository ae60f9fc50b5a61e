"""Build recipe for the C oracle (test infrastructure only).

Compiles ``oracle/c/f5_oracle.c`` into ``oracle/_build/libf5oracle.so``
with gcc + OpenMP.  No reference source is compiled: the reference is
Python, so the oracle is a restatement, pinned by ``tests/golden``.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "c", "f5_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "libf5oracle.so")


def build(force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= os.path.getmtime(SRC)):
        return OUT
    cmd = ["gcc", "-O3", "-mavx2", "-fopenmp", "-shared", "-fPIC",
           "-o", OUT + ".tmp", SRC]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
