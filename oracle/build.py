"""Build the C oracle (asa_oracle.c) into oracle/libasa_oracle.so.

TEST INFRASTRUCTURE ONLY.  -ffp-contract=off keeps the host compiler from
adding FMA contractions the source does not spell out; the source writes the
FMAs nvcc would emit for the reference explicitly.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "asa_oracle.c")
LIB = os.path.join(HERE, "libasa_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c11",
           "-shared", "-fPIC", SRC, "-o", LIB + ".tmp", "-lm"]
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
