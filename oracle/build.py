"""Build the CPU oracle (test infrastructure) into oracle/_build/liboracle.so.

    python oracle/build.py
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_build", "liboracle.so")
SOURCES = [os.path.join(HERE, "radix_oracle.c")]
CXX_SOURCES = [os.path.join(HERE, "cpu_sorts.cpp")]
DEPS = SOURCES + CXX_SOURCES + [os.path.join(HERE, "radix_oracle.h"), os.path.abspath(__file__)]


def build(force: bool = False) -> str:
    if (not force and os.path.exists(OUT)
            and all(os.path.getmtime(d) <= os.path.getmtime(OUT) for d in DEPS)):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    tmp = OUT + ".tmp"
    obj = os.path.join(os.path.dirname(OUT), "radix_oracle.o")
    subprocess.run(["gcc", "-O2", "-std=c11", "-fPIC", "-pthread", "-c", "-o", obj, *SOURCES],
                   check=True)
    subprocess.run(["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-o", tmp,
                    obj, *CXX_SOURCES], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
