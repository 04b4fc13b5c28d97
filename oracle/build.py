"""Build the oracle's C restatement (test infrastructure): oracle/liboracle.so.

    python oracle/build.py

gcc -O2 -fopenmp -ffp-contract=off: every float expression rounds as written.
The reference (SimonDanisch/Mantle.jl) is pure Julia with no C sources, so
there is no oracle/_ref build of the reference itself.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRCS = [HERE / "mantle_oracle.c", HERE / "showcase_oracle.c", HERE / "raster_oracle.c"]
OUT = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    if not force and OUT.exists() and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in SRCS):
        return OUT
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(OUT), *map(str, SRCS), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
