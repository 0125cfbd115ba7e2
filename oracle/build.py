"""Build recipe for the oracle's C restatement (test infrastructure only).

Compiles ``oracle/gdn_recurrent.c`` into ``oracle/_build/libgdn_oracle.so`` with gcc + OpenMP.
Generic x86-64-v2 code and no floating-point contraction, so the same binary gives the same
results on this container and on the GPU hosts.
"""

from __future__ import annotations

import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_build" / "libgdn_oracle.so"


def build_oracle(force: bool = False) -> pathlib.Path:
    src = HERE / "gdn_recurrent.c"
    if OUT.exists() and not force and OUT.stat().st_mtime >= src.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-o", str(OUT),
           str(src), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build_oracle(force=True))
