"""Build libmoc_b200.so in-tree: ``python -m moc.build`` (runs ``make -C csrc``)."""
from __future__ import annotations

import os
import subprocess
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(_HERE), "csrc")


def build(jobs: int | None = None, verbose: bool = False) -> str:
    jobs = jobs or os.cpu_count() or 4
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError(f"building libmoc_b200.so failed:\n{out[-4000:]}")
    return os.path.join(_HERE, "libmoc_b200.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
