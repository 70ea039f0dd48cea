"""Build libdw_moe.so in-tree for sm_100a: ``python dw_tpu_b200/build.py``
(or ``python __graft_entry__.py``). Run it as a script: importing the
package loads the library, which a fresh checkout does not have yet."""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(jobs: int | None = None, verbose: bool = False) -> str:
    jobs = jobs or min(8, os.cpu_count() or 1)
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError(f"building libdw_moe.so failed:\n{out[-4000:]}")
    return os.path.join(HERE, "libdw_moe.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
