"""Build libqres.so (sm_100a) in-tree: ``python -m tt_qwen_resident_b200.build``."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs=8, verbose=False):
    csrc = os.path.join(HERE, "csrc")
    cmd = ["make", "-C", csrc, f"-j{jobs}"]
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        sys.stderr.write((r.stdout or "") + (r.stderr or ""))
        raise RuntimeError("building libqres.so failed")
    return os.path.join(HERE, "libqres.so")


if __name__ == "__main__":
    print(build(verbose=True))
