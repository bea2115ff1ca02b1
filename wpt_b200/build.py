"""Builds libwpt_b200.so in-tree for sm_100a with nvcc (no torch headers:
the library is plain CUDA behind a C ABI, include/wpt_attn.h).

    python -m wpt_b200.build            # build if a source is newer
    python -m wpt_b200.build --force
"""

import argparse
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
TARGET = os.path.join(HERE, "libwpt_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    home = os.environ.get("CUDA_HOME") or "/usr/local/cuda"
    found = shutil.which("nvcc") or os.path.join(home, "bin", "nvcc")
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  [os.path.join(ROOT, "include", "wpt_attn.h")])


def stale():
    if not os.path.exists(TARGET):
        return True
    built = os.path.getmtime(TARGET)
    return any(os.path.getmtime(s) > built for s in sources())


def build(force=False, verbose=False):
    """Compiles the library when a source is newer than it (or force)."""
    if not force and not stale():
        return TARGET
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", os.path.join(ROOT, "include"), "-o", TARGET + ".tmp", os.path.join(CSRC, "wpt_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(TARGET + ".tmp", TARGET)
    return TARGET


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.verbose))
