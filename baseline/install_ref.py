"""Installs the reference (Workers-Intelligence-Commons/wpt) into
baseline/_ref, for bench.py's reference legs and the end-to-end decode
(config 5). Nothing in the product imports it.

    python baseline/install_ref.py --reference <the reference repository>

First it runs the offline pip install the build prescribes:

    python -m pip install --no-index --no-build-isolation \\
        --find-links /opt/wheelhouse --target baseline/_ref <reference>

In this image that fails: the reference's packages are built by uv_build
(packages/*/pyproject.toml), which the offline wheelhouse does not hold, so
pip cannot even read their metadata. The packages this build needs
(wpt-model, wpt-inference, wpt-utils, wpt-tokenizer) are pure Python, so
the script then does what pip --target would have done with them: it
places each package's source tree, unmodified, at baseline/_ref/<name>.
baseline/_ref is git-ignored (never committed) and travels to the GPU box
with the working tree.
"""

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
PACKAGES = {"wpt_model": "wpt-model", "wpt_inference": "wpt-inference", "wpt_utils": "wpt-utils",
            "wpt_tokenizer": "wpt-tokenizer"}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("WPT_REFERENCE"),
                        required="WPT_REFERENCE" not in os.environ,
                        help="the reference repository's root (or set WPT_REFERENCE)")
    parser.add_argument("--wheelhouse", default="/opt/wheelhouse")
    args = parser.parse_args()
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           args.wheelhouse, "--target", TARGET, args.reference]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode == 0:
        print("pip install: ok")
        return
    reason = "uv_build" if "uv_build" in (done.stdout + done.stderr) else f"exit {done.returncode}"
    print(f"pip install failed ({reason}); placing the pure-Python packages' source trees instead")
    os.makedirs(TARGET, exist_ok=True)
    for name, package in PACKAGES.items():
        source = os.path.join(args.reference, "packages", package, "src", name)
        if not os.path.isdir(source):
            raise SystemExit(f"{source} is missing")
        dest = os.path.join(TARGET, name)
        if os.path.isdir(dest):
            shutil.rmtree(dest)
        shutil.copytree(source, dest, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        print(f"{name}: {source} -> {dest}")


if __name__ == "__main__":
    main()
