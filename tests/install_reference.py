"""Install the reference package, unmodified, into ``baseline/_ref`` (git-ignored).

    python tests/install_reference.py --reference <path to the Aryagm/maxsim source tree>
    (or set MAXSIM_REFERENCE)

The drop-in tests (``tests/test_reference_dropin.py``) import that package and
bind its ``maxsim._maxsim_cuda`` to this library's extension module.  The
source tree is copied to a temporary directory first (the build writes next to
its sources) and installed offline with pip: ``--no-index --no-build-isolation
--no-deps`` (its one runtime dependency, NumPy, is already present).  Only the
reference's CPU extension is compiled (its CMake builds the CUDA extension only
when MAXSIM_BUILD_CUDA is set, which this recipe leaves unset).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
TARGET = REPO / "baseline" / "_ref"


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MAXSIM_REFERENCE"),
                    help="path of the reference source tree (or MAXSIM_REFERENCE)")
    ap.add_argument("--wheelhouse", default=os.environ.get("PIP_FIND_LINKS"),
                    help="extra --find-links directory for build requirements")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MAXSIM_REFERENCE")
    src = Path(args.reference)
    if not (src / "pyproject.toml").exists():
        ap.error(f"{src} is not the reference source tree (no pyproject.toml)")
    env = dict(os.environ)
    env.pop("MAXSIM_BUILD_CUDA", None)
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "maxsim-src"
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "output", "paper"))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--target", str(TARGET), str(copy)]
        if args.wheelhouse:
            cmd[4:4] = ["--find-links", args.wheelhouse]
        subprocess.run(cmd, check=True, env=env)
    print(f"installed the reference package into {TARGET}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
