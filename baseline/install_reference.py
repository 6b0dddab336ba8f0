"""Install the reference's Python package (mantisnet) into baseline/_ref.

    python baseline/install_reference.py --reference <path to the reference checkout>

The package's declared build backend (hatchling) is not in this image's
offline wheelhouse, so the package directory is copied to a temporary folder
whose pyproject names setuptools as the backend instead (same package, same
files installed), and pip installs it offline, without dependencies, into
baseline/_ref (git-ignored; it travels to GPU boxes with the working tree).
Its one compiled dependency, the hexo_py extension, is not buildable here;
the importing code installs a stub module carrying MODEL_REPR_VERSION, the
only attribute the package reads at import time (builder.py:26).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HEXO_REFERENCE"),
                    help="the reference checkout (the directory holding python/mantisnet)")
    ap.add_argument("--wheelhouse", default="/opt/wheelhouse")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <checkout> or set HEXO_REFERENCE")
    src = Path(args.reference) / "python" / "mantisnet"
    with tempfile.TemporaryDirectory() as tmp:
        pkg = Path(tmp) / "mantisnet"
        shutil.copytree(src, pkg)
        meta = (pkg / "pyproject.toml").read_text()
        meta = meta.replace('requires = ["hatchling"]\nbuild-backend = "hatchling.build"',
                            'requires = ["setuptools"]\nbuild-backend = "setuptools.build_meta"')
        meta = meta.replace('[tool.hatch.build.targets.wheel]\npackages = ["mantisnet"]',
                            '[tool.setuptools]\npackages = { find = { include = ["mantisnet", "mantisnet.*"] } }')
        (pkg / "pyproject.toml").write_text(meta)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", args.wheelhouse, "--target", str(HERE / "_ref"), "--upgrade", str(pkg)]
        return subprocess.call(cmd)


if __name__ == "__main__":
    sys.exit(main())
