"""Installs the reference's own kernels, unmodified, into baseline/_ref for the GPU
comparison legs of bench.py (`--impl triton-reference`).

    python baseline/install_reference.py [--reference PATH]

The reference checkout has no packaging (`pip install --target baseline/_ref <checkout>`
stops with "Neither 'setup.py' nor 'pyproject.toml' found").  This copies the checkout to a
temporary directory, adds a pyproject.toml that only lists the modules of its kernels/
directory (no source file is changed), and installs that copy with pip's offline options
(--no-index --no-build-isolation --find-links /opt/wheelhouse --target baseline/_ref).
baseline/_ref is not committed; it travels to the GPU box with the working tree.  Nothing
in the product package imports it.
"""

from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"

PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "dory-vllm-experiments-reference-kernels"
version = "0"

[tool.setuptools]
package-dir = {{"" = "kernels"}}
py-modules = [{modules}]
"""


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default="/root/reference",
                    help="checkout of chrisbennight/dory-vllm-experiments (read only)")
    args = ap.parse_args()
    src = Path(args.reference)
    if not (src / "kernels").is_dir():
        print(f"no kernels/ directory under {src}", file=sys.stderr)
        return 1
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "reference"
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "results", "docs"))
        modules = sorted(p.stem for p in (copy / "kernels").glob("*.py"))
        (copy / "pyproject.toml").write_text(
            PYPROJECT.format(modules=", ".join(f'"{m}"' for m in modules)))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--find-links", "/opt/wheelhouse", "--no-deps", "--target", str(TARGET),
               str(copy)]
        print(" ".join(cmd), flush=True)
        return subprocess.run(cmd).returncode


if __name__ == "__main__":
    sys.exit(main())
