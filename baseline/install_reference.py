"""Installs the reference's GPU kernels for the Triton baseline leg of bench.py.

The reference is a Rust crate whose GPU arithmetic is one Triton module,
kernels/ops.py; its Rust runtime cannot be built in this image (no cargo), and the
crate has no Python packaging, so `pip install --target baseline/_ref <reference>`
fails ("Neither 'setup.py' nor 'pyproject.toml' found").  This script copies that
module, unmodified, to baseline/_ref/kernels/ops.py (git-ignored; it travels with
the working tree to the machine that runs the benchmark) and records its SHA-256.

Usage: python baseline/install_reference.py <reference tree>
"""
from __future__ import annotations

import hashlib
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    source = Path(sys.argv[1]) / "kernels" / "ops.py"
    if not source.exists():
        sys.exit(f"{source} not found")
    target = HERE / "_ref" / "kernels"
    target.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(source, target / "ops.py")
    digest = hashlib.sha256(source.read_bytes()).hexdigest()
    (HERE / "_ref" / "INSTALLED.json").write_text(json.dumps({"module": "kernels/ops.py", "sha256": digest}) + "\n")
    print(f"installed {source} -> {target / 'ops.py'} (sha256 {digest})")


if __name__ == "__main__":
    main()
