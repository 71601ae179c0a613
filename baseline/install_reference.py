"""Install the unmodified reference into baseline/_ref (git-ignored; it travels with the tree).

The reference checkout has neither setup.py nor pyproject.toml, so
``pip install --target baseline/_ref <reference>`` refuses it ("Directory is
not installable").  This recipe tries that command first and, when it fails,
copies the reference's Python packages unchanged into baseline/_ref, which is
what the pip install would have placed there.  bench.py's GPU comparator leg
loads kernels/flash_attention.py from there.

Usage:  python baseline/install_reference.py REFERENCE_ROOT
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def main(src: str) -> int:
    src = os.path.abspath(src)
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
                        "/opt/wheelhouse", "--target", DEST, src], capture_output=True, text=True)
    if r.returncode == 0:
        print("pip install succeeded")
        return 0
    print("pip install failed:", (r.stderr.strip().splitlines() or ["?"])[-1])
    os.makedirs(DEST, exist_ok=True)
    for pkg in ("kernels", "core", "transformer"):
        dst = os.path.join(DEST, pkg)
        if os.path.exists(dst):
            shutil.rmtree(dst)
        shutil.copytree(os.path.join(src, pkg), dst, ignore=shutil.ignore_patterns("__pycache__", "*.pt"))
    with open(os.path.join(DEST, "SOURCE"), "w") as f:
        f.write(f"copied unchanged from {src}\n")
    print(f"copied kernels/, core/, transformer/ into {DEST}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PIE_REFERENCE_ROOT", "")))
