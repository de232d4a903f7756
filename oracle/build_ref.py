"""Recipe: compile the reference's own C MX accumulator into oracle/_ref/.

The reference keeps its C loop as a string constant ``_SRC`` in
src/sf/_fastmx.py (lines 41-85) and compiles it at import time with
``cc -O3 -shared -fPIC -std=c99`` (src/sf/_fastmx.py:87).  This recipe reads
that constant from the reference tree (parsed, not imported), writes it to a
temporary file outside the repository and compiles it with the same flags
into ``oracle/_ref/libmx_ref.so``.  Nothing from the reference is copied into
the repository; ``oracle/_ref/`` is git-ignored.

Usage: python oracle/build_ref.py [reference_root]
The root (the directory holding src/sf) is the argument, else the
SF_REFERENCE_ROOT environment variable, else the checkout this build
container mounts read-only beside the repository.  Exits 0 without building
when no reference tree is found (the GPU machines have none; they use the
library built here).
"""
from __future__ import annotations

import ast
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "libmx_ref.so")


def extract(ref_root: str) -> str:
    path = os.path.join(ref_root, "src", "sf", "_fastmx.py")
    tree = ast.parse(open(path).read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "_SRC" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError(f"no _SRC constant in {path}")


# where this build container mounts the reference checkout
MOUNTED_CHECKOUT = "/root/reference"


def main(ref_root: str | None = None) -> int:
    ref_root = ref_root or os.environ.get("SF_REFERENCE_ROOT") or MOUNTED_CHECKOUT
    if not os.path.isdir(os.path.join(ref_root, "src", "sf")):
        print(f"build_ref: no reference tree at {ref_root}; oracle/_ref not built")
        return 0
    src = extract(ref_root)
    cc = shutil.which(os.environ.get("CC", "gcc")) or shutil.which("cc")
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "mx_acc.c")
        with open(c, "w") as f:
            f.write(src)
        subprocess.run([cc, "-O3", "-shared", "-fPIC", "-std=c99", c, "-o", OUT], check=True)
    print(f"build_ref: built {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main(*sys.argv[1:]))
