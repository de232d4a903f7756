"""Where the fixture generators find the reference checkout: the
``reference_root`` argument, else the SF_REFERENCE_ROOT environment variable
(the directory holding src/sf)."""
from __future__ import annotations

import os
import sys


def reference_root(arg: str | None = None) -> str:
    root = arg or os.environ.get("SF_REFERENCE_ROOT")
    if not root or not os.path.isdir(os.path.join(root, "src", "sf")):
        sys.exit("pass the reference checkout (the directory holding src/sf) as the argument or in "
                 "SF_REFERENCE_ROOT")
    return root
