"""Copy the reference's digests of its format tables into
tests/golden/format_tables.json.

    python tests/golden/make_signmag.py [reference_root]

The reference's tests/golden/checksums.json holds, for every width sf4..sf16,
the sha256 of the canonical table "code<TAB>sign-magnitude word in hex<TAB>
repr(code / 2^(N-1))" over every code (tests/test_1_0_1_types_casts.py:311-335
in the reference); tests/test_signmag_oracle.py rebuilds the table from the
oracle and checks the digest.
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref: str | None = None) -> None:
    ref = reference_root(ref)
    with open(os.path.join(ref, "tests", "golden", "checksums.json")) as f:
        sums = json.load(f)
    out = {"source": "reference tests/golden/checksums.json", "line": "{code}\\t{word:0{(N+3)//4}x}\\t{value!r}\\n",
           "sha256": sums}
    with open(os.path.join(HERE, "format_tables.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote format_tables.json")


if __name__ == "__main__":
    main(*sys.argv[1:])
