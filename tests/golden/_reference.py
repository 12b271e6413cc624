"""Where the fixture generators find the reference kvcompress sources.

The generators import the reference package (never copy it) to record its
outputs.  Its source tree is named on the command line
(``--reference PATH``) or in the ``KVCOMPRESS_REFERENCE`` environment
variable: the directory that contains the ``kvcompress`` package.
"""

from __future__ import annotations

import os
import sys

ENV = "KVCOMPRESS_REFERENCE"


def reference_root(argv: list[str] | None = None) -> str:
    """The reference source tree from ``--reference PATH`` or ``$KVCOMPRESS_REFERENCE``."""
    argv = sys.argv[1:] if argv is None else argv
    root = None
    for i, a in enumerate(argv):
        if a == "--reference" and i + 1 < len(argv):
            root = argv[i + 1]
        elif a.startswith("--reference="):
            root = a.split("=", 1)[1]
    root = root or os.environ.get(ENV)
    if not root:
        raise SystemExit(f"name the reference source tree: --reference PATH or {ENV}=PATH")
    if not os.path.isdir(os.path.join(root, "kvcompress")):
        raise SystemExit(f"{root!r} has no kvcompress package")
    return os.path.abspath(root)


def import_reference(argv: list[str] | None = None) -> str:
    """Put the reference first on ``sys.path`` (and this repository after it)."""
    root = reference_root(argv)
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, root)
    sys.path.insert(1, os.path.abspath(os.path.join(here, "..", "..")))
    return root
