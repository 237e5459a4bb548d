"""Location of the reference checkout read by the checker build recipes.

One environment variable, FALCOM_REFERENCE_ROOT, names it; the recipes here
(oracle/Makefile, oracle/build_ref_gpu.py, the manifest generator) take it
from this function.  Nothing that runs on a GPU box reads the reference: the
checker binaries it produces travel as built files under oracle/_ref/.
"""
from __future__ import annotations

import os

DEFAULT = "/root/reference"


def reference_root() -> str:
    """The reference checkout: $FALCOM_REFERENCE_ROOT, else the recipe
    default; "" when neither exists."""
    root = os.environ.get("FALCOM_REFERENCE_ROOT", DEFAULT)
    return root if os.path.isdir(root) else ""
