"""Where the reference project's sources are, for CPU tests that read them as text or
build them (schemas, contract scripts, consumer programs).

XVRAM_REFERENCE_DIR in the environment names the directory; by default it is a
directory called `reference` beside this repository.  The GPU boxes have no copy, so
every test that needs it skips when it is absent."""
from __future__ import annotations

import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def reference_dir() -> Path:
    return Path(os.environ.get("XVRAM_REFERENCE_DIR") or (ROOT.parent / "reference"))


def reference_file(*parts: str) -> Path | None:
    """The file under the reference tree, or None when the tree (or the file) is absent."""
    p = reference_dir().joinpath(*parts)
    return p if p.exists() else None
