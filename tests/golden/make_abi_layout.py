#!/usr/bin/env python3
"""Regenerate tests/golden/abi_layout.json from the reference's public headers.

    python tests/golden/make_abi_layout.py [/path/to/reference]

Compiles abi_layout_dump.c against <reference>/include and stores what it prints.  The
reference directory defaults to XVRAM_REFERENCE_DIR, else `reference` beside this
repository.  tests/test_abi_layout.py compiles the same program against
this repository's include/ and requires identical output.
"""
from __future__ import annotations

import json
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def dump(include_args: list[str], defines: list[str]) -> dict:
    with tempfile.TemporaryDirectory() as tmp:
        exe = Path(tmp) / "dump"
        subprocess.run(["gcc", "-std=c11", "-O0", *defines, *include_args, "-o", str(exe),
                        str(HERE / "abi_layout_dump.c")], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return json.loads(out)


def main() -> None:
    sys.path.insert(0, str(HERE.parent))
    from reference_tree import reference_dir
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_dir()
    layout = dump(["-I", str(ref / "include")], [])
    (HERE / "abi_layout.json").write_text(json.dumps(layout, indent=1, sort_keys=True) + "\n")
    print(f"{len(layout)} entries")


if __name__ == "__main__":
    main()
